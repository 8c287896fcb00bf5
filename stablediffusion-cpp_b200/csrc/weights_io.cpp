// weights_io.cpp - checkpoints in the .safetensors format, read on the host the way the
// reference reads them (safetensors.cpp:80-168, Weights::load_model :170-194) and, for
// tensor parallelism, cut to one rank's shard before anything is uploaded.
//
// File layout: an 8-byte little-endian header length N, N bytes of JSON
// {name: {"dtype", "shape", "data_offsets": [begin, end]}, "__metadata__": {...}}, then
// the tensor bytes (offsets relative to that section). The file is memory-mapped.
// F32 / F16 / BF16 tensors are read (other dtypes are skipped): with keep_bf16 a tensor
// of at least bf16_min_numel elements is kept as BF16 (F16 and F32 rounded to nearest
// even), anything smaller as F32 - the reference's rule. Shards of one model are found
// as load_model finds them: <dir>/<base>.safetensors, the files named by
// <dir>/<base>.safetensors.index.json, or <dir>/<base>.fp16.safetensors.
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <cstdint>
#include <cstring>
#include <fstream>
#include <functional>
#include <map>
#include <memory>
#include <sstream>
#include <stdexcept>
#include <string>
#include <thread>
#include <vector>

#include "weights_io.h"

namespace sdb {
namespace {

// ---- a small JSON reader (objects, arrays, strings, numbers, literals) -------------
struct JVal {
  enum Kind { Null, Bool, Num, Str, Arr, Obj } kind = Null;
  double num = 0.0;
  bool b = false;
  std::string str;
  std::vector<JVal> arr;
  std::vector<std::pair<std::string, JVal>> obj;
  const JVal* find(const std::string& k) const {
    for (const auto& kv : obj)
      if (kv.first == k) return &kv.second;
    return nullptr;
  }
};

struct JParser {
  const char* p;
  const char* end;
  [[noreturn]] void bad(const char* what) const { throw std::runtime_error(std::string("json: ") + what); }
  void ws() {
    while (p < end && (*p == ' ' || *p == '\n' || *p == '\r' || *p == '\t')) ++p;
  }
  JVal value() {
    ws();
    if (p >= end) bad("unexpected end");
    JVal v;
    if (*p == '{') {
      v.kind = JVal::Obj;
      ++p;
      ws();
      if (p < end && *p == '}') {
        ++p;
        return v;
      }
      for (;;) {
        ws();
        if (p >= end || *p != '"') bad("expected a key");
        std::string k = string();
        ws();
        if (p >= end || *p != ':') bad("expected ':'");
        ++p;
        v.obj.emplace_back(std::move(k), value());
        ws();
        if (p < end && *p == ',') {
          ++p;
          continue;
        }
        if (p < end && *p == '}') {
          ++p;
          return v;
        }
        bad("expected ',' or '}'");
      }
    }
    if (*p == '[') {
      v.kind = JVal::Arr;
      ++p;
      ws();
      if (p < end && *p == ']') {
        ++p;
        return v;
      }
      for (;;) {
        v.arr.push_back(value());
        ws();
        if (p < end && *p == ',') {
          ++p;
          continue;
        }
        if (p < end && *p == ']') {
          ++p;
          return v;
        }
        bad("expected ',' or ']'");
      }
    }
    if (*p == '"') {
      v.kind = JVal::Str;
      v.str = string();
      return v;
    }
    if (end - p >= 4 && !std::strncmp(p, "true", 4)) {
      p += 4;
      v.kind = JVal::Bool;
      v.b = true;
      return v;
    }
    if (end - p >= 5 && !std::strncmp(p, "false", 5)) {
      p += 5;
      v.kind = JVal::Bool;
      return v;
    }
    if (end - p >= 4 && !std::strncmp(p, "null", 4)) {
      p += 4;
      return v;
    }
    // number
    const char* s = p;
    while (p < end && (std::strchr("+-0123456789.eE", *p) != nullptr)) ++p;
    if (p == s) bad("unexpected character");
    v.kind = JVal::Num;
    v.num = std::stod(std::string(s, p));
    return v;
  }
  std::string string() {
    ++p;  // opening quote
    std::string out;
    while (p < end && *p != '"') {
      if (*p == '\\') {
        ++p;
        if (p >= end) bad("bad escape");
        const char c = *p++;
        switch (c) {
          case 'n': out += '\n'; break;
          case 't': out += '\t'; break;
          case 'r': out += '\r'; break;
          case 'b': out += '\b'; break;
          case 'f': out += '\f'; break;
          case 'u': {
            if (end - p < 4) bad("bad \\u escape");
            const unsigned cp = (unsigned)std::stoul(std::string(p, p + 4), nullptr, 16);
            p += 4;
            if (cp < 0x80) {
              out += (char)cp;
            } else if (cp < 0x800) {
              out += (char)(0xC0 | (cp >> 6));
              out += (char)(0x80 | (cp & 0x3F));
            } else {
              out += (char)(0xE0 | (cp >> 12));
              out += (char)(0x80 | ((cp >> 6) & 0x3F));
              out += (char)(0x80 | (cp & 0x3F));
            }
            break;
          }
          default: out += c;  // \" \\ \/
        }
      } else {
        out += *p++;
      }
    }
    if (p >= end) bad("unterminated string");
    ++p;
    return out;
  }
};

JVal parse_json(const std::string& text) {
  JParser j{text.data(), text.data() + text.size()};
  return j.value();
}

// ---- memory-mapped file ----------------------------------------------------------
struct Mapped {
  void* base = nullptr;
  size_t size = 0;
  explicit Mapped(const std::string& path) {
    const int fd = ::open(path.c_str(), O_RDONLY);
    if (fd < 0) throw std::runtime_error("cannot open " + path);
    struct stat st;
    if (fstat(fd, &st) != 0) {
      ::close(fd);
      throw std::runtime_error("cannot stat " + path);
    }
    size = (size_t)st.st_size;
    base = size ? mmap(nullptr, size, PROT_READ, MAP_PRIVATE, fd, 0) : nullptr;
    ::close(fd);
    if (base == MAP_FAILED) {
      base = nullptr;
      throw std::runtime_error("mmap failed for " + path);
    }
  }
  ~Mapped() {
    if (base) munmap(base, size);
  }
  Mapped(const Mapped&) = delete;
  Mapped& operator=(const Mapped&) = delete;
};

bool exists(const std::string& p) {
  struct stat st;
  return stat(p.c_str(), &st) == 0;
}

// ---- element conversions -----------------------------------------------------------
// IEEE half -> single, exact (subnormals renormalised, inf / NaN payload kept).
inline float half_to_float(uint16_t h) {
  const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
  uint32_t e = (h >> 10) & 0x1Fu, m = h & 0x3FFu, bits;
  if (e == 0x1F) {
    bits = sign | 0x7F800000u | (m << 13);
  } else if (e != 0) {
    bits = sign | ((e + (127 - 15)) << 23) | (m << 13);
  } else if (m == 0) {
    bits = sign;
  } else {
    int shift = 0;  // normalise: the leading one of m moves to bit 10
    while (!(m & 0x400u)) {
      m <<= 1;
      ++shift;
    }
    bits = sign | ((uint32_t)(127 - 15 + 1 - shift) << 23) | ((m & 0x3FFu) << 13);
  }
  float f;
  std::memcpy(&f, &bits, 4);
  return f;
}
inline float bf16_to_float(uint16_t h) {
  const uint32_t bits = (uint32_t)h << 16;
  float f;
  std::memcpy(&f, &bits, 4);
  return f;
}
// Round to nearest even; NaN and infinity keep their top bits (the reference's
// f32_to_bf16, tensor.cpp:114-121).
inline uint16_t float_to_bf16(float f) {
  uint32_t u;
  std::memcpy(&u, &f, 4);
  if ((u & 0x7F800000u) == 0x7F800000u) return (uint16_t)(u >> 16);
  u += 0x7FFFu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}

// Runs f(lo, hi) over [0, n) on a few host threads.
void par(int64_t n, const std::function<void(int64_t, int64_t)>& f) {
  const int64_t kMin = 1 << 20;
  const int hw = std::max(1u, std::thread::hardware_concurrency());
  const int64_t parts = std::max<int64_t>(1, std::min<int64_t>(std::min(hw, 16), n / kMin));
  if (parts == 1) {
    f(0, n);
    return;
  }
  std::vector<std::thread> ts;
  for (int64_t t = 0; t < parts; ++t) ts.emplace_back(f, n * t / parts, n * (t + 1) / parts);
  for (auto& t : ts) t.join();
}

// ---- tensor-parallel sharding (same rules as sdb200/tp.py) ----------------------------
std::pair<int64_t, int64_t> even_split(int64_t n, int world, int rank) {
  const int64_t base = n / world, extra = n % world;
  const int64_t lo = rank * base + std::min<int64_t>(rank, extra);
  return {lo, lo + base + (rank < extra ? 1 : 0)};
}

bool is_block_param(const std::string& n) {
  return n.rfind("layers.", 0) == 0 || n.rfind("noise_refiner.", 0) == 0 || n.rfind("context_refiner.", 0) == 0;
}

std::string leaf_of(const std::string& n) {  // "layers.3.attention.to_q.weight" -> "attention.to_q.weight"
  const size_t a = n.find('.');
  const size_t b = a == std::string::npos ? a : n.find('.', a + 1);
  return b == std::string::npos ? n : n.substr(b + 1);
}

enum class Cut { None, Rows, Cols, Drop };

struct Plan {
  Cut cut = Cut::None;
  int64_t lo = 0, hi = 0;  // rows or columns kept
};

// `rows_of` gives the first dimension of another tensor of the same block (the FFN width).
Plan plan_shard(const std::string& name, const std::vector<int64_t>& shape, const TpShard* tp,
                const std::function<int64_t(const std::string&)>& rows_of) {
  Plan p;
  if (!tp || tp->world <= 1 || !is_block_param(name)) return p;
  const std::string leaf = leaf_of(name);
  const std::string block = name.substr(0, name.size() - leaf.size());
  auto heads_cut = [&]() {
    const int64_t D = rows_of(block + "attention.to_q.weight");
    if (D % tp->heads) throw std::runtime_error("zimage_load: to_q rows not divisible by heads");
    const int64_t hd = D / tp->heads;
    const auto h = even_split(tp->heads, tp->world, tp->rank);
    return std::make_pair(h.first * hd, h.second * hd);
  };
  auto ffn_cut = [&]() {
    const int64_t F = rows_of(block + "feed_forward.w1.weight");
    if (F % 16) throw std::runtime_error("zimage_load: FFN width not a multiple of 16");
    const auto b = even_split(F / 16, tp->world, tp->rank);
    return std::make_pair(b.first * 16, b.second * 16);
  };
  if (leaf == "attention.to_q.weight" || leaf == "attention.to_k.weight" || leaf == "attention.to_v.weight" ||
      leaf == "attention.to_q.bias" || leaf == "attention.to_k.bias" || leaf == "attention.to_v.bias") {
    const auto c = heads_cut();
    p.cut = Cut::Rows;
    p.lo = c.first;
    p.hi = c.second;
  } else if (leaf == "attention.to_out.0.weight") {
    const auto c = heads_cut();
    p.cut = Cut::Cols;
    p.lo = c.first;
    p.hi = c.second;
  } else if (leaf == "attention.to_out.0.bias" || leaf == "feed_forward.w2.bias") {
    if (tp->rank != 0) p.cut = Cut::Drop;
  } else if (leaf == "feed_forward.w1.weight" || leaf == "feed_forward.w3.weight" || leaf == "feed_forward.w1.bias" ||
             leaf == "feed_forward.w3.bias") {
    const auto c = ffn_cut();
    p.cut = Cut::Rows;
    p.lo = c.first;
    p.hi = c.second;
  } else if (leaf == "feed_forward.w2.weight") {
    const auto c = ffn_cut();
    p.cut = Cut::Cols;
    p.lo = c.first;
    p.hi = c.second;
  }
  if ((p.cut == Cut::Cols && shape.size() != 2) || (p.cut == Cut::Rows && shape.empty()))
    throw std::runtime_error("zimage_load: unexpected rank for " + name);
  return p;
}

struct Entry {
  std::string name, dtype;
  std::vector<int64_t> shape;
  size_t begin = 0, end = 0;
};

struct File {
  std::unique_ptr<Mapped> map;
  const uint8_t* data = nullptr;
  size_t data_size = 0;
  std::vector<Entry> entries;
};

File open_file(const std::string& path) {
  File f;
  f.map.reset(new Mapped(path));
  if (f.map->size < 8) throw std::runtime_error("safetensors: file too small: " + path);
  uint64_t hlen = 0;
  std::memcpy(&hlen, f.map->base, 8);
  if (hlen + 8 > f.map->size) throw std::runtime_error("safetensors: bad header length in " + path);
  const JVal meta = parse_json(std::string((const char*)f.map->base + 8, (size_t)hlen));
  if (meta.kind != JVal::Obj) throw std::runtime_error("safetensors: header is not an object in " + path);
  f.data = (const uint8_t*)f.map->base + 8 + hlen;
  f.data_size = f.map->size - 8 - (size_t)hlen;
  for (const auto& kv : meta.obj) {
    if (kv.first == "__metadata__") continue;
    const JVal* dt = kv.second.find("dtype");
    const JVal* sh = kv.second.find("shape");
    const JVal* off = kv.second.find("data_offsets");
    if (!dt || !sh || !off || off->arr.size() != 2) throw std::runtime_error("safetensors: bad entry " + kv.first);
    Entry e;
    e.name = kv.first;
    e.dtype = dt->str;
    for (const JVal& d : sh->arr) e.shape.push_back((int64_t)d.num);
    e.begin = (size_t)off->arr[0].num;
    e.end = (size_t)off->arr[1].num;
    if (e.end > f.data_size || e.begin > e.end) throw std::runtime_error("safetensors: bad offsets for " + e.name);
    f.entries.push_back(std::move(e));
  }
  return f;
}

int64_t numel(const std::vector<int64_t>& s) {
  int64_t n = 1;
  for (int64_t d : s) n *= d;
  return n;
}

// Converts one entry (optionally cut) into `out`; false for dtypes the reference skips.
bool convert(const File& f, const Entry& e, bool keep_bf16, int64_t min_numel, const Plan& plan, HostTensor& out) {
  if (e.dtype != "F32" && e.dtype != "F16" && e.dtype != "BF16") return false;
  const int64_t n = numel(e.shape);
  const size_t esz = e.dtype == "F32" ? 4 : 2;
  if (e.end - e.begin != (size_t)n * esz) throw std::runtime_error("safetensors: size mismatch for " + e.name);
  out.name = e.name;
  out.bf16 = keep_bf16 && n >= min_numel;  // decided on the whole tensor, as the reference does
  out.shape = e.shape;
  int64_t rows = e.shape.empty() ? 1 : e.shape[0];
  const int64_t cols = rows ? n / rows : 0;
  int64_t r0 = 0, r1 = rows, c0 = 0, c1 = cols;
  if (plan.cut == Cut::Rows) {
    r0 = plan.lo;
    r1 = plan.hi;
    out.shape[0] = r1 - r0;
  } else if (plan.cut == Cut::Cols) {
    c0 = plan.lo;
    c1 = plan.hi;
    out.shape[1] = c1 - c0;
  }
  const int64_t orows = r1 - r0, ocols = c1 - c0;
  out.data.assign((size_t)(orows * ocols) * (out.bf16 ? 2 : 4), 0);
  const uint8_t* src = f.data + e.begin;
  par(orows * ocols, [&](int64_t lo, int64_t hi) {
    for (int64_t i = lo; i < hi; ++i) {
      const int64_t r = r0 + i / std::max<int64_t>(ocols, 1), c = c0 + i % std::max<int64_t>(ocols, 1);
      const size_t s = (size_t)(r * cols + c);
      float v;
      uint16_t h = 0;
      if (e.dtype == "F32") {
        std::memcpy(&v, src + 4 * s, 4);
      } else {
        std::memcpy(&h, src + 2 * s, 2);
        v = e.dtype == "BF16" ? bf16_to_float(h) : half_to_float(h);
      }
      if (out.bf16) {
        const uint16_t b = e.dtype == "BF16" ? h : float_to_bf16(v);
        std::memcpy(out.data.data() + 2 * i, &b, 2);
      } else {
        std::memcpy(out.data.data() + 4 * i, &v, 4);
      }
    }
  });
  return true;
}

}  // namespace

std::vector<std::string> checkpoint_files(const std::string& dir, const std::string& base) {
  const std::string single = dir + "/" + base + ".safetensors";
  const std::string fp16 = dir + "/" + base + ".fp16.safetensors";
  const std::string index = dir + "/" + base + ".safetensors.index.json";
  if (exists(single)) return {single};
  if (exists(index)) {
    std::ifstream in(index);
    std::stringstream ss;
    ss << in.rdbuf();
    const JVal j = parse_json(ss.str());
    const JVal* wm = j.find("weight_map");
    if (!wm || wm->kind != JVal::Obj) throw std::runtime_error("index without weight_map: " + index);
    std::vector<std::string> shards;
    for (const auto& kv : wm->obj)
      if (std::find(shards.begin(), shards.end(), kv.second.str) == shards.end()) shards.push_back(kv.second.str);
    std::sort(shards.begin(), shards.end());
    for (auto& s : shards) s = dir + "/" + s;
    return shards;
  }
  if (exists(fp16)) return {fp16};
  throw std::runtime_error("cannot find " + single + " (or a .fp16 / sharded .index.json variant)");
}

void read_checkpoint(const std::vector<std::string>& files, bool keep_bf16, int64_t min_numel, const TpShard* tp,
                     const std::function<void(HostTensor&&)>& sink, const std::string* only) {
  std::vector<File> fs;
  std::map<std::string, int64_t> rows;  // first dimension of every tensor (sharding needs D and F)
  for (const auto& path : files) {
    fs.push_back(open_file(path));
    for (const Entry& e : fs.back().entries) rows[e.name] = e.shape.empty() ? 1 : e.shape[0];
  }
  auto rows_of = [&](const std::string& n) -> int64_t {
    const auto it = rows.find(n);
    if (it == rows.end()) throw std::runtime_error("zimage_load: sharding needs " + n);
    return it->second;
  };
  for (const File& f : fs)
    for (const Entry& e : f.entries) {
      if (only && e.name != *only) continue;
      const Plan plan = plan_shard(e.name, e.shape, tp, rows_of);
      if (plan.cut == Cut::Drop) continue;
      HostTensor t;
      if (convert(f, e, keep_bf16, min_numel, plan, t)) sink(std::move(t));
    }
}

bool read_tensor(const std::string& path, const std::string& name, bool keep_bf16, int64_t min_numel, HostTensor& out) {
  const File f = open_file(path);
  for (const Entry& e : f.entries)
    if (e.name == name) return convert(f, e, keep_bf16, min_numel, Plan{}, out);
  throw std::runtime_error("safetensors: no tensor " + name + " in " + path);
}

}  // namespace sdb
