// operand_cache.cu - packed copies of constant operands, kept across calls (opt-in).
//
// The op-level interface of the reference backend (backend_cuda.h) hands the fp32
// weights to every call: gemm_nt_f32's B (the linear layers of tensor.cpp:481-501) and
// conv2d's w (tensor.cpp:529-586). This library repacks them per call - B rounded to tf32
// with 16-byte rows, conv weights to [Cout, tap, Cin rounded up to 32] - which is 15% of
// an SD 1.5 UNet step through the drop-in link. With the cache on, the first call packs a
// weight into a buffer of its own and later calls reuse it.
//
// Contract (why it is opt-in): a cached operand must not change while it stays allocated,
// except through this library's sdb200_upload / sdb200_copy / sdb200_zero (and their
// sd::cuda counterparts), which drop the entries whose source they overwrite; freeing the
// buffer through sdb200_free / sd::cuda::free drops its entries too. Buffers from another
// allocator are not tracked. Weights uploaded once (Weights::to_device in the reference,
// safetensors.cpp:195-200) meet it. Only the C-ABI gemm_nt_f32 (its B) and conv2d (its w)
// use the cache; the library's internal GEMMs pass activations or scratch and never do.
// Enable with sdb200_set_operand_cache(1) or the environment variable SDB200_OPERAND_CACHE=1
// (read on the first such call). Entries are per device; the packs are stream-ordered on the
// caller's stream like every other op.
#include <cstdlib>
#include <map>
#include <mutex>
#include <tuple>
#include <vector>

#include "internal.h"

namespace sdb {
namespace {

enum Kind : int { kTf32Rows = 0, kConvWeight = 1 };

struct Key {
  int dev, kind;
  uintptr_t src;
  int64_t a, b, c, d;  // shape and pitch parameters of the pack
  bool operator<(const Key& o) const {
    return std::tie(dev, kind, src, a, b, c, d) < std::tie(o.dev, o.kind, o.src, o.a, o.b, o.c, o.d);
  }
};
struct Entry {
  void* packed = nullptr;
  int dev = 0;
  size_t bytes = 0;
  uintptr_t lo = 0, hi = 0;  // source byte range [lo, hi)
};
struct Victim {
  void* p;
  int dev;
};

std::mutex g_mutex;
std::map<Key, Entry> g_entries;
size_t g_bytes = 0;
int g_enabled = -1;  // -1: not decided yet (environment default)
constexpr size_t kMaxBytes = (size_t)16 << 30;

bool enabled_locked() {
  if (g_enabled < 0) {
    const char* e = std::getenv("SDB200_OPERAND_CACHE");
    g_enabled = (e && e[0] == '1') ? 1 : 0;
  }
  return g_enabled == 1;
}

// Removes entries matching `pred` and returns their packed buffers (freed by the caller
// after the lock is released: pool_free calls back into operand_cache_invalidate).
template <class Pred>
std::vector<Victim> take_locked(Pred pred) {
  std::vector<Victim> out;
  for (auto it = g_entries.begin(); it != g_entries.end();) {
    if (pred(it->second)) {
      out.push_back({it->second.packed, it->second.dev});
      g_bytes -= it->second.bytes;
      it = g_entries.erase(it);
    } else {
      ++it;
    }
  }
  return out;
}

// Returns packed buffers to the pool of the device that owns them.
void release(const std::vector<Victim>& bufs) {
  if (bufs.empty()) return;
  int cur = 0;
  check_cuda(cudaGetDevice(&cur), "cudaGetDevice");
  for (const Victim& v : bufs) {
    if (v.dev != cur) check_cuda(cudaSetDevice(v.dev), "cudaSetDevice");
    pool_free(v.p);
    if (v.dev != cur) check_cuda(cudaSetDevice(cur), "cudaSetDevice");
  }
}

// The packed copy for `key`, made by `pack(dst)` on a miss.
template <class Pack>
const float* lookup(const Key& key, size_t bytes, uintptr_t lo, uintptr_t hi, Pack&& pack) {
  std::vector<Victim> victims;
  {
    std::lock_guard<std::mutex> lk(g_mutex);
    const auto it = g_entries.find(key);
    if (it != g_entries.end()) return static_cast<const float*>(it->second.packed);
    if (g_bytes + bytes > kMaxBytes) victims = take_locked([](const Entry&) { return true; });
  }
  release(victims);
  victims.clear();
  void* dst = pool_malloc(bytes);
  try {
    pack(static_cast<float*>(dst));
  } catch (...) {
    pool_free(dst);
    throw;
  }
  {
    std::lock_guard<std::mutex> lk(g_mutex);
    const auto it = g_entries.find(key);
    if (it == g_entries.end()) {
      Entry e;
      e.packed = dst;
      e.dev = key.dev;
      e.bytes = bytes;
      e.lo = lo;
      e.hi = hi;
      g_entries.emplace(key, e);
      g_bytes += bytes;
      return static_cast<const float*>(dst);
    }
    victims.assign(1, Victim{dst, key.dev});  // another thread packed it meanwhile: use its copy
    dst = it->second.packed;
  }
  release(victims);
  return static_cast<const float*>(dst);
}

}  // namespace

bool operand_cache_on() {
  std::lock_guard<std::mutex> lk(g_mutex);
  return enabled_locked();
}

void operand_cache_enable(bool on) {
  std::vector<Victim> victims;
  {
    std::lock_guard<std::mutex> lk(g_mutex);
    g_enabled = on ? 1 : 0;
    if (!on) victims = take_locked([](const Entry&) { return true; });
  }
  release(victims);
}

int64_t operand_cache_entries() {
  std::lock_guard<std::mutex> lk(g_mutex);
  return (int64_t)g_entries.size();
}

void operand_cache_invalidate(const void* p, size_t bytes) {
  if (!p || !bytes) return;
  const uintptr_t lo = reinterpret_cast<uintptr_t>(p), hi = lo + bytes;
  std::vector<Victim> victims;
  {
    std::lock_guard<std::mutex> lk(g_mutex);
    if (g_entries.empty()) return;
    victims = take_locked([&](const Entry& e) { return e.lo < hi && lo < e.hi; });
  }
  release(victims);
}

const float* cached_tf32_rows(const float* B, int64_t rows, int64_t cols, int64_t ld, int64_t ldo) {
  const int dev = ctx().device;
  const Key key{dev, kTf32Rows, reinterpret_cast<uintptr_t>(B), rows, cols, ld, ldo};
  const uintptr_t lo = reinterpret_cast<uintptr_t>(B);
  const uintptr_t hi = lo + (size_t)((rows - 1) * ld + cols) * 4;
  const size_t bytes = (size_t)(rows * ldo) * 4;
  return lookup(key, bytes, lo, hi, [&](float* dst) { launch_pack_tf32(B, ld, dst, ldo, rows, cols); });
}

const float* cached_conv_weight(const float* w, int64_t Cout, int64_t Cin, int64_t taps, int64_t cq) {
  const int dev = ctx().device;
  const Key key{dev, kConvWeight, reinterpret_cast<uintptr_t>(w), Cout, Cin, taps, cq};
  const uintptr_t lo = reinterpret_cast<uintptr_t>(w);
  const uintptr_t hi = lo + (size_t)(Cout * Cin * taps) * 4;
  const size_t bytes = (size_t)(Cout * taps * cq) * 4;
  return lookup(key, bytes, lo, hi, [&](float* dst) { launch_conv_pack_w(w, dst, Cout, Cin, taps, cq); });
}

}  // namespace sdb
