// vae.cu - the AutoencoderKL decoder (reference: src/vae.{h,cpp}, VAEDecoder::decode;
// ResnetBlock and VAEAttention in src/modules.cpp:27-49, :119-141) as one device program
// on the implicit-GEMM convolution (gemm_tc.cu) and the split-statistics GroupNorm.
//
// The reference runs each layer as separate ops (group_norm, silu_, conv2d = im2col + GEMM,
// add_, upsample_nearest2x, nchw_to_nlc ...), each a full pass over the activation. Here
// activations stay NCHW fp32 between layers, and every convolution input is produced in
// the kernel's own layout (NHWC, tf32) by a single pass that also applies what precedes the
// convolution in the reference:
//   resnet   conv1(silu(norm1(x)))     GroupNorm stats -> pack(x * a + b, SiLU) -> conv
//            conv2(silu(norm2(h))) + x same, the residual added in the conv epilogue (in place)
//            shortcut(x)              pack(x) -> 1x1 conv, then the residual of conv2
//   upsample conv(upsample2x(h))      pack reads (y / 2, x / 2): no upsampled copy
//   latents  conv_in(z / s + shift)   the affine inside the first pack
//   attention h = nchw_to_nlc(norm(x)) pack with the GroupNorm affine (NHWC = tokens)
//            q|k|v = h W^T + b         one tf32 GEMM, N = 3C
//            attention(q, k, v), 1 head  attention_gemm.cu (head dim = C)
//            x += nlc_to_nchw(o W_out^T + b)  a 1x1 implicit conv of o with the residual
//   out      conv_out(silu(norm_out(h)))
// Weights are fp32 (the reference's VAE weights load as fp32, pipeline.cpp:86, and its
// conv2d takes no bf16 weights, tensor.cpp:538); finalize() keeps tf32-rounded copies in
// the convolution layout.
#include <algorithm>
#include <cmath>
#include <map>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

#include "internal.h"
#include "sdb200.h"
#include "weights_io.h"

namespace sdb {
namespace {

constexpr float kVaeEps = 1e-6f;  // every GroupNorm of the decoder (vae.cpp:11)
constexpr int kGroups = 32;

struct WRef {
  const float* p = nullptr;
  std::vector<int64_t> shape;
};

// Device buffer owned by the model (pool allocator), grown on demand.
struct Buf {
  void* p = nullptr;
  size_t bytes = 0;
  Buf() = default;
  Buf(const Buf&) = delete;
  Buf& operator=(const Buf&) = delete;
  Buf(Buf&& o) noexcept : p(o.p), bytes(o.bytes) {
    o.p = nullptr;
    o.bytes = 0;
  }
  ~Buf() { reset(); }
  void reset() {
    if (p) {
      try {
        pool_free(p);
      } catch (...) {
      }
    }
    p = nullptr;
    bytes = 0;
  }
  void ensure(size_t b) {
    if (b <= bytes) return;
    reset();
    p = pool_malloc(b);
    bytes = b;
  }
  float* f() const { return static_cast<float*>(p); }
};

struct Conv {
  const float* bias = nullptr;
  int64_t cout = 0, cin = 0, k = 1, cq = 0;
  Buf wp;  // [cout, k*k, cq] tf32
  bool valid() const { return cout > 0; }
};
struct Norm {
  const float* g = nullptr;
  const float* b = nullptr;
};
struct Resnet {
  Norm n1, n2;
  Conv c1, c2, sc;
};
struct Attn {
  Norm n;
  int64_t C = 0;
  Buf wqkv, bqkv;  // [3C, C] tf32, [3C]
  Conv out;        // to_out as a 1x1 convolution
};
struct Up {
  std::vector<Resnet> res;
  Conv up;
};

int64_t cp_of(int64_t c) { return (c + 3) / 4 * 4; }

struct Vae {
  float scale, shift;
  std::map<std::string, WRef> w;
  std::vector<Buf> owned;  // device copies made by sdb200_vae_load
  bool finalized = false;
  Conv post_quant, conv_in, conv_out;
  Resnet mid0, mid1;
  Attn attn;
  std::vector<Up> ups;
  Norm norm_out;
  int64_t latent_ch = 0;
  // activations
  Buf cur, tmp, sc, xh, ab, qkv, att;
  // GroupNorm partial statistics of cur / tmp written by the convolution that produced them
  // (tiles per image, or -1 when the producer did not write them)
  Buf part_cur, part_tmp;
  int64_t part_cap = 0, cur_tiles = -1, tmp_tiles = -1;

  // Optional timing of the tensor-core work (CUDA events on the stream): category 0 the
  // convolutions, 1 the attention (projections, scores, softmax, output); FLOPs are
  // algorithmic (2 Cout Cin k^2 H W per conv, 2 S C (3C) + 4 S^2 C for the attention).
  bool prof_on = false;
  struct Mark {
    cudaEvent_t a, b;
    int cat;
    double flop;
  };
  std::vector<Mark> marks;
  template <class Fn>
  void timed(int cat, double flop, Fn&& fn) {
    if (!prof_on) return fn();
    Mark m{nullptr, nullptr, cat, flop};
    check_cuda(cudaEventCreate(&m.a), "cudaEventCreate");
    check_cuda(cudaEventCreate(&m.b), "cudaEventCreate");
    check_cuda(cudaEventRecord(m.a, ctx().stream), "cudaEventRecord");
    fn();
    check_cuda(cudaEventRecord(m.b, ctx().stream), "cudaEventRecord");
    marks.push_back(m);
  }
  void prof_clear() {
    for (Mark& m : marks) {
      cudaEventDestroy(m.a);
      cudaEventDestroy(m.b);
    }
    marks.clear();
  }
  // out[0..4]: conv ms, conv flop, conv launches, attention ms, attention flop.
  void prof_read(double* out) {
    check_cuda(cudaStreamSynchronize(ctx().stream), "vae profile sync");
    for (int i = 0; i < 5; ++i) out[i] = 0.0;
    for (Mark& m : marks) {
      float ms = 0.0f;
      check_cuda(cudaEventElapsedTime(&ms, m.a, m.b), "cudaEventElapsedTime");
      if (m.cat == 0) {
        out[0] += ms;
        out[1] += m.flop;
        out[2] += 1.0;
      } else {
        out[3] += ms;
        out[4] += m.flop;
      }
    }
    prof_clear();
  }

  Vae(float s, float sh) : scale(s), shift(sh) {}
  ~Vae() { prof_clear(); }

  bool has(const std::string& n) const { return w.count(n) != 0; }
  const WRef& get(const std::string& n) const {
    auto it = w.find(n);
    if (it == w.end()) fail(kErrInvalidArg, "vae: missing weight " + n);
    return it->second;
  }
  const float* opt(const std::string& n) const {
    auto it = w.find(n);
    return it == w.end() ? nullptr : it->second.p;
  }

  void bind_conv(Conv& c, const std::string& p) {
    const WRef& W = get(p + ".weight");
    if (W.shape.size() != 4 || W.shape[2] != W.shape[3] || W.shape[2] % 2 == 0)
      fail(kErrInvalidArg, "vae: " + p + ".weight must be [Cout, Cin, k, k] with odd k");
    c.cout = W.shape[0];
    c.cin = W.shape[1];
    c.k = W.shape[2];
    c.cq = (c.cin + 31) / 32 * 32;
    c.bias = opt(p + ".bias");
    c.wp.ensure((size_t)(c.cout * c.k * c.k * c.cq) * 4);
    launch_conv_pack_w(W.p, c.wp.f(), c.cout, c.cin, c.k * c.k, c.cq);
  }
  void bind_norm(Norm& n, const std::string& p) {
    n.g = get(p + ".weight").p;
    n.b = get(p + ".bias").p;
  }
  void bind_resnet(Resnet& r, const std::string& p) {
    bind_norm(r.n1, p + ".norm1");
    bind_norm(r.n2, p + ".norm2");
    bind_conv(r.c1, p + ".conv1");
    bind_conv(r.c2, p + ".conv2");
    if (has(p + ".conv_shortcut.weight")) bind_conv(r.sc, p + ".conv_shortcut");
    if (r.c2.cin != r.c1.cout || (!r.sc.valid() && r.c1.cin != r.c2.cout))
      fail(kErrInvalidArg, "vae: " + p + ": channel counts do not chain");
  }
  void bind_attn(const std::string& p) {
    bind_norm(attn.n, p + ".group_norm");
    const bool diffusers = has(p + ".to_q.weight");
    const std::string nq = diffusers ? ".to_q" : ".query", nk = diffusers ? ".to_k" : ".key",
                      nv = diffusers ? ".to_v" : ".value", no = diffusers ? ".to_out.0" : ".proj_attn";
    const WRef& Wq = get(p + nq + ".weight");
    const int64_t C = Wq.shape[0];
    attn.C = C;
    if (C % 4 != 0) fail(kErrInvalidArg, "vae: attention width must be a multiple of 4");
    attn.wqkv.ensure((size_t)(3 * C * C) * 4);
    attn.bqkv.ensure((size_t)(3 * C) * 4);
    const std::string names[3] = {nq, nk, nv};
    for (int i = 0; i < 3; ++i) {
      const WRef& W = get(p + names[i] + ".weight");
      int64_t numel = 1;
      for (int64_t d : W.shape) numel *= d;
      if (numel != C * C) fail(kErrInvalidArg, "vae: attention projections must be C x C");
      launch_pack_tf32(W.p, C, attn.wqkv.f() + (int64_t)i * C * C, C, C, C);
      const float* b = opt(p + names[i] + ".bias");
      if (b)
        check_cuda(cudaMemcpyAsync(attn.bqkv.f() + i * C, b, (size_t)C * 4, cudaMemcpyDeviceToDevice, ctx().stream),
                   "vae: bias copy");
      else
        check_cuda(cudaMemsetAsync(attn.bqkv.f() + i * C, 0, (size_t)C * 4, ctx().stream), "vae: bias zero");
    }
    const WRef& Wo = get(p + no + ".weight");
    Conv& o = attn.out;
    o.cout = C;
    o.cin = C;
    o.k = 1;
    o.cq = (C + 31) / 32 * 32;
    o.bias = opt(p + no + ".bias");
    o.wp.ensure((size_t)(C * o.cq) * 4);
    launch_conv_pack_w(Wo.p, o.wp.f(), C, C, 1, o.cq);
  }

  void finalize() {
    if (finalized) fail(kErrInvalidArg, "vae: already finalized");
    if (has("post_quant_conv.weight")) bind_conv(post_quant, "post_quant_conv");
    bind_conv(conv_in, "decoder.conv_in");
    bind_conv(conv_out, "decoder.conv_out");
    bind_norm(norm_out, "decoder.conv_norm_out");
    bind_resnet(mid0, "decoder.mid_block.resnets.0");
    bind_resnet(mid1, "decoder.mid_block.resnets.1");
    bind_attn("decoder.mid_block.attentions.0");
    for (int i = 0;; ++i) {
      const std::string bp = "decoder.up_blocks." + std::to_string(i);
      if (!has(bp + ".resnets.0.conv1.weight")) break;
      Up u;
      for (int j = 0; has(bp + ".resnets." + std::to_string(j) + ".conv1.weight"); ++j) {
        u.res.emplace_back();
        bind_resnet(u.res.back(), bp + ".resnets." + std::to_string(j));
      }
      if (has(bp + ".upsamplers.0.conv.weight")) bind_conv(u.up, bp + ".upsamplers.0.conv");
      ups.push_back(std::move(u));
    }
    if (ups.empty()) fail(kErrInvalidArg, "vae: no decoder up blocks found");
    latent_ch = post_quant.valid() ? post_quant.cin : conv_in.cin;
    finalized = true;
  }

  // ---- layers ----------------------------------------------------------------------
  // conv over an NHWC input already in xh (channel pitch cp_of(c.cin)), NCHW output. With
  // part, the epilogue also writes the output's GroupNorm statistics there; returns the
  // tiles per image, or -1 when it did not (widths the epilogue form does not take).
  int64_t conv(const Conv& c, int64_t N, int64_t H, int64_t W, const float* res, float* out, Buf* part = nullptr) {
    const int pad = (int)(c.k - 1) / 2;
    ConvStats st{nullptr, part_cap, kGroups, -1};
    const bool stats = part && c.cout % 32 == 0 && 32 % (c.cout / kGroups) == 0;
    if (stats) st.part = static_cast<float4*>(part->p);
    timed(0, 2.0 * N * c.cout * c.cin * c.k * c.k * H * W, [&] {
      launch_conv_tc(xh.f(), N, c.cin, cp_of(c.cin), H, W, c.wp.f(), c.cq, c.cout, (int)c.k, (int)c.k, pad, c.bias,
                     res, out, H, W, stats ? &st : nullptr);
    });
    return stats ? st.tiles_img : -1;
  }
  // xh = pack(silu?(norm(x))); the statistics from the producer's partials when it wrote them
  void norm_pack(const Norm& n, const float* x, int64_t N, int64_t C, int64_t H, int64_t W, bool silu,
                 const Buf* part = nullptr, int64_t tiles = -1) {
    float2* abp = static_cast<float2*>(ab.p);
    if (part && tiles >= 0)
      gn_scale_shift_parts(static_cast<const float4*>(part->p), tiles, N, C, kGroups, n.g, n.b, kVaeEps, abp);
    else
      gn_scale_shift(x, N, C, H * W, kGroups, n.g, n.b, kVaeEps, abp);
    launch_pack_nhwc(x, xh.f(), N, C, H, W, cp_of(C), abp, 1.0f, 0.0f, silu, false);
  }
  // cur [N, cin, H, W] -> cur [N, cout, H, W]
  void resnet(const Resnet& r, int64_t N, int64_t H, int64_t W) {
    const float* res = cur.f();
    if (r.sc.valid()) {
      launch_pack_nhwc(cur.f(), xh.f(), N, r.sc.cin, H, W, cp_of(r.sc.cin), nullptr, 1.0f, 0.0f, false, false);
      conv(r.sc, N, H, W, nullptr, sc.f());
      res = sc.f();
    }
    norm_pack(r.n1, cur.f(), N, r.c1.cin, H, W, true, &part_cur, cur_tiles);
    tmp_tiles = conv(r.c1, N, H, W, nullptr, tmp.f(), &part_tmp);
    norm_pack(r.n2, tmp.f(), N, r.c2.cin, H, W, true, &part_tmp, tmp_tiles);
    // in place when res == cur: each element read, then written
    cur_tiles = conv(r.c2, N, H, W, res, cur.f(), &part_cur);
  }
  void attention(int64_t N, int64_t H, int64_t W) {
    const int64_t C = attn.C, S = H * W;
    float2* abp = static_cast<float2*>(ab.p);
    if (cur_tiles >= 0)
      gn_scale_shift_parts(static_cast<const float4*>(part_cur.p), cur_tiles, N, C, kGroups, attn.n.g, attn.n.b,
                           kVaeEps, abp);
    else
      gn_scale_shift(cur.f(), N, C, S, kGroups, attn.n.g, attn.n.b, kVaeEps, abp);
    launch_pack_nhwc(cur.f(), xh.f(), N, C, H, W, C, abp, 1.0f, 0.0f, false, false);  // tokens [N*S, C]
    timed(1, 2.0 * N * S * C * 3 * C + 4.0 * N * S * S * C, [&] {
      gemm_tf32_direct(N * S, 3 * C, C, xh.f(), C, attn.wqkv.f(), C, qkv.f(), 3 * C, attn.bqkv.f(), false);
      launch_round_tf32_inplace(qkv.f(), 3 * C, N * S, 2 * C);  // q | k onto the tf32 grid
      const float* q = qkv.f();
      launch_attention_gemm(q, q + C, q + 2 * C, att.f(), N, S, S, 1, 1, C, false, 3 * C, 3 * C, C, true);
      launch_pack_tf32(att.f(), C, xh.f(), C, N * S, C);  // the 1x1 conv's NHWC operand
    });
    cur_tiles = conv(attn.out, N, H, W, cur.f(), cur.f(), &part_cur);
  }

  // Largest NCHW activation and NHWC convolution input over the decode (elements).
  void plan(int64_t N, int64_t h, int64_t w, size_t& nchw, size_t& nhwc, size_t& ch_max) const {
    nchw = nhwc = ch_max = 0;
    auto act = [&](int64_t c, int64_t H, int64_t W) {
      nchw = std::max(nchw, (size_t)(N * c * H * W));
      ch_max = std::max(ch_max, (size_t)(N * c));
    };
    auto in = [&](int64_t c, int64_t H, int64_t W) { nhwc = std::max(nhwc, (size_t)(N * cp_of(c) * H * W)); };
    int64_t H = h, W = w;
    if (post_quant.valid()) {
      in(post_quant.cin, H, W);
      act(post_quant.cout, H, W);
    }
    in(conv_in.cin, H, W);
    act(conv_in.cout, H, W);
    auto res = [&](const Resnet& r) {
      in(r.c1.cin, H, W);
      act(r.c1.cout, H, W);
      in(r.c2.cin, H, W);
      act(r.c2.cout, H, W);
      act(r.c1.cin, H, W);
    };
    res(mid0);
    in(attn.C, H, W);
    res(mid1);
    for (const Up& u : ups) {
      for (const Resnet& r : u.res) res(r);
      if (u.up.valid()) {
        H *= 2;
        W *= 2;
        in(u.up.cin, H, W);
        act(u.up.cout, H, W);
      }
    }
    in(conv_out.cin, H, W);
  }

  // latents [N, latent_ch, h, w] -> out [N, conv_out.cout, h * 2^ups, w * 2^ups]
  void decode(const float* z, int64_t N, int64_t C, int64_t h, int64_t w, float* out) {
    if (!finalized) fail(kErrInvalidArg, "vae: decode before finalize");
    if (C != latent_ch) fail(kErrInvalidArg, "vae: latent channel count mismatch");
    if (N <= 0 || h <= 0 || w <= 0) return;
    size_t nchw, nhwc, chs;
    plan(N, h, w, nchw, nhwc, chs);
    cur.ensure(nchw * 4);
    tmp.ensure(nchw * 4);
    sc.ensure(nchw * 4);
    xh.ensure(nhwc * 4);
    ab.ensure(chs * sizeof(float2));
    {
      // the largest statistics buffer: N x 32 groups x Ho x ceil(Wo / 32) tiles bounds every layer
      const int64_t f = upscale();
      part_cap = N * kGroups * (h * f) * ((w * f + 31) / 32);
      part_cur.ensure((size_t)part_cap * sizeof(float4));
      part_tmp.ensure((size_t)part_cap * sizeof(float4));
      cur_tiles = tmp_tiles = -1;
    }
    const int64_t S = h * w;
    qkv.ensure((size_t)(N * S * 3 * attn.C) * 4);
    att.ensure((size_t)(N * S * attn.C) * 4);
    int64_t H = h, W = w;
    // z / scaling_factor + shift_factor (vae.cpp:37-38), inside the first pack
    launch_pack_nhwc(z, xh.f(), N, C, H, W, cp_of(C), nullptr, 1.0f / scale, shift, false, false);
    if (post_quant.valid()) {
      conv(post_quant, N, H, W, nullptr, tmp.f());
      launch_pack_nhwc(tmp.f(), xh.f(), N, post_quant.cout, H, W, cp_of(post_quant.cout), nullptr, 1.0f, 0.0f, false,
                       false);
    }
    cur_tiles = conv(conv_in, N, H, W, nullptr, cur.f(), &part_cur);
    resnet(mid0, N, H, W);
    attention(N, H, W);
    resnet(mid1, N, H, W);
    for (const Up& u : ups) {
      for (const Resnet& r : u.res) resnet(r, N, H, W);
      if (u.up.valid()) {
        launch_pack_nhwc(cur.f(), xh.f(), N, u.up.cin, H, W, cp_of(u.up.cin), nullptr, 1.0f, 0.0f, false, true);
        H *= 2;
        W *= 2;
        cur_tiles = conv(u.up, N, H, W, nullptr, cur.f(), &part_cur);
      }
    }
    norm_pack(norm_out, cur.f(), N, conv_out.cin, H, W, true, &part_cur, cur_tiles);
    conv(conv_out, N, H, W, nullptr, out);
  }
  int64_t upscale() const {
    int64_t f = 1;
    for (const Up& u : ups)
      if (u.up.valid()) f *= 2;
    return f;
  }
};

}  // namespace
}  // namespace sdb

// ===================================================================================
using sdb::Vae;

#define SDB_GUARD(body)                 \
  try {                                 \
    body;                               \
    return sdb::kOk;                    \
  } catch (const sdb::Error& e) {       \
    sdb::set_last_error(e.msg);         \
    return e.code;                      \
  } catch (const std::exception& e) {   \
    sdb::set_last_error(e.what());      \
    return sdb::kErrCuda;               \
  }

extern "C" {

void* sdb200_vae_create(float scaling_factor, float shift_factor) {
  try {
    if (!(scaling_factor != 0.0f)) sdb::fail(sdb::kErrInvalidArg, "vae_create: scaling factor must be non-zero");
    return new Vae(scaling_factor, shift_factor);
  } catch (const sdb::Error& e) {
    sdb::set_last_error(e.msg);
  } catch (const std::exception& e) {
    sdb::set_last_error(e.what());
  }
  return nullptr;
}

int sdb200_vae_set_weight(void* m, const char* name, const float* dev_ptr, const int64_t* shape, int ndim) {
  SDB_GUARD({
    if (!m || !name || !dev_ptr || !shape || ndim <= 0 || ndim > 8)
      sdb::fail(sdb::kErrInvalidArg, "vae_set_weight: bad argument");
    Vae* v = static_cast<Vae*>(m);
    if (v->finalized) sdb::fail(sdb::kErrInvalidArg, "vae_set_weight: model already finalized");
    sdb::WRef r;
    r.p = dev_ptr;
    r.shape.assign(shape, shape + ndim);
    v->w[name] = r;
  })
}

int sdb200_vae_load(void* m, const char* dir, const char* base) {
  SDB_GUARD({
    if (!m || !dir || !base) sdb::fail(sdb::kErrInvalidArg, "vae_load: null argument");
    Vae* v = static_cast<Vae*>(m);
    if (v->finalized) sdb::fail(sdb::kErrInvalidArg, "vae_load: model already finalized");
    try {
      // Weights::load_model(dir, base) with keep_bf16 = false (pipeline.cpp:86): all fp32.
      const std::vector<std::string> files = sdb::checkpoint_files(dir, base);
      sdb::read_checkpoint(files, false, (int64_t)1 << 62, nullptr, [&](sdb::HostTensor&& t) {
        sdb::Buf buf;
        buf.ensure(t.data.size());
        sdb::check_cuda(cudaMemcpy(buf.p, t.data.data(), t.data.size(), cudaMemcpyHostToDevice), "vae_load: upload");
        sdb::WRef r;
        r.p = buf.f();
        r.shape = t.shape;
        v->owned.push_back(std::move(buf));
        v->w[t.name] = r;
      });
    } catch (const std::runtime_error& e) {
      sdb::fail(sdb::kErrInvalidArg, std::string("vae_load: ") + e.what());
    }
  })
}

int sdb200_vae_finalize(void* m) {
  SDB_GUARD({
    if (!m) sdb::fail(sdb::kErrInvalidArg, "vae_finalize: null model");
    static_cast<Vae*>(m)->finalize();
  })
}

int sdb200_vae_info(void* m, int64_t* latent_channels, int64_t* out_channels, int64_t* upscale) {
  SDB_GUARD({
    if (!m) sdb::fail(sdb::kErrInvalidArg, "vae_info: null model");
    Vae* v = static_cast<Vae*>(m);
    if (!v->finalized) sdb::fail(sdb::kErrInvalidArg, "vae_info: model not finalized");
    if (latent_channels) *latent_channels = v->latent_ch;
    if (out_channels) *out_channels = v->conv_out.cout;
    if (upscale) *upscale = v->upscale();
  })
}

int sdb200_vae_decode(void* m, const float* latents, int64_t N, int64_t C, int64_t h, int64_t w, float* out) {
  SDB_GUARD({
    if (!m || !latents || !out) sdb::fail(sdb::kErrInvalidArg, "vae_decode: null argument");
    static_cast<Vae*>(m)->decode(latents, N, C, h, w, out);
  })
}

int sdb200_vae_profile(void* m, int on) {
  SDB_GUARD({
    if (!m) sdb::fail(sdb::kErrInvalidArg, "vae_profile: null model");
    Vae* v = static_cast<Vae*>(m);
    v->prof_clear();
    v->prof_on = on != 0;
  })
}

int sdb200_vae_profile_read(void* m, double* out5) {
  SDB_GUARD({
    if (!m || !out5) sdb::fail(sdb::kErrInvalidArg, "vae_profile_read: null argument");
    static_cast<Vae*>(m)->prof_read(out5);
  })
}

void sdb200_vae_destroy(void* m) { delete static_cast<Vae*>(m); }

}  // extern "C"
