// zimage.cu - the Z-Image single-stream DiT forward (reference: src/zimage.{h,cpp},
// ZImageTransformer::forward / run_block) on the B200 kernels, every activation kept
// on the device from the latent in to the prediction out.
//
// Per block (zimage.cpp:90-136), with the reference op each step replaces:
//   mod  = adaLN(t_emb)               GEMV, M=1 (bf16 W)        -> k_gemm_skinny
//          1 + s, tanh(g)             affine_/tanh_             -> k_adaln_split
//   h    = bf16(rms_norm(x)*scale)    rms_norm + mul_rows_      -> k_rms_mod_bf16
//   qkv  = h Wqkv^T                   to_q / to_k / to_v (3 GEMMs) -> one tcgen05 GEMM, N = 3D,
//   q,k,v -> fp16 heads               rms_norm_heads_ + rope_      whose epilogue normalises,
//                                                                  rotates and packs (kQkvRope)
//   o    = attention(q,k,v)           attention                  -> k_attention_tc (bf16 out)
//   a    = o Wout^T                   to_out                     -> tcgen05 GEMM
//   x   += g_msa * rms_norm(a)        rms_norm + add_rows_scaled_ -> k_post_norm_residual
//   h    = bf16(rms_norm(x)*scale)    (as above)
//   f    = silu(h W1^T) * (h W3^T)    w1, w3, swiglu             -> one GEMM, SwiGLU epilogue
//   a    = f W2^T                     w2                         -> tcgen05 GEMM
//   x   += g_mlp * rms_norm(a)        (as above)
// The forward takes a batch of B images that share the timestep (a sampler step):
// row-wise ops and GEMMs run over all B*S rows at once (larger GEMM M), attention over
// N = B samples. The reference forward is batch-1; for B = 1 the math is identical.
//
// Weights are the caller's device buffers under the checkpoint names
// (zimage.cpp:38-67). Block linears must be bf16 (the loader keeps tensors of >= 2^20
// elements in bf16, safetensors.cpp:119); small layers (x_embed, t_mlp, final) may be
// fp32 or bf16. finalize() builds the fused QKV and interleaved w1/w3 weights it owns.
#include <algorithm>
#include <array>
#include <cmath>
#include <cstring>
#include <stdexcept>
#include <map>
#include <memory>
#include <string>
#include <unordered_map>
#include <vector>

#include "internal.h"
#include "sdb200.h"
#include "weights_io.h"

namespace sdb {

namespace {

struct WRef {
  const void* p = nullptr;
  bool bf16 = false;
  std::vector<int64_t> shape;
  int64_t dim(int i) const { return shape[i < 0 ? i + (int)shape.size() : i]; }
};

// Device buffer owned by the model (pool allocator).
struct DBuf {
  void* p = nullptr;
  size_t bytes = 0;
  DBuf() = default;
  DBuf(const DBuf&) = delete;
  DBuf& operator=(const DBuf&) = delete;
  DBuf(DBuf&& o) noexcept : p(o.p), bytes(o.bytes) {
    o.p = nullptr;
    o.bytes = 0;
  }
  DBuf& operator=(DBuf&& o) noexcept {
    if (this != &o) {
      reset();
      p = o.p;
      bytes = o.bytes;
      o.p = nullptr;
      o.bytes = 0;
    }
    return *this;
  }
  ~DBuf() { reset(); }
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
  template <class T>
  T* as() const {
    return static_cast<T*>(p);
  }
};

struct Block {
  const float *attn_norm1 = nullptr, *attn_norm2 = nullptr, *ffn_norm1 = nullptr, *ffn_norm2 = nullptr;
  const float *norm_q = nullptr, *norm_k = nullptr;
  DBuf wqkv, bqkv, w13, b13;  // fused, owned
  bool has_bqkv = false, has_b13 = false;
  const uint16_t* wout = nullptr;
  const float* bout = nullptr;
  const uint16_t* w2 = nullptr;
  const float* b2 = nullptr;
  const uint16_t* adaln = nullptr;  // [4D, tdim] or null (context refiner)
  const float* adaln_b = nullptr;
  int64_t F = 0;       // FFN width held by this rank (all of it without tensor parallelism)
  int64_t Dq = 0;      // q/k/v width held by this rank = heads_local * 128
  int heads_local = 0;
};

// Generic linear on fp32 activations: bf16 or fp32 weights (tensor.cpp:481-501).
void linear(const float* x, int64_t rows, int64_t in, const WRef& W, const WRef* b, float* y) {
  const int64_t out = W.dim(0);
  if (W.dim(1) != in) fail(kErrInvalidArg, "zimage: linear input width mismatch");
  const float* bias = b ? static_cast<const float*>(b->p) : nullptr;
  if (W.bf16)
    gemm_nt_bf16_impl(rows, out, in, x, in, static_cast<const uint16_t*>(W.p), in, y, out, bias, false);
  else
    gemm_nt_f32_impl(rows, out, in, x, in, static_cast<const float*>(W.p), in, y, out, bias, false);
}

}  // namespace

// Flow-matching schedule of FlowMatchScheduler::set_timesteps (scheduler.cpp:117-127):
// sigma_i = shift s / (1 + (shift - 1) s), s running linearly from 1 to 1/steps, and
// sigma_steps = 0. The denominator is one fused multiply-add: the reference is built
// for x86-64-v3 and its compiler contracts exactly that term, so this reproduces the
// reference's values bit for bit.
void flow_sigmas(int steps, float shift, float* sig) {
  for (int i = 0; i < steps; ++i) {
    const float s = steps == 1 ? 1.0f : 1.0f - (float)i * (1.0f - 1.0f / (float)steps) / (float)(steps - 1);
    sig[i] = shift * s / std::fma(shift - 1.0f, s, 1.0f);
  }
  sig[steps] = 0.0f;
}

class ZImage {
 public:
  int heads, patch;
  float norm_eps, rope_theta, t_scale;
  int axes[3];
  std::unordered_map<std::string, WRef> w;
  std::vector<DBuf> owned;  // device copies made by sdb200_zimage_load
  bool finalized = false;
  int64_t D = 0, head_dim = 0, in_ch = 0, tdim = 0;
  std::vector<Block> noise, context, layers;

  ZImage(int h, int p, float eps, float theta, float ts, int a0, int a1, int a2)
      : heads(h), patch(p), norm_eps(eps), rope_theta(theta), t_scale(ts), axes{a0, a1, a2} {}
  ~ZImage() {
    prof_clear();
    release_tp();
  }

  // ---- optional per-kernel timing (CUDA events on the stream) ------------------------
  // Category 0: tensor-core GEMMs, 1: attention, 2: whole forward, 3: tensor-parallel
  // all-reduce. FLOPs are the algorithmic 2*M*N*K (GEMM) and 4*Sq*Skv*d*heads (attention).
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
  // out[0..n): gemm ms, gemm flop, gemm launches, attention ms, attention flop,
  // attention launches, forward ms, forwards, all-reduce ms, all-reduces, then (n = 16)
  // post-norm ms, post-norm bytes, post-norm launches, adaLN GEMV ms, adaLN bytes, adaLN
  // launches. Bytes are the algorithmic minimum (inputs read once, outputs written once).
  // Synchronises; resets the record.
  static constexpr int kProfValues = 16;
  void prof_read(double* out, int n) {
    double v[kProfValues] = {};
    check_cuda(cudaStreamSynchronize(ctx().stream), "profile sync");
    for (Mark& m : marks) {
      float ms = 0.0f;
      check_cuda(cudaEventElapsedTime(&ms, m.a, m.b), "cudaEventElapsedTime");
      switch (m.cat) {
        case 0: case 1: {  // GEMM, attention: ms, FLOP, launches
          const int base = m.cat == 0 ? 0 : 3;
          v[base] += ms;
          v[base + 1] += m.flop;
          v[base + 2] += 1.0;
          break;
        }
        case 2: v[6] += ms; v[7] += 1.0; break;          // whole forward
        case 3: v[8] += ms; v[9] += 1.0; break;          // collectives and barriers
        case 4: case 5: {  // post-norm, adaLN GEMV: ms, bytes, launches
          const int base = m.cat == 4 ? 10 : 13;
          v[base] += ms;
          v[base + 1] += m.flop;
          v[base + 2] += 1.0;
          break;
        }
        default: break;
      }
    }
    for (int i = 0; i < n && i < kProfValues; ++i) out[i] = v[i];
    prof_clear();
  }

  const WRef& get(const std::string& n) const {
    auto it = w.find(n);
    if (it == w.end()) fail(kErrInvalidArg, "zimage: missing weight: " + n);
    return it->second;
  }
  const WRef* try_get(const std::string& n) const {
    auto it = w.find(n);
    return it == w.end() ? nullptr : &it->second;
  }
  const float* f32(const std::string& n) const {
    const WRef& r = get(n);
    if (r.bf16) fail(kErrInvalidArg, "zimage: " + n + " must be fp32");
    return static_cast<const float*>(r.p);
  }
  const uint16_t* bf16w(const std::string& n) const {
    const WRef& r = get(n);
    if (!r.bf16) fail(kErrInvalidArg, "zimage: " + n + " must be bf16 (block linears run on the bf16 path)");
    return static_cast<const uint16_t*>(r.p);
  }

  Block load_block(const std::string& p, bool modulated) {
    Block b;
    b.attn_norm1 = f32(p + ".attention_norm1.weight");
    b.attn_norm2 = f32(p + ".attention_norm2.weight");
    b.ffn_norm1 = f32(p + ".ffn_norm1.weight");
    b.ffn_norm2 = f32(p + ".ffn_norm2.weight");
    b.norm_q = f32(p + ".attention.norm_q.weight");
    b.norm_k = f32(p + ".attention.norm_k.weight");
    const uint16_t* wq = bf16w(p + ".attention.to_q.weight");
    const uint16_t* wk = bf16w(p + ".attention.to_k.weight");
    const uint16_t* wv = bf16w(p + ".attention.to_v.weight");
    // With tensor parallelism the caller registers this rank's column shards: the rows
    // of to_q / to_k / to_v for its heads, the matching columns of to_out.
    b.Dq = get(p + ".attention.to_q.weight").dim(0);
    if (b.Dq % head_dim || get(p + ".attention.to_q.weight").dim(1) != D) fail(kErrInvalidArg, "zimage: to_q shape");
    b.heads_local = (int)(b.Dq / head_dim);
    if (get(p + ".attention.to_out.0.weight").dim(1) != b.Dq) fail(kErrInvalidArg, "zimage: to_out shard mismatch");
    const size_t mat = (size_t)(b.Dq * D) * 2;
    b.wqkv.ensure(3 * mat);
    cudaStream_t s = ctx().stream;
    check_cuda(cudaMemcpyAsync(b.wqkv.as<uint8_t>(), wq, mat, cudaMemcpyDeviceToDevice, s), "zimage wqkv");
    check_cuda(cudaMemcpyAsync(b.wqkv.as<uint8_t>() + mat, wk, mat, cudaMemcpyDeviceToDevice, s), "zimage wqkv");
    check_cuda(cudaMemcpyAsync(b.wqkv.as<uint8_t>() + 2 * mat, wv, mat, cudaMemcpyDeviceToDevice, s), "zimage wqkv");
    const WRef* bq = try_get(p + ".attention.to_q.bias");
    const WRef* bk = try_get(p + ".attention.to_k.bias");
    const WRef* bv = try_get(p + ".attention.to_v.bias");
    if (bq || bk || bv) {
      b.has_bqkv = true;
      b.bqkv.ensure((size_t)(3 * b.Dq) * 4);
      check_cuda(cudaMemsetAsync(b.bqkv.p, 0, (size_t)(3 * b.Dq) * 4, s), "zimage bqkv");
      const WRef* bb[3] = {bq, bk, bv};
      for (int i = 0; i < 3; ++i)
        if (bb[i])
          check_cuda(cudaMemcpyAsync(b.bqkv.as<float>() + i * b.Dq, bb[i]->p, (size_t)b.Dq * 4,
                                     cudaMemcpyDeviceToDevice, s),
                     "zimage bqkv");
    }
    b.wout = bf16w(p + ".attention.to_out.0.weight");
    const WRef* bo = try_get(p + ".attention.to_out.0.bias");
    b.bout = bo ? static_cast<const float*>(bo->p) : nullptr;
    const WRef& w1 = get(p + ".feed_forward.w1.weight");
    b.F = w1.dim(0);
    if (b.F % 16) fail(kErrInvalidArg, "zimage: FFN width must be a multiple of 16");
    b.w13.ensure((size_t)(2 * b.F * D) * 2);
    dit_interleave_rows16(bf16w(p + ".feed_forward.w1.weight"), bf16w(p + ".feed_forward.w3.weight"), b.w13.p, b.F, D,
                          2);
    const WRef* b1 = try_get(p + ".feed_forward.w1.bias");
    const WRef* b3 = try_get(p + ".feed_forward.w3.bias");
    if (b1 || b3) {
      if (!b1 || !b3) fail(kErrUnsupported, "zimage: w1/w3 must both have biases or neither");
      b.has_b13 = true;
      b.b13.ensure((size_t)(2 * b.F) * 4);
      dit_interleave_rows16(b1->p, b3->p, b.b13.p, b.F, 1, 4);
    }
    b.w2 = bf16w(p + ".feed_forward.w2.weight");
    const WRef* b2 = try_get(p + ".feed_forward.w2.bias");
    b.b2 = b2 ? static_cast<const float*>(b2->p) : nullptr;
    if (modulated) {
      b.adaln = bf16w(p + ".adaLN_modulation.0.weight");
      const WRef* ab = try_get(p + ".adaLN_modulation.0.bias");
      b.adaln_b = ab ? static_cast<const float*>(ab->p) : nullptr;
      if (get(p + ".adaLN_modulation.0.weight").dim(0) != 4 * D) fail(kErrInvalidArg, "zimage: adaLN width != 4*dim");
    }
    return b;
  }

  void finalize() {
    const WRef& xe = get("all_x_embedder.2-1.weight");
    D = xe.dim(0);
    if (D % heads) fail(kErrInvalidArg, "zimage: dim not divisible by heads");
    head_dim = D / heads;
    if (head_dim != 128) fail(kErrUnsupported, "zimage: head dim must be 128 (Z-Image)");
    if (axes[0] + axes[1] + axes[2] != head_dim) fail(kErrInvalidArg, "zimage: axes_dims must sum to the head dim");
    in_ch = xe.dim(1) / (patch * patch);
    tdim = get("t_embedder.mlp.0.weight").dim(1);
    for (int i = 0; has("noise_refiner." + std::to_string(i) + ".attention_norm1.weight"); ++i)
      noise.push_back(load_block("noise_refiner." + std::to_string(i), true));
    for (int i = 0; has("context_refiner." + std::to_string(i) + ".attention_norm1.weight"); ++i)
      context.push_back(load_block("context_refiner." + std::to_string(i), false));
    for (int i = 0; has("layers." + std::to_string(i) + ".attention_norm1.weight"); ++i)
      layers.push_back(load_block("layers." + std::to_string(i), true));
    if (layers.empty()) fail(kErrInvalidArg, "zimage: no transformer layers found");
    finalized = true;
  }
  bool has(const std::string& n) const { return w.count(n) != 0; }

  // ---- activations (grown on demand) ----------------------------------------------
  DBuf tok, img, cap, uni, h, q16, k16, v16, ao, a, g, mod, temb, thid, adaln, fscale, capn, outtok, fin;
  std::map<std::array<int64_t, 3>, std::unique_ptr<DBuf[]>> tables;  // (Ht, Wt, n_cap_pad) -> cos/sin sets

  // Rotary tables for (axis0, h, w) positions, interleaved layout (zimage.cpp:71-88):
  // freq = theta^(-2k/d_a) in double, angle = (float)(pos * freq), cos/sin in float.
  // cs holds cos at both columns of a rotary pair, sn holds (-sin, +sin), the operand
  // layout of the QKV epilogue's packed rotation (Epi::kQkvRope).
  void rope_tables(const std::vector<std::array<int, 3>>& pos, std::vector<float>& cs, std::vector<float>& sn) const {
    const int64_t S = (int64_t)pos.size(), d = head_dim;
    cs.assign((size_t)(S * d), 0.0f);
    sn.assign((size_t)(S * d), 0.0f);
    for (int64_t s = 0; s < S; ++s) {
      int64_t off = 0;
      for (int a = 0; a < 3; ++a) {
        const int da = axes[a];
        for (int k = 0; k < da / 2; ++k) {
          const double freq = 1.0 / std::pow((double)rope_theta, (double)(2 * k) / (double)da);
          const float ang = (float)((double)pos[s][a] * freq);
          const float c = std::cos(ang), si = std::sin(ang);
          cs[s * d + off + 2 * k] = cs[s * d + off + 2 * k + 1] = c;
          sn[s * d + off + 2 * k] = -si;
          sn[s * d + off + 2 * k + 1] = si;
        }
        off += da;
      }
    }
  }

  // Returns [img cos, img sin, cap cos, cap sin, uni cos, uni sin] on the device.
  DBuf* get_tables(int64_t Ht, int64_t Wt, int64_t n_img_pad, int64_t n_cap_pad) {
    auto key = std::array<int64_t, 3>{Ht, Wt, n_cap_pad};
    auto it = tables.find(key);
    if (it != tables.end()) return it->second.get();
    std::vector<std::array<int, 3>> cap_pos(n_cap_pad), img_pos(n_img_pad, {0, 0, 0});
    for (int64_t i = 0; i < n_cap_pad; ++i) cap_pos[i] = {(int)(1 + i), 0, 0};
    for (int64_t hh = 0; hh < Ht; ++hh)
      for (int64_t ww = 0; ww < Wt; ++ww) img_pos[hh * Wt + ww] = {(int)(n_cap_pad + 1), (int)hh, (int)ww};
    std::vector<std::array<int, 3>> uni_pos = img_pos;
    uni_pos.insert(uni_pos.end(), cap_pos.begin(), cap_pos.end());
    std::unique_ptr<DBuf[]> t(new DBuf[6]);
    const std::vector<std::array<int, 3>>* sets[3] = {&img_pos, &cap_pos, &uni_pos};
    for (int i = 0; i < 3; ++i) {
      std::vector<float> c, s;
      rope_tables(*sets[i], c, s);
      const size_t bytes = c.size() * 4;
      t[2 * i].ensure(bytes);
      t[2 * i + 1].ensure(bytes);
      check_cuda(cudaMemcpy(t[2 * i].p, c.data(), bytes, cudaMemcpyHostToDevice), "zimage tables");
      check_cuda(cudaMemcpy(t[2 * i + 1].p, s.data(), bytes, cudaMemcpyHostToDevice), "zimage tables");
    }
    DBuf* raw = t.get();
    tables[key] = std::move(t);
    return raw;
  }

  // Tensor-parallel group (null or world 1: the whole model on this GPU).
  Comm* comm = nullptr;
  // 1: stages run through run_stage_sp (on one GPU too, where the scatter is a local
  // store and the post-norm also forms the next GEMM input); world > 1 then shares the
  // row-parallel outputs through the owners' memory. 0: run_block per block, with an
  // NCCL all-reduce of the full partial outputs under tensor parallelism.
  int tp_mode = 1;
  SymBuf tp_slots, tp_h;  // per rank: world partial slots of its rows (fp32), the full bf16 GEMM input
  DBuf mods;              // modulation vectors of every block of a stage [blocks, 4D]

  void release_tp() {
    comm_sym_free(comm, tp_slots);
    comm_sym_free(comm, tp_h);
  }
  int64_t rows_alloc(int64_t R) const {
    const int64_t w = comm_world(comm);
    return (R + w - 1) / w * w;
  }

  // Algorithmic bytes of one post-norm launch over `own` rows: the world partial rows and
  // x read, x written, the next GEMM's bf16 row stored into nh buffers.
  double post_norm_bytes(int64_t own, int world, int nh) const {
    return (double)own * (double)D * (4.0 * world + 8.0 + 2.0 * nh);
  }
  // Algorithmic bytes of one adaLN GEMV: the bf16 weights [4D, tdim], the fp32 input,
  // bias and output.
  double adaln_bytes() const { return 2.0 * 4 * D * tdim + 4.0 * tdim + 8.0 * 4 * D; }

  void run_stage(const std::vector<Block>& blocks, float* x, int64_t B, int64_t S, const float* cs, const float* sn,
                 bool modulated) {
    if (blocks.empty()) return;
    if (tp_mode == 1) {
      run_stage_sp(blocks, x, B, S, cs, sn, modulated);
      return;
    }
    for (const Block& b : blocks) run_block(b, x, B, S, cs, sn, modulated);
  }

  // A stage of blocks under tensor parallelism with the exchange fused into the kernels.
  // Rank rk owns rows [rk * Rs, rk * Rs + Rs) of the B*S rows. Per block:
  //   QKV GEMM (column-parallel, this rank's heads) + attention on all rows, then
  //   to_out GEMM whose epilogue stores each partial row into its owner's slot;
  //   barrier; the owner sums the world slots of its rows, applies post-norm + gated
  //   residual to its rows of x, and stores the FFN's bf16 input row on every rank;
  //   barrier; w1/w3 SwiGLU and w2 the same way; the second post-norm stores the next
  //   block's attention input. x is exact on owned rows only; the stage ends with an
  //   all-gather of x. NCCL moves no activation data inside the stage.
  void run_stage_sp(const std::vector<Block>& blocks, float* x, int64_t B, int64_t S, const float* cs, const float* sn,
                    bool modulated) {
    const int w = comm_world(comm), rk = comm_rank(comm);
    const int64_t R = B * S, Rs = (R + w - 1) / w, row0 = (int64_t)rk * Rs;
    const int64_t own = std::max<int64_t>(0, std::min<int64_t>(Rs, R - row0));
    // Symmetric buffers; every rank runs the same shapes, so growth is collective.
    const size_t slot_bytes = (size_t)(w * Rs * D) * 4, h_bytes = (size_t)(w * Rs * D) * 2;
    if (tp_slots.bytes < slot_bytes) comm_sym_alloc(comm, tp_slots, slot_bytes);
    if (tp_h.bytes < h_bytes) comm_sym_alloc(comm, tp_h, h_bytes);
    const int64_t nb = (int64_t)blocks.size();
    mods.ensure((size_t)(nb * 4 * D) * 4);
    if (modulated)
      for (int64_t i = 0; i < nb; ++i) {
        float* mi = mods.as<float>() + i * 4 * D;
        timed(5, adaln_bytes(), [&] {
          gemm_nt_bf16_impl(1, 4 * D, tdim, adaln.as<float>(), tdim, blocks[i].adaln, tdim, mi, 4 * D,
                            blocks[i].adaln_b, false);
        });
        dit_adaln_split(mi, (int)D);
      }
    auto part = [&](int64_t i, int k) -> const float* {  // 0 scale_msa, 1 gate_msa, 2 scale_mlp, 3 gate_mlp
      return modulated ? mods.as<float>() + i * 4 * D + k * D : nullptr;
    };
    uint16_t* hloc = static_cast<uint16_t*>(tp_h.local);
    uint16_t* hall[kMaxTpRanks] = {};
    ScatterOut so{};
    for (int q = 0; q < w; ++q) {
      hall[q] = static_cast<uint16_t*>(tp_h.peer[q]);
      so.base[q] = static_cast<float*>(tp_slots.peer[q]);
    }
    so.slot_rows = Rs;
    so.rs = (int)Rs;
    so.rank = rk;
    const float* slots = static_cast<const float*>(tp_slots.local);
    const double gf = 2.0 * (double)R;
    // The stage's first input: x is complete on every rank here.
    dit_rms_mod_bf16(x, hloc, R, (int)D, blocks[0].attn_norm1, part(0, 0), norm_eps);
    for (int64_t i = 0; i < nb; ++i) {
      const Block& b = blocks[i];
      const int64_t Dq = b.Dq;
      const int Hl = b.heads_local;
      QkvRope rp{};
      rp.S = (int)S;
      rp.Dq = (int)Dq;
      rp.gq = b.norm_q;
      rp.gk = b.norm_k;
      rp.cs = cs;
      rp.sn = sn;
      rp.eps = 1e-5f;
      rp.q16 = q16.p;
      rp.k16 = k16.p;
      rp.v16 = v16.p;
      timed(0, gf * 3 * Dq * D, [&] {
        gemm_bf16_qkv_rope_impl(R, D, hloc, D, true, b.wqkv.as<uint16_t>(), D, b.has_bqkv ? b.bqkv.as<float>() : nullptr,
                                rp);
      });
      timed(1, 4.0 * (double)B * S * S * Dq, [&] {
        launch_attention_f16(q16.p, k16.p, v16.p, ao.p, Dq, S * Dq, true, B, S, S, Hl, Hl, head_dim, 128, false);
      });
      timed(0, gf * D * Dq, [&] { gemm_bf16_scatter_impl(R, D, Dq, ao.p, Dq, true, b.wout, Dq, b.bout, so); });
      timed(3, 0.0, [&] { comm_barrier(comm); });
      timed(4, post_norm_bytes(own, w, w), [&] {
        dit_post_norm_mod_bcast(slots, Rs, w, row0, own, x, (int)D, b.attn_norm2, part(i, 1), b.ffn_norm1, part(i, 2),
                                hall, w, norm_eps);
      });
      timed(3, 0.0, [&] { comm_barrier(comm); });
      timed(0, gf * 2 * b.F * D, [&] {
        gemm_bf16_epilogue_impl(R, 2 * b.F, D, hloc, D, true, b.w13.as<uint16_t>(), D, g.p, b.F, true,
                                b.has_b13 ? b.b13.as<float>() : nullptr, 1);
      });
      timed(0, gf * b.F * D, [&] { gemm_bf16_scatter_impl(R, D, b.F, g.p, b.F, true, b.w2, b.F, b.b2, so); });
      timed(3, 0.0, [&] { comm_barrier(comm); });
      if (i + 1 < nb) {
        timed(4, post_norm_bytes(own, w, w), [&] {
          dit_post_norm_mod_bcast(slots, Rs, w, row0, own, x, (int)D, b.ffn_norm2, part(i, 3), blocks[i + 1].attn_norm1,
                                  part(i + 1, 0), hall, w, norm_eps);
        });
        timed(3, 0.0, [&] { comm_barrier(comm); });
      } else {
        timed(4, post_norm_bytes(own, w, 0), [&] {
          dit_post_norm_mod_bcast(slots, Rs, w, row0, own, x, (int)D, b.ffn_norm2, part(i, 3), nullptr, nullptr, hall,
                                  0, norm_eps);
        });
      }
    }
    // Every rank gets every row of x (the buffer holds w * Rs rows).
    timed(3, 0.0, [&] { comm_allgather(comm, x + row0 * D, x, (size_t)(Rs * D) * 4); });
  }

  // One block on x [B*S, D] (B sequences of S rows), rotary tables [S, 128]. Under tensor
  // parallelism this rank holds heads_local heads and F of the FFN; the row-parallel
  // outputs of to_out and w2 are summed over the group before the post-norm.
  void run_block(const Block& b, float* x, int64_t B, int64_t S, const float* cs, const float* sn, bool modulated) {
    const int64_t R = B * S;
    const float *scale_msa = nullptr, *gate_msa = nullptr, *scale_mlp = nullptr, *gate_mlp = nullptr;
    if (modulated) {
      timed(5, adaln_bytes(), [&] {
        gemm_nt_bf16_impl(1, 4 * D, tdim, adaln.as<float>(), tdim, b.adaln, tdim, mod.as<float>(), 4 * D, b.adaln_b,
                          false);
      });
      dit_adaln_split(mod.as<float>(), (int)D);
      scale_msa = mod.as<float>();
      gate_msa = scale_msa + D;
      scale_mlp = scale_msa + 2 * D;
      gate_mlp = scale_msa + 3 * D;
    }
    // attention
    dit_rms_mod_bf16(x, h.as<uint16_t>(), R, (int)D, b.attn_norm1, scale_msa, norm_eps);
    const int64_t Dq = b.Dq;
    const int Hl = b.heads_local;
    const double gf = 2.0 * (double)R;  // 2*M, times N*K per GEMM below
    // QKV projection with the QK norm, rotary embedding and fp16 head packing in the GEMM
    // epilogue (q16 / k16 / v16 = [B*S, Dq] = [B, S, heads, 128]).
    QkvRope rp{};
    rp.S = (int)S;
    rp.Dq = (int)Dq;
    rp.gq = b.norm_q;
    rp.gk = b.norm_k;
    rp.cs = cs;
    rp.sn = sn;
    rp.eps = 1e-5f;
    rp.q16 = q16.p;
    rp.k16 = k16.p;
    rp.v16 = v16.p;
    timed(0, gf * 3 * Dq * D, [&] {
      gemm_bf16_qkv_rope_impl(R, D, h.p, D, true, b.wqkv.as<uint16_t>(), D, b.has_bqkv ? b.bqkv.as<float>() : nullptr,
                              rp);
    });
    timed(1, 4.0 * (double)B * S * S * Dq, [&] {
      launch_attention_f16(q16.p, k16.p, v16.p, ao.p, Dq, S * Dq, true, B, S, S, Hl, Hl, head_dim, 128, false);
    });
    timed(0, gf * D * Dq, [&] { gemm_bf16_epilogue_impl(R, D, Dq, ao.p, Dq, true, b.wout, Dq, a.p, D, false, b.bout, 0); });
    if (comm_world(comm) > 1) timed(3, 0.0, [&] { comm_allreduce_sum(comm, a.as<float>(), (size_t)(R * D)); });
    timed(4, 12.0 * (double)(R * D), [&] { dit_post_norm_residual(x, a.as<float>(), R, (int)D, b.attn_norm2, gate_msa, norm_eps); });
    // feed-forward
    dit_rms_mod_bf16(x, h.as<uint16_t>(), R, (int)D, b.ffn_norm1, scale_mlp, norm_eps);
    timed(0, gf * 2 * b.F * D, [&] {
      gemm_bf16_epilogue_impl(R, 2 * b.F, D, h.p, D, true, b.w13.as<uint16_t>(), D, g.p, b.F, true,
                              b.has_b13 ? b.b13.as<float>() : nullptr, 1);
    });
    timed(0, gf * b.F * D, [&] { gemm_bf16_epilogue_impl(R, D, b.F, g.p, b.F, true, b.w2, b.F, a.p, D, false, b.b2, 0); });
    if (comm_world(comm) > 1) timed(3, 0.0, [&] { comm_allreduce_sum(comm, a.as<float>(), (size_t)(R * D)); });
    timed(4, 12.0 * (double)(R * D), [&] { dit_post_norm_residual(x, a.as<float>(), R, (int)D, b.ffn_norm2, gate_mlp, norm_eps); });
  }

  static int64_t pad_to(int64_t n) { return (n + 31) / 32 * 32; }

  // The sampler of the Z-Image pipeline (pipeline.cpp:229-244) with every step on the
  // device: steps flow-matching Euler steps from the latent x (in place) under the
  // text states cap (and cap_neg with guidance cfg > 0). Model time of step i is
  // 1 - sigma_i; the update is x += (sigma_i - sigma_(i+1)) * prediction.
  void sample(float* x, int64_t B, int64_t C, int64_t H, int64_t W, const float* cap, const float* cap_neg, int64_t L,
              int64_t capdim, float cfg, int steps, float shift) {
    if (!finalized) fail(kErrInvalidArg, "zimage: finalize() not called");
    if (steps < 1) fail(kErrInvalidArg, "zimage_sample: steps must be >= 1");
    const bool use_cfg = cfg > 0.0f;
    if (use_cfg && !cap_neg) fail(kErrInvalidArg, "zimage_sample: cfg > 0 needs the negative text states");
    std::vector<float> sig((size_t)steps + 1);
    flow_sigmas(steps, shift, sig.data());
    const int64_t n = B * C * H * W;
    pred.ensure((size_t)n * 4);
    if (use_cfg) pred_neg.ensure((size_t)n * 4);
    for (int i = 0; i < steps; ++i) {
      const float t = 1.0f - sig[(size_t)i];
      forward(x, B, C, H, W, t, cap, L, capdim, pred.as<float>());
      if (use_cfg) forward(x, B, C, H, W, t, cap_neg, L, capdim, pred_neg.as<float>());
      dit_flow_step(x, pred.as<float>(), use_cfg ? pred_neg.as<float>() : nullptr, cfg,
                    sig[(size_t)i] - sig[(size_t)i + 1], n);
    }
  }
  DBuf pred, pred_neg;

  // x [B, C, H, W], cap [B, L, capdim] -> out [B, C, H, W] (zimage.cpp:138-228).
  void forward(const float* x_in, int64_t B, int64_t C, int64_t H, int64_t W, float t, const float* cap_in, int64_t L,
               int64_t capdim, float* out) {
    if (!finalized) fail(kErrInvalidArg, "zimage: finalize() not called");
    timed(2, 0.0, [&] { forward_impl(x_in, B, C, H, W, t, cap_in, L, capdim, out); });
  }

  void forward_impl(const float* x_in, int64_t B, int64_t C, int64_t H, int64_t W, float t, const float* cap_in,
                    int64_t L, int64_t capdim, float* out) {
    const int64_t p = patch;
    if (C != in_ch || H % p || W % p || B < 1) fail(kErrInvalidArg, "zimage: bad latent shape");
    const int64_t Ht = H / p, Wt = W / p, n_img = Ht * Wt, n_img_pad = pad_to(n_img);
    const int64_t n_cap_pad = pad_to(L), S = n_img_pad + n_cap_pad;
    int64_t F = 0, Dq = 0;
    for (const std::vector<Block>* v : {&noise, &context, &layers})
      for (const Block& b : *v) {
        F = std::max(F, b.F);
        Dq = std::max(Dq, b.Dq);
      }
    cudaStream_t st = ctx().stream;
    DBuf* tb = get_tables(Ht, Wt, n_img_pad, n_cap_pad);
    // activations
    const int64_t Rmax = B * S;
    tok.ensure((size_t)(B * n_img * p * p * C) * 4);
    // x buffers hold a whole number of per-rank row blocks (tensor parallelism gathers them)
    img.ensure((size_t)(rows_alloc(B * n_img_pad) * D) * 4);
    cap.ensure((size_t)(rows_alloc(B * n_cap_pad) * D) * 4);
    uni.ensure((size_t)(rows_alloc(Rmax) * D) * 4);
    if (tp_mode == 0) h.ensure((size_t)(Rmax * D) * 2);  // run_block's GEMM input
    q16.ensure((size_t)(Rmax * Dq) * 2);
    k16.ensure((size_t)(Rmax * Dq) * 2);
    v16.ensure((size_t)(Rmax * Dq) * 2);
    ao.ensure((size_t)(Rmax * Dq) * 2);
    if (tp_mode == 0) a.ensure((size_t)(Rmax * D) * 4);  // run_block's row-parallel outputs
    g.ensure((size_t)(Rmax * F) * 2);
    mod.ensure((size_t)(4 * D) * 4);
    const WRef& t0 = get("t_embedder.mlp.0.weight");
    temb.ensure((size_t)tdim * 4);
    thid.ensure((size_t)t0.dim(0) * 4);
    adaln.ensure((size_t)tdim * 4);
    fscale.ensure((size_t)D * 4);
    capn.ensure((size_t)(B * L * capdim) * 4);
    outtok.ensure((size_t)(B * n_img * p * p * C) * 4);
    fin.ensure((size_t)(B * n_img * D) * 4);

    // Tensor parallelism with fused exchange: size the symmetric buffers once for the
    // largest stage (collective; every rank runs the same shapes).
    if (tp_mode == 1) {
      const int64_t w = comm_world(comm), Rs = (Rmax + w - 1) / w;
      if (tp_slots.bytes < (size_t)(w * Rs * D) * 4) comm_sym_alloc(comm, tp_slots, (size_t)(w * Rs * D) * 4);
      if (tp_h.bytes < (size_t)(w * Rs * D) * 2) comm_sym_alloc(comm, tp_h, (size_t)(w * Rs * D) * 2);
    }
    // 1. timestep embedding -> adaln [1, tdim]
    dit_timestep_embed(temb.as<float>(), (int)tdim, t * t_scale);
    linear(temb.as<float>(), 1, tdim, t0, try_get("t_embedder.mlp.0.bias"), thid.as<float>());
    op_unary(thid.as<float>(), t0.dim(0), 0);  // silu
    linear(thid.as<float>(), 1, t0.dim(0), get("t_embedder.mlp.2.weight"), try_get("t_embedder.mlp.2.bias"),
           adaln.as<float>());
    // 2. image tokens: patchify, embed, pad
    const int64_t tokw = p * p * C;
    for (int64_t n = 0; n < B; ++n) {
      op_patchify(x_in + n * C * H * W, tok.as<float>() + n * n_img * tokw, C, H, W, (int)p);
      linear(tok.as<float>() + n * n_img * tokw, n_img, tokw, get("all_x_embedder.2-1.weight"),
             try_get("all_x_embedder.2-1.bias"), img.as<float>() + n * n_img_pad * D);
      dit_fill_rows(img.as<float>() + n * n_img_pad * D, f32("x_pad_token"), n_img, n_img_pad, (int)D);
    }
    // 3. text tokens: RMSNorm, embed, pad
    op_row_norm(cap_in, capn.as<float>(), B * L, capdim, f32("cap_embedder.0.weight"), nullptr, norm_eps, true);
    for (int64_t n = 0; n < B; ++n) {
      linear(capn.as<float>() + n * L * capdim, L, capdim, get("cap_embedder.1.weight"), try_get("cap_embedder.1.bias"),
             cap.as<float>() + n * n_cap_pad * D);
      dit_fill_rows(cap.as<float>() + n * n_cap_pad * D, f32("cap_pad_token"), L, n_cap_pad, (int)D);
    }
    // refiners
    run_stage(noise, img.as<float>(), B, n_img_pad, tb[0].as<float>(), tb[1].as<float>(), true);
    run_stage(context, cap.as<float>(), B, n_cap_pad, tb[2].as<float>(), tb[3].as<float>(), false);
    // 4. unified [image, text] per sample, main stack
    for (int64_t n = 0; n < B; ++n) {
      check_cuda(cudaMemcpyAsync(uni.as<float>() + n * S * D, img.as<float>() + n * n_img_pad * D,
                                 (size_t)(n_img_pad * D) * 4, cudaMemcpyDeviceToDevice, st),
                 "zimage concat");
      check_cuda(cudaMemcpyAsync(uni.as<float>() + (n * S + n_img_pad) * D, cap.as<float>() + n * n_cap_pad * D,
                                 (size_t)(n_cap_pad * D) * 4, cudaMemcpyDeviceToDevice, st),
                 "zimage concat");
    }
    run_stage(layers, uni.as<float>(), B, S, tb[4].as<float>(), tb[5].as<float>(), true);
    // 5. final layer on the image tokens: LayerNorm * (1 + adaLN(silu(t_emb))), linear, unpatchify
    {
      check_cuda(cudaMemcpyAsync(temb.p, adaln.p, (size_t)tdim * 4, cudaMemcpyDeviceToDevice, st), "zimage final");
      op_unary(temb.as<float>(), tdim, 0);  // silu(adaln) (the reference silus a copy)
      linear(temb.as<float>(), 1, tdim, get("all_final_layer.2-1.adaLN_modulation.1.weight"),
             try_get("all_final_layer.2-1.adaLN_modulation.1.bias"), fscale.as<float>());
      op_affine(fscale.as<float>(), 1.0f, 1.0f, D);
    }
    for (int64_t n = 0; n < B; ++n) {
      dit_layer_norm_mod(uni.as<float>() + n * S * D, fin.as<float>() + n * n_img * D, n_img, (int)D,
                         fscale.as<float>(), 1e-6f);
    }
    linear(fin.as<float>(), B * n_img, D, get("all_final_layer.2-1.linear.weight"),
           try_get("all_final_layer.2-1.linear.bias"), outtok.as<float>());
    for (int64_t n = 0; n < B; ++n)
      op_unpatchify(outtok.as<float>() + n * n_img * tokw, out + n * C * H * W, C, H, W, (int)p);
  }
};

}  // namespace sdb

// ===================================================================================
using sdb::ZImage;

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

void* sdb200_zimage_create(int heads, int patch, float norm_eps, float rope_theta, float t_scale, int ax0, int ax1,
                           int ax2) {
  try {
    if (heads <= 0 || patch <= 0) sdb::fail(sdb::kErrInvalidArg, "zimage_create: bad config");
    return new ZImage(heads, patch, norm_eps, rope_theta, t_scale, ax0, ax1, ax2);
  } catch (const sdb::Error& e) {
    sdb::set_last_error(e.msg);
    return nullptr;
  }
}

int sdb200_zimage_set_weight(void* m, const char* name, const void* dev_ptr, int is_bf16, const int64_t* shape,
                             int ndim) {
  SDB_GUARD({
    if (!m || !name || !dev_ptr || !shape || ndim <= 0) sdb::fail(sdb::kErrInvalidArg, "zimage_set_weight: bad args");
    ZImage* z = static_cast<ZImage*>(m);
    if (z->finalized) sdb::fail(sdb::kErrInvalidArg, "zimage_set_weight: model already finalized");
    sdb::WRef r;
    r.p = dev_ptr;
    r.bf16 = is_bf16 != 0;
    r.shape.assign(shape, shape + ndim);
    z->w[name] = r;
  })
}

int sdb200_zimage_finalize(void* m) {
  SDB_GUARD({
    if (!m) sdb::fail(sdb::kErrInvalidArg, "zimage_finalize: null model");
    static_cast<ZImage*>(m)->finalize();
  })
}

int sdb200_zimage_forward(void* m, const float* x, int64_t B, int64_t C, int64_t H, int64_t W, float t,
                          const float* cap, int64_t L, int64_t capdim, float* out) {
  SDB_GUARD({
    if (!m || !x || !cap || !out) sdb::fail(sdb::kErrInvalidArg, "zimage_forward: null pointer");
    static_cast<ZImage*>(m)->forward(x, B, C, H, W, t, cap, L, capdim, out);
  })
}

int sdb200_zimage_profile(void* m, int enable) {
  SDB_GUARD({
    if (!m) sdb::fail(sdb::kErrInvalidArg, "zimage_profile: null model");
    ZImage* z = static_cast<ZImage*>(m);
    z->prof_clear();
    z->prof_on = enable != 0;
  })
}

int sdb200_zimage_profile_read(void* m, double* out10) {
  SDB_GUARD({
    if (!m || !out10) sdb::fail(sdb::kErrInvalidArg, "zimage_profile_read: null pointer");
    static_cast<ZImage*>(m)->prof_read(out10, 10);
  })
}

int sdb200_zimage_profile_read_ex(void* m, double* out, int n) {
  SDB_GUARD({
    if (!m || !out || n < 0) sdb::fail(sdb::kErrInvalidArg, "zimage_profile_read_ex: null pointer or n < 0");
    static_cast<ZImage*>(m)->prof_read(out, n);
  })
}

int sdb200_zimage_set_tp(void* m, void* comm) {
  SDB_GUARD({
    if (!m) sdb::fail(sdb::kErrInvalidArg, "zimage_set_tp: null model");
    ZImage* z = static_cast<ZImage*>(m);
    z->release_tp();
    z->comm = static_cast<sdb::Comm*>(comm);
  })
}

int sdb200_zimage_sample(void* m, float* x, int64_t B, int64_t C, int64_t H, int64_t W, const float* cap,
                         const float* cap_neg, int64_t L, int64_t capdim, float cfg, int steps, float shift) {
  SDB_GUARD({
    if (!m || !x || !cap) sdb::fail(sdb::kErrInvalidArg, "zimage_sample: null pointer");
    static_cast<ZImage*>(m)->sample(x, B, C, H, W, cap, cap_neg, L, capdim, cfg, steps, shift);
  })
}

int sdb200_zimage_load(void* m, const char* dir, const char* base, int rank, int world, int64_t bf16_min_numel) {
  SDB_GUARD({
    if (!m || !dir || !base) sdb::fail(sdb::kErrInvalidArg, "zimage_load: null argument");
    if (world < 1 || rank < 0 || rank >= world) sdb::fail(sdb::kErrInvalidArg, "zimage_load: bad rank / world");
    ZImage* z = static_cast<ZImage*>(m);
    if (z->finalized) sdb::fail(sdb::kErrInvalidArg, "zimage_load: model already finalized");
    sdb::TpShard tp;
    tp.rank = rank;
    tp.world = world;
    tp.heads = z->heads;
    try {
      const std::vector<std::string> files = sdb::checkpoint_files(dir, base);
      sdb::read_checkpoint(files, true, bf16_min_numel > 0 ? bf16_min_numel : ((int64_t)1 << 20),
                           world > 1 ? &tp : nullptr, [&](sdb::HostTensor&& t) {
                             sdb::DBuf buf;
                             buf.ensure(t.data.size());
                             sdb::check_cuda(cudaMemcpy(buf.p, t.data.data(), t.data.size(), cudaMemcpyHostToDevice),
                                             "zimage_load: upload");
                             sdb::WRef r;
                             r.p = buf.p;
                             r.bf16 = t.bf16;
                             r.shape = t.shape;
                             z->owned.push_back(std::move(buf));
                             z->w[t.name] = r;
                           });
    } catch (const std::runtime_error& e) {
      sdb::fail(sdb::kErrInvalidArg, std::string("zimage_load: ") + e.what());
    }
  })
}

int sdb200_checkpoint_read_shard(const char* dir, const char* base, const char* name, int rank, int world, int heads,
                                 int64_t bf16_min_numel, void* dst, int64_t dst_bytes, int64_t* shape, int* ndim,
                                 int* is_bf16) {
  SDB_GUARD({
    if (!dir || !base || !name || !shape || !ndim || !is_bf16)
      sdb::fail(sdb::kErrInvalidArg, "checkpoint_read_shard: null argument");
    if (world < 1 || world > sdb::kMaxTpRanks || rank < 0 || rank >= world || heads < 1)
      sdb::fail(sdb::kErrInvalidArg, "checkpoint_read_shard: bad rank / world / heads");
    sdb::TpShard tp;
    tp.rank = rank;
    tp.world = world;
    tp.heads = heads;
    const std::string want(name);
    *ndim = -1;  // no part of the tensor on this rank (or not read)
    try {
      const std::vector<std::string> files = sdb::checkpoint_files(dir, base);
      sdb::read_checkpoint(
          files, true, bf16_min_numel > 0 ? bf16_min_numel : ((int64_t)1 << 20), world > 1 ? &tp : nullptr,
          [&](sdb::HostTensor&& t) {
            if (t.shape.size() > 8) throw std::runtime_error("more than 8 dimensions");
            *ndim = (int)t.shape.size();
            for (size_t i = 0; i < t.shape.size(); ++i) shape[i] = t.shape[i];
            *is_bf16 = t.bf16 ? 1 : 0;
            if (dst) {
              if ((int64_t)t.data.size() > dst_bytes) throw std::runtime_error("dst too small");
              std::memcpy(dst, t.data.data(), t.data.size());
            }
          },
          &want);
    } catch (const std::runtime_error& e) {
      sdb::fail(sdb::kErrInvalidArg, std::string("checkpoint_read_shard: ") + e.what());
    }
  })
}

int sdb200_zimage_get_weight(void* m, const char* name, void* dst, int64_t dst_bytes, int64_t* shape, int* ndim,
                             int* is_bf16) {
  SDB_GUARD({
    if (!m || !name || !shape || !ndim || !is_bf16) sdb::fail(sdb::kErrInvalidArg, "zimage_get_weight: null argument");
    ZImage* z = static_cast<ZImage*>(m);
    const auto it = z->w.find(name);
    if (it == z->w.end()) sdb::fail(sdb::kErrInvalidArg, std::string("zimage_get_weight: no weight ") + name);
    const sdb::WRef& r = it->second;
    if (r.shape.size() > 8) sdb::fail(sdb::kErrUnsupported, "zimage_get_weight: more than 8 dimensions");
    int64_t n = 1;
    for (size_t i = 0; i < r.shape.size(); ++i) {
      shape[i] = r.shape[i];
      n *= r.shape[i];
    }
    *ndim = (int)r.shape.size();
    *is_bf16 = r.bf16 ? 1 : 0;
    if (dst) {
      const int64_t bytes = n * (r.bf16 ? 2 : 4);
      if (bytes > dst_bytes) sdb::fail(sdb::kErrInvalidArg, "zimage_get_weight: dst too small");
      sdb::check_cuda(cudaStreamSynchronize(sdb::ctx().stream), "zimage_get_weight: sync");
      sdb::check_cuda(cudaMemcpy(dst, r.p, (size_t)bytes, cudaMemcpyDeviceToHost), "zimage_get_weight: copy");
    }
  })
}

int sdb200_safetensors_read(const char* path, const char* name, int keep_bf16, int64_t bf16_min_numel, void* dst,
                            int64_t dst_bytes, int64_t* shape, int* ndim, int* is_bf16) {
  SDB_GUARD({
    if (!path || !name || !shape || !ndim || !is_bf16) sdb::fail(sdb::kErrInvalidArg, "safetensors_read: null argument");
    sdb::HostTensor t;
    bool ok = false;
    try {
      ok = sdb::read_tensor(path, name, keep_bf16 != 0, bf16_min_numel > 0 ? bf16_min_numel : ((int64_t)1 << 20), t);
    } catch (const std::runtime_error& e) {
      sdb::fail(sdb::kErrInvalidArg, std::string("safetensors_read: ") + e.what());
    }
    if (!ok) sdb::fail(sdb::kErrUnsupported, "safetensors_read: dtype not read (F32 / F16 / BF16 only)");
    if (t.shape.size() > 8) sdb::fail(sdb::kErrUnsupported, "safetensors_read: more than 8 dimensions");
    *ndim = (int)t.shape.size();
    for (size_t i = 0; i < t.shape.size(); ++i) shape[i] = t.shape[i];
    if (dst) {
      if ((int64_t)t.data.size() > dst_bytes) sdb::fail(sdb::kErrInvalidArg, "safetensors_read: dst too small");
      std::memcpy(dst, t.data.data(), t.data.size());
    }
    *is_bf16 = t.bf16 ? 1 : 0;
  })
}

int sdb200_flow_sigmas(int steps, float shift, float* sigmas) {
  SDB_GUARD({
    if (steps < 1 || !sigmas) sdb::fail(sdb::kErrInvalidArg, "flow_sigmas: steps must be >= 1 and sigmas non-null");
    sdb::flow_sigmas(steps, shift, sigmas);
  })
}

int sdb200_zimage_set_tp_mode(void* m, int mode) {
  SDB_GUARD({
    if (!m || mode < 0 || mode > 1) sdb::fail(sdb::kErrInvalidArg, "zimage_set_tp_mode: null model or mode not 0/1");
    static_cast<ZImage*>(m)->tp_mode = mode;
  })
}

void sdb200_zimage_destroy(void* m) { delete static_cast<ZImage*>(m); }

}  // extern "C"
