// dit_ops.cu - the memory-bound glue of one Z-Image DiT block, fused around the
// tensor-core GEMMs so activations cross HBM as few times as possible. Each kernel
// names the chain of reference ops it replaces (zimage.cpp:90-136 run_block, built on
// tensor.cpp's rms_norm / mul_rows_ / add_rows_scaled_). The per-head QK norm and the
// rotary embedding (rms_norm_heads_ / rope_) run in the QKV GEMM's epilogue (gemm_tc.cu).
//
//   k_rms_mod_bf16       h = bf16( rms_norm(x, gamma) * scale )   (GEMM A operand)
//   k_post_norm_residual x += gate * rms_norm(a, gamma2)           (or x += rms_norm(a))
//   k_adaln_split        mod[4D] -> (1 + scale_msa, tanh gate_msa, 1 + scale_mlp, tanh gate_mlp)
//   k_timestep_embed     the 256-d sinusoid of t * t_scale (zimage.cpp:151-157)
//   k_layer_norm_mod     y = layer_norm(x, eps) * scale (final layer, zimage.cpp:221-223)
//
// Row kernels run one CTA per token row with 256 threads and float4 loads (D = 3840 =
// 256 x 15, so each thread owns 15 values = 3.75 float4; a scalar tail covers any D).
// Reductions are fp32 warp-shuffle trees.
#include <cuda_fp16.h>

#include <algorithm>
#include <cmath>

#include "internal.h"
#include "ptx.cuh"

namespace sdb {
namespace {

constexpr int kRowThreads = 256;

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float block_sum256(float v, float* red) {
  v = warp_sum(v);
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  __syncthreads();
  if (lane == 0) red[w] = v;
  __syncthreads();
  float t = lane < (kRowThreads / 32) ? red[lane] : 0.0f;
  return warp_sum(t);
}

// h[r, :] = bf16(x[r, :] * rstd * gamma * scale); scale may be null (unmodulated
// blocks). Reference: rms_norm (tensor.cpp:660-679) then mul_rows_ (:889-901), then
// the A-operand rounding of gemm_nt_bf16 (backend_cuda.cu:466-467).
__global__ void __launch_bounds__(kRowThreads) k_rms_mod_bf16(const float* __restrict__ x, uint16_t* __restrict__ h,
                                                              int D, const float* __restrict__ gamma,
                                                              const float* __restrict__ scale, float eps) {
  __shared__ float red[32];
  const float* p = x + (int64_t)blockIdx.x * D;
  uint16_t* q = h + (int64_t)blockIdx.x * D;
  float ss = 0.0f;
  for (int i = threadIdx.x; i < D; i += kRowThreads) ss += p[i] * p[i];
  const float rstd = rsqrtf(block_sum256(ss, red) / (float)D + eps);
  for (int i = threadIdx.x * 2; i < D; i += kRowThreads * 2) {
    float a = p[i] * rstd * (gamma ? gamma[i] : 1.0f);
    if (scale) a *= scale[i];
    if (i + 1 < D) {
      float b = p[i + 1] * rstd * (gamma ? gamma[i + 1] : 1.0f);
      if (scale) b *= scale[i + 1];
      *reinterpret_cast<uint32_t*>(q + i) = pack_bf16x2(a, b);
    } else {
      q[i] = f32_to_bf16_rne(a);
    }
  }
}

// x[r, :] += g * (a[r, :] * rstd(a[r, :]) * gamma); g null means 1 (plain residual).
// Reference: rms_norm (attn_norm2 / ffn_norm2) then add_rows_scaled_ or add_
// (zimage.cpp:122-126, :131-135).
__global__ void __launch_bounds__(kRowThreads) k_post_norm_residual(float* __restrict__ x, const float* __restrict__ a,
                                                                    int D, const float* __restrict__ gamma,
                                                                    const float* __restrict__ g, float eps) {
  __shared__ float red[32];
  const float* p = a + (int64_t)blockIdx.x * D;
  float* y = x + (int64_t)blockIdx.x * D;
  float ss = 0.0f;
  for (int i = threadIdx.x; i < D; i += kRowThreads) ss += p[i] * p[i];
  const float rstd = rsqrtf(block_sum256(ss, red) / (float)D + eps);
  for (int i = threadIdx.x; i < D; i += kRowThreads) {
    const float v = p[i] * rstd * (gamma ? gamma[i] : 1.0f);
    y[i] += g ? g[i] * v : v;
  }
}

// Destinations of a broadcast row: the same buffer on every rank of the group.
struct BcastDst {
  uint16_t* p[kMaxTpRanks];
  int n;
};

// Tensor-parallel post-norm on this rank's rows, fused with the reduction of the
// row-parallel partial outputs and with the next GEMM's input. Owned row lr (global row
// row0 + lr):
//   a   = sum over s of slots[(s * slot_rows + lr) * D + :]   (every rank's partial row,
//         stored there by the GEMM's scatter epilogue; the bias came with rank 0's)
//   x  += g * (a * rstd(a) * gamma2)                          (as k_post_norm_residual)
//   h   = bf16(x * rstd(x) * gamma_n * scale_n) at row row0 + lr of every rank's h,
//         when hd.n > 0 (then hd.n == W)                        (as k_rms_mod_bf16)
// The row lives in shared memory between the passes (D * 4 bytes).
template <int W>
__global__ void __launch_bounds__(kRowThreads) k_post_norm_mod_bcast(
    const float* __restrict__ slots, long long slot_rows, long long row0, float* __restrict__ x, int D,
    const float* __restrict__ gamma2, const float* __restrict__ g, const float* __restrict__ gamma_n,
    const float* __restrict__ scale_n, BcastDst hd, float eps) {
  extern __shared__ float rowbuf[];
  __shared__ float red[32];
  const long long lr = blockIdx.x, row = row0 + lr;
  float ss = 0.0f;
  const float* src = slots + lr * D;
  const long long sstride = slot_rows * D;
#pragma unroll 4
  for (int i = threadIdx.x; i < D; i += kRowThreads) {
    float a = src[i];
#pragma unroll
    for (int s = 1; s < W; ++s) a += src[s * sstride + i];
    rowbuf[i] = a;
    ss += a * a;
  }
  const float rstd = rsqrtf(block_sum256(ss, red) / (float)D + eps);
  float* y = x + row * D;
  float ss2 = 0.0f;
  for (int i = threadIdx.x; i < D; i += kRowThreads) {
    const float v = rowbuf[i] * rstd * (gamma2 ? gamma2[i] : 1.0f);
    const float xn = y[i] + (g ? g[i] * v : v);
    y[i] = xn;
    rowbuf[i] = xn;
    ss2 += xn * xn;
  }
  if (hd.n == 0) return;
  const float rstd2 = rsqrtf(block_sum256(ss2, red) / (float)D + eps);  // also orders the rowbuf writes
  for (int i = threadIdx.x * 2; i < D; i += kRowThreads * 2) {
    float a = rowbuf[i] * rstd2 * (gamma_n ? gamma_n[i] : 1.0f);
    if (scale_n) a *= scale_n[i];
    if (i + 1 < D) {
      float b = rowbuf[i + 1] * rstd2 * (gamma_n ? gamma_n[i + 1] : 1.0f);
      if (scale_n) b *= scale_n[i + 1];
      const uint32_t w = pack_bf16x2(a, b);
#pragma unroll
      for (int q = 0; q < W; ++q) *reinterpret_cast<uint32_t*>(hd.p[q] + row * D + i) = w;
    } else {
      const uint16_t w = f32_to_bf16_rne(a);
#pragma unroll
      for (int q = 0; q < W; ++q) hd.p[q][row * D + i] = w;
    }
  }
  // Stores into peers' memory are visible system-wide before this kernel completes (with
  // one rank every destination is local).
  if (W > 1) __threadfence_system();
}

// Register-resident form of k_post_norm_mod_bcast for D % 4 == 0 and D <= 4096: thread t
// owns the float4 chunks t, t + 256, t + 512, t + 768 of the row, kept in registers across
// the three passes; every global access is 16 bytes (8 for the bf16 rows). Same
// arithmetic per element as the scalar form.
constexpr int kPnChunks = 4;  // float4 chunks per thread: D <= 256 * 4 * 4
template <int W>
__global__ void __launch_bounds__(kRowThreads) k_post_norm_mod_bcast_v4(
    const float* __restrict__ slots, long long slot_rows, long long row0, float* __restrict__ x, int D,
    const float* __restrict__ gamma2, const float* __restrict__ g, const float* __restrict__ gamma_n,
    const float* __restrict__ scale_n, BcastDst hd, float eps, long long rows, int rpb) {
  __shared__ float red[32];
  const int D4 = D >> 2;
  // rpb consecutive rows per block: with peers to write (W > 1) one system-scope fence then
  // covers rpb rows instead of one.
  const long long r_end = min(rows, ((long long)blockIdx.x + 1) * rpb);
  for (long long lr = (long long)blockIdx.x * rpb; lr < r_end; ++lr) {
  const long long row = row0 + lr;
  const float4* src = reinterpret_cast<const float4*>(slots + lr * D);
  const long long sstride4 = (slot_rows * D) >> 2;
  float4* y = reinterpret_cast<float4*>(x + row * D);
  // The residual row is loaded together with the partial rows, so that both are in flight
  // before the first reduction.
  float4 a[kPnChunks], xo[kPnChunks];
#pragma unroll
  for (int k = 0; k < kPnChunks; ++k) {
    const int i4 = threadIdx.x + k * kRowThreads;
    xo[k] = i4 < D4 ? y[i4] : make_float4(0.f, 0.f, 0.f, 0.f);
  }
  float ss = 0.0f;
#pragma unroll
  for (int k = 0; k < kPnChunks; ++k) {
    const int i4 = threadIdx.x + k * kRowThreads;
    a[k] = make_float4(0.f, 0.f, 0.f, 0.f);
    if (i4 < D4) {
      a[k] = src[i4];
#pragma unroll
      for (int s = 1; s < W; ++s) {
        const float4 t = src[s * sstride4 + i4];
        a[k].x += t.x;
        a[k].y += t.y;
        a[k].z += t.z;
        a[k].w += t.w;
      }
      ss += a[k].x * a[k].x + a[k].y * a[k].y + a[k].z * a[k].z + a[k].w * a[k].w;
    }
  }
  const float rstd = rsqrtf(block_sum256(ss, red) / (float)D + eps);
  const float4* g2 = reinterpret_cast<const float4*>(gamma2);
  const float4* gt = reinterpret_cast<const float4*>(g);
  float ss2 = 0.0f;
#pragma unroll
  for (int k = 0; k < kPnChunks; ++k) {
    const int i4 = threadIdx.x + k * kRowThreads;
    if (i4 < D4) {
      const float4 gm = gamma2 ? g2[i4] : make_float4(1.f, 1.f, 1.f, 1.f);
      float4 v = make_float4(a[k].x * rstd * gm.x, a[k].y * rstd * gm.y, a[k].z * rstd * gm.z, a[k].w * rstd * gm.w);
      if (g) {
        const float4 gg = gt[i4];
        v = make_float4(gg.x * v.x, gg.y * v.y, gg.z * v.z, gg.w * v.w);
      }
      const float4 xn = make_float4(xo[k].x + v.x, xo[k].y + v.y, xo[k].z + v.z, xo[k].w + v.w);
      y[i4] = xn;
      a[k] = xn;
      ss2 += xn.x * xn.x + xn.y * xn.y + xn.z * xn.z + xn.w * xn.w;
    }
  }
  if (hd.n == 0) continue;
  const float rstd2 = rsqrtf(block_sum256(ss2, red) / (float)D + eps);
  const float4* gn = reinterpret_cast<const float4*>(gamma_n);
  const float4* sc = reinterpret_cast<const float4*>(scale_n);
#pragma unroll
  for (int k = 0; k < kPnChunks; ++k) {
    const int i4 = threadIdx.x + k * kRowThreads;
    if (i4 < D4) {
      const float4 gm = gamma_n ? gn[i4] : make_float4(1.f, 1.f, 1.f, 1.f);
      float4 hv = make_float4(a[k].x * rstd2 * gm.x, a[k].y * rstd2 * gm.y, a[k].z * rstd2 * gm.z, a[k].w * rstd2 * gm.w);
      if (scale_n) {
        const float4 sv = sc[i4];
        hv = make_float4(hv.x * sv.x, hv.y * sv.y, hv.z * sv.z, hv.w * sv.w);
      }
      uint2 w;
      w.x = pack_bf16x2(hv.x, hv.y);
      w.y = pack_bf16x2(hv.z, hv.w);
#pragma unroll
      for (int q = 0; q < W; ++q) *reinterpret_cast<uint2*>(hd.p[q] + row * D + 4 * i4) = w;
    }
  }
  }
  // Stores into peers' memory are visible system-wide before this kernel completes (with
  // one rank every destination is local and kernel completion orders the stores).
  if (W > 1) __threadfence_system();
}

// One flow-matching Euler step of the sampler on the device (pipeline.cpp:237-243,
// scheduler.cpp:129-134): with classifier-free guidance (neg != null) the prediction is
// out + cfg (out - neg), then x += dt * prediction, dt = sigma_i - sigma_(i+1). Rounded
// as the reference's loops compile for x86-64-v3: the guidance mix as a separate
// multiply and add (no contraction), the Euler update as one fused multiply-add.
__global__ void k_flow_step(float* __restrict__ x, const float* __restrict__ out, const float* __restrict__ neg,
                            float cfg, float dt, int64_t n) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    float o = out[i];
    if (neg) o = __fadd_rn(o, __fmul_rn(cfg, __fsub_rn(o, neg[i])));
    x[i] = fmaf(dt, o, x[i]);
  }
}

// mod [4D] = scale_msa | gate_msa | scale_mlp | gate_mlp -> 1 + s, tanh(g) in place
// (zimage.cpp:97-112: affine_(1, 1) and tanh_).
__global__ void k_adaln_split(float* __restrict__ mod, int D) {
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < 4 * D; i += gridDim.x * blockDim.x) {
    const int part = i / D;
    const float v = mod[i];
    mod[i] = (part == 0 || part == 2) ? v * 1.0f + 1.0f : tanhf(v);
  }
}

// freq[i] = cos(tt * f_i), freq[half + i] = sin(tt * f_i), f_i = exp(-ln(10000) i / half)
// (zimage.cpp:151-157).
__global__ void k_timestep_embed(float* __restrict__ out, int F, float tt) {
  const int half = F / 2;
  for (int i = threadIdx.x; i < half; i += blockDim.x) {
    const float f = expf(-logf(10000.0f) * (float)i / (float)half);
    out[i] = cosf(tt * f);
    out[half + i] = sinf(tt * f);
  }
}

// y = layer_norm(x) (no affine) * scale, two-pass mean / variance
// (tensor.cpp:628-658 then mul_rows_; zimage.cpp:221-223).
__global__ void __launch_bounds__(kRowThreads) k_layer_norm_mod(const float* __restrict__ x, float* __restrict__ y,
                                                                int D, const float* __restrict__ scale, float eps) {
  __shared__ float red[32];
  const float* p = x + (int64_t)blockIdx.x * D;
  float* q = y + (int64_t)blockIdx.x * D;
  float s = 0.0f;
  for (int i = threadIdx.x; i < D; i += kRowThreads) s += p[i];
  const float mean = block_sum256(s, red) / (float)D;
  float v = 0.0f;
  for (int i = threadIdx.x; i < D; i += kRowThreads) {
    const float d = p[i] - mean;
    v += d * d;
  }
  const float rstd = rsqrtf(block_sum256(v, red) / (float)D + eps);
  for (int i = threadIdx.x; i < D; i += kRowThreads) q[i] = (p[i] - mean) * rstd * (scale ? scale[i] : 1.0f);
}

// Copies `src` [1, D] into rows [r0, r1) of y [*, D] (pad tokens, zimage.cpp:31-36).
__global__ void k_fill_rows(float* __restrict__ y, const float* __restrict__ src, int64_t r0, int64_t r1, int D) {
  const int64_t n = (r1 - r0) * D;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    y[r0 * D + i] = src[i % D];
}

// out rows [32j, 32j+16) = a rows [16j, 16j+16), out rows [32j+16, 32j+32) = b rows
// [16j, 16j+16): the gate/up (or value/gate) interleave the fused gated epilogue of
// the GEMM reads (gemm_tc.cu). Works for 2-byte and 4-byte elements (weights, biases).
template <typename T>
__global__ void k_interleave_rows16(const T* __restrict__ a, const T* __restrict__ b, T* __restrict__ out,
                                    int64_t rows, int64_t cols) {
  const int64_t n = 2 * rows * cols;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / cols, c = i - r * cols;
    const int64_t blk = r / 32, w = r % 32;
    const int64_t src = blk * 16 + (w & 15);
    out[i] = (w < 16 ? a : b)[src * cols + c];
  }
}

}  // namespace

void dit_interleave_rows16(const void* a, const void* b, void* out, int64_t rows, int64_t cols, int esize) {
  const int64_t n = 2 * rows * cols;
  if (n <= 0) return;
  const unsigned blocks = (unsigned)std::min<int64_t>((n + 255) / 256, (int64_t)ctx().num_sms * 16);
  if (esize == 2)
    k_interleave_rows16<uint16_t><<<blocks, 256, 0, ctx().stream>>>((const uint16_t*)a, (const uint16_t*)b,
                                                                     (uint16_t*)out, rows, cols);
  else
    k_interleave_rows16<float><<<blocks, 256, 0, ctx().stream>>>((const float*)a, (const float*)b, (float*)out, rows,
                                                                 cols);
  check_launch("interleave_rows16");
}

// ---------------------------------------------------------------------------------
void dit_rms_mod_bf16(const float* x, uint16_t* h, int64_t rows, int D, const float* gamma, const float* scale,
                      float eps) {
  if (rows <= 0) return;
  k_rms_mod_bf16<<<(unsigned)rows, kRowThreads, 0, ctx().stream>>>(x, h, D, gamma, scale, eps);
  check_launch("rms_mod_bf16");
}
void dit_post_norm_residual(float* x, const float* a, int64_t rows, int D, const float* gamma, const float* g,
                            float eps) {
  if (rows <= 0) return;
  k_post_norm_residual<<<(unsigned)rows, kRowThreads, 0, ctx().stream>>>(x, a, D, gamma, g, eps);
  check_launch("post_norm_residual");
}

void dit_flow_step(float* x, const float* out, const float* neg, float cfg, float dt, int64_t n) {
  if (n <= 0) return;
  const int64_t blocks = std::min<int64_t>((n + 255) / 256, (int64_t)ctx().num_sms * 8);
  k_flow_step<<<(unsigned)blocks, 256, 0, ctx().stream>>>(x, out, neg, cfg, dt, n);
  check_launch("flow_step");
}

void dit_post_norm_mod_bcast(const float* slots, int64_t slot_rows, int world, int64_t row0, int64_t rows, float* x,
                             int D, const float* gamma2, const float* g, const float* gamma_n, const float* scale_n,
                             uint16_t* const* hdst, int nh, float eps) {
  if (rows <= 0) return;
  if ((size_t)D * 4 > 48 * 1024) fail(kErrUnsupported, "post_norm_mod_bcast: row of more than 12288 values");
  if (world < 1 || world > kMaxTpRanks || (nh != 0 && nh != world))
    fail(kErrInvalidArg, "post_norm_mod_bcast: ranks (the row goes to every rank or to none)");
  BcastDst hd{};
  hd.n = nh;
  for (int q = 0; q < nh; ++q) hd.p[q] = hdst[q];
  const dim3 grid((unsigned)rows);
  // Rows per block of the register-resident form: 4 when peers are written (one fence per
  // block), else 1.
  const int rpb = (world > 1 && nh > 0) ? 4 : 1;
  const dim3 grid4((unsigned)((rows + rpb - 1) / rpb));
  const size_t sm = (size_t)D * 4;
  cudaStream_t st = ctx().stream;
  // The register-resident form needs 16-byte rows and vectors (all cudaMalloc'd / pool).
  const bool v4 = D % 4 == 0 && D <= 4 * kRowThreads * kPnChunks &&
                  ((reinterpret_cast<uintptr_t>(slots) | reinterpret_cast<uintptr_t>(x) |
                    reinterpret_cast<uintptr_t>(gamma2) | reinterpret_cast<uintptr_t>(g) |
                    reinterpret_cast<uintptr_t>(gamma_n) | reinterpret_cast<uintptr_t>(scale_n)) & 15) == 0;
  bool hd_ok = true;
  for (int q = 0; q < nh; ++q) hd_ok = hd_ok && (reinterpret_cast<uintptr_t>(hdst[q]) & 7) == 0;
  switch (world) {
#define SDB_PNMB(W)                                                                                             \
  case W:                                                                                                       \
    if (v4 && hd_ok)                                                                                            \
      k_post_norm_mod_bcast_v4<W><<<grid4, kRowThreads, 0, st>>>(slots, slot_rows, row0, x, D, gamma2, g, gamma_n, \
                                                                 scale_n, hd, eps, rows, rpb);                  \
    else                                                                                                        \
      k_post_norm_mod_bcast<W><<<grid, kRowThreads, sm, st>>>(slots, slot_rows, row0, x, D, gamma2, g, gamma_n,   \
                                                             scale_n, hd, eps);                                 \
    break;
    SDB_PNMB(1) SDB_PNMB(2) SDB_PNMB(3) SDB_PNMB(4) SDB_PNMB(5) SDB_PNMB(6) SDB_PNMB(7) SDB_PNMB(8)
#undef SDB_PNMB
  }
  check_launch("post_norm_mod_bcast");
}
void dit_adaln_split(float* mod, int D) {
  k_adaln_split<<<(unsigned)((4 * D + 255) / 256), 256, 0, ctx().stream>>>(mod, D);
  check_launch("adaln_split");
}
void dit_timestep_embed(float* out, int F, float tt) {
  k_timestep_embed<<<1, 128, 0, ctx().stream>>>(out, F, tt);
  check_launch("timestep_embed");
}
void dit_layer_norm_mod(const float* x, float* y, int64_t rows, int D, const float* scale, float eps) {
  if (rows <= 0) return;
  k_layer_norm_mod<<<(unsigned)rows, kRowThreads, 0, ctx().stream>>>(x, y, D, scale, eps);
  check_launch("layer_norm_mod");
}
void dit_fill_rows(float* y, const float* src, int64_t r0, int64_t r1, int D) {
  if (r1 <= r0) return;
  const int64_t n = (r1 - r0) * D;
  k_fill_rows<<<(unsigned)std::min<int64_t>((n + 255) / 256, 4096), 256, 0, ctx().stream>>>(y, src, r0, r1, D);
  check_launch("fill_rows");
}

}  // namespace sdb
