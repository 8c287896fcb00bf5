// layers.cu - the memory-bound kernels of the backend: operand packing for the
// tensor-core GEMM, the small-M GEMM, and every layer / elementwise / layout op of
// the reference backend API (backend_cuda.h:45-80) that is not a contraction.
//
// These are HBM-bound (a few flops per byte), so they are written as plain SIMT
// kernels: 16-byte vector loads/stores where the layout allows, grids sized in
// multiples of the SM count, fp32 warp-shuffle reductions. Numerics follow the
// reference CPU loops in tensor.cpp (cited per kernel); reductions that the CPU
// does in double are done here in fp32 tree order, well inside the reference's own
// GPU-vs-CPU tolerances (test_ops.cpp:356-477).
#include <algorithm>
#include <cmath>

#include "internal.h"
#include "ptx.cuh"

namespace sdb {
namespace {

constexpr int kT = 256;

unsigned blocks_for(int64_t n, int per_thread = 1) {
  const int64_t blocks = (n / per_thread + kT - 1) / kT;
  const int64_t cap = (int64_t)std::max(1, ctx().num_sms) * 16;
  return (unsigned)std::max<int64_t>(1, std::min<int64_t>(blocks, cap));
}

#define FOR_GRID_ITEMS(i, n) \
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < (n); i += (int64_t)gridDim.x * blockDim.x)

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
// Block-wide sum; every thread gets the result. `red` holds >= 32 floats.
__device__ __forceinline__ float block_sum(float v, float* red) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
  v = warp_sum(v);
  __syncthreads();
  if (lane == 0) red[w] = v;
  __syncthreads();
  float t = lane < nw ? red[lane] : 0.0f;
  t = warp_sum(t);
  return t;
}
__device__ __forceinline__ float block_max(float v, float* red) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
  v = warp_max(v);
  __syncthreads();
  if (lane == 0) red[w] = v;
  __syncthreads();
  float t = lane < nw ? red[lane] : -INFINITY;
  t = warp_max(t);
  return t;
}

// ---------------------------------------------------------------------------------
// Packing
// ---------------------------------------------------------------------------------
// fp32 -> bf16 (reference rounding), 8 elements per thread when rows allow it.
__global__ void k_pack_bf16_vec(const float* __restrict__ src, int64_t ld, uint16_t* __restrict__ dst, int64_t ldo,
                                int64_t rows, int64_t cols8) {
  FOR_GRID_ITEMS(i, rows * cols8) {
    const int64_t r = i / cols8, c = (i - r * cols8) * 8;
    const float4 a = *reinterpret_cast<const float4*>(src + r * ld + c);
    const float4 b = *reinterpret_cast<const float4*>(src + r * ld + c + 4);
    uint4 o;
    o.x = pack_bf16x2(a.x, a.y);
    o.y = pack_bf16x2(a.z, a.w);
    o.z = pack_bf16x2(b.x, b.y);
    o.w = pack_bf16x2(b.z, b.w);
    *reinterpret_cast<uint4*>(dst + r * ldo + c) = o;
  }
}
__global__ void k_pack_bf16(const float* __restrict__ src, int64_t ld, uint16_t* __restrict__ dst, int64_t ldo,
                            int64_t rows, int64_t cols) {
  FOR_GRID_ITEMS(i, rows * cols) {
    const int64_t r = i / cols, c = i - r * cols;
    dst[r * ldo + c] = f32_to_bf16_rne(src[r * ld + c]);
  }
}
// fp32 -> fp32 rounded to the tf32 grid (10 explicit mantissa bits, nearest even), so
// that kind::tf32 sees an unbiased operand whatever the hardware does with low bits.
__device__ __forceinline__ float round_tf32(float f) {
  uint32_t b = __float_as_uint(f);
  if ((b & 0x7F800000u) == 0x7F800000u) return f;
  b += 0xFFFu + ((b >> 13) & 1u);
  return __uint_as_float(b & 0xFFFFE000u);
}
// NCHW -> NHWC (channel pitch cp) through a 32-channel x 128-pixel shared-memory tile:
// 128-byte reads along pixels (16 in flight per thread), 128-byte writes along channels;
// tf32-rounded, zero past C. On the way each value may be transformed, in this order:
//   y = x * a + b    per channel (a, b) = ab[n * C + c] (GroupNorm), or the constants
//                    (a0, b0) when ab is null (the VAE's latent un-scaling)
//   y = silu(y)      when silu != 0 (y / (1 + e^-y), tensor.cpp:843-849)
// With UP, the output is the nearest-neighbour 2x upsampling of x (tensor.cpp:982-990):
// output pixel (oy, ox) of the 2H x 2W image reads input (oy / 2, ox / 2).
constexpr int kPackPx = 128;
template <bool UP>
__global__ void __launch_bounds__(256) k_pack_nhwc(const float* __restrict__ x, float* __restrict__ xh, int64_t C,
                                                   int64_t H, int64_t W, int64_t cp, const float2* __restrict__ ab,
                                                   float a0, float b0, int silu) {
  __shared__ float tile[32][kPackPx + 1];
  const int64_t Wo = UP ? 2 * W : W, HWo = (UP ? 2 * H : H) * Wo, HWs = H * W;
  const int64_t n = blockIdx.z, p0 = (int64_t)blockIdx.x * kPackPx, c0 = (int64_t)blockIdx.y * 32;
  const int tx = threadIdx.x, ty = threadIdx.y;
  // Source pixel of each of this thread's output pixels (the launcher keeps HWo < 2^31,
  // so 32-bit division suffices).
  int64_t src[kPackPx / 32];
#pragma unroll
  for (int j = 0; j < kPackPx / 32; ++j) {
    const int64_t p = p0 + tx + 32 * j;
    src[j] = p;
    if (UP) {
      const uint32_t oy = (uint32_t)p / (uint32_t)Wo, ox = (uint32_t)p - oy * (uint32_t)Wo;
      src[j] = (int64_t)(oy >> 1) * W + (ox >> 1);
    }
  }
  float v[4][kPackPx / 32];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int64_t c = c0 + ty + 8 * i;
    const float* xc = x + (n * C + c) * HWs;
#pragma unroll
    for (int j = 0; j < kPackPx / 32; ++j) {
      const int64_t p = p0 + tx + 32 * j;
      v[i][j] = (c < C && p < HWo) ? __ldg(xc + src[j]) : 0.0f;
    }
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int64_t c = c0 + ty + 8 * i;
    float a = a0, b = b0;
    if (ab && c < C) {
      const float2 t = ab[n * C + c];
      a = t.x;
      b = t.y;
    }
#pragma unroll
    for (int j = 0; j < kPackPx / 32; ++j) {
      float y = v[i][j] * a + b;
      // The result is rounded to tf32 (13 low bits dropped) next, so the fast exponential
      // and division are exact enough: their error is below that rounding.
      if (silu) y = __fdividef(y, 1.0f + __expf(-y));
      tile[ty + 8 * i][tx + 32 * j] = c < C ? round_tf32(y) : 0.0f;
    }
  }
  __syncthreads();
  const int64_t c = c0 + tx;
  if (c >= cp) return;
#pragma unroll 4
  for (int i = 0; i < kPackPx / 8; ++i) {
    const int64_t p = p0 + ty + 8 * i;
    if (p < HWo) xh[(n * HWo + p) * cp + c] = tile[tx][ty + 8 * i];
  }
}
__global__ void k_conv_pack_w(const float* __restrict__ w, float* __restrict__ wp, int64_t Cin, int64_t taps,
                              int64_t cq, int64_t total) {
  FOR_GRID_ITEMS(i, total) {
    const int64_t ci = i % cq, r = i / cq, t = r % taps, co = r / taps;
    wp[i] = ci < Cin ? round_tf32(__ldg(w + (co * Cin + ci) * taps + t)) : 0.0f;
  }
}
// The same pack, one block per output channel: the channel's [Cin, taps] slab is read
// contiguously into shared memory, then written as [taps, cq] with contiguous stores (the
// gather above reads with a stride of `taps` floats and re-reads each line once per tap).
// Shared-memory reads at stride taps are conflict-free for odd taps. Each thread keeps 8
// loads in flight (16-byte loads when the slab is 16-byte aligned).
template <bool VEC>
__global__ void __launch_bounds__(256) k_conv_pack_w_slab(const float* __restrict__ w, float* __restrict__ wp,
                                                          int Cin, int taps, int cq) {
  extern __shared__ float4 slab4[];
  float* slab = reinterpret_cast<float*>(slab4);
  const int64_t co = blockIdx.x;
  const int n = Cin * taps;
  const float* src = w + co * n;
  constexpr int kU = 8;
  if (VEC) {
    const float4* s4 = reinterpret_cast<const float4*>(src);
    const int n4 = n >> 2;
    for (int j0 = threadIdx.x; j0 < n4; j0 += kU * 256) {
      float4 v[kU];
#pragma unroll
      for (int u = 0; u < kU; ++u) {
        const int j = j0 + u * 256;
        if (j < n4) v[u] = __ldg(s4 + j);
      }
#pragma unroll
      for (int u = 0; u < kU; ++u) {
        const int j = j0 + u * 256;
        if (j < n4) slab4[j] = v[u];
      }
    }
  } else {
    for (int j0 = threadIdx.x; j0 < n; j0 += kU * 256) {
      float v[kU];
#pragma unroll
      for (int u = 0; u < kU; ++u) {
        const int j = j0 + u * 256;
        if (j < n) v[u] = __ldg(src + j);
      }
#pragma unroll
      for (int u = 0; u < kU; ++u) {
        const int j = j0 + u * 256;
        if (j < n) slab[j] = v[u];
      }
    }
  }
  __syncthreads();
  float* dst = wp + co * (int64_t)taps * cq;
  const int m = taps * cq;
  for (int i = threadIdx.x; i < m; i += blockDim.x) {
    const int t = i / cq, ci = i - t * cq;
    dst[i] = ci < Cin ? round_tf32(slab[ci * taps + t]) : 0.0f;
  }
}
// Direct convolution for layers with few output channels (the VAE's conv_out, 128 -> 3):
// on the tensor cores such a layer would fill 3 of a tile's 128 rows. Operands are the
// implicit-GEMM path's: xh NHWC (channel pitch cp, tf32 values), wp [Cout, taps, cq].
// A block computes a 16 x 32 tile of output pixels for all CO channels, each thread two
// pixels 16 rows apart. 8-channel slices of the input tile with its halo are staged
// channel-major in shared memory (conflict-free reads along x), and the slice's weights
// as [channel][tap][CO], so one 16-byte load gives four output channels' weights, used for
// both pixels; fp32 FMA accumulation.
constexpr int kDirTX = 16, kDirTY = 32, kDirCh = 8;
template <int CO, int KC>  // KC: the kernel size at compile time, or 0 (runtime k)
__global__ void __launch_bounds__(256) k_conv_direct_nhwc(
    const float* __restrict__ xh, int64_t cp, int Cin, int H, int W, const float* __restrict__ wp, int64_t cq,
    int Cout, int k_rt, int pad, const float* __restrict__ bias, const float* res, float* out, int Ho, int Wo) {
  const int k = KC ? KC : k_rt;
  extern __shared__ float4 dsm4[];
  float* dsm = reinterpret_cast<float*>(dsm4);
  const int TWx = kDirTX + k - 1, TWy = kDirTY + k - 1, TT = TWx * TWy, taps = k * k;
  float* tin = dsm;                        // [kDirCh][TT]
  float* tw = dsm + ((kDirCh * TT + 3) & ~3);  // [kDirCh][taps][CO], 16-byte aligned
  const int n = blockIdx.z, oy0 = blockIdx.y * kDirTY, ox0 = blockIdx.x * kDirTX;
  const int tx = threadIdx.x % kDirTX, ty = threadIdx.x / kDirTX;  // ty < 16: rows ty and ty + 16
  float acc0[CO], acc1[CO];
#pragma unroll
  for (int co = 0; co < CO; ++co) acc0[co] = acc1[co] = 0.0f;
  for (int c0 = 0; c0 < Cin; c0 += kDirCh) {
    __syncthreads();
    // One pixel's 8 channels per step: two 16-byte loads (cp % 4 == 0, c0 % 8 == 0), or
    // element loads for a slice that runs past Cin.
    const bool full = c0 + kDirCh <= Cin;
    for (int p = threadIdx.x; p < TT; p += blockDim.x) {
      const int py = p / TWx, iy = oy0 - pad + py, ix = ox0 - pad + (p - py * TWx);
      float v[kDirCh];
#pragma unroll
      for (int c = 0; c < kDirCh; ++c) v[c] = 0.0f;
      if (iy >= 0 && iy < H && ix >= 0 && ix < W) {
        const float* src = xh + (((int64_t)n * H + iy) * W + ix) * cp + c0;
        if (full) {
          const float4 a0 = __ldg(reinterpret_cast<const float4*>(src));
          const float4 a1 = __ldg(reinterpret_cast<const float4*>(src + 4));
          v[0] = a0.x; v[1] = a0.y; v[2] = a0.z; v[3] = a0.w;
          v[4] = a1.x; v[5] = a1.y; v[6] = a1.z; v[7] = a1.w;
        } else {
#pragma unroll
          for (int c = 0; c < kDirCh; ++c)
            if (c0 + c < Cin) v[c] = __ldg(src + c);
        }
      }
#pragma unroll
      for (int c = 0; c < kDirCh; ++c) tin[c * TT + p] = v[c];
    }
    for (int i = threadIdx.x; i < kDirCh * taps * CO; i += blockDim.x) {
      const int co = i % CO, r = i / CO, t = r % taps, c = r / taps;
      tw[i] = (co < Cout && c0 + c < Cin) ? __ldg(wp + ((int64_t)co * taps + t) * cq + c0 + c) : 0.0f;
    }
    __syncthreads();
    for (int c = 0; c < kDirCh; ++c) {
      const float* tc = tin + c * TT;
#pragma unroll
      for (int ky = 0; ky < k; ++ky) {
        const float* r0 = tc + (ty + ky) * TWx + tx;
        const float* r1 = r0 + 16 * TWx;
        const float4* wrow = reinterpret_cast<const float4*>(tw + ((c * taps) + ky * k) * CO);
#pragma unroll
        for (int kx = 0; kx < k; ++kx) {
          const float v0 = r0[kx], v1 = r1[kx];
#pragma unroll
          for (int q = 0; q < CO / 4; ++q) {
            const float4 w4 = wrow[kx * (CO / 4) + q];
            acc0[4 * q] = fmaf(v0, w4.x, acc0[4 * q]);
            acc0[4 * q + 1] = fmaf(v0, w4.y, acc0[4 * q + 1]);
            acc0[4 * q + 2] = fmaf(v0, w4.z, acc0[4 * q + 2]);
            acc0[4 * q + 3] = fmaf(v0, w4.w, acc0[4 * q + 3]);
            acc1[4 * q] = fmaf(v1, w4.x, acc1[4 * q]);
            acc1[4 * q + 1] = fmaf(v1, w4.y, acc1[4 * q + 1]);
            acc1[4 * q + 2] = fmaf(v1, w4.z, acc1[4 * q + 2]);
            acc1[4 * q + 3] = fmaf(v1, w4.w, acc1[4 * q + 3]);
          }
        }
      }
    }
  }
  const int ox = ox0 + tx;
  if (ox >= Wo) return;
#pragma unroll
  for (int half = 0; half < 2; ++half) {
    const int oy = oy0 + ty + 16 * half;
    if (oy >= Ho) break;
#pragma unroll
    for (int co = 0; co < CO; ++co) {
      if (co >= Cout) break;
      const int64_t o = (((int64_t)n * Cout + co) * Ho + oy) * Wo + ox;
      float r = (half ? acc1[co] : acc0[co]) + (bias ? __ldg(bias + co) : 0.0f);
      if (res) r += res[o];
      out[o] = r;
    }
  }
}
// Split-K reduction (deterministic: the splits are summed in order).
__global__ void k_split_reduce(const float* __restrict__ part, int splits, int64_t total, int64_t C, int64_t hw,
                               const float* __restrict__ bias, const float* res, float* out) {
  FOR_GRID_ITEMS(i, total) {
    float s = part[i];
    for (int k = 1; k < splits; ++k) s += part[k * total + i];
    if (bias) s += __ldg(bias + (i / hw) % C);
    if (res) s += res[i];
    out[i] = s;
  }
}
// Two matrices packed to the tf32 grid by one launch (the A and B operands of one GEMM).
// dst = tf32(src) for one matrix ([r0, cols], strides ld0 / ldo0) or two at once (the
// second [r1, cols]): the fp32 GEMM's A and B operands in one launch. One warp per row: no
// per-element 64-bit division, and with VEC (16-byte rows, strides and bases) 16-byte
// accesses, four in flight per lane.
template <bool VEC>
__global__ void __launch_bounds__(256) k_pack_tf32_rows(const float* __restrict__ s0, int64_t ld0,
                                                        float* __restrict__ d0, int64_t ldo0, int64_t r0,
                                                        const float* __restrict__ s1, int64_t ld1,
                                                        float* __restrict__ d1, int64_t ldo1, int64_t r1,
                                                        int64_t cols) {
  const int lane = threadIdx.x & 31;
  const int64_t rows = r0 + r1;
  for (int64_t row = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5); row < rows; row += (int64_t)gridDim.x * 8) {
    const bool first = row < r0;
    const int64_t r = first ? row : row - r0;
    const float* s = first ? s0 + r * ld0 : s1 + r * ld1;
    float* d = first ? d0 + r * ldo0 : d1 + r * ldo1;
    if (VEC) {
      const int64_t c4 = cols >> 2;
      const float4* s4 = reinterpret_cast<const float4*>(s);
      float4* d4 = reinterpret_cast<float4*>(d);
      for (int64_t c0 = lane; c0 < c4; c0 += 4 * 32) {
        float4 v[4];
#pragma unroll
        for (int u = 0; u < 4; ++u)
          if (c0 + 32 * u < c4) v[u] = __ldg(s4 + c0 + 32 * u);
#pragma unroll
        for (int u = 0; u < 4; ++u)
          if (c0 + 32 * u < c4)
            d4[c0 + 32 * u] = make_float4(round_tf32(v[u].x), round_tf32(v[u].y), round_tf32(v[u].z),
                                          round_tf32(v[u].w));
      }
    } else {
      for (int64_t c0 = lane; c0 < cols; c0 += 4 * 32) {
        float v[4];
#pragma unroll
        for (int u = 0; u < 4; ++u)
          if (c0 + 32 * u < cols) v[u] = __ldg(s + c0 + 32 * u);
#pragma unroll
        for (int u = 0; u < 4; ++u)
          if (c0 + 32 * u < cols) d[c0 + 32 * u] = round_tf32(v[u]);
      }
    }
  }
}
// In place (no restrict): x[r * ld + c] = tf32(x[r * ld + c]).
__global__ void k_round_tf32_inplace(float* x, int64_t ld, int64_t rows, int64_t cols) {
  FOR_GRID_ITEMS(i, rows * cols) {
    const int64_t r = i / cols, c = i - r * cols;
    x[r * ld + c] = round_tf32(x[r * ld + c]);
  }
}
__global__ void k_copy2d_16(const uint16_t* __restrict__ src, int64_t ld, uint16_t* __restrict__ dst, int64_t ldo,
                            int64_t rows, int64_t cols) {
  FOR_GRID_ITEMS(i, rows * cols) {
    const int64_t r = i / cols, c = i - r * cols;
    dst[r * ldo + c] = src[r * ld + c];
  }
}
__global__ void k_copy2d_32(const float* __restrict__ src, int64_t ld, float* __restrict__ dst, int64_t ldo,
                            int64_t rows, int64_t cols) {
  FOR_GRID_ITEMS(i, rows * cols) {
    const int64_t r = i / cols, c = i - r * cols;
    dst[r * ldo + c] = src[r * ld + c];
  }
}
__global__ void k_bias_fill(float* C, int64_t ldc, int64_t M, int64_t N, const float* bias, int acc) {
  FOR_GRID_ITEMS(i, M * N) {
    const int64_t r = i / N, c = i - r * N;
    const float b = bias ? bias[c] : 0.0f;
    float* p = C + r * ldc + c;
    *p = acc ? *p + b : b;
  }
}

// ---------------------------------------------------------------------------------
// Small-M GEMM: C[M,N] = A[M,K] B[N,K]^T (+bias) (+C), M <= 16. HBM-bound on the
// weights B, which are read once. A (fp32) is staged in shared memory once per CTA; each
// warp then owns groups of kGemvRows consecutive rows of B and, per K chunk, issues the
// 16-byte loads of all of them before any arithmetic, so that every warp keeps
// kGemvRows x 512 bytes in flight. The 32 lane partial sums of each (row of B, row of A)
// are combined by one shuffle tree at the end. MMAX (1, 4 or 16) bounds M at compile
// time, so the M = 1 GEMV of the adaLN modulation carries no unused accumulators.
// ---------------------------------------------------------------------------------
constexpr int kGemvRows = 4;
constexpr int kGemvWarps = 8;

__device__ __forceinline__ void widen_bf16x8(const uint4 w, float (&b)[8]) {
  b[0] = __uint_as_float(w.x << 16); b[1] = __uint_as_float(w.x & 0xFFFF0000u);
  b[2] = __uint_as_float(w.y << 16); b[3] = __uint_as_float(w.y & 0xFFFF0000u);
  b[4] = __uint_as_float(w.z << 16); b[5] = __uint_as_float(w.z & 0xFFFF0000u);
  b[6] = __uint_as_float(w.w << 16); b[7] = __uint_as_float(w.w & 0xFFFF0000u);
}

// ASMEM: A staged in shared memory (M up to 16 rows); otherwise each lane reads its A
// values straight from global memory (small M x K, cached in L1 / L2 after the first warp),
// so that the weight loads are issued at once instead of after an A staging round trip.
template <bool BF16, int MMAX, bool ASMEM>
__global__ void __launch_bounds__(256) k_gemv_rows(int M, int N, int K, const float* __restrict__ A, int64_t lda,
                                                   const void* __restrict__ Bv, int64_t ldb, float* __restrict__ C,
                                                   int64_t ldc, const float* __restrict__ bias, int acc, int vec) {
  constexpr int R = kGemvRows;
  constexpr int E = BF16 ? 8 : 4;  // elements of B per 16-byte load
  extern __shared__ float sa[];    // A as [M][K] (ASMEM)
  if (ASMEM) {
    for (int i = threadIdx.x; i < M * K; i += blockDim.x) {
      const int m = i / K;
      sa[i] = A[(int64_t)m * lda + (i - m * K)];
    }
    __syncthreads();
  }
  const float* Ab = ASMEM ? sa : A;
  const int64_t ald = ASMEM ? K : lda;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int groups = (N + R - 1) / R;
  for (int grp = blockIdx.x * kGemvWarps + warp; grp < groups; grp += gridDim.x * kGemvWarps) {
    const int n0 = grp * R;
    float s[R][MMAX];
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
      for (int m = 0; m < MMAX; ++m) s[r][m] = 0.0f;
    int k0 = 0;
    if (vec) {
      const int kv = K / (32 * E) * (32 * E);
      for (int k = lane * E; k < kv; k += 32 * E) {
        uint4 w[R];
#pragma unroll
        for (int r = 0; r < R; ++r) {
          const int n = min(n0 + r, N - 1);  // rows past N repeat the last row; never stored
          const char* row = reinterpret_cast<const char*>(Bv) + (int64_t)n * ldb * (BF16 ? 2 : 4);
          w[r] = __ldg(reinterpret_cast<const uint4*>(row) + k / E);
        }
        // Direct A: this lane's A values of the chunk, loaded alongside the weights.
        float a[ASMEM ? 1 : MMAX][E];
        if constexpr (!ASMEM) {
#pragma unroll
          for (int m = 0; m < MMAX; ++m)
            if (m < M) {
              const float4* ap = reinterpret_cast<const float4*>(A + m * lda + k);
#pragma unroll
              for (int e = 0; e < E; e += 4) {
                const float4 v = __ldg(ap + e / 4);
                a[m][e] = v.x;
                a[m][e + 1] = v.y;
                a[m][e + 2] = v.z;
                a[m][e + 3] = v.w;
              }
            }
        }
#pragma unroll
        for (int r = 0; r < R; ++r) {
          float b[8];
          if (BF16) {
            widen_bf16x8(w[r], b);
          } else {
            b[0] = __uint_as_float(w[r].x); b[1] = __uint_as_float(w[r].y);
            b[2] = __uint_as_float(w[r].z); b[3] = __uint_as_float(w[r].w);
          }
#pragma unroll
          for (int m = 0; m < MMAX; ++m)
            if (m < M) {
#pragma unroll
              for (int e = 0; e < E; ++e) s[r][m] = fmaf(ASMEM ? sa[m * K + k + e] : a[ASMEM ? 0 : m][e], b[e], s[r][m]);
            }
        }
      }
      k0 = kv;
    }
    for (int k = k0 + lane; k < K; k += 32) {
#pragma unroll
      for (int r = 0; r < R; ++r) {
        const int n = min(n0 + r, N - 1);
        const float b = BF16 ? bf16_to_f32(reinterpret_cast<const uint16_t*>(Bv)[(int64_t)n * ldb + k])
                             : reinterpret_cast<const float*>(Bv)[(int64_t)n * ldb + k];
#pragma unroll
        for (int m = 0; m < MMAX; ++m)
          if (m < M) s[r][m] = fmaf(Ab[m * ald + k], b, s[r][m]);
      }
    }
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const int n = n0 + r;
#pragma unroll
      for (int m = 0; m < MMAX; ++m) {
        if (m < M) {
          const float t = warp_sum(s[r][m]);
          if (lane == 0 && n < N) {
            float* c = C + (int64_t)m * ldc + n;
            const float v = t + (bias ? bias[n] : 0.0f);
            *c = acc ? *c + v : v;
          }
        }
      }
    }
  }
}

// ---------------------------------------------------------------------------------
// Norms (tensor.cpp:588-679, :681-699)
// ---------------------------------------------------------------------------------
// GroupNorm (tensor.cpp:603-624) in three steps over the N * groups contiguous segments
// of cg * HW values:
//   1. k_gn_stats: one block per 8192-value chunk keeps its chunk in registers and
//      writes the chunk's mean and sum of squared deviations (two passes, fp32);
//   2. k_gn_finalize: one warp per segment combines its chunks in double (Chan et al.'s
//      pairwise update: M2 = sum M2_c + n_c (mean_c - mean)^2), the counterpart of the
//      reference's double two-pass statistics, and folds normalisation and the affine
//      transform into a per-channel scale a = rstd * gamma and shift b = beta - mean * a;
//   3. k_gn_apply: y = x * a + b over every (sample, channel) row, optionally SiLU.
constexpr int kGnThreads = 256;
constexpr int kGnPer = 32;  // values per thread per chunk
constexpr int kGnChunk = kGnThreads * kGnPer;
__global__ void __launch_bounds__(kGnThreads) k_gn_stats(const float* __restrict__ x, int64_t len, int chunks,
                                                         float2* __restrict__ part) {
  __shared__ float red[32];
  const int64_t seg = blockIdx.y;
  const int64_t c0 = (int64_t)blockIdx.x * kGnChunk;
  const float* p = x + seg * len + c0;
  const int64_t n = (len - c0 < (int64_t)kGnChunk ? len - c0 : (int64_t)kGnChunk);
  float v[kGnPer];
  float s = 0.0f;
#pragma unroll
  for (int j = 0; j < kGnPer; ++j) {
    const int64_t i = (int64_t)j * kGnThreads + threadIdx.x;
    v[j] = i < n ? __ldg(p + i) : 0.0f;
    s += v[j];
  }
  const float mean = block_sum(s, red) / (float)n;
  float m2 = 0.0f;
#pragma unroll
  for (int j = 0; j < kGnPer; ++j) {
    const int64_t i = (int64_t)j * kGnThreads + threadIdx.x;
    const float d = v[j] - mean;
    if (i < n) m2 = fmaf(d, d, m2);
  }
  m2 = block_sum(m2, red);
  if (threadIdx.x == 0) part[seg * chunks + blockIdx.x] = make_float2(mean, m2);
}
__global__ void k_gn_finalize(const float2* __restrict__ part, int chunks, int64_t len, int64_t C, int groups,
                              const float* __restrict__ gamma, const float* __restrict__ beta, float eps,
                              float2* __restrict__ ab, int64_t segs) {
  const int64_t seg = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (seg >= segs) return;
  const float2* q = part + seg * chunks;
  double sum = 0.0;
  for (int c = lane; c < chunks; c += 32) {
    const double nc = (double)(len - (int64_t)c * kGnChunk < (int64_t)kGnChunk ? len - (int64_t)c * kGnChunk : (int64_t)kGnChunk);
    sum += nc * (double)q[c].x;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
  const double mean = sum / (double)len;
  double m2 = 0.0;
  for (int c = lane; c < chunks; c += 32) {
    const double nc = (double)(len - (int64_t)c * kGnChunk < (int64_t)kGnChunk ? len - (int64_t)c * kGnChunk : (int64_t)kGnChunk);
    const double d = (double)q[c].x - mean;
    m2 += (double)q[c].y + nc * d * d;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m2 += __shfl_xor_sync(0xffffffffu, m2, o);
  const float rstd = (float)(1.0 / sqrt(m2 / (double)len + (double)eps));
  const int64_t n = seg / groups, g = seg % groups, cg = C / groups;
  for (int64_t c = lane; c < cg; c += 32) {
    const int64_t ch = g * cg + c;
    const float a = rstd * gamma[ch];
    ab[n * C + ch] = make_float2(a, beta[ch] - (float)mean * a);
  }
}
// The same from a convolution epilogue's per-tile partials: one block per (sample, group)
// merges its tiles' (count, mean, M2) in double, pairwise, then writes the affine of the
// group's channels.
__global__ void __launch_bounds__(256) k_gn_finalize_parts(const float4* __restrict__ part, int64_t tiles, int64_t C,
                                                           int groups, const float* __restrict__ gamma,
                                                           const float* __restrict__ beta, float eps,
                                                           float2* __restrict__ ab) {
  __shared__ double sn[256], smean[256], sm2[256];
  const int64_t seg = blockIdx.x;
  const float4* q = part + seg * tiles;
  double N = 0.0, mean = 0.0, m2 = 0.0;
  auto merge = [](double& Na, double& ma, double& qa, double Nb, double mb, double qb) {
    if (Nb == 0.0) return;
    if (Na == 0.0) {
      Na = Nb;
      ma = mb;
      qa = qb;
      return;
    }
    const double n = Na + Nb, d = mb - ma;
    ma += d * (Nb / n);
    qa += qb + d * d * (Na * Nb / n);
    Na = n;
  };
  for (int64_t t = threadIdx.x; t < tiles; t += blockDim.x) {
    const float4 v = q[t];
    merge(N, mean, m2, (double)v.x, (double)v.y, (double)v.z);
  }
  sn[threadIdx.x] = N;
  smean[threadIdx.x] = mean;
  sm2[threadIdx.x] = m2;
  __syncthreads();
  for (int s = 128; s > 0; s >>= 1) {
    if ((int)threadIdx.x < s) {
      double a = sn[threadIdx.x], b = smean[threadIdx.x], c = sm2[threadIdx.x];
      merge(a, b, c, sn[threadIdx.x + s], smean[threadIdx.x + s], sm2[threadIdx.x + s]);
      sn[threadIdx.x] = a;
      smean[threadIdx.x] = b;
      sm2[threadIdx.x] = c;
    }
    __syncthreads();
  }
  const double tot = sn[0], mu = smean[0];
  const float rstd = (float)(1.0 / sqrt(sm2[0] / (tot > 0.0 ? tot : 1.0) + (double)eps));
  const int64_t n = seg / groups, g = seg % groups, cg = C / groups;
  for (int64_t c = threadIdx.x; c < cg; c += blockDim.x) {
    const int64_t ch = g * cg + c;
    const float a = rstd * gamma[ch];
    ab[n * C + ch] = make_float2(a, beta[ch] - (float)mu * a);
  }
}
// GroupNorm in one launch for groups that fit in shared memory (cg x HW <= kGnFusedMax
// values; every group of the SD 1.x UNet at 512^2): one 1024-thread block per (group,
// sample) reads the group's values (contiguous in NCHW) once into shared memory, eight
// 16-byte loads in flight per thread; mean, then the mean of squared deviations, are fp32
// block reductions over shared memory; y = (x - mean) * rstd * gamma[c] + beta[c], then
// SiLU when asked. Groups too large for it use the split statistics below.
constexpr int kGnFusedMax = 48 * 1024;
__global__ void __launch_bounds__(1024) k_gn_fused(const float* __restrict__ x, float* __restrict__ y, int64_t C,
                                                   int HW, int cg, const float* __restrict__ gamma,
                                                   const float* __restrict__ beta, float eps, int silu) {
  extern __shared__ float4 gsm4[];
  __shared__ float red[32];
  const int g = blockIdx.x, n = blockIdx.y, cnt = cg * HW, c4n = cnt >> 2;
  const int64_t base = ((int64_t)n * C + (int64_t)g * cg) * HW;
  const float4* src = reinterpret_cast<const float4*>(x + base);
  constexpr int kU = 8;
  float s = 0.0f;
  for (int i0 = threadIdx.x; i0 < c4n; i0 += kU * 1024) {
    float4 v[kU];
#pragma unroll
    for (int u = 0; u < kU; ++u)
      if (i0 + u * 1024 < c4n) v[u] = __ldg(src + i0 + u * 1024);
#pragma unroll
    for (int u = 0; u < kU; ++u)
      if (i0 + u * 1024 < c4n) {
        gsm4[i0 + u * 1024] = v[u];
        s += (v[u].x + v[u].y) + (v[u].z + v[u].w);
      }
  }
  const float mean = block_sum(s, red) / (float)cnt;
  float q = 0.0f;
  for (int i = threadIdx.x; i < c4n; i += 1024) {
    const float4 v = gsm4[i];
    const float a = v.x - mean, b = v.y - mean, c = v.z - mean, d = v.w - mean;
    q += (a * a + b * b) + (c * c + d * d);
  }
  const float rstd = rsqrtf(block_sum(q, red) / (float)cnt + eps);
  float4* dst = reinterpret_cast<float4*>(y + base);
  for (int i = threadIdx.x; i < c4n; i += 1024) {
    const int c = g * cg + (4 * i) / HW;  // HW % 4 == 0: the four values share a channel
    const float ga = gamma ? __ldg(gamma + c) : 1.0f, be = beta ? __ldg(beta + c) : 0.0f;
    const float4 v = gsm4[i];
    float o[4] = {(v.x - mean) * rstd * ga + be, (v.y - mean) * rstd * ga + be, (v.z - mean) * rstd * ga + be,
                  (v.w - mean) * rstd * ga + be};
    if (silu) {
#pragma unroll
      for (int e = 0; e < 4; ++e) o[e] = o[e] / (1.0f + expf(-o[e]));
    }
    dst[i] = make_float4(o[0], o[1], o[2], o[3]);
  }
}
template <bool VEC>
__global__ void k_gn_apply(const float* __restrict__ x, float* __restrict__ y, int64_t HW,
                           const float2* __restrict__ ab, int silu) {
  const int64_t row = blockIdx.y;
  const float2 t = ab[row];
  const float* p = x + row * HW;
  float* q = y + row * HW;
  auto f = [&](float v) {
    const float o = v * t.x + t.y;
    return silu ? o / (1.0f + expf(-o)) : o;
  };
  if (VEC) {
    const int64_t n4 = HW >> 2;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += (int64_t)gridDim.x * blockDim.x) {
      const float4 v = __ldg(reinterpret_cast<const float4*>(p) + i);
      reinterpret_cast<float4*>(q)[i] = make_float4(f(v.x), f(v.y), f(v.z), f(v.w));
    }
  } else {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < HW; i += (int64_t)gridDim.x * blockDim.x)
      q[i] = f(__ldg(p + i));
  }
}
// LayerNorm / RMSNorm over rows of C (tensor.cpp:628-679).
__global__ void k_row_norm(const float* __restrict__ x, float* __restrict__ y, int64_t C, const float* __restrict__ gamma,
                           const float* __restrict__ beta, float eps, int rms) {
  __shared__ float red[32];
  const float* p = x + (int64_t)blockIdx.x * C;
  float* q = y + (int64_t)blockIdx.x * C;
  float mean = 0.0f;
  if (!rms) {
    float s = 0.0f;
    for (int64_t i = threadIdx.x; i < C; i += blockDim.x) s += p[i];
    mean = block_sum(s, red) / (float)C;
  }
  float v = 0.0f;
  for (int64_t i = threadIdx.x; i < C; i += blockDim.x) {
    const float d = p[i] - mean;
    v += d * d;
  }
  const float rstd = rsqrtf(block_sum(v, red) / (float)C + eps);
  for (int64_t i = threadIdx.x; i < C; i += blockDim.x) {
    float o = (p[i] - mean) * rstd;
    if (gamma) o *= gamma[i];
    if (beta) o += beta[i];
    q[i] = o;
  }
}
// The same for rows of C <= 128 NV floats (C % 4 == 0, 16-byte rows): one warp per row,
// the row held in registers as NV float4 per lane, so it is read once and the two
// reductions are warp shuffles (the UNet's LayerNorms: C = 320 ... 1280).
template <int NV>
__global__ void __launch_bounds__(256) k_row_norm_warp(const float* __restrict__ x, float* __restrict__ y, int64_t rows,
                                                       int C, const float* __restrict__ gamma,
                                                       const float* __restrict__ beta, float eps, int rms) {
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  if (row >= rows) return;
  const int C4 = C >> 2;
  const float4* p = reinterpret_cast<const float4*>(x + row * C);
  float4 v[NV];
  float s = 0.0f;
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    const int c = lane + 32 * j;
    v[j] = c < C4 ? p[c] : make_float4(0.f, 0.f, 0.f, 0.f);
    s += (v[j].x + v[j].y) + (v[j].z + v[j].w);
  }
  const float mean = rms ? 0.0f : warp_sum(s) / (float)C;
  float q = 0.0f;
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    if (lane + 32 * j < C4) {
      const float a = v[j].x - mean, b = v[j].y - mean, c = v[j].z - mean, d = v[j].w - mean;
      q += (a * a + b * b) + (c * c + d * d);
    }
  }
  const float rstd = rsqrtf(warp_sum(q) / (float)C + eps);
  float4* o = reinterpret_cast<float4*>(y + row * C);
  const float4* g4 = reinterpret_cast<const float4*>(gamma);
  const float4* b4 = reinterpret_cast<const float4*>(beta);
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    const int c = lane + 32 * j;
    if (c < C4) {
      float4 r = make_float4((v[j].x - mean) * rstd, (v[j].y - mean) * rstd, (v[j].z - mean) * rstd,
                             (v[j].w - mean) * rstd);
      if (gamma) {
        const float4 g = __ldg(g4 + c);
        r = make_float4(r.x * g.x, r.y * g.y, r.z * g.z, r.w * g.w);
      }
      if (beta) {
        const float4 b = __ldg(b4 + c);
        r = make_float4(r.x + b.x, r.y + b.y, r.z + b.z, r.w + b.w);
      }
      o[c] = r;
    }
  }
}
// Per-head RMSNorm in place: one warp per group of `dim` values (tensor.cpp:681-699).
__global__ void k_rms_norm_heads(float* __restrict__ x, int64_t groups, int64_t dim, const float* __restrict__ gamma,
                                 float eps) {
  const int lane = threadIdx.x & 31;
  const int64_t w = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (w >= groups) return;
  float* p = x + w * dim;
  float s = 0.0f;
  for (int64_t i = lane; i < dim; i += 32) s += p[i] * p[i];
  const float rstd = rsqrtf(warp_sum(s) / (float)dim + eps);
  for (int64_t i = lane; i < dim; i += 32) p[i] = p[i] * rstd * (gamma ? gamma[i] : 1.0f);
}


// Scaled, max-subtracted softmax per row; causal rows keep (row0 + r % rows_per_head) + 1
// entries and zero the rest (tensor.cpp:752-769). Rows are ld apart; with round_out the
// probabilities are stored rounded to tf32 (the A operand of a tf32 GEMM).
__global__ void k_softmax_rows(float* __restrict__ x, int64_t cols, int64_t ld, float scale, int causal,
                               int64_t rows_per_head, int64_t row0, int round_out) {
  __shared__ float red[32];
  float* p = x + (int64_t)blockIdx.x * ld;
  const int64_t r = row0 + (int64_t)blockIdx.x % rows_per_head;
  const int64_t valid = causal ? min(cols, r + 1) : cols;
  float m = -INFINITY;
  for (int64_t j = threadIdx.x; j < valid; j += blockDim.x) m = fmaxf(m, p[j] * scale);
  m = block_max(m, red);
  float s = 0.0f;
  for (int64_t j = threadIdx.x; j < valid; j += blockDim.x) {
    const float e = expf(p[j] * scale - m);
    p[j] = e;
    s += e;
  }
  const float inv = 1.0f / block_sum(s, red);
  for (int64_t j = threadIdx.x; j < cols; j += blockDim.x) {
    const float o = j < valid ? p[j] * inv : 0.0f;
    p[j] = round_out ? round_tf32(o) : o;
  }
}
// The same softmax with the row held in registers (kSmxThreads x kSmxPer values): one
// read and one write of the row instead of three passes. Rows of up to 16384 columns.
constexpr int kSmxThreads = 512, kSmxPer = 32;
__global__ void __launch_bounds__(kSmxThreads) k_softmax_rows_reg(float* __restrict__ x, int64_t cols, int64_t ld,
                                                                  float scale, int causal, int64_t rows_per_head,
                                                                  int64_t row0, int round_out) {
  __shared__ float red[32];
  float* p = x + (int64_t)blockIdx.x * ld;
  const int64_t r = row0 + (int64_t)blockIdx.x % rows_per_head;
  const int64_t valid = causal ? min(cols, r + 1) : cols;
  float v[kSmxPer];
  float m = -INFINITY;
#pragma unroll
  for (int k = 0; k < kSmxPer; ++k) {
    const int64_t j = threadIdx.x + (int64_t)k * kSmxThreads;
    v[k] = j < valid ? p[j] * scale : -INFINITY;
    m = fmaxf(m, v[k]);
  }
  m = block_max(m, red);
  float s = 0.0f;
#pragma unroll
  for (int k = 0; k < kSmxPer; ++k) {
    v[k] = v[k] == -INFINITY ? 0.0f : expf(v[k] - m);
    s += v[k];
  }
  const float inv = 1.0f / block_sum(s, red);
#pragma unroll
  for (int k = 0; k < kSmxPer; ++k) {
    const int64_t j = threadIdx.x + (int64_t)k * kSmxThreads;
    if (j < cols) {
      const float o = v[k] * inv;
      p[j] = round_out ? round_tf32(o) : o;
    }
  }
}
// dst[c, r] = tf32(src[r, c]) for a rows x cols block (ld_src, ld_dst in elements), through
// a 32 x 32 shared-memory tile.
__global__ void k_transpose_tf32(const float* __restrict__ src, int64_t ld_src, float* __restrict__ dst,
                                 int64_t ld_dst, int64_t rows, int64_t cols) {
  __shared__ float tile[32][33];
  const int64_t r0 = (int64_t)blockIdx.y * 32, c0 = (int64_t)blockIdx.x * 32;
  const int tx = threadIdx.x, ty = threadIdx.y;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int64_t r = r0 + ty + 8 * i, c = c0 + tx;
    tile[ty + 8 * i][tx] = (r < rows && c < cols) ? round_tf32(__ldg(src + r * ld_src + c)) : 0.0f;
  }
  __syncthreads();
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int64_t c = c0 + ty + 8 * i, r = r0 + tx;
    if (c < cols && r < rows) dst[c * ld_dst + r] = tile[tx][ty + 8 * i];
  }
}

// im2col rows for pixels p0..p0+P-1: cols[p, (ci, ky, kx)] (tensor.cpp:551-575).
__global__ void k_im2col(const float* __restrict__ x, float* __restrict__ cols, int64_t Cin, int64_t H, int64_t W,
                         int64_t kh, int64_t kw, int64_t Wo, int stride, int pad, int64_t p0, int64_t P, int64_t K,
                         int64_t ldk) {
  FOR_GRID_ITEMS(i, P * K) {
    const int64_t p = i / K, k = i - p * K;
    const int64_t ci = k / (kh * kw), r = k - ci * kh * kw, ky = r / kw, kx = r - ky * kw;
    const int64_t oy = (p0 + p) / Wo, ox = (p0 + p) % Wo;
    const int64_t iy = oy * stride - pad + ky, ix = ox * stride - pad + kx;
    cols[p * ldk + k] = (iy >= 0 && iy < H && ix >= 0 && ix < W) ? x[(ci * H + iy) * W + ix] : 0.0f;
  }
}

}  // namespace

// ---------------------------------------------------------------------------------
// Launchers
// ---------------------------------------------------------------------------------
void launch_pack_bf16(const float* src, int64_t ld, uint16_t* dst, int64_t ldo, int64_t rows, int64_t cols) {
  if (rows <= 0 || cols <= 0) return;
  const bool vec = (cols % 8 == 0) && (ld % 4 == 0) && (ldo % 8 == 0) && ((uintptr_t)src % 16 == 0) &&
                   ((uintptr_t)dst % 16 == 0);
  if (vec)
    k_pack_bf16_vec<<<blocks_for(rows * cols, 8), kT, 0, ctx().stream>>>(src, ld, dst, ldo, rows, cols / 8);
  else
    k_pack_bf16<<<blocks_for(rows * cols), kT, 0, ctx().stream>>>(src, ld, dst, ldo, rows, cols);
  check_launch("pack_bf16");
}
void launch_conv_direct(const float* xh, int64_t N, int64_t Cin, int64_t cp, int64_t H, int64_t W, const float* wp,
                        int64_t cq, int64_t Cout, int k, int pad, const float* bias, const float* res, float* out,
                        int64_t Ho, int64_t Wo) {
  if (Cout > 8 || k > 15 || N > 65535 || (Ho + kDirTY - 1) / kDirTY > 65535)
    fail(kErrInvalidArg, "conv_direct: unsupported shape");
  const int TT = (kDirTX + k - 1) * (kDirTY + k - 1);
  const size_t smem = (size_t)(((kDirCh * TT + 3) & ~3) + 8 * kDirCh * k * k) * sizeof(float);
  const dim3 grid((unsigned)((Wo + kDirTX - 1) / kDirTX), (unsigned)((Ho + kDirTY - 1) / kDirTY), (unsigned)N);
  auto go = [&](auto kern) {
    if (smem > 48 * 1024)
      check_cuda(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem), "conv_direct attr");
    kern<<<grid, 256, smem, ctx().stream>>>(xh, cp, (int)Cin, (int)H, (int)W, wp, cq, (int)Cout, k, pad,
                                                            bias, res, out, (int)Ho, (int)Wo);
  };
  if (cp % 4 != 0 || (reinterpret_cast<uintptr_t>(xh) & 15) != 0)
    fail(kErrInvalidArg, "conv_direct: NHWC input must have 16-byte pixel rows");
  if (Cout <= 4)
    k == 3 ? go(k_conv_direct_nhwc<4, 3>) : go(k_conv_direct_nhwc<4, 0>);
  else
    k == 3 ? go(k_conv_direct_nhwc<8, 3>) : go(k_conv_direct_nhwc<8, 0>);
  check_launch("conv_direct");
}
void launch_split_reduce(const float* part, int splits, int64_t total, int64_t C, int64_t hw, const float* bias,
                         const float* res, float* out) {
  if (total <= 0) return;
  k_split_reduce<<<blocks_for(total), kT, 0, ctx().stream>>>(part, splits, total, C, hw, bias, res, out);
  check_launch("split_reduce");
}
void launch_conv_pack_x(const float* x, float* xh, int64_t N, int64_t C, int64_t HW, int64_t cp) {
  launch_pack_nhwc(x, xh, N, C, 1, HW, cp, nullptr, 1.0f, 0.0f, false, false);
}
void launch_pack_nhwc(const float* x, float* xh, int64_t N, int64_t C, int64_t H, int64_t W, int64_t cp,
                      const float2* ab, float a0, float b0, bool silu, bool up2) {
  if (N <= 0 || H <= 0 || W <= 0) return;
  if (N > 65535 || (cp + 31) / 32 > 65535) fail(kErrInvalidArg, "pack_nhwc: too many samples or channels");
  const int64_t HWo = (up2 ? 4 : 1) * H * W;
  if (HWo >= ((int64_t)1 << 31)) fail(kErrInvalidArg, "pack_nhwc: image too large");
  const dim3 grid((unsigned)((HWo + kPackPx - 1) / kPackPx), (unsigned)((cp + 31) / 32), (unsigned)N);
  if (up2)
    k_pack_nhwc<true><<<grid, dim3(32, 8), 0, ctx().stream>>>(x, xh, C, H, W, cp, ab, a0, b0, silu ? 1 : 0);
  else
    k_pack_nhwc<false><<<grid, dim3(32, 8), 0, ctx().stream>>>(x, xh, C, H, W, cp, ab, a0, b0, silu ? 1 : 0);
  check_launch("pack_nhwc");
}
void launch_conv_pack_w(const float* w, float* wp, int64_t Cout, int64_t Cin, int64_t taps, int64_t cq) {
  const int64_t total = Cout * taps * cq;
  if (total <= 0) return;
  const size_t slab = (size_t)(Cin * taps) * sizeof(float);
  constexpr size_t kSlabMax = 128 * 1024;
  if (slab <= kSlabMax && Cout <= 0x7fffffff && taps * cq < ((int64_t)1 << 31)) {
    auto go = [&](auto kern) {
      if (slab > 48 * 1024)
        check_cuda(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSlabMax),
                   "conv_pack_w attr");
      kern<<<(unsigned)Cout, 256, slab, ctx().stream>>>(w, wp, (int)Cin, (int)taps, (int)cq);
    };
    if ((Cin * taps) % 4 == 0 && (reinterpret_cast<uintptr_t>(w) & 15) == 0)
      go(k_conv_pack_w_slab<true>);
    else
      go(k_conv_pack_w_slab<false>);
  } else {
    k_conv_pack_w<<<blocks_for(total), kT, 0, ctx().stream>>>(w, wp, Cin, taps, cq, total);
  }
  check_launch("conv_pack_w");
}
void launch_pack_tf32(const float* src, int64_t ld, float* dst, int64_t ldo, int64_t rows, int64_t cols) {
  if (rows <= 0 || cols <= 0) return;
  launch_pack_tf32_pair(src, ld, dst, ldo, rows, nullptr, 0, nullptr, 0, 0, cols);
}
void launch_pack_tf32_pair(const float* s0, int64_t ld0, float* d0, int64_t ldo0, int64_t r0, const float* s1,
                           int64_t ld1, float* d1, int64_t ldo1, int64_t r1, int64_t cols) {
  if (cols <= 0 || r0 + r1 <= 0) return;
  auto a16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
  const bool vec = cols % 4 == 0 && ld0 % 4 == 0 && ldo0 % 4 == 0 && a16(s0) && a16(d0) &&
                   (r1 == 0 || (ld1 % 4 == 0 && ldo1 % 4 == 0 && a16(s1) && a16(d1)));
  const int64_t blocks = std::min<int64_t>((r0 + r1 + 7) / 8, (int64_t)std::max(1, ctx().num_sms) * 16);
  if (vec)
    k_pack_tf32_rows<true><<<(unsigned)blocks, 256, 0, ctx().stream>>>(s0, ld0, d0, ldo0, r0, s1, ld1, d1, ldo1, r1,
                                                                       cols);
  else
    k_pack_tf32_rows<false><<<(unsigned)blocks, 256, 0, ctx().stream>>>(s0, ld0, d0, ldo0, r0, s1, ld1, d1, ldo1, r1,
                                                                        cols);
  check_launch("pack_tf32_pair");
}
void launch_round_tf32_inplace(float* x, int64_t ld, int64_t rows, int64_t cols) {
  if (rows <= 0 || cols <= 0) return;
  k_round_tf32_inplace<<<blocks_for(rows * cols), kT, 0, ctx().stream>>>(x, ld, rows, cols);
  check_launch("round_tf32");
}
void launch_copy2d(const void* src, int64_t ld, void* dst, int64_t ldo, int64_t rows, int64_t cols, int esize) {
  if (rows <= 0 || cols <= 0) return;
  if (esize == 2)
    k_copy2d_16<<<blocks_for(rows * cols), kT, 0, ctx().stream>>>((const uint16_t*)src, ld, (uint16_t*)dst, ldo, rows,
                                                                 cols);
  else
    k_copy2d_32<<<blocks_for(rows * cols), kT, 0, ctx().stream>>>((const float*)src, ld, (float*)dst, ldo, rows, cols);
  check_launch("copy2d");
}
void launch_bias_fill(float* C, int64_t ldc, int64_t M, int64_t N, const float* bias, bool accumulate) {
  if (M <= 0 || N <= 0) return;
  k_bias_fill<<<blocks_for(M * N), kT, 0, ctx().stream>>>(C, ldc, M, N, bias, accumulate ? 1 : 0);
  check_launch("bias_fill");
}
void launch_gemm_skinny(int64_t M, int64_t N, int64_t K, const float* A, int64_t lda, const void* B, int64_t ldb,
                        bool b_bf16, float* C, int64_t ldc, const float* bias, bool accumulate) {
  DeviceContext& c = ctx();
  launch_gemm_skinny_on(M, N, K, A, lda, B, ldb, b_bf16, C, ldc, bias, accumulate, c.num_sms, c.stream);
}
void launch_gemm_skinny_on(int64_t M, int64_t N, int64_t K, const float* A, int64_t lda, const void* B, int64_t ldb,
                           bool b_bf16, float* C, int64_t ldc, const float* bias, bool accumulate, int num_sms,
                           cudaStream_t stream) {
  const int esz = b_bf16 ? 2 : 4;
  const bool vec = ((ldb * esz) % 16 == 0) && ((uintptr_t)B % 16 == 0);
  // A read in place when it is 16-byte aligned row by row and M <= 4; otherwise staged.
  const bool a_direct = M <= 4 && (lda % 4 == 0) && ((uintptr_t)A % 16 == 0);
  const size_t smem = a_direct ? 0 : (size_t)(M * K) * sizeof(float);
  const int64_t groups = (N + kGemvRows - 1) / kGemvRows;
  const int64_t per_sm =
      std::max<int64_t>(1, std::min<int64_t>(8, (int64_t)(200 * 1024) / (int64_t)std::max<size_t>(smem, 1)));
  const int64_t blocks = std::max<int64_t>(
      1, std::min<int64_t>((groups + kGemvWarps - 1) / kGemvWarps, (int64_t)num_sms * per_sm));
  auto go = [&](auto kern) {
    if (smem > 48 * 1024)
      check_cuda(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem), "gemv attr");
    kern<<<(unsigned)blocks, kGemvWarps * 32, smem, stream>>>((int)M, (int)N, (int)K, A, lda, B, ldb, C, ldc, bias,
                                                              accumulate ? 1 : 0, vec ? 1 : 0);
  };
  if (b_bf16) {
    if (a_direct) {
      if (M == 1) go(k_gemv_rows<true, 1, false>);
      else go(k_gemv_rows<true, 4, false>);
    } else if (M <= 4) {
      go(k_gemv_rows<true, 4, true>);
    } else {
      go(k_gemv_rows<true, 16, true>);
    }
  } else {
    if (a_direct) {
      if (M == 1) go(k_gemv_rows<false, 1, false>);
      else go(k_gemv_rows<false, 4, false>);
    } else if (M <= 4) {
      go(k_gemv_rows<false, 4, true>);
    } else {
      go(k_gemv_rows<false, 16, true>);
    }
  }
  check_launch("gemm_skinny");
}

// Public layer ops (called from runtime.cu's C ABI after argument checks).
void gn_scale_shift(const float* x, int64_t N, int64_t C, int64_t HW, int groups, const float* gamma,
                    const float* beta, float eps, float2* ab) {
  const int64_t segs = N * groups, len = (C / groups) * HW;
  const int64_t chunks = (len + kGnChunk - 1) / kGnChunk;
  if (segs > 65535 || chunks > (1ll << 31) - 1) fail(kErrInvalidArg, "group_norm: too many samples or groups");
  float2* part = static_cast<float2*>(pool_malloc((size_t)(segs * chunks) * sizeof(float2)));
  cudaStream_t st = ctx().stream;
  k_gn_stats<<<dim3((unsigned)chunks, (unsigned)segs), kGnThreads, 0, st>>>(x, len, (int)chunks, part);
  k_gn_finalize<<<(unsigned)((segs + 7) / 8), 256, 0, st>>>(part, (int)chunks, len, C, groups, gamma, beta, eps, ab,
                                                            segs);
  check_launch("group_norm_stats");
  pool_free(part);  // stream-ordered reuse
}
void gn_scale_shift_parts(const float4* part, int64_t tiles_img, int64_t N, int64_t C, int groups,
                          const float* gamma, const float* beta, float eps, float2* ab) {
  if (N * groups > (1ll << 31) - 1) fail(kErrInvalidArg, "group_norm: too many groups");
  k_gn_finalize_parts<<<(unsigned)(N * groups), 256, 0, ctx().stream>>>(part, tiles_img, C, groups, gamma, beta, eps,
                                                                        ab);
  check_launch("group_norm_parts");
}
void op_group_norm(const float* x, float* y, int64_t N, int64_t C, int64_t HW, int groups, const float* gamma,
                   const float* beta, float eps, bool silu) {
  if (N <= 0 || C <= 0 || HW <= 0) return;
  if (N * C > 65535) fail(kErrInvalidArg, "group_norm: too many samples x channels");
  if (groups > 0 && C % groups == 0 && HW % 4 == 0 && (C / groups) * HW <= kGnFusedMax &&
      (reinterpret_cast<uintptr_t>(x) & 15) == 0 && (reinterpret_cast<uintptr_t>(y) & 15) == 0) {
    const int cg = (int)(C / groups);
    const size_t smem = (size_t)cg * HW * sizeof(float);
    static bool attr_set[64] = {};  // per device ordinal (ctx() keeps ordinals below 64)
    DeviceContext& c = ctx();
    if (smem > 48 * 1024 && !attr_set[c.device]) {
      check_cuda(cudaFuncSetAttribute(k_gn_fused, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      (int)(kGnFusedMax * sizeof(float))),
                 "group_norm attr");
      attr_set[c.device] = true;
    }
    k_gn_fused<<<dim3((unsigned)groups, (unsigned)N), 1024, smem, c.stream>>>(x, y, C, (int)HW, cg, gamma, beta, eps,
                                                                             silu ? 1 : 0);
    check_launch("group_norm");
    return;
  }
  float2* ab = static_cast<float2*>(pool_malloc((size_t)(N * C) * sizeof(float2)));
  uint8_t* ws = reinterpret_cast<uint8_t*>(ab);
  cudaStream_t st = ctx().stream;
  gn_scale_shift(x, N, C, HW, groups, gamma, beta, eps, ab);
  const bool vec = HW % 4 == 0 && (reinterpret_cast<uintptr_t>(x) & 15) == 0 && (reinterpret_cast<uintptr_t>(y) & 15) == 0;
  const int64_t per_row = vec ? HW / 4 : HW;
  const unsigned bx = (unsigned)std::max<int64_t>(1, std::min<int64_t>((per_row + 4 * 256 - 1) / (4 * 256), 64));
  if (vec)
    k_gn_apply<true><<<dim3(bx, (unsigned)(N * C)), 256, 0, st>>>(x, y, HW, ab, silu ? 1 : 0);
  else
    k_gn_apply<false><<<dim3(bx, (unsigned)(N * C)), 256, 0, st>>>(x, y, HW, ab, silu ? 1 : 0);
  check_launch("group_norm");
  // Stream-ordered: the next user of this pool block is issued on the same stream.
  pool_free(ws);
}
void op_row_norm(const float* x, float* y, int64_t rows, int64_t C, const float* gamma, const float* beta, float eps,
                 bool rms) {
  if (rows <= 0) return;
  auto a16 = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15) == 0; };
  const int nv = (int)((C + 127) / 128);
  if (C % 4 == 0 && nv <= 16 && a16(x) && a16(y) && a16(gamma) && a16(beta) && (rows + 7) / 8 < (1ll << 31)) {
    const unsigned blocks = (unsigned)((rows + 7) / 8);
    const int r = rms ? 1 : 0;
    cudaStream_t st = ctx().stream;
    switch (nv) {
#define SDB_RN(V) \
  case V: k_row_norm_warp<V><<<blocks, 256, 0, st>>>(x, y, rows, (int)C, gamma, beta, eps, r); break;
      SDB_RN(1) SDB_RN(2) SDB_RN(3) SDB_RN(4) SDB_RN(5) SDB_RN(6) SDB_RN(7) SDB_RN(8)
      SDB_RN(9) SDB_RN(10) SDB_RN(11) SDB_RN(12) SDB_RN(13) SDB_RN(14) SDB_RN(15) SDB_RN(16)
#undef SDB_RN
    }
  } else {
    k_row_norm<<<(unsigned)rows, kT, 0, ctx().stream>>>(x, y, C, gamma, beta, eps, rms ? 1 : 0);
  }
  check_launch(rms ? "rms_norm" : "layer_norm");
}
void op_rms_norm_heads(float* x, int64_t groups, int64_t dim, const float* gamma, float eps) {
  if (groups <= 0) return;
  const int64_t blocks = (groups + 7) / 8;
  k_rms_norm_heads<<<(unsigned)blocks, kT, 0, ctx().stream>>>(x, groups, dim, gamma, eps);
  check_launch("rms_norm_heads");
}
void op_softmax_rows(float* x, int64_t rows, int64_t cols, float scale, bool causal, int64_t rows_per_head) {
  op_softmax_rows_ex(x, rows, cols, cols, scale, causal, rows_per_head, 0, false);
}
void op_softmax_rows_ex(float* x, int64_t rows, int64_t cols, int64_t ld, float scale, bool causal,
                        int64_t rows_per_head, int64_t row0, bool round_out) {
  if (rows <= 0 || cols <= 0) return;
  if (cols <= (int64_t)kSmxThreads * kSmxPer)
    k_softmax_rows_reg<<<(unsigned)rows, kSmxThreads, 0, ctx().stream>>>(x, cols, ld, scale, causal ? 1 : 0,
                                                                          rows_per_head, row0, round_out ? 1 : 0);
  else
    k_softmax_rows<<<(unsigned)rows, kT, 0, ctx().stream>>>(x, cols, ld, scale, causal ? 1 : 0, rows_per_head, row0,
                                                            round_out ? 1 : 0);
  check_launch("softmax_rows");
}
void launch_transpose_tf32(const float* src, int64_t ld_src, float* dst, int64_t ld_dst, int64_t rows, int64_t cols) {
  if (rows <= 0 || cols <= 0) return;
  const dim3 grid((unsigned)((cols + 31) / 32), (unsigned)((rows + 31) / 32));
  k_transpose_tf32<<<grid, dim3(32, 8), 0, ctx().stream>>>(src, ld_src, dst, ld_dst, rows, cols);
  check_launch("transpose_tf32");
}
void op_im2col(const float* x, float* cols, int64_t Cin, int64_t H, int64_t W, int64_t kh, int64_t kw, int64_t Wo,
               int stride, int pad, int64_t p0, int64_t P, int64_t K, int64_t ldk) {
  if (P * K <= 0) return;
  k_im2col<<<blocks_for(P * K), kT, 0, ctx().stream>>>(x, cols, Cin, H, W, kh, kw, Wo, stride, pad, p0, P, K, ldk);
  check_launch("im2col");
}

}  // namespace sdb
