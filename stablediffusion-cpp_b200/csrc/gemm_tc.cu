// gemm_tc.cu - the dense contraction C[M,N] = A[M,K] * B[N,K]^T on 5th-generation
// tensor cores (sm_100a), the B200 replacement for the cuBLAS call inside the
// reference's gemm_nt_bf16 / gemm_nt_f32 (backend_cuda.cu:453-477).
//
// Design
//   * Persistent kernel, one CTA per SM, 192 threads in four roles:
//       warp 0   TMA producer: streams 128-byte-wide K slices of A and B into a
//                ring of shared-memory stages (128B swizzle), one mbarrier per stage
//       warp 1   MMA issuer: allocates TMEM, issues tcgen05.mma (M=128, N=BN) from
//                the stages into one of two TMEM accumulators, commits each stage
//                back to the producer and each finished tile to the epilogue
//       warps 2-5 epilogue: tcgen05.ld the accumulator (warp w owns TMEM lanes
//                32*(w%4)...), apply bias / gated activation / accumulate and store
//                with 16-byte vector stores; the TMEM buffer is released after the
//                last load so the next tile's MMAs overlap this tile's stores
//   * Operands: kind::f16 (bf16 x bf16) or kind::tf32 (fp32 x fp32), both K-major,
//     fp32 accumulation in TMEM. 128 B of K per stage = 64 bf16 or 32 fp32.
//   * Tiles are walked in groups of 16 M-blocks so that the CTAs running at the same
//     time share A and B tiles through L2.
//   * Edges: TMA zero-fills out-of-range rows/columns/K; the epilogue masks stores.
//   * Every mbarrier wait is bounded (ptx.cuh): a stuck pipeline sets the device error
//     word and the CTA drains and frees TMEM instead of hanging the GPU.
#include <algorithm>
#include <cstdio>
#include <cuda_fp16.h>

#include <string>

#include "internal.h"
#include "ptx.cuh"

namespace sdb {
namespace {

constexpr int kBM = 128;
constexpr int kThreads = 192;
constexpr int kGroupM = 16;

// Implicit-GEMM convolution, stride 1: out[img, co, oy, ox] = sum over taps (ky, kx) and
// channels ci of w[co, ky, kx, ci] * x[img, oy - pad + ky, ox - pad + kx, ci] (+ bias[co])
// (+ res[img, co, oy, ox]; res may be the output itself: each element is read, then
// written, by one thread). GEMM rows are output channels; a tile's BN columns are a
// BW x BH rectangle of output pixels of one image (column j -> (oy0 + j / BW, ox0 + j % BW)).
// One K block is 32 channels of one tap, loaded as a 4-D TMA box of the NHWC input that the
// hardware zero-fills outside the image (the padding).
struct ConvGeom {
  int Ho, Wo, BW, BH, tiles_x, tiles_y;
  int kw, pad, cblocks;
  int b_bytes;             // bytes of one B box (BW * BH rows of 128 B; half of that on SM pairs)
  int half_dx, half_dy;    // SM pairs: offset of the second CTA's half of the pixel rectangle
  long long img_stride;    // elements between images of the output (Cout * Ho * Wo)
  const float* res;        // residual added in the epilogue (output layout), or null
  // GroupNorm statistics of the output (null: off): per (image, group, pixel tile) the
  // count, mean and sum of squared deviations, at gn_part[(img * groups + g) * tiles_img +
  // tile]. Groups are gn_cg consecutive channels, gn_cg a divisor of 32.
  float4* gn_part;
  int gn_cg, gn_groups, tiles_img;
};

struct GemmParams {
  int M, N, K;
  int m_tiles, n_tiles, num_tiles, k_blocks;
  void* C;
  long long ldc;
  const float* bias;
  int accumulate;
  int epi;       // Epi
  int out_bf16;  // store bf16 instead of fp32
  int vec_ok;    // C base and ldc allow 16-byte stores
  int* err;
  QkvRope rope;  // Epi::kQkvRope
  ScatterOut sc;  // Epi::kScatter
  ConvGeom cv;    // implicit-GEMM convolution (k_gemm_tc<BN, true, true>)
  // Split-K (convolution only): work item t is split t / base_tiles of tile t % base_tiles,
  // K blocks [split * kb_split, +kb_split); the epilogue stores split s's partial tile at
  // C + s * split_stride (no bias or residual; a reduction kernel adds them).
  int splits, base_tiles, kb_split;
  long long split_stride;
  int bias_vec;   // bias is 16-byte aligned: float4 loads in the epilogue
};

// Work item t -> tile index and K-block range.
__device__ __forceinline__ void split_item(const GemmParams& p, int t, int& tile, int& kb0, int& kb1, int& split) {
  if (p.splits > 1) {
    split = t / p.base_tiles;
    tile = t - split * p.base_tiles;
    kb0 = split * p.kb_split;
    kb1 = min(p.k_blocks, kb0 + p.kb_split);
  } else {
    split = 0;
    tile = t;
    kb0 = 0;
    kb1 = p.k_blocks;
  }
}

constexpr int kStgPitch = 36;  // floats per staged row: 16-byte aligned, spreads banks

template <int BN>
struct Cfg {
  static constexpr int A_BYTES = kBM * 128;
  static constexpr int B_BYTES = BN * 128;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int STAGES_RAW = (200 * 1024) / STAGE_BYTES;
  static constexpr int STAGES = STAGES_RAW > 8 ? 8 : STAGES_RAW;
  static constexpr uint32_t TMEM_COLS =
      (2 * BN <= 32) ? 32 : (2 * BN <= 64) ? 64 : (2 * BN <= 128) ? 128 : (2 * BN <= 256) ? 256 : 512;
  static constexpr int STG_BYTES = 4 * 32 * kStgPitch * 4;  // scatter staging, one 32x32 block per epilogue warp
  static constexpr int SMEM = STAGES * STAGE_BYTES + 1024 /*align*/ + 256 /*barriers*/ + STG_BYTES;
};

__device__ __forceinline__ void tile_coords(int t, int m_tiles, int n_tiles, int& mb, int& nb) {
  const int per_group = kGroupM * n_tiles;
  const int g = t / per_group;
  const int first = g * kGroupM;
  const int gs = min(m_tiles - first, kGroupM);
  const int r = t - g * per_group;
  mb = first + r % gs;
  nb = r / gs;
}

// silu(g) = g * 1 / (1 + 2^(-g log2 e)) for a pair, on the MUFU pipe (ex2.approx and
// rcp.approx, each within 2 ulp of the exact fp32 value per the PTX ISA) with packed fp32
// multiplies and adds around them. The SwiGLU product differs from the reference's
// g / (1 + expf(-g)) (tensor.cpp:732-748) by a few fp32 ulp, below the bf16 rounding of
// the output. g -> -inf gives 2^+inf = inf, rcp(inf) = 0 and a (-)0 result, as the exact
// form does. The epilogue shares the SM sub-partitions with the MMA issuer and the power
// budget with the tensor core, so its instruction count shows in the GEMM's time: packed,
// the w1/w3 GEMM launches of the DiT step run about 1% faster than with the same math
// unpacked.
__device__ __forceinline__ float2 silu2(float2 g) {
  const float2 a = fmul2(g, make_float2(-1.4426950408889634f, -1.4426950408889634f));
  float e0, e1, r0, r1;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e0) : "f"(a.x));
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e1) : "f"(a.y));
  const float2 d = fadd2(make_float2(e0, e1), make_float2(1.0f, 1.0f));
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r0) : "f"(d.x));
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r1) : "f"(d.y));
  return fmul2(g, make_float2(r0, r1));
}
__device__ __forceinline__ float gelu_erf_f(float g) { return 0.5f * g * (1.0f + erff(g * 0.70710678118654752f)); }

// Stores 32 consecutive fp32 results of one row (columns col0..col0+31).
__device__ __forceinline__ void store_row32(const GemmParams& p, int row, int col0, float (&v)[32],
                                            long long off = 0) {
  if (p.out_bf16) {
    uint16_t* c = reinterpret_cast<uint16_t*>(p.C) + (long long)row * p.ldc + col0;
    if (p.vec_ok && col0 + 32 <= p.N) {
#pragma unroll
      for (int j = 0; j < 32; j += 8) {
        uint4 w;
        w.x = pack_bf16x2(v[j], v[j + 1]);
        w.y = pack_bf16x2(v[j + 2], v[j + 3]);
        w.z = pack_bf16x2(v[j + 4], v[j + 5]);
        w.w = pack_bf16x2(v[j + 6], v[j + 7]);
        *reinterpret_cast<uint4*>(c + j) = w;
      }
    } else {
      const int n = min(32, p.N - col0);
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (j < n) c[j] = f32_to_bf16_rne(v[j]);
    }
    return;
  }
  float* c = reinterpret_cast<float*>(p.C) + off + (long long)row * p.ldc + col0;
  if (p.vec_ok && col0 + 32 <= p.N) {
#pragma unroll
    for (int j = 0; j < 32; j += 4) {
      float4 o = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
      if (p.accumulate) {
        const float4 old = *reinterpret_cast<const float4*>(c + j);
        o.x += old.x; o.y += old.y; o.z += old.z; o.w += old.w;
      }
      *reinterpret_cast<float4*>(c + j) = o;
    }
  } else {
    const int n = min(32, p.N - col0);
#pragma unroll
    for (int j = 0; j < 32; ++j)
      if (j < n) c[j] = p.accumulate ? c[j] + v[j] : v[j];
  }
}

// Adds bias[col0 .. col0 + 31] to v. With p.bias_vec (16-byte aligned bias) by float4
// loads and packed adds; otherwise per element, masked at N. The sums are the same.
__device__ __forceinline__ void add_bias32(const GemmParams& p, int col0, float (&v)[32]) {
  if (!p.bias) return;
  if (p.bias_vec && col0 + 32 <= p.N) {
#pragma unroll
    for (int j = 0; j < 32; j += 4) {
      const float4 b = __ldg(reinterpret_cast<const float4*>(p.bias + col0 + j));
      const float2 x0 = fadd2(make_float2(v[j], v[j + 1]), make_float2(b.x, b.y));
      const float2 x1 = fadd2(make_float2(v[j + 2], v[j + 3]), make_float2(b.z, b.w));
      v[j] = x0.x;
      v[j + 1] = x0.y;
      v[j + 2] = x1.x;
      v[j + 3] = x1.y;
    }
  } else {
#pragma unroll
    for (int j = 0; j < 32; ++j)
      if (col0 + j < p.N) v[j] += __ldg(p.bias + col0 + j);
  }
}

// Epi::kQkvRope for one row and one 128-column head of the accumulator at TMEM address
// `hcol` (lane of this thread), head columns [col0, col0 + 128) of the GEMM output.
// q and k: two passes over TMEM (sum of squares, then normalise, gamma, rotate, store);
// v: one pass. The rotary pair (x0, x1) = columns (2i, 2i+1) maps to
// (x0 c - x1 s, x1 c + x0 s). The tables hold cos at both 2i and 2i + 1 (cs) and
// (-sin, +sin) at (2i, 2i + 1) (sn), so a pair is x * (c, c) + (x1, x0) * (-s, s): one
// packed multiply and one packed FMA. The normalisation scale rstd * gamma is applied to
// x first, so the pair costs four packed instructions in all. This epilogue runs beside
// the MMA issuer on the same SM sub-partitions; against scalar math with per-element
// gamma loads the packed form takes 2-4% off the fused-QKV GEMM launches of the DiT step
// (ncu launch times at 32768 and 33792 rows).
__device__ __forceinline__ void qkv_rope_head(const GemmParams& p, uint32_t hcol, int row, bool row_ok, int col0) {
  const QkvRope& q = p.rope;
  const int which = col0 / q.Dq;  // 0 q, 1 k, 2 v
  const int hc = col0 - which * q.Dq;
  __half* dst = reinterpret_cast<__half*>(which == 0 ? q.q16 : which == 1 ? q.k16 : q.v16) +
                (long long)row * q.Dq + hc;
  auto load = [&](int cc, float (&v)[32]) {
    uint32_t r[32];
    __syncwarp();  // tcgen05.ld is .sync.aligned: reconverge after the masked stores
    tmem_ld_32x32b_x32(hcol + (uint32_t)(cc * 32), r);
    tmem_wait_ld();
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
    add_bias32(p, col0 + cc * 32, v);
  };
  auto store32 = [&](int cc, const float (&o)[32]) {
    if (!row_ok) return;
    uint4* d4 = reinterpret_cast<uint4*>(dst + cc * 32);
#pragma unroll
    for (int j = 0; j < 32; j += 8) {
      uint4 w;
      __half2 h0 = __floats2half2_rn(o[j], o[j + 1]), h1 = __floats2half2_rn(o[j + 2], o[j + 3]);
      __half2 h2 = __floats2half2_rn(o[j + 4], o[j + 5]), h3 = __floats2half2_rn(o[j + 6], o[j + 7]);
      w.x = *reinterpret_cast<uint32_t*>(&h0);
      w.y = *reinterpret_cast<uint32_t*>(&h1);
      w.z = *reinterpret_cast<uint32_t*>(&h2);
      w.w = *reinterpret_cast<uint32_t*>(&h3);
      d4[j / 8] = w;
    }
  };
  if (which == 2) {
#pragma unroll 1
    for (int cc = 0; cc < 4; ++cc) {
      float v[32];
      load(cc, v);
      store32(cc, v);
    }
    return;
  }
  float2 ssa = make_float2(0.0f, 0.0f), ssb = make_float2(0.0f, 0.0f);
#pragma unroll 1
  for (int cc = 0; cc < 4; ++cc) {
    float v[32];
    load(cc, v);
#pragma unroll
    for (int j = 0; j < 32; j += 4) {
      ssa = ffma2(make_float2(v[j], v[j + 1]), make_float2(v[j], v[j + 1]), ssa);
      ssb = ffma2(make_float2(v[j + 2], v[j + 3]), make_float2(v[j + 2], v[j + 3]), ssb);
    }
  }
  const float rstd = rsqrtf(((ssa.x + ssa.y) + (ssb.x + ssb.y)) / 128.0f + q.eps);
  const float2 r2 = make_float2(rstd, rstd);
  const float* gam = which == 0 ? q.gq : q.gk;
  const int s = row_ok ? row % q.S : 0;
  const float* cr = q.cs + (long long)s * 128;
  const float* sr = q.sn + (long long)s * 128;
#pragma unroll 1
  for (int cc = 0; cc < 4; ++cc) {
    float v[32], o[32];
    load(cc, v);
#pragma unroll
    for (int j = 0; j < 32; j += 4) {
      float4 g4 = make_float4(1.0f, 1.0f, 1.0f, 1.0f);
      if (gam) {
        if (q.gamma_vec) {
          g4 = __ldg(reinterpret_cast<const float4*>(gam + cc * 32 + j));
        } else {
          g4.x = __ldg(gam + cc * 32 + j);
          g4.y = __ldg(gam + cc * 32 + j + 1);
          g4.z = __ldg(gam + cc * 32 + j + 2);
          g4.w = __ldg(gam + cc * 32 + j + 3);
        }
      }
      const float4 c4 = __ldg(reinterpret_cast<const float4*>(cr + cc * 32 + j));
      const float4 s4 = __ldg(reinterpret_cast<const float4*>(sr + cc * 32 + j));
      const float2 xa = fmul2(make_float2(v[j], v[j + 1]), fmul2(make_float2(g4.x, g4.y), r2));
      const float2 xb = fmul2(make_float2(v[j + 2], v[j + 3]), fmul2(make_float2(g4.z, g4.w), r2));
      const float2 oa = ffma2(make_float2(xa.y, xa.x), make_float2(s4.x, s4.y), fmul2(xa, make_float2(c4.x, c4.y)));
      const float2 ob = ffma2(make_float2(xb.y, xb.x), make_float2(s4.z, s4.w), fmul2(xb, make_float2(c4.z, c4.w)));
      o[j] = oa.x;
      o[j + 1] = oa.y;
      o[j + 2] = ob.x;
      o[j + 3] = ob.y;
    }
    store32(cc, o);
  }
}

// Epi::kScatter for one 32-column chunk of the warp's 32 rows (row_base..+31): each lane
// stages its row in shared memory, then the warp stores four full 128-byte row segments
// per instruction, so stores to a peer cross NVLink as whole lines rather than 16-byte
// pieces of 32 different rows.
__device__ __forceinline__ void scatter_chunk(const GemmParams& p, float* stg, const uint32_t (&r)[32], int row_base,
                                              int col0, int lane) {
  float* mine = stg + lane * kStgPitch;
#pragma unroll
  for (int j = 0; j < 32; j += 4) {
    float4 o = make_float4(__uint_as_float(r[j]), __uint_as_float(r[j + 1]), __uint_as_float(r[j + 2]),
                           __uint_as_float(r[j + 3]));
    if (p.bias) {
      if (col0 + j + 3 < p.N) {
        o.x += __ldg(p.bias + col0 + j);
        o.y += __ldg(p.bias + col0 + j + 1);
        o.z += __ldg(p.bias + col0 + j + 2);
        o.w += __ldg(p.bias + col0 + j + 3);
      }
    }
    *reinterpret_cast<float4*>(mine + j) = o;
  }
  __syncwarp();
  const int sub = lane >> 3, c4 = (lane & 7) * 4;
#pragma unroll
  for (int r0 = 0; r0 < 32; r0 += 4) {
    const int rr = r0 + sub, grow = row_base + rr;
    if (grow < p.M && col0 + c4 < p.N) {
      const int o = grow / p.sc.rs;
      float* dst = p.sc.base[o] + ((long long)p.sc.rank * p.sc.slot_rows + (grow - o * p.sc.rs)) * p.ldc + col0 + c4;
      *reinterpret_cast<float4*>(dst) = *reinterpret_cast<const float4*>(stg + rr * kStgPitch + c4);
    }
  }
  __syncwarp();
}

// Stores 16 gated results (from 16 gate + 16 up columns) at output column ocol0.
__device__ __forceinline__ void store_row16(const GemmParams& p, int row, int ocol0, const float (&y)[16]) {
  const int on = p.N / 2;
  if (p.out_bf16) {
    uint16_t* c = reinterpret_cast<uint16_t*>(p.C) + (long long)row * p.ldc + ocol0;
    if (p.vec_ok && ocol0 + 16 <= on) {
#pragma unroll
      for (int j = 0; j < 16; j += 8) {
        uint4 w;
        w.x = pack_bf16x2(y[j], y[j + 1]);
        w.y = pack_bf16x2(y[j + 2], y[j + 3]);
        w.z = pack_bf16x2(y[j + 4], y[j + 5]);
        w.w = pack_bf16x2(y[j + 6], y[j + 7]);
        *reinterpret_cast<uint4*>(c + j) = w;
      }
    } else {
      const int n = min(16, on - ocol0);
#pragma unroll
      for (int j = 0; j < 16; ++j)
        if (j < n) c[j] = f32_to_bf16_rne(y[j]);
    }
    return;
  }
  float* c = reinterpret_cast<float*>(p.C) + (long long)row * p.ldc + ocol0;
  if (p.vec_ok && ocol0 + 16 <= on) {
#pragma unroll
    for (int j = 0; j < 16; j += 4) *reinterpret_cast<float4*>(c + j) = make_float4(y[j], y[j + 1], y[j + 2], y[j + 3]);
  } else {
    const int n = min(16, on - ocol0);
#pragma unroll
    for (int j = 0; j < 16; ++j)
      if (j < n) c[j] = y[j];
  }
}

// The epilogue of one accumulator tile for one warp: TMEM lanes of rows
// row_base..row_base+31 (this thread: row_base + lane) at TMEM address tbase, tile column
// block nb. stg is this warp's 32 x kStgPitch staging block (Epi::kScatter).
// With split-K (p.splits > 1, Epi::kStore only) the raw partial tile of K split `split`
// goes to C + split * split_stride; bias and accumulate are applied by the reduction.
template <int BN>
__device__ __forceinline__ void epilogue_tile(const GemmParams& p, float* stg, uint32_t tbase, int row_base, int nb,
                                              int lane, int split = 0) {
  const int row = row_base + lane;
  const bool row_ok = row < p.M;
  if constexpr (BN % 128 == 0) {
    if (p.epi == (int)Epi::kQkvRope) {
      // The launcher only pairs this epilogue with 128- or 256-column tiles, which
      // hold whole heads; N = 3 Dq is a multiple of 128.
#pragma unroll 1
      for (int hg = 0; hg < BN / 128; ++hg) {
        const int col0 = nb * BN + hg * 128;
        if (col0 >= p.N) break;  // uniform over the warp
        qkv_rope_head(p, tbase + (uint32_t)(hg * 128), row, row_ok, col0);
      }
      return;
    }
  }
#pragma unroll 1
  for (int c = 0; c < BN / 32; ++c) {
    uint32_t r[32];
    __syncwarp();  // tcgen05.ld is .sync.aligned: reconverge after the masked stores
    tmem_ld_32x32b_x32(tbase + (uint32_t)(c * 32), r);
    tmem_wait_ld();
    const int col0 = nb * BN + c * 32;
    if (p.epi == (int)Epi::kScatter) {
      if (col0 < p.N) scatter_chunk(p, stg, r, row_base, col0, lane);
      continue;
    }
    if (!row_ok || col0 >= p.N) continue;
    float v[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
    add_bias32(p, col0, v);
    if (p.epi == (int)Epi::kStore) {
      store_row32(p, row, col0, v, (long long)split * p.split_stride);
    } else {
      // Interleaved pairs: columns [16j, 16j+16) are gates (SwiGLU) / values
      // (GEGLU) and [16j+16, 16j+32) the matching up / gate columns.
      float y[16];
      if (p.epi == (int)Epi::kSwiglu) {
#pragma unroll
        for (int j = 0; j < 16; j += 2) {
          const float2 y2 = fmul2(silu2(make_float2(v[j], v[j + 1])), make_float2(v[16 + j], v[17 + j]));
          y[j] = y2.x;
          y[j + 1] = y2.y;
        }
      } else {
#pragma unroll
        for (int j = 0; j < 16; ++j) y[j] = v[j] * gelu_erf_f(v[16 + j]);
      }
      store_row16(p, row, col0 / 2, y);
    }
  }
}

// Pixel tile nb of the implicit convolution -> image and top-left output pixel.
__device__ __forceinline__ void conv_tile(const ConvGeom& g, int nb, int& img, int& oy0, int& ox0) {
  const int tx = nb % g.tiles_x;
  const int r = nb / g.tiles_x;
  const int ty = r % g.tiles_y;
  img = r / g.tiles_y;
  oy0 = ty * g.BH;
  ox0 = tx * g.BW;
}

// Chan et al.'s pairwise update of (count, mean, sum of squared deviations).
__device__ __forceinline__ void chan_merge(float& N, float& mean, float& m2, float n2, float mean2, float m22) {
  if (n2 == 0.0f) return;
  if (N == 0.0f) {
    N = n2;
    mean = mean2;
    m2 = m22;
    return;
  }
  const float n = N + n2, d = mean2 - mean;
  mean += d * (n2 / n);
  m2 += m22 + d * d * (N * n2 / n);
  N = n;
}

// Epilogue of the implicit convolution for one warp: rows (output channels) row_base..+31,
// this thread's channel row_base + lane. Each 32-column chunk is 32 consecutive pixels of
// one output row (BW a multiple of 32), or of the flattened image when BW == Wo < 32. The
// warp's 32 x 32 block goes through shared memory (stg, pitch kStgPitch) so that each
// store instruction writes four whole 128-byte channel-row segments instead of 32 lines
// one channel plane (Ho * Wo * 4 bytes) apart.
template <int BN>
__device__ __forceinline__ void epilogue_conv(const GemmParams& p, float* stg, uint32_t tbase, int row_base, int nb,
                                              int lane, int split = 0) {
  const ConvGeom& g = p.cv;
  int img, oy0, ox0;
  conv_tile(g, nb, img, oy0, ox0);
  const long long hw = (long long)g.Ho * g.Wo;
  const int co = row_base + lane;
  const float bias = (co < p.M && p.bias) ? __ldg(p.bias + co) : 0.0f;
  float* out = reinterpret_cast<float*>(p.C) + (long long)split * p.split_stride + (long long)img * g.img_stride;
  const float* res = g.res ? g.res + (long long)img * g.img_stride : nullptr;
  const int sub = lane >> 3, c4 = (lane & 7) * 4;
  const bool stats = g.gn_part != nullptr;
  float sN = 0.0f, sMean = 0.0f, sM2 = 0.0f;  // this lane's channel over the tile's pixels
#pragma unroll 1
  for (int c = 0; c < BN / 32; ++c) {
    const int j0 = c * 32;
    if (j0 >= g.BW * g.BH) break;  // uniform: columns past the pixel rectangle are unused
    long long pix0;
    int n;
    if (g.BW >= 32) {
      const int oy = oy0 + j0 / g.BW, ox = ox0 + j0 % g.BW;
      pix0 = (long long)oy * g.Wo + ox;
      n = (oy < g.Ho && ox < g.Wo) ? min(32, g.Wo - ox) : 0;
    } else {
      pix0 = (long long)oy0 * g.Wo + j0;
      n = (int)min((long long)min(32, g.BW * g.BH - j0), hw - pix0);
    }
    if (n <= 0) continue;  // uniform over the warp
    uint32_t r[32];
    __syncwarp();
    tmem_ld_32x32b_x32(tbase + (uint32_t)(c * 32), r);
    tmem_wait_ld();
    float* mine = stg + lane * kStgPitch;
#pragma unroll
    for (int j = 0; j < 32; j += 4)
      *reinterpret_cast<float4*>(mine + j) =
          make_float4(__uint_as_float(r[j]) + bias, __uint_as_float(r[j + 1]) + bias,
                      __uint_as_float(r[j + 2]) + bias, __uint_as_float(r[j + 3]) + bias);
    __syncwarp();
    const bool vec = n == 32 && p.vec_ok && (pix0 & 3) == 0;
    if (vec && res) {
      // All eight residual loads of this lane first (eight in flight instead of one per
      // store), then the stores. res may alias out: each element is loaded before this
      // lane stores it, and no other lane touches it; plain loads, not the .nc path.
      float4 a4[8];
#pragma unroll
      for (int r0 = 0; r0 < 32; r0 += 4) {
        const int ch = row_base + r0 + sub;
        a4[r0 / 4] = ch < p.M ? *reinterpret_cast<const float4*>(res + (long long)ch * hw + pix0 + c4)
                              : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
      }
#pragma unroll
      for (int r0 = 0; r0 < 32; r0 += 4) {
        const int rr = r0 + sub, ch = row_base + rr;
        if (ch >= p.M) continue;
        float4 o = *reinterpret_cast<const float4*>(stg + rr * kStgPitch + c4);
        const float4 a = a4[r0 / 4];
        o.x += a.x; o.y += a.y; o.z += a.z; o.w += a.w;
        *reinterpret_cast<float4*>(out + (long long)ch * hw + pix0 + c4) = o;
        if (stats) *reinterpret_cast<float4*>(stg + rr * kStgPitch + c4) = o;  // final values, for the statistics
      }
    } else {
#pragma unroll
      for (int r0 = 0; r0 < 32; r0 += 4) {
        const int rr = r0 + sub, ch = row_base + rr;
        if (ch >= p.M) continue;
        const long long off = (long long)ch * hw + pix0 + c4;
        float* src = stg + rr * kStgPitch + c4;
        if (vec) {
          *reinterpret_cast<float4*>(out + off) = *reinterpret_cast<const float4*>(src);
        } else {
#pragma unroll
          for (int e = 0; e < 4; ++e)
            if (c4 + e < n) {
              const float o = res ? src[e] + res[off + e] : src[e];
              out[off + e] = o;
              if (stats) src[e] = o;
            }
        }
      }
    }
    __syncwarp();
    if (stats) {
      // This lane's channel over the chunk's n pixels (two passes over registers), merged
      // into the tile's running statistics.
      float v[32];
#pragma unroll
      for (int j = 0; j < 32; j += 4) {
        const float4 t = *reinterpret_cast<const float4*>(mine + j);
        v[j] = t.x; v[j + 1] = t.y; v[j + 2] = t.z; v[j + 3] = t.w;
      }
      float s = 0.0f;
#pragma unroll
      for (int j = 0; j < 32; ++j) s += j < n ? v[j] : 0.0f;
      const float mc = s / (float)n;
      float q = 0.0f;
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        const float d = v[j] - mc;
        q += j < n ? d * d : 0.0f;
      }
      chan_merge(sN, sMean, sM2, (float)n, mc, q);
      __syncwarp();
    }
  }
  if (stats) {
    // The group's channels are consecutive lanes (gn_cg divides 32): combine them, and the
    // group's first lane writes the tile's partial.
    for (int off = 1; off < g.gn_cg; off <<= 1) {
      const float n2 = __shfl_xor_sync(0xffffffffu, sN, off);
      const float mean2 = __shfl_xor_sync(0xffffffffu, sMean, off);
      const float m22 = __shfl_xor_sync(0xffffffffu, sM2, off);
      chan_merge(sN, sMean, sM2, n2, mean2, m22);
    }
    if (co < p.M && lane % g.gn_cg == 0) {
      const int tile = nb - img * g.tiles_x * g.tiles_y;
      g.gn_part[((long long)img * g.gn_groups + co / g.gn_cg) * g.tiles_img + tile] = make_float4(sN, sMean, sM2, 0.0f);
    }
  }
}

template <int BN, bool TF32, bool CONV = false>
__global__ void __launch_bounds__(kThreads, 1)
    k_gemm_tc(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, const GemmParams p) {
  using C_ = Cfg<BN>;
  constexpr int STAGES = C_::STAGES;
  constexpr int ESZ = TF32 ? 4 : 2;
  constexpr int BK = 128 / ESZ;        // K elements per stage (one swizzle row)
  constexpr int KSTEPS = 4;            // MMAs per stage: 32 bytes of K each
  constexpr uint32_t IDESC = make_idesc(TF32 ? 2u : 1u, 0, 0, kBM, BN);

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * C_::A_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(sB + STAGES * C_::B_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* acc_full = empty + STAGES;   // [2]
  uint64_t* acc_empty = acc_full + 2;    // [2]
  uint64_t* drain = acc_empty + 2;       // [1] MMA completion before TMEM is freed
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  float* stg = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(full) + 256);  // scatter staging

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], 4);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, C_::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      uint32_t issued = 0;  // bit s: stage s has a load whose completion was not yet observed
      uint32_t last_par = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < p.num_tiles && ok; t += gridDim.x) {
        int mb, nb, tile, kb0, kb1, split;
        split_item(p, t, tile, kb0, kb1, split);
        tile_coords(tile, p.m_tiles, p.n_tiles, mb, nb);
        int img = 0, oy0 = 0, ox0 = 0;
        if constexpr (CONV) conv_tile(p.cv, nb, img, oy0, ox0);
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag, p.err, kErrWaitEmpty)) {
            ok = false;
            break;
          }
          if constexpr (CONV) {
            const int tap = kb / p.cv.cblocks, cb = kb - tap * p.cv.cblocks;
            const int ky = tap / p.cv.kw, kx = tap - ky * p.cv.kw;
            mbar_arrive_expect_tx(&full[stage], C_::A_BYTES + p.cv.b_bytes);
            tma_load_2d(sA + stage * C_::A_BYTES, &tmA, &full[stage], kb * BK, mb * kBM);
            tma_load_4d(sB + stage * C_::B_BYTES, &tmB, &full[stage], cb * 32, ox0 + kx - p.cv.pad,
                        oy0 + ky - p.cv.pad, img);
          } else {
            mbar_arrive_expect_tx(&full[stage], C_::STAGE_BYTES);
            tma_load_2d(sA + stage * C_::A_BYTES, &tmA, &full[stage], kb * BK, mb * kBM);
            tma_load_2d(sB + stage * C_::B_BYTES, &tmB, &full[stage], kb * BK, nb * BN);
          }
          issued |= 1u << stage;
          last_par = (last_par & ~(1u << stage)) | (phase << stage);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (!ok) {
        // Aborted: wait (bounded) for this CTA's loads still in flight before exiting.
        for (int s = 0; s < STAGES; ++s)
          if (issued & (1u << s)) {
            const uint64_t t0 = globaltimer_ns();
            while (!mbar_try_wait(&full[s], (last_par >> s) & 1u))
              if (globaltimer_ns() - t0 > kWaitLimitNs) {
                atomicOr(p.err, kErrWaitDrain);
                break;
              }
          }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < p.num_tiles && ok; t += gridDim.x) {
        if (!mbar_wait(&acc_empty[acc], acc_phase ^ 1u, abort_flag, p.err, kErrWaitAccEmpty)) break;
        tc_fence_after();
        const uint32_t d = tmem_base + (uint32_t)(acc * BN);
        int tile, kb0, kb1, split;
        split_item(p, t, tile, kb0, kb1, split);
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&full[stage], phase, abort_flag, p.err, kErrWaitFull)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a0 = smem_u32(sA + stage * C_::A_BYTES);
          const uint32_t b0 = smem_u32(sB + stage * C_::B_BYTES);
#pragma unroll
          for (int k = 0; k < KSTEPS; ++k) {
            const uint64_t ad = sdesc_k_sw128(a0 + k * 32);
            const uint64_t bd = sdesc_k_sw128(b0 + k * 32);
            if (TF32)
              umma_tf32_ss(d, ad, bd, IDESC, (kb != kb0 || k != 0) ? 1u : 0u);
            else
              umma_f16_ss(d, ad, bd, IDESC, (kb != kb0 || k != 0) ? 1u : 0u);
          }
          umma_commit(&empty[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        umma_commit(&acc_full[acc]);
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1u;
      }
      // Every MMA this thread issued must have completed before TMEM is freed. In the
      // normal path the epilogue already observed the last tile's commit; after an
      // abort, wait (bounded) for a final commit.
      umma_commit(drain);
      const uint64_t t0 = globaltimer_ns();
      while (!mbar_try_wait(drain, 0))
        if (globaltimer_ns() - t0 > kWaitLimitNs) {
          atomicOr(p.err, kErrWaitDrain);
          break;
        }
    }
  } else {
    // ---------------- epilogue (warps 2..5) ----------------
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int t = blockIdx.x; t < p.num_tiles; t += gridDim.x) {
      int mb, nb, tile, kb0, kb1, split;
      split_item(p, t, tile, kb0, kb1, split);
      tile_coords(tile, p.m_tiles, p.n_tiles, mb, nb);
      if (!mbar_wait(&acc_full[acc], acc_phase, abort_flag, p.err, kErrWaitAccFull)) break;
      tc_fence_after();
      const uint32_t tbase = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * BN);
      if constexpr (CONV)
        epilogue_conv<BN>(p, stg + q * (32 * kStgPitch), tbase, mb * kBM + q * 32, nb, lane, split);
      else
        epilogue_tile<BN>(p, stg + q * (32 * kStgPitch), tbase, mb * kBM + q * 32, nb, lane, split);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[acc]);
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1u;
    }
    // Stores into peers' memory are visible system-wide before this kernel completes.
    if (p.epi == (int)Epi::kScatter) __threadfence_system();
  }

  // Teardown: all roles are done; the MMA thread has seen its final commit.
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();  // lane 0 ran the MMA loop alone; dealloc is .sync.aligned
    tc_fence_after();
    tmem_dealloc(tmem_base, C_::TMEM_COLS);
  }
}

// ------------------------------------------------------------------------------------
// Pair kernel: a cluster of two CTAs (on two SMs of one TPC) computes 256 x 256 tiles
// with M = 256 tcgen05 MMAs (.cta_group::2) issued by the leader (cluster rank 0). Each
// CTA stages its own 128 rows of A and its own 128 rows (half) of B, so the pair reads
// each operand tile once per 256 x 256 outputs instead of twice per two 128 x 256 tiles
// (a third less L2 -> shared memory traffic per FLOP), and each CTA's TMEM holds its 128
// rows of the accumulator (double-buffered, 2 x 256 columns). Both CTAs' loads complete
// on the leader's "full" barrier; the leader's MMA commits arrive on both CTAs' "empty" /
// accumulator barriers (tcgen05.commit multicast); both CTAs' epilogue warps release the
// leader's accumulator barrier. No load uses cluster multicast. bf16 operands only.
struct PairCfg {
  static constexpr int BN = 256;
  static constexpr int A_BYTES = kBM * 128;       // 128 rows x 64 bf16
  static constexpr int B_BYTES = (BN / 2) * 128;  // this CTA's half of the B tile
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int STAGES = 6;
  static constexpr uint32_t TMEM_COLS = 512;
  static constexpr int STG_BYTES = 4 * 32 * kStgPitch * 4;
  static constexpr int SMEM = STAGES * STAGE_BYTES + 1024 + 256 + STG_BYTES;
};

template <bool CONV>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
    k_gemm_tc_pair(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const GemmParams p) {
  using C_ = PairCfg;
  constexpr int BN = C_::BN;
  constexpr int STAGES = C_::STAGES;
  constexpr int BK = CONV ? 32 : 64;  // one 128-byte swizzle row of K: tf32 (conv) or bf16
  constexpr int KSTEPS = 4;
  constexpr uint32_t IDESC = make_idesc(CONV ? 2u : 1u, 0, 0, 2 * kBM, BN);

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = sA + STAGES * C_::A_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(sB + STAGES * C_::B_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* acc_full = empty + STAGES;  // [2]
  uint64_t* acc_empty = acc_full + 2;   // [2] (the leader's are the ones used)
  uint64_t* drain = acc_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  float* stg = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(full) + 256);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const int cluster = (int)(blockIdx.x >> 1), nclusters = (int)(gridDim.x >> 1);

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], 8);  // 4 epilogue warps in each CTA
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, C_::TMEM_COLS);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();  // both CTAs' barriers exist before any signal crosses the pair
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ---------------- TMA producer (both CTAs) ----------------
    if (lane == 0) {
      const uint32_t full0 = mapa_shared(&full[0], 0);  // the leader's barriers
      int stage = 0;
      uint32_t phase = 0;
      uint32_t issued = 0, last_par = 0;
      bool ok = true;
      for (int t = cluster; t < p.num_tiles && ok; t += nclusters) {
        int mb, nb;
        tile_coords(t, p.m_tiles, p.n_tiles, mb, nb);
        int img = 0, oy0 = 0, ox0 = 0;
        if constexpr (CONV) {
          conv_tile(p.cv, nb, img, oy0, ox0);
          oy0 += (int)rank * p.cv.half_dy;  // this CTA's half of the pixel rectangle
          ox0 += (int)rank * p.cv.half_dx;
        }
        for (int kb = 0; kb < p.k_blocks; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag, p.err, kErrWaitEmpty)) {
            ok = false;
            break;
          }
          const uint32_t fb = full0 + (uint32_t)(stage * 8);
          if constexpr (CONV) {
            const int tap = kb / p.cv.cblocks, cb = kb - tap * p.cv.cblocks;
            const int ky = tap / p.cv.kw, kx = tap - ky * p.cv.kw;
            if (rank == 0) mbar_arrive_expect_tx(&full[stage], 2 * (C_::A_BYTES + p.cv.b_bytes));
            tma_load_2d_pair(sA + stage * C_::A_BYTES, &tmA, fb, kb * BK, mb * 2 * kBM + (int)rank * kBM);
            tma_load_4d_pair(sB + stage * C_::B_BYTES, &tmB, fb, cb * 32, ox0 + kx - p.cv.pad, oy0 + ky - p.cv.pad,
                             img);
          } else {
            if (rank == 0) mbar_arrive_expect_tx(&full[stage], 2 * C_::STAGE_BYTES);
            tma_load_2d_pair(sA + stage * C_::A_BYTES, &tmA, fb, kb * BK, mb * 2 * kBM + (int)rank * kBM);
            tma_load_2d_pair(sB + stage * C_::B_BYTES, &tmB, fb, kb * BK, nb * BN + (int)rank * (BN / 2));
          }
          issued |= 1u << stage;
          last_par = (last_par & ~(1u << stage)) | (phase << stage);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (!ok && rank == 0) {
        // Aborted: wait (bounded) for loads still in flight (both CTAs' complete here).
        for (int s = 0; s < STAGES; ++s)
          if (issued & (1u << s)) {
            const uint64_t t0 = globaltimer_ns();
            while (!mbar_try_wait(&full[s], (last_par >> s) & 1u))
              if (globaltimer_ns() - t0 > kWaitLimitNs) {
                atomicOr(p.err, kErrWaitDrain);
                break;
              }
          }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer (leader only) ----------------
    if (lane == 0 && rank == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int t = cluster; t < p.num_tiles && ok; t += nclusters) {
        if (!mbar_wait(&acc_empty[acc], acc_phase ^ 1u, abort_flag, p.err, kErrWaitAccEmpty)) break;
        tc_fence_after();
        const uint32_t d = tmem_base + (uint32_t)(acc * BN);
        for (int kb = 0; kb < p.k_blocks; ++kb) {
          if (!mbar_wait(&full[stage], phase, abort_flag, p.err, kErrWaitFull)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a0 = smem_u32(sA + stage * C_::A_BYTES);
          const uint32_t b0 = smem_u32(sB + stage * C_::B_BYTES);
#pragma unroll
          for (int k = 0; k < KSTEPS; ++k) {
            if constexpr (CONV)
              umma_tf32_ss_pair(d, sdesc_k_sw128(a0 + k * 32), sdesc_k_sw128(b0 + k * 32), IDESC, (kb | k) != 0);
            else
              umma_f16_ss_pair(d, sdesc_k_sw128(a0 + k * 32), sdesc_k_sw128(b0 + k * 32), IDESC, (kb | k) != 0);
          }
          umma_commit_pair(&empty[stage], 0x3);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        umma_commit_pair(&acc_full[acc], 0x3);
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1u;
      }
      umma_commit_pair(drain, 0x3);
    }
    if (lane == 0) {
      // Both CTAs: every pair MMA has completed before TMEM and shared memory go away.
      const uint64_t t0 = globaltimer_ns();
      while (!mbar_try_wait(drain, 0))
        if (globaltimer_ns() - t0 > kWaitLimitNs) {
          atomicOr(p.err, kErrWaitDrain);
          break;
        }
    }
  } else {
    // ---------------- epilogue (warps 2..5, both CTAs) ----------------
    const int q = warp & 3;
    const uint32_t acc_empty0 = mapa_shared(&acc_empty[0], 0);
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int t = cluster; t < p.num_tiles; t += nclusters) {
      int mb, nb;
      tile_coords(t, p.m_tiles, p.n_tiles, mb, nb);
      if (!mbar_wait(&acc_full[acc], acc_phase, abort_flag, p.err, kErrWaitAccFull)) break;
      tc_fence_after();
      const uint32_t tbase = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * BN);
      if constexpr (CONV)
        epilogue_conv<BN>(p, stg + q * (32 * kStgPitch), tbase, mb * 2 * kBM + (int)rank * kBM + q * 32, nb, lane);
      else
        epilogue_tile<BN>(p, stg + q * (32 * kStgPitch), tbase, mb * 2 * kBM + (int)rank * kBM + q * 32, nb, lane);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(acc_empty0 + (uint32_t)(acc * 8));
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1u;
    }
    if (p.epi == (int)Epi::kScatter) __threadfence_system();
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync();  // both CTAs are done with TMEM, shared memory and each other's barriers
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, C_::TMEM_COLS);
  }
}

// Clusters of the pair kernel that fit on the device at once (cached per device).
int pair_clusters(int dev) {
  static int cached[64] = {};
  if (dev >= 0 && dev < 64 && cached[dev]) return cached[dev];
  check_cuda(cudaFuncSetAttribute(k_gemm_tc_pair<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, PairCfg::SMEM),
             "cudaFuncSetAttribute(gemm pair)");
  check_cuda(cudaFuncSetAttribute(k_gemm_tc_pair<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, PairCfg::SMEM),
             "cudaFuncSetAttribute(conv pair)");
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(2, 1, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = PairCfg::SMEM;
  cudaLaunchAttribute attr{};
  attr.id = cudaLaunchAttributeClusterDimension;
  attr.val.clusterDim.x = 2;
  attr.val.clusterDim.y = 1;
  attr.val.clusterDim.z = 1;
  cfg.attrs = &attr;
  cfg.numAttrs = 1;
  int n = 0;
  check_cuda(cudaOccupancyMaxActiveClusters(&n, k_gemm_tc_pair<false>, &cfg), "cudaOccupancyMaxActiveClusters");
  if (n <= 0) fail(kErrUnsupported, "gemm pair kernel: no cluster of 2 fits");
  if (dev >= 0 && dev < 64) cached[dev] = n;
  return n;
}

void launch_pair(const GemmCall& g, GemmParams p, int dev, cudaStream_t stream) {
  using C_ = PairCfg;
  CUtensorMap ta, tb;
  {
    const uint64_t dims[2] = {(uint64_t)g.K, (uint64_t)g.M};
    const uint64_t strides[1] = {(uint64_t)g.lda * 2};
    const uint32_t box[2] = {64, (uint32_t)kBM};
    encode_tmap(&ta, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, g.A, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
  }
  {
    const uint64_t dims[2] = {(uint64_t)g.K, (uint64_t)g.N};
    const uint64_t strides[1] = {(uint64_t)g.ldb * 2};
    const uint32_t box[2] = {64, (uint32_t)(C_::BN / 2)};
    encode_tmap(&tb, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, g.B, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
  }
  p.m_tiles = (int)((g.M + 2 * kBM - 1) / (2 * kBM));
  p.n_tiles = (int)((g.N + C_::BN - 1) / C_::BN);
  p.num_tiles = p.m_tiles * p.n_tiles;
  const int clusters = std::min(pair_clusters(dev), p.num_tiles);
  k_gemm_tc_pair<false><<<(unsigned)(2 * clusters), kThreads, C_::SMEM, stream>>>(ta, tb, p);
  check_launch("gemm_tc_pair");
}

template <int BN, bool TF32>
void launch_bn(const GemmCall& g, const GemmParams& p, int num_sms) {
  using C_ = Cfg<BN>;
  const int esz = TF32 ? 4 : 2;
  const uint32_t bk = 128 / esz;
  CUtensorMap ta, tb;
  const CUtensorMapDataType dt = TF32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  {
    const uint64_t dims[2] = {(uint64_t)g.K, (uint64_t)g.M};
    const uint64_t strides[1] = {(uint64_t)g.lda * esz};
    const uint32_t box[2] = {bk, (uint32_t)kBM};
    encode_tmap(&ta, dt, 2, g.A, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
  }
  {
    const uint64_t dims[2] = {(uint64_t)g.K, (uint64_t)g.N};
    const uint64_t strides[1] = {(uint64_t)g.ldb * esz};
    const uint32_t box[2] = {bk, (uint32_t)BN};
    encode_tmap(&tb, dt, 2, g.B, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
  }
  auto kern = k_gemm_tc<BN, TF32>;
  static bool attr_set[64] = {};
  const int dev = ctx().device;
  if (dev >= 0 && dev < 64 && !attr_set[dev]) {
    check_cuda(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C_::SMEM),
               "cudaFuncSetAttribute(gemm)");
    attr_set[dev] = true;
  }
  const int grid = std::min(p.num_tiles, num_sms);
  kern<<<grid, kThreads, C_::SMEM, ctx().stream>>>(ta, tb, p);
  check_launch("gemm_tc");
}

// Same launch with the device facts passed in instead of read from the device
// context, for callers that must not create one (the context allocates its error word).
template <int BN, bool TF32>
void launch_bn_explicit(const GemmCall& g, const GemmParams& p, int num_sms, cudaStream_t stream, int dev) {
  using C_ = Cfg<BN>;
  const int esz = TF32 ? 4 : 2;
  const uint32_t bk = 128 / esz;
  CUtensorMap ta, tb;
  const CUtensorMapDataType dt = TF32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  {
    const uint64_t dims[2] = {(uint64_t)g.K, (uint64_t)g.M};
    const uint64_t strides[1] = {(uint64_t)g.lda * esz};
    const uint32_t box[2] = {bk, (uint32_t)kBM};
    encode_tmap(&ta, dt, 2, g.A, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
  }
  {
    const uint64_t dims[2] = {(uint64_t)g.K, (uint64_t)g.N};
    const uint64_t strides[1] = {(uint64_t)g.ldb * esz};
    const uint32_t box[2] = {bk, (uint32_t)BN};
    encode_tmap(&tb, dt, 2, g.B, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
  }
  auto kern = k_gemm_tc<BN, TF32>;
  static bool attr_set[64] = {};
  if (dev >= 0 && dev < 64 && !attr_set[dev]) {
    check_cuda(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C_::SMEM),
               "cudaFuncSetAttribute(gemm)");
    attr_set[dev] = true;
  }
  const int grid = std::min(p.num_tiles, num_sms);
  kern<<<grid, kThreads, C_::SMEM, stream>>>(ta, tb, p);
  check_launch("gemm_tc");
}

// C[m, n] = sum over s < S of part[s][m][n] (+ bias[n]) (+ C[m, n] when acc): the
// reduction of a split-K GEMM, partial tiles dense [S][M][N]; the sum runs in split order,
// so results are deterministic. Four columns per thread when N, ldc and C allow it.
__global__ void __launch_bounds__(256) k_split_k_sum(const float* __restrict__ part, int S, int64_t M, int64_t N,
                                                     float* __restrict__ C, int64_t ldc, const float* __restrict__ bias,
                                                     int acc, int vec) {
  const int64_t stride = M * N;
  const int64_t step = (int64_t)gridDim.x * blockDim.x;
  if (vec) {
    const int64_t n4 = N / 4;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < M * n4; i += step) {
      const int64_t m = i / n4, c = (i - m * n4) * 4;
      float4 t = *reinterpret_cast<const float4*>(part + m * N + c);
      for (int s = 1; s < S; ++s) {
        const float4 u = *reinterpret_cast<const float4*>(part + s * stride + m * N + c);
        t.x += u.x; t.y += u.y; t.z += u.z; t.w += u.w;
      }
      if (bias) {
        const float4 b = *reinterpret_cast<const float4*>(bias + c);
        t.x += b.x; t.y += b.y; t.z += b.z; t.w += b.w;
      }
      float4* d = reinterpret_cast<float4*>(C + m * ldc + c);
      if (acc) {
        const float4 o = *d;
        t.x += o.x; t.y += o.y; t.z += o.z; t.w += o.w;
      }
      *d = t;
    }
    return;
  }
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < M * N; i += step) {
    const int64_t m = i / N, c = i - m * N;
    float t = part[i];
    for (int s = 1; s < S; ++s) t += part[s * stride + i];
    if (bias) t += bias[c];
    float* d = C + m * ldc + c;
    *d = acc ? *d + t : t;
  }
}

int choose_bn(int64_t M, int64_t N, int num_sms, Epi epi) {
  // Every candidate BN is a multiple of the 32-column gated chunk; the QKV epilogue
  // needs whole 128-column heads per tile.
  const int cands[4] = {256, 192, 128, 64};
  int best = 256;
  double best_cost = 1e30;
  const int64_t m_tiles = (M + kBM - 1) / kBM;
  for (int bn : cands) {
    if (epi == Epi::kQkvRope && bn % 128 != 0) continue;
    const int64_t tiles = m_tiles * ((N + bn - 1) / bn);
    const int64_t waves = (tiles + num_sms - 1) / num_sms;
    // Per-tile time grows with BN; 48 columns of fixed cost model the lower
    // efficiency of narrow tiles (more A traffic per FLOP, more epilogue overhead).
    const double cost = (double)waves * (bn + 48);
    if (cost < best_cost - 1e-9) {
      best_cost = cost;
      best = bn;
    }
  }
  return best;
}

}  // namespace



// Tile-width override for tuning and tests (0 = automatic choice).
static int g_forced_bn = 0;
void set_gemm_tile(int bn) { g_forced_bn = bn; }

// 256 x 256 tiles on CTA pairs (k_gemm_tc_pair) for bf16 GEMMs with 256-column
// tiles and for implicit-GEMM convolutions with >= 256 output channels.
// Mode 0: never; 1: when the cost model prefers them (default); 2: whenever eligible.
static int g_gemm_pair = 1;
void set_gemm_pair(int mode) { g_gemm_pair = mode; }

void launch_gemm_tc(const GemmCall& g) {
  DeviceContext& c = ctx();
  GemmParams p{};
  p.M = (int)g.M;
  p.N = (int)g.N;
  p.K = (int)g.K;
  int bn = g.bn ? g.bn : g_forced_bn ? g_forced_bn : choose_bn(g.M, g.N, c.num_sms, g.epi);
  if (g.epi == Epi::kQkvRope) {
    if (!g.rope || g.tf32 || g.N % 128 != 0 || g.N != 3 * (int64_t)g.rope->Dq)
      fail(kErrInvalidArg, "gemm_tc: QKV epilogue needs bf16 operands and N = 3 * Dq, Dq % 128 == 0");
    if (bn % 128 != 0) bn = choose_bn(g.M, g.N, c.num_sms, g.epi);
  }
  if (g.epi == Epi::kScatter) {
    if (!g.scatter || g.scatter->rs <= 0 || g.accumulate || g.out_bf16 || g.ldc % 4 != 0)
      fail(kErrInvalidArg, "gemm_tc: scatter epilogue needs fp32 rows of 16-byte pitch and no accumulate");
    for (int64_t o = 0; o * g.scatter->rs < g.M; ++o)
      if (o >= 8 || !g.scatter->base[o] || (reinterpret_cast<uintptr_t>(g.scatter->base[o]) & 15))
        fail(kErrInvalidArg, "gemm_tc: scatter epilogue: missing or misaligned owner slot");
  }
  p.m_tiles = (int)((g.M + kBM - 1) / kBM);
  p.n_tiles = (int)((g.N + bn - 1) / bn);
  p.num_tiles = p.m_tiles * p.n_tiles;
  const int bk = g.tf32 ? 32 : 64;
  p.k_blocks = (int)((g.K + bk - 1) / bk);
  p.C = g.C;
  p.ldc = g.ldc;
  p.bias = g.bias;
  p.bias_vec = g.bias && (reinterpret_cast<uintptr_t>(g.bias) & 15) == 0;
  p.accumulate = g.accumulate ? 1 : 0;
  p.epi = (int)g.epi;
  p.out_bf16 = g.out_bf16 ? 1 : 0;
  const int oesz = g.out_bf16 ? 2 : 4;
  p.vec_ok = ((reinterpret_cast<uintptr_t>(g.C) & 15) == 0) && ((g.ldc * oesz) % 16 == 0);
  p.err = c.err_word;
  if (g.rope) p.rope = *g.rope;
  if (g.scatter) p.sc = *g.scatter;
  if (!g.tf32 && g_gemm_pair && g.M >= 2 * kBM && (bn == 256 || (!g.bn && !g_forced_bn))) {
    // Same wave-count cost model as choose_bn; a pair tile (256 x 256 over two SMs)
    // costs one 128 x 256 tile-time at about 8% better efficiency (measured on the DiT
    // shapes), so narrow single-SM tiles win only where they fill the last wave better.
    const int64_t single_tiles = ((g.M + kBM - 1) / kBM) * ((g.N + bn - 1) / bn);
    const double single_cost = (double)((single_tiles + c.num_sms - 1) / c.num_sms) * (bn + 48);
    const int64_t pair_tiles = ((g.M + 2 * kBM - 1) / (2 * kBM)) * ((g.N + 255) / 256);
    const int64_t clusters = pair_clusters(c.device);
    const double pair_cost = (double)((pair_tiles + clusters - 1) / clusters) * (256 + 48) * 0.92;
    if (pair_cost <= single_cost || g_gemm_pair == 2) {
      launch_pair(g, p, c.device, c.stream);
      return;
    }
  }
  // Split-K for few-tile, long-K plain GEMMs (M of a few hundred rows against large
  // weights: the context refiner and caption embedder at one image, the reference's
  // linear() on short sequences). A single pass would leave most SMs idle while the rest
  // stream the weights; instead each K split of each 128 x 256 tile runs on its own SM and
  // a reduction kernel adds the partial tiles in split order with the bias.
  // Taken when the 128 x 256 tiles fill at most half of the SMs and K has at least 16
  // blocks; every split keeps at least 4 K blocks.
  const int sbn = 256;
  const int64_t tiles256 = (int64_t)p.m_tiles * ((g.N + sbn - 1) / sbn);
  if (g.epi == Epi::kStore && !g.out_bf16 && !g.bn && !g_forced_bn && p.k_blocks >= 16 && tiles256 * 2 <= c.num_sms) {
    const int64_t want = std::min<int64_t>(c.num_sms / tiles256, p.k_blocks / 4);
    if (want >= 2) {
      const int kb_split = (int)((p.k_blocks + want - 1) / want);
      const int splits = (p.k_blocks + kb_split - 1) / kb_split;
      const size_t part_bytes = (size_t)splits * (size_t)(g.M * g.N) * 4;
      float* part = static_cast<float*>(split_workspace(part_bytes));
      GemmCall gs = g;
      gs.C = part;
      gs.ldc = g.N;
      gs.bias = nullptr;
      gs.accumulate = false;
      GemmParams ps = p;
      ps.n_tiles = (int)((g.N + sbn - 1) / sbn);
      ps.base_tiles = ps.m_tiles * ps.n_tiles;
      ps.splits = splits;
      ps.kb_split = kb_split;
      ps.num_tiles = ps.base_tiles * splits;
      ps.split_stride = (long long)(g.M * g.N);
      ps.C = part;
      ps.ldc = g.N;
      ps.bias = nullptr;
      ps.accumulate = 0;
      ps.vec_ok = (g.N % 4) == 0;
      if (g.tf32)
        launch_bn<256, true>(gs, ps, c.num_sms);
      else
        launch_bn<256, false>(gs, ps, c.num_sms);
      const bool vec = (g.N % 4 == 0) && (g.ldc % 4 == 0) && ((reinterpret_cast<uintptr_t>(g.C) & 15) == 0) &&
                       (!g.bias || (reinterpret_cast<uintptr_t>(g.bias) & 15) == 0);
      const int64_t work = vec ? g.M * (g.N / 4) : g.M * g.N;
      const int64_t blocks = std::max<int64_t>(1, std::min<int64_t>((work + 255) / 256, (int64_t)c.num_sms * 8));
      k_split_k_sum<<<(unsigned)blocks, 256, 0, c.stream>>>(part, splits, g.M, g.N, static_cast<float*>(g.C), g.ldc,
                                                            g.bias, g.accumulate ? 1 : 0, vec ? 1 : 0);
      check_launch("gemm split-K reduction");
      return;
    }
  }
  if (g.tf32) {
    switch (bn) {
      case 256: launch_bn<256, true>(g, p, c.num_sms); break;
      case 192: launch_bn<192, true>(g, p, c.num_sms); break;
      case 128: launch_bn<128, true>(g, p, c.num_sms); break;
      default: launch_bn<64, true>(g, p, c.num_sms); break;
    }
  } else {
    switch (bn) {
      case 256: launch_bn<256, false>(g, p, c.num_sms); break;
      case 192: launch_bn<192, false>(g, p, c.num_sms); break;
      case 128: launch_bn<128, false>(g, p, c.num_sms); break;
      default: launch_bn<64, false>(g, p, c.num_sms); break;
    }
  }
}


namespace {
template <int BN>
void launch_conv_bn(const CUtensorMap& ta, const CUtensorMap& tb, const GemmParams& p, int num_sms, int dev,
                    cudaStream_t stream) {
  using C_ = Cfg<BN>;
  auto kern = k_gemm_tc<BN, true, true>;
  static bool attr_set[64] = {};
  if (dev >= 0 && dev < 64 && !attr_set[dev]) {
    check_cuda(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C_::SMEM),
               "cudaFuncSetAttribute(conv)");
    attr_set[dev] = true;
  }
  const int grid = std::min(p.num_tiles, num_sms);
  kern<<<grid, kThreads, C_::SMEM, stream>>>(ta, tb, p);
  check_launch("conv_tc");
}

// Pixel rectangle of a BN-column tile: BW a power of two >= 32 (or the whole row when
// Wo < 32), BH rows, never more rows than the image has.
void conv_rect(int bn, int64_t Ho, int64_t Wo, int& bw, int& bh) {
  if (Wo >= 32) {
    bw = 32;
    while (bw < Wo && bw < bn) bw *= 2;
    bh = bn / bw;
  } else {
    bw = (int)Wo;
    bh = std::min(bn / (int)Wo, 256);
  }
  bh = (int)std::min<int64_t>(bh, Ho);
}
}  // namespace

void launch_conv_tc(const float* xh, int64_t N, int64_t Cin, int64_t cp, int64_t H, int64_t W, const float* wp,
                    int64_t cq, int64_t Cout, int kh, int kw, int pad, const float* bias, const float* res, float* out,
                    int64_t Ho, int64_t Wo, ConvStats* stats) {
  DeviceContext& c = ctx();
  if (stats) {
    const int cg = stats->groups > 0 ? (int)(Cout / stats->groups) : 0;
    if (cg <= 0 || Cout % stats->groups != 0 || 32 % cg != 0 || Cout % 32 != 0)
      fail(kErrInvalidArg, "conv_tc: GroupNorm statistics need groups of a divisor of 32 channels and Cout % 32 == 0");
  }
  if (cp % 4 != 0 || cq % 32 != 0 || cq < Cin || cp < Cin || N <= 0 || Ho <= 0 || Wo <= 0)
    fail(kErrInvalidArg, "conv_tc: bad packed layout");
  if (Cout > (1 << 30) || Ho * Wo > (1ll << 31) || N > 65535)
    fail(kErrInvalidArg, "conv_tc: shape too large");
  // A few output channels would fill a few of a tile's 128 MMA rows: direct kernel instead.
  if (!stats && Cout <= 8 && kh == kw && kh <= 15 && (Ho + 31) / 32 <= 65535 && H * W < (1ll << 31))
    return launch_conv_direct(xh, N, Cin, cp, H, W, wp, cq, Cout, kh, pad, bias, res, out, Ho, Wo);
  // Tile width by the wave-count cost model of choose_bn over the pixel rectangles.
  const int64_t m_tiles = (Cout + kBM - 1) / kBM;
  int bn = 256, bw = 0, bh = 0;
  double best = 1e30;
  for (int cand : {256, 128, 64}) {
    int w_, h_;
    conv_rect(cand, Ho, Wo, w_, h_);
    const int64_t tiles = m_tiles * N * ((Ho + h_ - 1) / h_) * ((Wo + w_ - 1) / w_);
    const double cost = (double)((tiles + c.num_sms - 1) / c.num_sms) * (cand + 48);
    if (cost < best - 1e-9) {
      best = cost;
      bn = cand;
      bw = w_;
      bh = h_;
    }
  }
  const bool forced = g_forced_bn == 256 || g_forced_bn == 128 || g_forced_bn == 64;
  if (forced) {
    bn = g_forced_bn;
    conv_rect(bn, Ho, Wo, bw, bh);
  }
  // SM pairs (k_gemm_tc_pair<true>): 256 channels x 256 pixels per pair, each CTA loading
  // 128 channels of the weights and half of the pixel rectangle; same cost model as the
  // GEMM's pair choice. Needs a full 256-pixel rectangle that splits into two halves.
  bool pair = false;
  int pw = 0, ph = 0;
  if (g_gemm_pair && !forced && Cout >= 2 * kBM) {
    conv_rect(256, Ho, Wo, pw, ph);
    if (pw * ph == 256 && (ph % 2 == 0 || pw == 256)) {
      const int64_t pair_tiles = ((Cout + 2 * kBM - 1) / (2 * kBM)) * N * ((Ho + ph - 1) / ph) * ((Wo + pw - 1) / pw);
      const int64_t clusters = pair_clusters(c.device);
      const double pair_cost = (double)((pair_tiles + clusters - 1) / clusters) * (256 + 48) * 0.92;
      pair = pair_cost <= best || g_gemm_pair == 2;
    }
  }
  if (pair) {
    bn = 256;
    bw = pw;
    bh = ph;
  }
  const int64_t kk = (int64_t)kh * kw * cq;
  // Split-K for outputs with fewer tiles than SMs and a long K (the UNet's 1280-channel 3x3
  // convolutions at 16 x 16 and 8 x 8 pixels, K up to 23040): the splits' partial outputs
  // go to a workspace and one pass adds them with the bias and residual. With few tiles each
  // SM is bound by its L2 -> SM load rate, about 64 bytes per clock: a K block (32 channels)
  // of a 128 x BN tile loads (128 + BN) x 128 bytes, so t_kb = 2 (128 + BN) clocks (a
  // 256 x 256 pair tile: 512 per SM). Cost of a choice = waves x K blocks per item x t_kb,
  // plus the reduction: (2 splits + 2) x the output's bytes at about 3400 bytes per clock and
  // a fixed 6000 clocks (the extra launch). The split is taken when it beats the plain
  // choice by 20%; the tile width is then chosen with it (kept when the width is forced).
  int splits = 1;
  {
    const int64_t kb = kk / 32;
    int w0, h0;
    conv_rect(bn, Ho, Wo, w0, h0);
    const int64_t tiles0 = pair ? ((Cout + 2 * kBM - 1) / (2 * kBM)) * N * ((Ho + h0 - 1) / h0) * ((Wo + w0 - 1) / w0)
                                : m_tiles * N * ((Ho + h0 - 1) / h0) * ((Wo + w0 - 1) / w0);
    const int64_t units0 = pair ? pair_clusters(c.device) : c.num_sms;
    if (!stats && !(pair && g_gemm_pair == 2) && tiles0 < units0 && kb >= 32) {
      const double out_bytes = (double)N * Cout * Ho * Wo * 4.0;
      const double base = (double)((tiles0 + units0 - 1) / units0) * (double)kb * (pair ? 512.0 : 2.0 * (128 + bn));
      double best_split = 0.8 * base;
      for (int cand : {256, 128, 64}) {
        if (forced && cand != bn) continue;
        int w_, h_;
        conv_rect(cand, Ho, Wo, w_, h_);
        const int64_t tiles = m_tiles * N * ((Ho + h_ - 1) / h_) * ((Wo + w_ - 1) / w_);
        for (int s = 2; s <= 16 && s * 8 <= kb; ++s) {
          const int64_t kbs = (kb + s - 1) / s;
          const int64_t used = (kb + kbs - 1) / kbs;
          const double cost = (double)((tiles * used + c.num_sms - 1) / c.num_sms) * (double)kbs * 2.0 * (128 + cand) +
                              (2.0 * used + 2.0) * out_bytes / 3400.0 + 6000.0;
          if (cost < best_split) {
            best_split = cost;
            splits = s;
            bn = cand;
            bw = w_;
            bh = h_;
          }
        }
      }
      if (splits > 1) pair = false;
    }
  }
  CUtensorMap ta, tb;
  {
    const uint64_t dims[2] = {(uint64_t)kk, (uint64_t)Cout};
    const uint64_t strides[1] = {(uint64_t)kk * 4};
    const uint32_t box[2] = {32, (uint32_t)kBM};
    encode_tmap(&ta, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, wp, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
  }
  // On SM pairs each CTA loads half of the rectangle: the top / bottom rows, or the left /
  // right half of a one-row rectangle.
  const int hx = (pair && bh == 1) ? bw / 2 : 0, hy = (pair && bh > 1) ? bh / 2 : 0;
  const int box_w = hx ? bw / 2 : bw, box_h = hy ? bh / 2 : bh;
  {
    const uint64_t dims[4] = {(uint64_t)Cin, (uint64_t)W, (uint64_t)H, (uint64_t)N};
    const uint64_t strides[3] = {(uint64_t)cp * 4, (uint64_t)(W * cp * 4), (uint64_t)(H * W * cp * 4)};
    const uint32_t box[4] = {32, (uint32_t)box_w, (uint32_t)box_h, 1};
    encode_tmap(&tb, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, xh, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
  }
  GemmParams p{};
  p.M = (int)Cout;
  p.N = bw * bh;  // columns used per tile (informational; the conv epilogue masks by geometry)
  p.K = (int)kk;
  p.cv.Ho = (int)Ho;
  p.cv.Wo = (int)Wo;
  p.cv.BW = bw;
  p.cv.BH = bh;
  p.cv.tiles_x = (int)((Wo + bw - 1) / bw);
  p.cv.tiles_y = (int)((Ho + bh - 1) / bh);
  p.cv.kw = kw;
  p.cv.pad = pad;
  p.cv.cblocks = (int)(cq / 32);
  p.cv.b_bytes = box_w * box_h * 128;
  p.cv.half_dx = hx;
  p.cv.half_dy = hy;
  p.cv.img_stride = Cout * Ho * Wo;
  p.cv.res = res;
  if (stats) {
    const int64_t tiles_img = (int64_t)p.cv.tiles_x * p.cv.tiles_y;
    if (N * stats->groups * tiles_img > stats->cap) fail(kErrInvalidArg, "conv_tc: statistics buffer too small");
    p.cv.gn_part = stats->part;
    p.cv.gn_groups = stats->groups;
    p.cv.gn_cg = (int)(Cout / stats->groups);
    p.cv.tiles_img = (int)tiles_img;
    stats->tiles_img = tiles_img;
  }
  p.m_tiles = pair ? (int)((Cout + 2 * kBM - 1) / (2 * kBM)) : (int)m_tiles;
  p.n_tiles = (int)(N * p.cv.tiles_x * p.cv.tiles_y);
  if ((int64_t)p.m_tiles * p.n_tiles > (1ll << 31) - 1) fail(kErrInvalidArg, "conv_tc: too many tiles");
  p.num_tiles = p.m_tiles * p.n_tiles;
  p.k_blocks = (int)(kk / 32);
  p.C = out;
  p.ldc = Ho * Wo;
  p.bias = bias;
  p.epi = (int)Epi::kStore;
  const bool al = (reinterpret_cast<uintptr_t>(out) & 15) == 0 &&
                  (!res || (reinterpret_cast<uintptr_t>(res) & 15) == 0);
  p.vec_ok = al && (Ho * Wo) % 4 == 0;
  p.err = c.err_word;
  if (pair) {
    const int clusters = std::min(pair_clusters(c.device), p.num_tiles);
    k_gemm_tc_pair<true><<<(unsigned)(2 * clusters), kThreads, PairCfg::SMEM, c.stream>>>(ta, tb, p);
    check_launch("conv_tc_pair");
    return;
  }
  // Split-K as chosen above.
  float* part = nullptr;
  if (splits > 1) {
    const int want = splits;
    {
      const int kb_split = (p.k_blocks + want - 1) / want;
      const int used = (p.k_blocks + kb_split - 1) / kb_split;
      const long long total = N * Cout * Ho * Wo;
      part = static_cast<float*>(pool_malloc((size_t)(used * total) * sizeof(float)));
      p.splits = used;
      p.base_tiles = p.num_tiles;
      p.kb_split = kb_split;
      p.split_stride = total;
      p.num_tiles = p.num_tiles * used;
      p.C = part;
      p.bias = nullptr;
      p.cv.res = nullptr;
      p.vec_ok = (Ho * Wo) % 4 == 0;
    }
  }
  switch (bn) {
    case 256: launch_conv_bn<256>(ta, tb, p, c.num_sms, c.device, c.stream); break;
    case 128: launch_conv_bn<128>(ta, tb, p, c.num_sms, c.device, c.stream); break;
    default: launch_conv_bn<64>(ta, tb, p, c.num_sms, c.device, c.stream); break;
  }
  if (part) {
    launch_split_reduce(part, p.splits, N * Cout * Ho * Wo, Cout, Ho * Wo, bias, res, out);
    pool_free(part);  // stream-ordered reuse
  }
}

// bf16 GEMM launch on an explicit device / stream / error word (no device context).
void launch_gemm_tc_explicit(const GemmCall& g, int num_sms, cudaStream_t stream, int* err_word, int dev) {
  GemmParams p{};
  p.M = (int)g.M;
  p.N = (int)g.N;
  p.K = (int)g.K;
  if (g.epi == Epi::kQkvRope || g.epi == Epi::kScatter)
    fail(kErrInvalidArg, "gemm_tc: the QKV and scatter epilogues need a device context");
  const int bn = g.bn ? g.bn : choose_bn(g.M, g.N, num_sms, g.epi);
  p.m_tiles = (int)((g.M + kBM - 1) / kBM);
  p.n_tiles = (int)((g.N + bn - 1) / bn);
  p.num_tiles = p.m_tiles * p.n_tiles;
  p.k_blocks = (int)((g.K + 63) / 64);
  p.C = g.C;
  p.ldc = g.ldc;
  p.bias = g.bias;
  p.bias_vec = g.bias && (reinterpret_cast<uintptr_t>(g.bias) & 15) == 0;
  p.accumulate = g.accumulate ? 1 : 0;
  p.epi = (int)g.epi;
  p.out_bf16 = g.out_bf16 ? 1 : 0;
  const int oesz = g.out_bf16 ? 2 : 4;
  p.vec_ok = ((reinterpret_cast<uintptr_t>(g.C) & 15) == 0) && ((g.ldc * oesz) % 16 == 0);
  p.err = err_word;
  switch (bn) {
    case 256: launch_bn_explicit<256, false>(g, p, num_sms, stream, dev); break;
    case 192: launch_bn_explicit<192, false>(g, p, num_sms, stream, dev); break;
    case 128: launch_bn_explicit<128, false>(g, p, num_sms, stream, dev); break;
    default: launch_bn_explicit<64, false>(g, p, num_sms, stream, dev); break;
  }
}

}  // namespace sdb
