// attention_tc.cu - flash attention on 5th-generation tensor cores (sm_100a):
// softmax(q k^T / sqrt(d)) v per head with grouped key/value heads and an optional
// causal mask, replacing the reference's score-matrix attention
// (backend_cuda.cu:550-586: two batched SGEMMs around a softmax, the full Sq x Skv
// matrix in HBM) and the CPU path it is checked against (tensor.cpp:771-810).
//
// One CTA owns 128 query rows of one (sample, head); 224 threads in four roles:
//   warp 0     TMA: Q once, then K and V tiles of 128 keys through separate 2-stage
//              rings (K is freed when QK^T is done, so it runs ahead of the PV chain)
//   warp 1     QK^T issuer: S_j = Q K_j^T into one of two TMEM score buffers
//              (ping-pong: the next tile's QK^T overlaps this tile's softmax)
//   warp 2     PV issuer: O += P_j V_j into a TMEM accumulator as soon as P_j and V_j
//              are ready; two issuer threads keep one role's wait from blocking the other
//   warps 3-6  softmax: one query row per thread (TMEM lane). Loads S_j, applies the
//              scale (in log2 units) and the masks, keeps the running max m and sum l,
//              writes P_j = 2^(s - m) as fp16 into a swizzled shared-memory tile for
//              the PV MMA, and at the end normalises O by 1/l and stores it.
// O is rescaled only when a row's max grows by more than 2^8 since the value used so
// far (P stays <= 256, fine for fp16 and fp32); the stale max cancels in O / l.
//
// Operands are fp16 (10-bit mantissa, as tf32), not bf16: with bf16 Q/K/V/P the result
// misses the 2e-3 relative-Frobenius parity gate (about 3e-3 at d = 128); with fp16 it
// lands near 5e-4. Inputs are packed to fp16 [N, S, heads, dp] (dp = 64 or 128, zero
// padded) by the caller; |x| > 65504 saturates.
#include <cuda_fp16.h>

#include <algorithm>
#include <cmath>

#include "internal.h"
#include "ptx.cuh"

namespace sdb {
namespace {

constexpr int kBQ = 128;
constexpr int kBK = 128;
constexpr int kThreads = 224;  // TMA, QK^T issuer, PV issuer, 4 softmax warps
constexpr float kRescaleThreshold = 8.0f;  // log2 units

struct AttnParams {
  int N, Sq, Skv, heads, kv_heads, d, dp, causal;
  float scale_log2;
  void* out;
  long long out_row;    // elements between consecutive query rows of one sample
  long long out_batch;  // elements between samples
  int out_bf16;
  int* err;
};

template <int DP>
struct ACfg {
  static constexpr int ATOM = kBQ * 128;  // one 128-byte-wide swizzle atom of 128 rows
  static constexpr int ATOMS = DP / 64;
  static constexpr int Q_BYTES = ATOMS * ATOM;
  static constexpr int KV_BYTES = ATOMS * ATOM;  // one K or one V tile
  static constexpr int P_BYTES = 2 * ATOM;       // 128 x 128 fp16
  static constexpr int SMEM = Q_BYTES + 2 * 2 * KV_BYTES + 2 * P_BYTES + 1024 + 256;  // Q | K[2] | V[2] | P[2]
  static constexpr uint32_t TMEM_COLS = 512;     // S0 | S1 | O
  static constexpr uint32_t O_COL = 256;
};

// 2^x on the MUFU pipe (PTX ex2.approx.ftz.f32; 2^-inf = +0).
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ uint32_t pack_half2(float a, float b) {
  const __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<const uint32_t*>(&h);
}

template <int DP>
__global__ void __launch_bounds__(kThreads, 1)
    k_attention_tc(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                   const __grid_constant__ CUtensorMap tmV, const AttnParams p) {
  using C_ = ACfg<DP>;
  constexpr uint32_t IDESC_S = make_idesc(0u /*f16*/, 0, 0, kBQ, kBK);
  constexpr uint32_t IDESC_O = make_idesc(0u /*f16*/, 0, 1 /*V is MN-major*/, kBQ, DP);

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;
  uint8_t* sK = sQ + C_::Q_BYTES;          // [2 stages]
  uint8_t* sV = sK + 2 * C_::KV_BYTES;     // [2 stages]
  uint8_t* sP = sV + 2 * C_::KV_BYTES;     // [2 buffers]
  uint64_t* bars = reinterpret_cast<uint64_t*>(sP + 2 * C_::P_BYTES);
  uint64_t* q_full = bars + 0;
  uint64_t* k_full = bars + 1;     // [2]
  uint64_t* k_empty = bars + 3;    // [2]
  uint64_t* v_full = bars + 5;     // [2]
  uint64_t* v_empty = bars + 7;    // [2]
  uint64_t* s_full = bars + 9;     // [2]
  uint64_t* p_full = bars + 11;    // [2]
  uint64_t* p_free = bars + 13;    // [2]
  uint64_t* o_final = bars + 15;
  uint64_t* drain = bars + 16;     // [2] one per MMA thread
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 18);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int q0 = blockIdx.x * kBQ, h = blockIdx.y, n = blockIdx.z;
  const int kvh = h / (p.heads / p.kv_heads);
  int nkv = (p.Skv + kBK - 1) / kBK;
  if (p.causal) nkv = min(nkv, (q0 + kBQ - 1) / kBK + 1);

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1);
      mbar_init(&v_full[i], 1);
      mbar_init(&v_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], 4);
      mbar_init(&p_free[i], 1);
      mbar_init(&drain[i], 1);
    }
    mbar_init(o_final, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, C_::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ------------------------------ TMA producer ------------------------------
    // K_j and V_j have separate 2-stage rings: K_j is released as soon as S_j is
    // computed, V_j only after PV_j, so K loads run ahead of the PV chain.
    if (lane == 0) {
      mbar_arrive_expect_tx(q_full, C_::Q_BYTES);
      for (int a = 0; a < C_::ATOMS; ++a)
        tma_load_3d(sQ + a * C_::ATOM, &tmQ, q_full, h * p.dp + a * 64, q0, n);
      int k_issued = -1, v_issued = -1;
      bool ok = true;
      for (int j = 0; j < nkv && ok; ++j) {
        const int st = j & 1;
        const uint32_t par = ((j >> 1) & 1) ^ 1u;
        if (!mbar_wait(&k_empty[st], par, abort_flag, p.err, kErrAttnWait)) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(&k_full[st], C_::KV_BYTES);
        for (int a = 0; a < C_::ATOMS; ++a)
          tma_load_3d(sK + st * C_::KV_BYTES + a * C_::ATOM, &tmK, &k_full[st], kvh * p.dp + a * 64, j * kBK, n);
        k_issued = j;
        if (!mbar_wait(&v_empty[st], par, abort_flag, p.err, kErrAttnWait)) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(&v_full[st], C_::KV_BYTES);
        for (int a = 0; a < C_::ATOMS; ++a)
          tma_load_3d(sV + st * C_::KV_BYTES + a * C_::ATOM, &tmV, &v_full[st], kvh * p.dp + a * 64, j * kBK, n);
        v_issued = j;
      }
      if (!ok) {
        // Aborted: wait (bounded) for the loads this CTA still has in flight.
        const uint64_t t0 = globaltimer_ns();
        while (!mbar_try_wait(q_full, 0) && globaltimer_ns() - t0 < kWaitLimitNs) {
        }
        for (int j = max(0, k_issued - 1); j <= k_issued; ++j)
          while (!mbar_try_wait(&k_full[j & 1], (j >> 1) & 1) && globaltimer_ns() - t0 < kWaitLimitNs) {
          }
        for (int j = max(0, v_issued - 1); j <= v_issued; ++j)
          while (!mbar_try_wait(&v_full[j & 1], (j >> 1) & 1) && globaltimer_ns() - t0 < kWaitLimitNs) {
          }
      }
    }
  } else if (warp == 1) {
    // ------------------------------ QK^T issuer -------------------------------
    if (lane == 0) {
      bool ok = mbar_wait(q_full, 0, abort_flag, p.err, kErrAttnWait);
      tc_fence_after();
      const uint32_t q_addr = smem_u32(sQ);
      for (int j = 0; ok && j < nkv; ++j) {
        const int st = j & 1;
        // S buffer j&1 is free once the softmax has consumed S_{j-2} (it posted P_{j-2}).
        if (j >= 2 && !mbar_wait(&p_full[st], ((j - 2) >> 1) & 1, abort_flag, p.err, kErrAttnWait)) break;
        if (!mbar_wait(&k_full[st], (j >> 1) & 1, abort_flag, p.err, kErrAttnWait)) break;
        tc_fence_after();
        const uint32_t k_addr = smem_u32(sK + st * C_::KV_BYTES);
        const uint32_t d_s = tmem + (uint32_t)(st * kBK);
#pragma unroll
        for (int ks = 0; ks < DP / 16; ++ks) {
          const uint32_t off = (uint32_t)((ks >> 2) * C_::ATOM + (ks & 3) * 32);
          umma_f16_ss(d_s, sdesc_k_sw128(q_addr + off), sdesc_k_sw128(k_addr + off), IDESC_S, ks > 0);
        }
        umma_commit(&s_full[st]);
        umma_commit(&k_empty[st]);
      }
      umma_commit(&drain[0]);
      const uint64_t t0 = globaltimer_ns();
      while (!mbar_try_wait(&drain[0], 0))
        if (globaltimer_ns() - t0 > kWaitLimitNs) {
          atomicOr(p.err, kErrWaitDrain);
          break;
        }
    }
  } else if (warp == 2) {
    // ------------------------------ PV issuer ---------------------------------
    if (lane == 0) {
      for (int j = 0; j < nkv; ++j) {
        const int b = j & 1;
        if (!mbar_wait(&p_full[b], (j >> 1) & 1, abort_flag, p.err, kErrAttnWait)) break;
        if (!mbar_wait(&v_full[b], (j >> 1) & 1, abort_flag, p.err, kErrAttnWait)) break;
        tc_fence_after();
        const uint32_t p_addr = smem_u32(sP + b * C_::P_BYTES);
        const uint32_t v_addr = smem_u32(sV + b * C_::KV_BYTES);
#pragma unroll
        for (int ks = 0; ks < kBK / 16; ++ks) {
          const uint64_t ad = sdesc_k_sw128(p_addr + (uint32_t)((ks >> 2) * C_::ATOM + (ks & 3) * 32));
          const uint64_t bd = sdesc_mn_sw128(v_addr + (uint32_t)(ks * 16 * 128), C_::ATOM, 1024);
          umma_f16_ss(tmem + C_::O_COL, ad, bd, IDESC_O, (j > 0 || ks > 0) ? 1u : 0u);
        }
        umma_commit(&p_free[b]);
        umma_commit(&v_empty[b]);
      }
      umma_commit(o_final);
      umma_commit(&drain[1]);
      const uint64_t t0 = globaltimer_ns();
      while (!mbar_try_wait(&drain[1], 0))
        if (globaltimer_ns() - t0 > kWaitLimitNs) {
          atomicOr(p.err, kErrWaitDrain);
          break;
        }
    }
  } else {
    // ------------------------------ softmax / epilogue ------------------------
    const int qq = warp & 3;
    const int r = qq * 32 + lane;     // tile row == TMEM lane
    const int row = q0 + r;           // query index
    const uint32_t lane_base = tmem + ((uint32_t)(qq * 32) << 16);
    float m_used = -INFINITY, l = 0.0f;
    bool ok = true;
    for (int j = 0; j < nkv; ++j) {
      const int b = j & 1;
      if (!mbar_wait(&s_full[b], (j >> 1) & 1, abort_flag, p.err, kErrAttnWait)) {
        ok = false;
        break;
      }
      tc_fence_after();
      // All 128 scores of this row in registers: four 32-column TMEM loads, one wait.
      uint32_t u[4][32];
      __syncwarp();
      tmem_ld_32x32b_x32(lane_base + (uint32_t)(b * kBK + 0), u[0]);
      tmem_ld_32x32b_x32(lane_base + (uint32_t)(b * kBK + 32), u[1]);
      tmem_ld_32x32b_x32(lane_base + (uint32_t)(b * kBK + 64), u[2]);
      tmem_ld_32x32b_x32(lane_base + (uint32_t)(b * kBK + 96), u[3]);
      tmem_wait_ld();
      const int kbase = j * kBK;
      const bool full_tile = (kbase + kBK <= p.Skv) && (!p.causal || kbase + kBK - 1 <= q0);
      if (!full_tile) {
#pragma unroll
        for (int c = 0; c < kBK; ++c) {
          const int key = kbase + c;
          if (key >= p.Skv || (p.causal && key > row)) u[c >> 5][c & 31] = __float_as_uint(-INFINITY);
        }
      }
      // Row max of the raw scores, 4 partial maxima (short dependency chains); the
      // scale is positive, so max(s) * scale = max(s * scale).
      float pm[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
      for (int c = 0; c < kBK; ++c) pm[c & 3] = fmaxf(pm[c & 3], __uint_as_float(u[c >> 5][c & 31]));
      const float mx = fmaxf(fmaxf(pm[0], pm[1]), fmaxf(pm[2], pm[3]));
      const float m_new = fmaxf(m_used, mx * p.scale_log2);
      const bool need = m_new > m_used + kRescaleThreshold;
      if (__any_sync(0xffffffffu, need)) {
        if (j > 0) {
          // O must hold PV_{j-1} before it is rescaled.
          if (!mbar_wait(&p_free[(j - 1) & 1], ((j - 1) >> 1) & 1, abort_flag, p.err, kErrAttnWait)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const float f = need ? ex2_approx(m_used - m_new) : 1.0f;
#pragma unroll 1
          for (int c = 0; c < DP; c += 32) {
            uint32_t o[32];
            __syncwarp();
            tmem_ld_32x32b_x32(lane_base + C_::O_COL + (uint32_t)c, o);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * f);
            tmem_st_32x32b_x32(lane_base + C_::O_COL + (uint32_t)c, o);
          }
          tmem_wait_st();
        }
        if (need) {
          l *= ex2_approx(m_used - m_new);
          m_used = m_new;
        }
      }
      // The P buffer of this tile must no longer be read by PV_{j-2}.
      if (j >= 2 && !mbar_wait(&p_free[b], ((j - 2) >> 1) & 1, abort_flag, p.err, kErrAttnWait)) {
        ok = false;
        break;
      }
      // p = 2^(s * scale_log2 - m): one FFMA + one MUFU ex2 per score, 4 partial sums,
      // written as fp16 into the 128B-swizzled K-major P tile: keys [64a, 64a+64) form
      // atom a; 16-byte chunk c of row r sits at chunk position c ^ (r & 7).
      const float neg_m = (m_used == -INFINITY) ? 0.0f : -m_used;
      float ps[4] = {0.0f, 0.0f, 0.0f, 0.0f};
      uint8_t* pb = sP + b * C_::P_BYTES + r * 128;
#pragma unroll
      for (int a = 0; a < 2; ++a)
#pragma unroll
        for (int cc = 0; cc < 8; ++cc) {
          float e[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const int c = a * 64 + cc * 8 + i;
            e[i] = ex2_approx(fmaf(__uint_as_float(u[c >> 5][c & 31]), p.scale_log2, neg_m));
            ps[i & 3] += e[i];
          }
          uint4 w;
          w.x = pack_half2(e[0], e[1]);
          w.y = pack_half2(e[2], e[3]);
          w.z = pack_half2(e[4], e[5]);
          w.w = pack_half2(e[6], e[7]);
          *reinterpret_cast<uint4*>(pb + a * C_::ATOM + ((cc ^ (r & 7)) << 4)) = w;
        }
      l += (ps[0] + ps[1]) + (ps[2] + ps[3]);
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[b]);
    }
    if (ok && mbar_wait(o_final, 0, abort_flag, p.err, kErrAttnWait)) {
      tc_fence_after();
      const float inv = l > 0.0f ? 1.0f / l : 0.0f;
      const bool row_ok = row < p.Sq;
#pragma unroll 1
      for (int c = 0; c < DP; c += 32) {
        uint32_t o[32];
        __syncwarp();
        tmem_ld_32x32b_x32(lane_base + C_::O_COL + (uint32_t)c, o);
        tmem_wait_ld();
        if (!row_ok || c >= p.d) continue;
        const long long base = (long long)n * p.out_batch + (long long)row * p.out_row + (long long)h * p.d + c;
        const int cnt = min(32, p.d - c);
        if (p.out_bf16) {
          uint16_t* dst = reinterpret_cast<uint16_t*>(p.out) + base;
#pragma unroll
          for (int i = 0; i < 32; ++i)
            if (i < cnt) dst[i] = f32_to_bf16_rne(__uint_as_float(o[i]) * inv);
        } else {
          float* dst = reinterpret_cast<float*>(p.out) + base;
          if (cnt == 32 && (reinterpret_cast<uintptr_t>(dst) & 15) == 0) {
#pragma unroll
            for (int i = 0; i < 32; i += 4)
              *reinterpret_cast<float4*>(dst + i) =
                  make_float4(__uint_as_float(o[i]) * inv, __uint_as_float(o[i + 1]) * inv,
                              __uint_as_float(o[i + 2]) * inv, __uint_as_float(o[i + 3]) * inv);
          } else {
#pragma unroll
            for (int i = 0; i < 32; ++i)
              if (i < cnt) dst[i] = __uint_as_float(o[i]) * inv;
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, C_::TMEM_COLS);
  }
}

// fp32 [N, S, H*d] -> fp16 [N, S, H, dp] (zero padded), saturating at +-65504.
__global__ void k_pack_heads_f16(const float* __restrict__ x, __half* __restrict__ y, int64_t rows, int H, int d,
                                 int dp) {
  const int64_t total = rows * H * dp;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int c = (int)(i % dp);
    const int64_t rh = i / dp;
    float v = 0.0f;
    if (c < d) {
      v = x[rh * d + c];
      if (!isnan(v)) v = fminf(fmaxf(v, -65504.0f), 65504.0f);
    }
    y[i] = __float2half_rn(v);
  }
}

template <int DP>
void launch_tc(const __half* q, const __half* k, const __half* v, void* out, long long out_row, long long out_batch,
               bool out_bf16, int64_t N, int64_t Sq, int64_t Skv, int heads, int kv_heads, int64_t d, bool causal,
               float scale) {
  using C_ = ACfg<DP>;
  CUtensorMap tq, tk, tv;
  const uint32_t box[3] = {64, (uint32_t)kBQ, 1};
  {
    const uint64_t dims[3] = {(uint64_t)heads * DP, (uint64_t)Sq, (uint64_t)N};
    const uint64_t str[2] = {(uint64_t)heads * DP * 2, (uint64_t)Sq * heads * DP * 2};
    encode_tmap(&tq, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, q, dims, str, box, CU_TENSOR_MAP_SWIZZLE_128B);
  }
  {
    const uint64_t dims[3] = {(uint64_t)kv_heads * DP, (uint64_t)Skv, (uint64_t)N};
    const uint64_t str[2] = {(uint64_t)kv_heads * DP * 2, (uint64_t)Skv * kv_heads * DP * 2};
    encode_tmap(&tk, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, k, dims, str, box, CU_TENSOR_MAP_SWIZZLE_128B);
    encode_tmap(&tv, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, v, dims, str, box, CU_TENSOR_MAP_SWIZZLE_128B);
  }
  AttnParams p{};
  p.N = (int)N;
  p.Sq = (int)Sq;
  p.Skv = (int)Skv;
  p.heads = heads;
  p.kv_heads = kv_heads;
  p.d = (int)d;
  p.dp = DP;
  p.causal = causal ? 1 : 0;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.out = out;
  p.out_row = out_row;
  p.out_batch = out_batch;
  p.out_bf16 = out_bf16 ? 1 : 0;
  p.err = ctx().err_word;
  auto kern = k_attention_tc<DP>;
  static bool attr_set[64] = {};
  const int dev = ctx().device;
  if (dev >= 0 && dev < 64 && !attr_set[dev]) {
    check_cuda(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C_::SMEM),
               "cudaFuncSetAttribute(attention)");
    attr_set[dev] = true;
  }
  dim3 grid((unsigned)((Sq + kBQ - 1) / kBQ), (unsigned)heads, (unsigned)N);
  kern<<<grid, kThreads, C_::SMEM, ctx().stream>>>(tq, tk, tv, p);
  check_launch("attention_tc");
}

}  // namespace

void launch_attention_simt(const float* q, const float* k, const float* v, float* out, int64_t N, int64_t Sq,
                           int64_t Skv, int heads, int kv_heads, int64_t d, bool causal);

// Tensor-core attention on fp16 operands already laid out [N, S, heads, dp].
void launch_attention_f16(const void* q, const void* k, const void* v, void* out, long long out_row,
                          long long out_batch, bool out_bf16, int64_t N, int64_t Sq, int64_t Skv, int heads,
                          int kv_heads, int64_t d, int64_t dp, bool causal) {
  const float scale = 1.0f / sqrtf((float)d);
  if (dp == 64)
    launch_tc<64>((const __half*)q, (const __half*)k, (const __half*)v, out, out_row, out_batch, out_bf16, N, Sq, Skv,
                  heads, kv_heads, d, causal, scale);
  else
    launch_tc<128>((const __half*)q, (const __half*)k, (const __half*)v, out, out_row, out_batch, out_bf16, N, Sq,
                   Skv, heads, kv_heads, d, causal, scale);
}

void launch_pack_heads_f16(const float* x, void* y, int64_t rows, int H, int64_t d, int64_t dp) {
  const int64_t total = rows * H * dp;
  if (total <= 0) return;
  const int64_t blocks = std::min<int64_t>((total + 255) / 256, (int64_t)ctx().num_sms * 16);
  k_pack_heads_f16<<<(unsigned)blocks, 256, 0, ctx().stream>>>(x, (__half*)y, rows, H, (int)d, (int)dp);
  check_launch("pack_heads_f16");
}

// Drop-in attention (backend_cuda.h:58-59): fp32 q/k/v/out [N, S, heads*d].
// Head dims up to 128 run on the tensor-core kernel (operands packed to fp16 in the
// workspace); larger head dims use the exact fp32 streaming kernel.
static bool g_attention_tc = true;
void set_attention_tc(bool on) { g_attention_tc = on; }

void launch_attention(const float* q, const float* k, const float* v, float* out, int64_t N, int64_t Sq, int64_t Skv,
                      int heads, int kv_heads, int64_t d, bool causal) {
  if (!g_attention_tc || d > 128) return launch_attention_simt(q, k, v, out, N, Sq, Skv, heads, kv_heads, d, causal);
  const int64_t dp = d <= 64 ? 64 : 128;
  const size_t qb = (size_t)(N * Sq * heads * dp) * 2, kb = (size_t)(N * Skv * kv_heads * dp) * 2;
  auto a256 = [](size_t b) { return (b + 255) & ~size_t(255); };
  uint8_t* ws = static_cast<uint8_t*>(workspace(a256(qb) + 2 * a256(kb)));
  void* q16 = ws;
  void* k16 = ws + a256(qb);
  void* v16 = ws + a256(qb) + a256(kb);
  launch_pack_heads_f16(q, q16, N * Sq, heads, d, dp);
  launch_pack_heads_f16(k, k16, N * Skv, kv_heads, d, dp);
  launch_pack_heads_f16(v, v16, N * Skv, kv_heads, d, dp);
  launch_attention_f16(q16, k16, v16, out, (long long)heads * d, (long long)Sq * heads * d, false, N, Sq, Skv, heads,
                       kv_heads, d, dp, causal);
}

}  // namespace sdb
