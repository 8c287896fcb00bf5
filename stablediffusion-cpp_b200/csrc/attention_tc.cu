// attention_tc.cu - flash attention on 5th-generation tensor cores (sm_100a):
// softmax(q k^T / sqrt(d)) v per head with grouped key/value heads and an optional
// causal mask, replacing the reference's score-matrix attention
// (backend_cuda.cu:550-586: two batched SGEMMs around a softmax, the full Sq x Skv
// matrix in HBM) and the CPU path it is checked against (tensor.cpp:771-810).
//
// One CTA owns two 128-row query tiles (A and B) of one (sample, head), 384 threads:
//   warp 0      TMA: Q_A and Q_B once, then K_0, V_0, K_1, V_1, ... (128 keys each) in
//               order through one 5-slot ring; a slot is free again once the MMAs of
//               both tiles that read it are done
//   warps 1, 2  MMA issuers of tiles A and B. Step j, once the tile's softmax has posted
//               P_t(j-1): O_t += P_t(j-1) V_(j-1), then S_t = Q_t K_j^T. P_t lives in TMEM
//               over the first 64 columns of S_t (fp16 pairs) and is the A operand of
//               the PV MMA; one thread's MMAs execute in issue order, so the PV has read
//               P before the next QK^T overwrites S_t, and when the softmax sees S_t(j)
//               the PV of step j-1 is complete too
//   warp 3      idle
//   warps 4-7   softmax of tile A, warps 8-11 softmax of tile B: one query row per thread
//               (TMEM lane). Loads S, applies the scale (in log2 units) and the masks,
//               keeps the running max m and sum l, writes P = 2^(s - m) as fp16 back into
//               TMEM, and at the end normalises O by 1/l and stores it.
// The two softmax warpgroups take turns at the exp pass, so that while one works the
// tensor core runs the other tile's MMAs. O is rescaled only when a row's max grows by
// more than 2^8 since the value used so far (P stays <= 256, fine for fp16 and fp32);
// the stale max cancels in O / l. TMEM: S_A | S_B | O_A | O_B = 512 columns.
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

constexpr int kBQ = 128;      // rows per query tile (TMEM lanes)
constexpr int kBK = 128;      // keys per K / V tile
constexpr int kTiles = 2;     // query tiles per CTA (ping-pong)
constexpr int kThreads = 384; // control warpgroup (TMA, 2 MMA issuers, idle) + 2 softmax warpgroups
// Register split by setmaxnreg: launched at kRegsLaunch per thread (384 x 168 = 64512),
// the control warpgroup gives registers back and the softmax warpgroups take them, so
// each softmax thread can hold a whole 128-column row of S. The shares add up to the
// launch total exactly (128 x 56 + 256 x 224 = 64512); the launcher checks the compiled
// register count so the increase can always be satisfied.
constexpr int kRegsLaunch = 168, kRegsControl = 56, kRegsSoftmax = 224;
static_assert(128 * kRegsControl + 256 * kRegsSoftmax <= kThreads * kRegsLaunch, "register split");
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
  static constexpr int Q_BYTES = ATOMS * ATOM;   // one query tile
  static constexpr int KV_BYTES = ATOMS * ATOM;  // one K or one V tile
  static constexpr int SLOTS = 5;                // K / V ring
  // Q[2] | ring[5] | barriers
  static constexpr int SMEM = kTiles * Q_BYTES + SLOTS * KV_BYTES + 1024 + 256;
  static constexpr uint32_t TMEM_COLS = 512;     // S_A | S_B | O_A | O_B
  static constexpr uint32_t O_COL = 256;
};

// 2^x on the MUFU pipe (PTX ex2.approx.ftz.f32; 2^-inf = +0).
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Three-input max (sm_100 max.f32 with two sources and a third operand).
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
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
  uint8_t* sQ = smem;                            // [2 tiles]
  uint8_t* sR = sQ + kTiles * C_::Q_BYTES;       // ring [5 slots]
  uint64_t* bars = reinterpret_cast<uint64_t*>(sR + C_::SLOTS * C_::KV_BYTES);
  uint64_t* q_full = bars + 0;
  uint64_t* r_full = bars + 1;     // [5 slots]
  uint64_t* r_empty = bars + 6;    // [5 slots]
  uint64_t* s_full = bars + 11;    // [2 tiles] S_t(j) ready (and PV_t(j-1) done)
  uint64_t* p_full = bars + 13;    // [2 tiles] P_t(j) in TMEM, O_t rescaled
  uint64_t* o_final = bars + 15;   // [2 tiles]
  uint64_t* drain = bars + 17;     // [2] one per MMA issuer
  uint64_t* turn = bars + 19;      // [2 tiles] the tile's softmax finished its exp pass
  uint64_t* p_half = bars + 21;    // [2 tiles] keys 0..63 of P_t(j) in TMEM, O_t rescaled
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 23);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int q0 = blockIdx.x * (kTiles * kBQ), h = blockIdx.y, n = blockIdx.z;
  const int kvh = h / (p.heads / p.kv_heads);
  int nkv = (p.Skv + kBK - 1) / kBK;
  if (p.causal) nkv = min(nkv, (q0 + kTiles * kBQ - 1) / kBK + 1);

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < C_::SLOTS; ++i) {
      mbar_init(&r_full[i], 1);
      mbar_init(&r_empty[i], 2);  // both MMA issuers
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], 4);
      mbar_init(&o_final[i], 1);
      mbar_init(&drain[i], 1);
      mbar_init(&turn[i], 4);
      mbar_init(&p_half[i], 4);
    }
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
  if (warp < 4) {
  // Control warpgroup: gives its registers back (all four warps, warp-group aligned).
  asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kRegsControl));
  if (warp == 0) {
    // ------------------------------ TMA producer ------------------------------
    if (lane == 0) {
      mbar_arrive_expect_tx(q_full, kTiles * C_::Q_BYTES);
      for (int t = 0; t < kTiles; ++t)
        for (int a = 0; a < C_::ATOMS; ++a)
          tma_load_3d(sQ + t * C_::Q_BYTES + a * C_::ATOM, &tmQ, q_full, h * p.dp + a * 64, q0 + t * kBQ, n);
      // Load i = 2j is K_j, i = 2j + 1 is V_j; slot i % SLOTS, use i / SLOTS of that slot.
      int issued = -1;
      for (int i = 0; i < 2 * nkv; ++i) {
        const int sl = i % C_::SLOTS, u = i / C_::SLOTS;
        if (!mbar_wait(&r_empty[sl], (u & 1) ^ 1u, abort_flag, p.err, kErrAttnWait)) break;
        mbar_arrive_expect_tx(&r_full[sl], C_::KV_BYTES);
        const CUtensorMap* tm = (i & 1) ? &tmV : &tmK;
        for (int a = 0; a < C_::ATOMS; ++a)
          tma_load_3d(sR + sl * C_::KV_BYTES + a * C_::ATOM, tm, &r_full[sl], kvh * p.dp + a * 64, (i >> 1) * kBK, n);
        issued = i;
      }
      if (issued < 2 * nkv - 1) {
        // Aborted: wait (bounded) for the loads this CTA still has in flight.
        const uint64_t t0 = globaltimer_ns();
        while (!mbar_try_wait(q_full, 0) && globaltimer_ns() - t0 < kWaitLimitNs) {
        }
        for (int i = max(0, issued - C_::SLOTS + 1); i <= issued; ++i)
          while (!mbar_try_wait(&r_full[i % C_::SLOTS], (i / C_::SLOTS) & 1) && globaltimer_ns() - t0 < kWaitLimitNs) {
          }
      }
    }
  } else if (warp == 1 || warp == 2) {
    // ------------------------------ MMA issuers -------------------------------
    const int t = warp - 1;
    if (lane == 0) {
      bool ok = mbar_wait(q_full, 0, abort_flag, p.err, kErrAttnWait);
      tc_fence_after();
      const uint32_t q_addr = smem_u32(sQ + t * C_::Q_BYTES);
      const uint32_t d_s = tmem + (uint32_t)(t * kBK);  // S_t; P_t over its first 64 columns
      const uint32_t d_o = tmem + C_::O_COL + (uint32_t)(t * DP);
      // Descriptors of the K steps (16 wide): Q_t (fixed), P_t in TMEM (8 columns per
      // step), K_j and V_(j-1) per step, all built before the waits so that the eight
      // MMAs of a product issue back to back.
      static_assert(DP == 64 || DP == 128, "head dim padded to 64 or 128");
      uint64_t qd[8] = {};
      uint32_t pa[8];
#pragma unroll
      for (int ks = 0; ks < 8; ++ks) {
        if (ks < DP / 16) qd[ks] = sdesc_k_sw128(q_addr + (uint32_t)((ks >> 2) * C_::ATOM + (ks & 3) * 32));
        pa[ks] = d_s + (uint32_t)(ks * 8);
      }
      for (int j = 0; ok && j <= nkv; ++j) {
        const int vsl = (2 * j - 1 + C_::SLOTS) % C_::SLOTS, ksl = (2 * j) % C_::SLOTS;
        const uint32_t v_addr = smem_u32(sR + vsl * C_::KV_BYTES), k_addr = smem_u32(sR + ksl * C_::KV_BYTES);
        uint64_t vd[8], kd[8] = {};
#pragma unroll
        for (int ks = 0; ks < 8; ++ks) {
          vd[ks] = sdesc_mn_sw128(v_addr + (uint32_t)(ks * 16 * 128), C_::ATOM, 1024);
          if (ks < DP / 16) kd[ks] = sdesc_k_sw128(k_addr + (uint32_t)((ks >> 2) * C_::ATOM + (ks & 3) * 32));
        }
        // K_j and V_(j-1) normally landed long ago; wait for them before P_t(j-1), so
        // the PV and the QK^T go out back to back once P is there.
        if (j > 0 && !mbar_wait(&r_full[vsl], ((2 * j - 1) / C_::SLOTS) & 1, abort_flag, p.err, kErrAttnWait)) break;
        if (j < nkv && !mbar_wait(&r_full[ksl], ((2 * j) / C_::SLOTS) & 1, abort_flag, p.err, kErrAttnWait)) break;
        if (j > 0) {
          // O_t += P_t(j-1) V_(j-1): A = P from TMEM, B = V (MN-major). Keys 0..63 go as
          // soon as the softmax has posted them, keys 64..127 once P is complete.
          if (!mbar_wait(&p_half[t], (j - 1) & 1, abort_flag, p.err, kErrAttnWait)) break;
          tc_fence_after();
          {
            const uint32_t a4[4] = {pa[0], pa[1], pa[2], pa[3]};
            const uint64_t b4[4] = {vd[0], vd[1], vd[2], vd[3]};
            umma4_f16_ts(d_o, a4, b4, IDESC_O, j > 1 ? 1u : 0u);
          }
          if (!mbar_wait(&p_full[t], (j - 1) & 1, abort_flag, p.err, kErrAttnWait)) break;
          tc_fence_after();
          {
            const uint32_t a4[4] = {pa[4], pa[5], pa[6], pa[7]};
            const uint64_t b4[4] = {vd[4], vd[5], vd[6], vd[7]};
            umma4_f16_ts(d_o, a4, b4, IDESC_O, 1u);
          }
          umma_commit(&r_empty[vsl]);
        }
        if (j < nkv) {
          // S_t = Q_t K_j^T
          tc_fence_after();
          if constexpr (DP == 128)
            umma8_f16_ss(d_s, qd, kd, IDESC_S, 0u);
          else {
            const uint64_t a4[4] = {qd[0], qd[1], qd[2], qd[3]};  // dp = 64: four K steps
            const uint64_t b4[4] = {kd[0], kd[1], kd[2], kd[3]};
            umma4_f16_ss(d_s, a4, b4, IDESC_S, 0u);
          }
          umma_commit(&s_full[t]);
          umma_commit(&r_empty[ksl]);
        }
      }
      umma_commit(&o_final[t]);
      umma_commit(&drain[t]);
      const uint64_t t0 = globaltimer_ns();
      while (!mbar_try_wait(&drain[t], 0))
        if (globaltimer_ns() - t0 > kWaitLimitNs) {
          atomicOr(p.err, kErrWaitDrain);
          break;
        }
    }
  }
  } else {
    // ------------------------------ softmax / epilogue ------------------------
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kRegsSoftmax));
    const int t = (warp - 4) >> 2;   // query tile of this warpgroup (warps 4..11)
    const int qq = warp & 3;         // TMEM lane quarter this warp may access
    const int r = qq * 32 + lane;    // tile row == TMEM lane
    const int row = q0 + t * kBQ + r;
    const int tile_q0 = q0 + t * kBQ;
    const uint32_t lane_base = tmem + ((uint32_t)(qq * 32) << 16);
    const uint32_t s_addr = lane_base + (uint32_t)(t * kBK);
    const uint32_t o_addr = lane_base + C_::O_COL + (uint32_t)(t * DP);
    float m_used = -INFINITY, l = 0.0f;
    bool ok = true;
    // Keys past Skv (and, if causal, past the row) read as -inf. full_tile is uniform
    // over the CTA, so the fast path runs no per-score mask code.
    auto mask_row = [&](uint32_t(&u)[4][32], int key0) {
#pragma unroll
      for (int c = 0; c < kBK; ++c) {
        const int key = key0 + c;
        if (key >= p.Skv || (p.causal && key > row)) u[c >> 5][c & 31] = 0xff800000u;
      }
    };
    for (int j = 0; j < nkv; ++j) {
      if (!mbar_wait(&s_full[t], j & 1, abort_flag, p.err, kErrAttnWait)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const int kbase = j * kBK;
      const bool full_tile = (kbase + kBK <= p.Skv) && (!p.causal || kbase + kBK - 1 <= tile_q0);
      // The whole 128-key row of S in registers: one TMEM round trip per step.
      uint32_t u[4][32];
      __syncwarp();
#pragma unroll
      for (int g = 0; g < 4; ++g) tmem_ld_32x32b_x32(s_addr + (uint32_t)(g * 32), u[g]);
      tmem_wait_ld();
      if (!full_tile) mask_row(u, kbase);
      // Row max of the raw scores, 4 partial maxima; the scale is positive, so
      // max(s) * scale = max(s * scale).
      float pm[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
      for (int c = 0; c < kBK; c += 8)
#pragma unroll
        for (int i = 0; i < 4; ++i)
          pm[i] = fmax3(pm[i], __uint_as_float(u[c >> 5][(c & 31) + 2 * i]), __uint_as_float(u[c >> 5][(c & 31) + 2 * i + 1]));
      const float mx = fmaxf(fmaxf(pm[0], pm[1]), fmaxf(pm[2], pm[3]));
      const float m_new = fmaxf(m_used, mx * p.scale_log2);
      const bool need = m_new > m_used + kRescaleThreshold;
      // PV_t(j-1) completed before S_t(j) was posted, so O_t can be rescaled here.
      if (__any_sync(0xffffffffu, need)) {
        if (j > 0) {
          const float f = need ? ex2_approx(m_used - m_new) : 1.0f;
#pragma unroll 1
          for (int c = 0; c < DP; c += 32) {
            uint32_t o[32];
            __syncwarp();
            tmem_ld_32x32b_x32(o_addr + (uint32_t)c, o);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * f);
            tmem_st_32x32b_x32(o_addr + (uint32_t)c, o);
          }
        }
        if (need) {
          l *= ex2_approx(m_used - m_new);
          m_used = m_new;
        }
      }
      // The two softmax warpgroups take turns at the exp pass (A(0), B(0), A(1), ...), so
      // that each has the MUFU pipes to itself while the tensor core runs the other
      // tile's MMAs; left alone they fall into lockstep and the MMAs of both tiles wait.
      if (!(t == 0 && j == 0) &&
          !mbar_wait(&turn[t ^ 1], (t == 0 ? j - 1 : j) & 1, abort_flag, p.err, kErrAttnWait)) {
        ok = false;
        break;
      }
      // p = 2^(s * scale_log2 - m), keys 2c and 2c + 1 as a pair: one packed FFMA2, two
      // MUFU ex2, one packed FADD2 into two partial sums and one fp16x2 pack. The pass runs
      // as one in-order warp per SM sub-partition, so its instruction count sets its
      // length (the packed forms took 4-6% off the kernel; moving some exponentials onto
      // an FMA polynomial added instructions and was slower). The pair goes to TMEM
      // column c of S_t, the layout of a 16-bit A operand in tensor memory.
      const float neg_m = (m_used == -INFINITY) ? 0.0f : -m_used;
      const float2 sc2 = make_float2(p.scale_log2, p.scale_log2), nm2 = make_float2(neg_m, neg_m);
      float2 psa = make_float2(0.0f, 0.0f), psb = make_float2(0.0f, 0.0f);
#pragma unroll
      for (int g = 0; g < 4; ++g) {
        uint32_t w[16];
#pragma unroll
        for (int c = 0; c < 16; ++c) {
          const float2 x = ffma2(make_float2(__uint_as_float(u[g][2 * c]), __uint_as_float(u[g][2 * c + 1])), sc2, nm2);
          const float e0 = ex2_approx(x.x);
          const float e1 = ex2_approx(x.y);
          if (c & 1)
            psb = fadd2(psb, make_float2(e0, e1));
          else
            psa = fadd2(psa, make_float2(e0, e1));
          w[c] = pack_half2(e0, e1);
        }
        tmem_st_32x32b_x16(s_addr + (uint32_t)(g * 16), w);
        if (g == 1) {
          // Keys 0..63 are in place: the PV of this half can start.
          tmem_wait_st();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&p_half[t]);
        }
      }
      l += (psa.x + psb.x) + (psa.y + psb.y);
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&p_full[t]);
        mbar_arrive(&turn[t]);
      }
    }
    if (ok && mbar_wait(&o_final[t], 0, abort_flag, p.err, kErrAttnWait)) {
      tc_fence_after();
      const float inv = l > 0.0f ? 1.0f / l : 0.0f;
      const bool row_ok = row < p.Sq;
#pragma unroll 1
      for (int c = 0; c < DP; c += 32) {
        uint32_t o[32];
        __syncwarp();
        tmem_ld_32x32b_x32(o_addr + (uint32_t)c, o);
        tmem_wait_ld();
        if (!row_ok || c >= p.d) continue;
        const long long base = (long long)n * p.out_batch + (long long)row * p.out_row + (long long)h * p.d + c;
        const int cnt = min(32, p.d - c);
        if (p.out_bf16) {
          uint16_t* dst = reinterpret_cast<uint16_t*>(p.out) + base;
          if (cnt == 32 && (reinterpret_cast<uintptr_t>(dst) & 15) == 0) {
#pragma unroll
            for (int i = 0; i < 32; i += 8) {
              uint4 w;
              w.x = pack_bf16x2(__uint_as_float(o[i]) * inv, __uint_as_float(o[i + 1]) * inv);
              w.y = pack_bf16x2(__uint_as_float(o[i + 2]) * inv, __uint_as_float(o[i + 3]) * inv);
              w.z = pack_bf16x2(__uint_as_float(o[i + 4]) * inv, __uint_as_float(o[i + 5]) * inv);
              w.w = pack_bf16x2(__uint_as_float(o[i + 6]) * inv, __uint_as_float(o[i + 7]) * inv);
              *reinterpret_cast<uint4*>(dst + i) = w;
            }
          } else {
#pragma unroll
            for (int i = 0; i < 32; ++i)
              if (i < cnt) dst[i] = f32_to_bf16_rne(__uint_as_float(o[i]) * inv);
          }
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

// q, k and v packed by one launch, two values per thread (one half2 store): segment 0 has
// qn2 = rows_q * Hq * dp / 2 pairs, segments 1 and 2 kn2 = rows_kv * Hkv * dp / 2 each.
// dp / 2 = 1 << sh (dp is 64 or 128), so a pair's row and column come from a shift and a
// mask. Columns d..dp-1 are zero; finite values saturate at the fp16 range.
__device__ __forceinline__ float f16_sat(float v) { return isnan(v) ? v : fminf(fmaxf(v, -65504.0f), 65504.0f); }
__global__ void k_pack_qkv_f16(const float* __restrict__ q, const float* __restrict__ k, const float* __restrict__ v,
                               __half* __restrict__ q16, __half* __restrict__ k16, __half* __restrict__ v16,
                               int64_t qn2, int64_t kn2, int d, int sh) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < qn2 + 2 * kn2;
       i += (int64_t)gridDim.x * blockDim.x) {
    const float* x = q;
    __half* y = q16;
    int64_t j = i;
    if (j >= qn2) {
      j -= qn2;
      x = k;
      y = k16;
      if (j >= kn2) {
        j -= kn2;
        x = v;
        y = v16;
      }
    }
    const int c = (int)(j & ((1 << sh) - 1)) * 2;
    const float* src = x + (j >> sh) * d + c;
    const float a = c < d ? f16_sat(src[0]) : 0.0f;
    const float b = c + 1 < d ? f16_sat(src[1]) : 0.0f;
    reinterpret_cast<__half2*>(y)[j] = __floats2half2_rn(a, b);
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
    // setmaxnreg.inc waits until the registers it asks for are free; the split only adds
    // up if the kernel was compiled to exactly kRegsLaunch registers per thread.
    cudaFuncAttributes fa{};
    check_cuda(cudaFuncGetAttributes(&fa, kern), "cudaFuncGetAttributes(attention)");
    if (fa.numRegs != kRegsLaunch)
      fail(kErrUnsupported, "attention_tc: compiled with " + std::to_string(fa.numRegs) +
                                " registers per thread, the register split needs " + std::to_string(kRegsLaunch));
    check_cuda(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C_::SMEM),
               "cudaFuncSetAttribute(attention)");
    attr_set[dev] = true;
  }
  dim3 grid((unsigned)((Sq + kTiles * kBQ - 1) / (kTiles * kBQ)), (unsigned)heads, (unsigned)N);
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
// Head dims up to 128 run on the flash kernel (operands packed to fp16 in the
// workspace); larger head dims on tf32 GEMMs around a softmax (attention_gemm.cu).
// set_attention_tc(false) selects the exact fp32 streaming kernel for every head dim.
static bool g_attention_tc = true;
void set_attention_tc(bool on) { g_attention_tc = on; }

void launch_attention(const float* q, const float* k, const float* v, float* out, int64_t N, int64_t Sq, int64_t Skv,
                      int heads, int kv_heads, int64_t d, bool causal) {
  if (!g_attention_tc) return launch_attention_simt(q, k, v, out, N, Sq, Skv, heads, kv_heads, d, causal);
  if (d > 128) {
    // The GEMM form launches about five kernels per (sample, head) and query chunk; with
    // small score matrices (the UNet's 64-256 tokens at its deepest levels) the exact
    // streaming kernel covers all heads in one launch and is faster.
    if (d <= 512 && (double)N * heads * Sq * (double)Skv <= (double)(1 << 24))
      return launch_attention_simt(q, k, v, out, N, Sq, Skv, heads, kv_heads, d, causal);
    return launch_attention_gemm(q, k, v, out, N, Sq, Skv, heads, kv_heads, d, causal);
  }
  const int64_t dp = d <= 64 ? 64 : 128;
  const size_t qb = (size_t)(N * Sq * heads * dp) * 2, kb = (size_t)(N * Skv * kv_heads * dp) * 2;
  auto a256 = [](size_t b) { return (b + 255) & ~size_t(255); };
  uint8_t* ws = static_cast<uint8_t*>(workspace(a256(qb) + 2 * a256(kb)));
  void* q16 = ws;
  void* k16 = ws + a256(qb);
  void* v16 = ws + a256(qb) + a256(kb);
  {
    const int64_t qn2 = N * Sq * heads * dp / 2, kn2 = N * Skv * kv_heads * dp / 2;
    const int sh = dp == 64 ? 5 : 6;  // log2(dp / 2)
    const int64_t blocks = std::min<int64_t>((qn2 + 2 * kn2 + 255) / 256, (int64_t)ctx().num_sms * 16);
    k_pack_qkv_f16<<<(unsigned)blocks, 256, 0, ctx().stream>>>(q, k, v, (__half*)q16, (__half*)k16, (__half*)v16, qn2,
                                                               kn2, (int)d, sh);
    check_launch("pack_qkv_f16");
  }
  launch_attention_f16(q16, k16, v16, out, (long long)heads * d, (long long)Sq * heads * d, false, N, Sq, Skv, heads,
                       kv_heads, d, dp, causal);
}

}  // namespace sdb
