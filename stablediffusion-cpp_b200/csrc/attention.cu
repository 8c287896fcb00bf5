// attention.cu - softmax(q k^T / sqrt(d)) v per head with grouped key/value heads and
// an optional causal mask: the replacement for the reference's attention
// (backend_cuda.cu:550-586, CPU tensor.cpp:771-810), which materialises the full
// Sq x Skv score matrix per head in HBM.
//
// This file holds the exact-fp32 streaming kernel (online softmax, no score matrix in
// memory): K/V tiles of 32 keys are staged in shared memory and shared by the query
// rows of a block; each warp owns one query row and keeps its running max, sum and
// output accumulator in registers. Lane r scores key r, so key rows sit at a stride that
// keeps the lanes on different banks. When d % 4 == 0 the rows are read as 16-byte vectors
// at a stride of d + 4 or d + 8, whichever makes stride / 4 odd: each 8-lane phase of a
// 128-bit load then covers 32 distinct banks. Otherwise the stride is d | 1, read as
// scalars. Both forms add the products in the same order. It serves head dims above 128, which the
// tensor-core kernel (attention_tc.cu) does not take, and is the exact reference the
// tensor-core path can be compared with on the device.
#include <algorithm>
#include <cmath>

#include "internal.h"
#include "ptx.cuh"

namespace sdb {
namespace {

constexpr int kRows = 8;   // query rows (warps) per block
constexpr int kKeys = 32;  // keys per shared-memory tile

// Key-row stride of the score loop's shared-memory tile (see above).
__host__ __device__ __forceinline__ int simt_key_stride(int d) {
  return d % 4 != 0 ? (d | 1) : (d / 4) % 2 == 0 ? d + 4 : d + 8;
}

template <int DV>  // DV = ceil(d / 32): output dims owned per lane
__global__ void __launch_bounds__(kRows * 32)
    k_attention_simt(const float* __restrict__ q, const float* __restrict__ k, const float* __restrict__ v,
                     float* __restrict__ out, int64_t Sq, int64_t Skv, int heads, int kv_heads, int d, int causal,
                     float scale, int vec_kv) {
  extern __shared__ float4 sm4[];
  float* sm = reinterpret_cast<float*>(sm4);
  const int dk = simt_key_stride(d);
  const bool vec = d % 4 == 0;      // then dk, d and every offset below are multiples of 4
  float* sk = sm;                   // [kKeys][dk]
  float* sv = sk + kKeys * dk;      // [kKeys][d]
  float* sq = sv + kKeys * d;       // [kRows][d]
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const int h = blockIdx.y, n = blockIdx.z;
  const int group = heads / kv_heads, kvh = h / group;
  const int64_t inner = (int64_t)heads * d, kv_inner = (int64_t)kv_heads * d;
  const int64_t i = (int64_t)blockIdx.x * kRows + w;  // query row of this warp
  const float* qb = q + (int64_t)n * Sq * inner + (int64_t)h * d;
  const float* kb = k + (int64_t)n * Skv * kv_inner + (int64_t)kvh * d;
  const float* vb = v + (int64_t)n * Skv * kv_inner + (int64_t)kvh * d;
  for (int t = lane; t < d; t += 32) sq[w * d + t] = i < Sq ? qb[i * inner + t] * scale : 0.0f;
  float m = -INFINITY, l = 0.0f, o[DV];
#pragma unroll
  for (int c = 0; c < DV; ++c) o[c] = 0.0f;
  // Keys needed by this block: all, or up to the last row's diagonal when causal.
  const int64_t last_row = std::min<int64_t>(Sq, (int64_t)(blockIdx.x + 1) * kRows) - 1;
  const int64_t kend = causal ? std::min<int64_t>(Skv, last_row + 1) : Skv;
  for (int64_t j0 = 0; j0 < kend; j0 += kKeys) {
    __syncthreads();
    if (vec_kv) {
      // 16-byte loads (k and v 16-byte aligned, d % 4 == 0), four of each in flight per thread.
      const int d4 = d >> 2, n4 = kKeys * d4;
      for (int e0 = threadIdx.x; e0 < n4; e0 += 4 * kRows * 32) {
        float4 kv[4], vv[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int e = e0 + u * kRows * 32;
          kv[u] = vv[u] = make_float4(0.f, 0.f, 0.f, 0.f);
          if (e < n4) {
            const int r = e / d4, t4 = e - r * d4;
            const int64_t j = j0 + r;
            if (j < Skv) {
              kv[u] = __ldg(reinterpret_cast<const float4*>(kb + j * kv_inner) + t4);
              vv[u] = __ldg(reinterpret_cast<const float4*>(vb + j * kv_inner) + t4);
            }
          }
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int e = e0 + u * kRows * 32;
          if (e < n4) {
            const int r = e / d4, t4 = e - r * d4;
            *reinterpret_cast<float4*>(sk + r * dk + 4 * t4) = kv[u];
            *reinterpret_cast<float4*>(sv + r * d + 4 * t4) = vv[u];
          }
        }
      }
    } else {
      for (int e = threadIdx.x; e < kKeys * d; e += blockDim.x) {
        const int r = e / d, t = e - r * d;
        const int64_t j = j0 + r;
        sk[r * dk + t] = j < Skv ? kb[j * kv_inner + t] : 0.0f;
        sv[e] = j < Skv ? vb[j * kv_inner + t] : 0.0f;
      }
    }
    __syncthreads();
    // lane r scores key j0 + r
    const int64_t j = j0 + lane;
    float s = 0.0f;
    if (vec) {
      const float4* q4 = reinterpret_cast<const float4*>(sq + w * d);
      const float4* k4 = reinterpret_cast<const float4*>(sk + lane * dk);
      for (int t = 0; t < (d >> 2); ++t) {
        const float4 a = q4[t], b = k4[t];
        s = fmaf(a.x, b.x, s);
        s = fmaf(a.y, b.y, s);
        s = fmaf(a.z, b.z, s);
        s = fmaf(a.w, b.w, s);
      }
    } else {
      for (int t = 0; t < d; ++t) s = fmaf(sq[w * d + t], sk[lane * dk + t], s);
    }
    const bool valid = (j < Skv) && (!causal || j <= i);
    s = valid ? s : -INFINITY;
    float mx = s;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
    const float m_new = fmaxf(m, mx);
    if (m_new == -INFINITY) continue;  // nothing valid yet for this row
    const float corr = expf(m - m_new);
    const float p = valid ? expf(s - m_new) : 0.0f;
    float ps = p;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) ps += __shfl_xor_sync(0xffffffffu, ps, off);
    l = l * corr + ps;
    m = m_new;
#pragma unroll
    for (int c = 0; c < DV; ++c) o[c] *= corr;
    for (int r = 0; r < kKeys; ++r) {
      const float pr = __shfl_sync(0xffffffffu, p, r);
#pragma unroll
      for (int c = 0; c < DV; ++c) {
        const int t = lane + 32 * c;
        if (t < d) o[c] = fmaf(pr, sv[r * d + t], o[c]);
      }
    }
  }
  if (i < Sq) {
    float* ob = out + (int64_t)n * Sq * inner + i * inner + (int64_t)h * d;
    const float inv = l > 0.0f ? 1.0f / l : 0.0f;
#pragma unroll
    for (int c = 0; c < DV; ++c) {
      const int t = lane + 32 * c;
      if (t < d) ob[t] = o[c] * inv;
    }
  }
}

template <int DV>
void launch_simt(const float* q, const float* k, const float* v, float* out, int64_t N, int64_t Sq, int64_t Skv,
                 int heads, int kv_heads, int64_t d, bool causal) {
  const size_t smem = (size_t)(kKeys * simt_key_stride((int)d) + (kKeys + kRows) * d) * sizeof(float);
  if (smem > 48 * 1024)
    check_cuda(cudaFuncSetAttribute(k_attention_simt<DV>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem),
               "attention attr");
  dim3 grid((unsigned)((Sq + kRows - 1) / kRows), (unsigned)heads, (unsigned)N);
  const int vec_kv = d % 4 == 0 && ((reinterpret_cast<uintptr_t>(k) | reinterpret_cast<uintptr_t>(v)) & 15) == 0;
  k_attention_simt<DV><<<grid, kRows * 32, smem, ctx().stream>>>(q, k, v, out, Sq, Skv, heads, kv_heads, (int)d,
                                                                 causal ? 1 : 0, 1.0f / sqrtf((float)d), vec_kv);
  check_launch("attention_simt");
}

}  // namespace

void launch_attention_simt(const float* q, const float* k, const float* v, float* out, int64_t N, int64_t Sq,
                           int64_t Skv, int heads, int kv_heads, int64_t d, bool causal) {
  switch ((d + 31) / 32) {
    case 1: return launch_simt<1>(q, k, v, out, N, Sq, Skv, heads, kv_heads, d, causal);
    case 2: return launch_simt<2>(q, k, v, out, N, Sq, Skv, heads, kv_heads, d, causal);
    case 3: return launch_simt<3>(q, k, v, out, N, Sq, Skv, heads, kv_heads, d, causal);
    case 4: return launch_simt<4>(q, k, v, out, N, Sq, Skv, heads, kv_heads, d, causal);
    case 5: return launch_simt<5>(q, k, v, out, N, Sq, Skv, heads, kv_heads, d, causal);
    case 6: return launch_simt<6>(q, k, v, out, N, Sq, Skv, heads, kv_heads, d, causal);
    case 7: return launch_simt<7>(q, k, v, out, N, Sq, Skv, heads, kv_heads, d, causal);
    case 8: return launch_simt<8>(q, k, v, out, N, Sq, Skv, heads, kv_heads, d, causal);
    case 9: case 10: case 11: case 12: return launch_simt<12>(q, k, v, out, N, Sq, Skv, heads, kv_heads, d, causal);
    case 13: case 14: case 15: case 16: return launch_simt<16>(q, k, v, out, N, Sq, Skv, heads, kv_heads, d, causal);
    default: fail(kErrInvalidArg, "attention: the exact fp32 kernel takes head dims up to 512");
  }
}

}  // namespace sdb
