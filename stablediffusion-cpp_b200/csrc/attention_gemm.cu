// attention_gemm.cu - attention as two tensor-core GEMMs around a softmax, the scheme of
// the reference's GPU backend (backend_cuda.cu:550-586: batched scores GEMM, row softmax,
// batched output GEMM), on kind::tf32 instead of fp32 SGEMM. It serves head dims above 128,
// which the flash kernel (attention_tc.cu) does not take: the VAE's single-head attention
// over 512 channels (modules.cpp:133-141) is the case that matters.
//
// Per (sample, query head) and chunk of query rows:
//   scores[R, Skv] = q_chunk k^T            (tf32 operands rounded from fp32, fp32 accumulate)
//   P = softmax(scores * 1/sqrt(d))          (causal rows masked; stored rounded to tf32)
//   out_chunk[R, d] = P v                    (v transposed once per kv head to [d, Skv])
// Chunks keep the score block at most 256 MB. Heads of one kv group share the transposed v.
#include <algorithm>
#include <cmath>

#include "internal.h"

namespace sdb {

void launch_attention_gemm(const float* q, const float* k, const float* v, float* out, int64_t N, int64_t Sq,
                           int64_t Skv, int heads, int kv_heads, int64_t d, bool causal, int64_t q_ld, int64_t kv_ld,
                           int64_t o_ld, bool qk_tf32) {
  if (N <= 0 || Sq <= 0 || heads <= 0) return;
  const float scale = 1.0f / std::sqrt((float)d);
  const int group = heads / kv_heads;
  const int64_t inner = q_ld ? q_ld : (int64_t)heads * d, kv_inner = kv_ld ? kv_ld : (int64_t)kv_heads * d;
  const int64_t o_inner = o_ld ? o_ld : (int64_t)heads * d;
  const int64_t ld = (std::max<int64_t>(Skv, 1) + 3) / 4 * 4;  // 16-byte rows for the TMA operands
  // Query rows per chunk: the score block stays within 512 MB, and where possible the
  // output GEMM's 128-row tiles x (d / 128) column tiles fill whole waves of the SMs.
  int64_t chunk = std::max<int64_t>(1, std::min<int64_t>(Sq, ((int64_t)1 << 27) / ld));
  const int64_t wave_rows = 128 * std::max<int64_t>(1, ctx().num_sms / ((d + 127) / 128));
  if (chunk >= wave_rows && chunk < Sq)
    chunk -= chunk % wave_rows;
  else if (chunk >= 128 && chunk < Sq)
    chunk -= chunk % 128;
  const bool direct = qk_tf32 && inner % 4 == 0 && kv_inner % 4 == 0 &&
                      (reinterpret_cast<uintptr_t>(q) & 15) == 0 && (reinterpret_cast<uintptr_t>(k) & 15) == 0 &&
                      (d * 4) % 16 == 0;
  const size_t sb = ((size_t)(chunk * ld) * 4 + 255) & ~(size_t)255;
  const size_t vb = ((size_t)(d * ld) * 4 + 255) & ~(size_t)255;
  uint8_t* buf = static_cast<uint8_t*>(pool_malloc(sb + vb));
  float* sc = reinterpret_cast<float*>(buf);
  float* vt = reinterpret_cast<float*>(buf + sb);
  try {
    for (int64_t n = 0; n < N; ++n) {
      for (int kvh = 0; kvh < kv_heads; ++kvh) {
        const float* kb = k + n * Skv * kv_inner + (int64_t)kvh * d;
        launch_transpose_tf32(v + n * Skv * kv_inner + (int64_t)kvh * d, kv_inner, vt, ld, Skv, d);
        for (int h = kvh * group; h < (kvh + 1) * group; ++h) {
          for (int64_t r0 = 0; r0 < Sq; r0 += chunk) {
            const int64_t R = std::min(chunk, Sq - r0);
            const float* qb = q + (n * Sq + r0) * inner + (int64_t)h * d;
            float* ob = out + (n * Sq + r0) * o_inner + (int64_t)h * d;
            if (Skv == 0) {
              launch_bias_fill(ob, o_inner, R, d, nullptr, false);
              continue;
            }
            if (direct)  // operands already on the tf32 grid: read in place
              gemm_tf32_direct(R, Skv, d, qb, inner, kb, kv_inner, sc, ld, nullptr, false);
            else
              gemm_nt_f32_impl(R, Skv, d, qb, inner, kb, kv_inner, sc, ld, nullptr, false);
            op_softmax_rows_ex(sc, R, Skv, ld, scale, causal, R, r0, true);
            gemm_tf32_direct(R, d, Skv, sc, ld, vt, ld, ob, o_inner, nullptr, false);
          }
        }
      }
    }
  } catch (...) {
    pool_free(buf);
    throw;
  }
  // Stream-ordered: the next user of this pool block is issued on the same stream.
  pool_free(buf);
}

}  // namespace sdb
