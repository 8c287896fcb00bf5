// internal.h - state shared by the library's translation units: the per-device
// context (stream, SM count, device error word, workspace), the thread-local error
// message, and the launch entry points each kernel file exports to runtime.cu.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include <atomic>
#include <string>

namespace sdb {

// Thrown inside the library; the C-ABI boundary converts it to a status code plus a
// message readable through sdb200_last_error().
struct Error {
  int code;
  std::string msg;
};
[[noreturn]] void fail(int code, const std::string& msg);
void check_cuda(cudaError_t e, const char* what);
// Checks the launch status of the last kernel (does not synchronise) and counts it.
void check_launch(const char* what);
unsigned long long launch_count();

// Status codes of the C ABI.
enum : int {
  kOk = 0,
  kErrInvalidArg = 1,   // bad size, leading dimension, alignment or null pointer
  kErrNoDevice = 2,     // no CUDA device / driver
  kErrCuda = 3,         // a CUDA runtime call failed
  kErrDeviceWait = 4,   // a kernel's bounded wait expired (device error word set)
  kErrOutOfMemory = 5,
  kErrUnsupported = 6,
};

struct DeviceContext {
  // Set (release) once every other field is filled; readers that skip the creation lock
  // load it with acquire before touching the rest.
  std::atomic<bool> ready{false};
  int device = -1;
  int num_sms = 0;
  int cc_major = 0, cc_minor = 0;
  size_t total_mem = 0;
  std::string name;
  cudaStream_t stream = nullptr;   // stream every op of this device is issued on
  int* err_word = nullptr;         // device int, OR-ed by kernels on bounded-wait expiry
  // Workspace for operand packing (grown on demand, never shrunk). Ops on one stream
  // run in order, so one workspace per context is safe.
  void* ws = nullptr;
  size_t ws_bytes = 0;
  // Split-K partial tiles of the GEMM (a second workspace: the first may hold the packed
  // operands of the same call).
  void* ws_split = nullptr;
  size_t ws_split_bytes = 0;
};

// Context of the calling thread's current device (created on first use).
DeviceContext& ctx();
// The context of device `dev` if one was already created, else null (never creates).
DeviceContext* ctx_if_created(int dev);
// Returns a workspace pointer of at least `bytes` bytes (256-byte aligned).
void* workspace(size_t bytes);
// The split-K partial-tile workspace (independent of workspace()).
void* split_workspace(size_t bytes);
// Encodes a 2-D/3-D tiled tensor map through the driver entry point.
void encode_tmap(CUtensorMap* map, CUtensorMapDataType dtype, int rank, const void* base, const uint64_t* dims,
                 const uint64_t* strides_bytes, const uint32_t* box, CUtensorMapSwizzle swizzle);

// ------------------------------------------------------------------------------
// Kernel entry points (host launchers). All take device pointers, validate their
// arguments, enqueue on ctx().stream and return without synchronising.
// ------------------------------------------------------------------------------
// GEMM core: C[M,N] = A[M,K] * B[N,K]^T (+bias[N]) (+C if accumulate).
// a_bf16/b_bf16 select the operand types: bf16 x bf16 -> kind::f16,
// fp32 x fp32 -> kind::tf32. Pointers must be 16-byte aligned and leading dimensions
// (in elements) must give 16-byte multiples; the callers in gemm_api.cu repack
// operands that do not.
enum class Epi : int {
  kStore = 0,      // C = acc (+bias) (+C)
  kSwiglu = 1,     // columns interleaved gate/up per 16: Y[m, n/2] = silu(g) * u
  kGeglu = 2,      // columns interleaved value/gate per 16: Y[m, n/2] = v * gelu_erf(g)
  kQkvRope = 3,    // fused-QKV output [rows, 3 Dq] -> fp16 q, k (RMS-normalised, rotated), v
  kScatter = 4,    // fp32 C (+bias) rows stored into their owner rank's slot (ScatterOut)
};
// Operands of Epi::kScatter (tensor parallelism, row-parallel partial outputs). Row r
// belongs to rank o = r / rs; it is stored at row (rank * slot_rows + r - o * rs) of
// base[o], a buffer of rank o mapped into this process (local for o == rank).
struct ScatterOut {
  float* base[8];
  long long slot_rows;
  int rs;
  int rank;
};
// Operands of Epi::kQkvRope. The GEMM output columns are q | k | v, Dq = heads * 128
// each; row r is token r % S of its sequence. Per 128-column head of q and k: RMS norm
// over the head (eps), times gamma, then interleaved rotary pairs (2i, 2i+1) with the
// token's cos / sin row; v is only converted. All three go to fp16 [rows, Dq].
struct QkvRope {
  int S;
  int Dq;
  const float* gq;  // [128] or null (1)
  const float* gk;  // [128] or null (1)
  const float* cs;  // [S, 128]: cos of angle i at 2i and 2i + 1
  const float* sn;  // [S, 128]: -sin of angle i at 2i, +sin at 2i + 1
  float eps;
  void* q16;
  void* k16;
  void* v16;
  int gamma_vec;    // gq and gk 16-byte aligned (set by gemm_bf16_qkv_rope_impl)
};
struct GemmCall {
  int64_t M, N, K;
  const void* A;
  int64_t lda;      // elements
  const void* B;
  int64_t ldb;      // elements
  void* C;
  int64_t ldc;      // elements of the output type
  const float* bias;
  bool accumulate;
  bool tf32;        // operands fp32 (kind::tf32) instead of bf16
  Epi epi;
  bool out_bf16;    // store C as bf16 (ldc in bf16 elements); no accumulate
  int bn;           // 0 = choose
  const QkvRope* rope = nullptr;  // Epi::kQkvRope only (C unused)
  const ScatterOut* scatter = nullptr;  // Epi::kScatter only (C unused, ldc = row length)
};
void launch_gemm_tc(const GemmCall& g);
// Implicit-GEMM convolution (stride 1) on kind::tf32: out NCHW [N, Cout, Ho, Wo] =
// conv(x, w) (+bias[Cout]) (+res, same layout as out). xh is the input in NHWC with a
// channel pitch cp (% 4 == 0; channels past Cin are ignored) and wp the weights as
// [Cout, kh, kw, cq] with cq = round_up(Cin, 32), zero past Cin; both tf32-rounded.
// With stats, the epilogue also writes the output's GroupNorm partial statistics
// (groups of Cout / groups channels, a divisor of 32; Cout % 32 == 0): per (image, group,
// pixel tile) float4 {count, mean, sum of squared deviations, 0} at
// part[(img * groups + g) * tiles_img + tile]; tiles_img is returned. cap is the buffer's
// capacity in float4; N * groups * Ho * ceil(Wo / 32) always suffices.
struct ConvStats {
  float4* part;
  int64_t cap;
  int groups;
  int64_t tiles_img;  // out
};
void launch_conv_tc(const float* xh, int64_t N, int64_t Cin, int64_t cp, int64_t H, int64_t W, const float* wp,
                    int64_t cq, int64_t Cout, int kh, int kw, int pad, const float* bias, const float* res, float* out,
                    int64_t Ho, int64_t Wo, ConvStats* stats = nullptr);
// GroupNorm scale / shift from a convolution's partial statistics (ConvStats):
// ab[n * C + c] = (rstd * gamma[c], beta[c] - mean * rstd * gamma[c]).
void gn_scale_shift_parts(const float4* part, int64_t tiles_img, int64_t N, int64_t C, int groups,
                          const float* gamma, const float* beta, float eps, float2* ab);
// NCHW [N, C, H, W] -> NHWC [N, Ho*Wo, cp] tf32, zero past C, with y = x * a + b per
// channel (ab[n * C + c] = (a, b), or the constants a0, b0 when ab is null), then SiLU if
// silu; with up2 the output is the nearest 2x upsampling (Ho = 2H, Wo = 2W).
void launch_pack_nhwc(const float* x, float* xh, int64_t N, int64_t C, int64_t H, int64_t W, int64_t cp,
                      const float2* ab, float a0, float b0, bool silu, bool up2);
// GroupNorm statistics of x [N, C, HW] as a per-(sample, channel) scale and shift:
// ab[n * C + c] = (rstd * gamma[c], beta[c] - mean * rstd * gamma[c]).
void gn_scale_shift(const float* x, int64_t N, int64_t C, int64_t HW, int groups, const float* gamma,
                    const float* beta, float eps, float2* ab);
// out[i] = sum over s < splits of part[s * total + i] (+ bias[(i / hw) % C]) (+ res[i]):
// the reduction of a split-K convolution (res may alias out).
void launch_split_reduce(const float* part, int splits, int64_t total, int64_t C, int64_t hw, const float* bias,
                         const float* res, float* out);
// The same convolution (square kernel k) as a direct fp32 SIMT kernel, for Cout <= 8.
void launch_conv_direct(const float* xh, int64_t N, int64_t Cin, int64_t cp, int64_t H, int64_t W, const float* wp,
                        int64_t cq, int64_t Cout, int k, int pad, const float* bias, const float* res, float* out,
                        int64_t Ho, int64_t Wo);
// NCHW fp32 [N, C, HW] -> NHWC [N, HW, cp], rounded to tf32, zero in channels C..cp-1.
void launch_conv_pack_x(const float* x, float* xh, int64_t N, int64_t C, int64_t HW, int64_t cp);
// Conv weights [Cout, Cin, taps] -> [Cout, taps, cq], rounded to tf32, zero past Cin.
void launch_conv_pack_w(const float* w, float* wp, int64_t Cout, int64_t Cin, int64_t taps, int64_t cq);
// Forces the tile width of later launch_gemm_tc calls (0 = automatic).
void set_gemm_tile(int bn);
// CTA-pair kernel for bf16 GEMMs and implicit convolutions: 0 never, 1 by the cost model
// (default), 2 whenever the shape allows (tests).
void set_gemm_pair(int mode);
// Enables (default) or disables the implicit-GEMM path of conv2d for stride 1.
void set_conv_implicit(bool on);
// bf16 tcgen05 GEMM on an explicit device / stream / error word; no device context.
void launch_gemm_tc_explicit(const GemmCall& g, int num_sms, cudaStream_t stream, int* err_word, int dev);
// Small-M (M <= 16) GEMM through a memory-bound SIMT kernel (weights streamed once).
void launch_gemm_skinny(int64_t M, int64_t N, int64_t K, const float* A, int64_t lda, const void* B, int64_t ldb,
                        bool b_bf16, float* C, int64_t ldc, const float* bias, bool accumulate);
// The same kernel on an explicit SM count and stream (no device context needed).
void launch_gemm_skinny_on(int64_t M, int64_t N, int64_t K, const float* A, int64_t lda, const void* B, int64_t ldb,
                           bool b_bf16, float* C, int64_t ldc, const float* bias, bool accumulate, int num_sms,
                           cudaStream_t stream);
// Whether (M, K) takes the skinny kernel in gemm_nt_bf16 / gemm_nt_f32.
inline bool skinny_shape(int64_t M, int64_t K) { return M <= 16 && (size_t)(M * K) * 4 <= 160 * 1024; }
// Bounded-wait status word of the no-allocation GEMM (noalloc.cu) on device `dev`: 0 when
// that entry point never ran there; cleared after the read when `clear`.
int noalloc_error_word(int dev, bool clear);

// fp32 [rows, cols] (ld) -> bf16 [rows, cols] (ldo), RNE as the reference rounds.
void launch_pack_bf16(const float* src, int64_t ld, uint16_t* dst, int64_t ldo, int64_t rows, int64_t cols);
// Strided 2-D copy of 16-bit or 32-bit elements into a dense destination.
void launch_copy2d(const void* src, int64_t ld, void* dst, int64_t ldo, int64_t rows, int64_t cols, int esize);
// C[m, n] = bias[n] (or += when accumulate), used when K == 0.
void launch_bias_fill(float* C, int64_t ldc, int64_t M, int64_t N, const float* bias, bool accumulate);

// Layer ops (layers.cu); arguments already validated by the caller.
void launch_pack_tf32(const float* src, int64_t ld, float* dst, int64_t ldo, int64_t rows, int64_t cols);
// launch_pack_tf32 of two matrices with the same column count, in one launch.
void launch_pack_tf32_pair(const float* s0, int64_t ld0, float* d0, int64_t ldo0, int64_t r0, const float* s1,
                           int64_t ld1, float* d1, int64_t ldo1, int64_t r1, int64_t cols);
// x[r, c] rounded to tf32 in place (rows x cols, ld elements apart).
void launch_round_tf32_inplace(float* x, int64_t ld, int64_t rows, int64_t cols);
// GroupNorm over N samples of C channels x HW values (optionally followed by SiLU).
void op_group_norm(const float*, float*, int64_t, int64_t, int64_t, int, const float*, const float*, float,
                   bool silu = false);
void op_row_norm(const float*, float*, int64_t, int64_t, const float*, const float*, float, bool);
void op_rms_norm_heads(float*, int64_t, int64_t, const float*, float);
void op_rope(float*, int64_t, int64_t, int64_t, int64_t, const float*, const float*, bool);
// rope() tables (cos / sin [S, 128], interleaved) -> the Epi::kQkvRope layout (QkvRope::cs / sn).
void op_rope_pair_tables(const float* cos, const float* sin, float* cs, float* sn, int64_t S);
void op_softmax_rows(float*, int64_t, int64_t, float, bool, int64_t);
// Softmax rows ld elements apart; causal row index = row0 + r % rows_per_head; with
// round_out the probabilities are stored rounded to tf32.
void op_softmax_rows_ex(float* x, int64_t rows, int64_t cols, int64_t ld, float scale, bool causal,
                        int64_t rows_per_head, int64_t row0, bool round_out);
// dst[c, r] = tf32(src[r, c]), rows x cols.
void launch_transpose_tf32(const float* src, int64_t ld_src, float* dst, int64_t ld_dst, int64_t rows, int64_t cols);
// tf32 tensor-core GEMM on operands already rounded to tf32, 16-byte aligned, with
// leading dimensions that are multiples of 4: C[M,N] = A[M,K] B[N,K]^T (+bias) (+C).
void gemm_tf32_direct(int64_t M, int64_t N, int64_t K, const float* A, int64_t lda, const float* B, int64_t ldb,
                      float* C, int64_t ldc, const float* bias, bool acc);
// Attention for any head dim as GEMM -> softmax -> GEMM on tf32 tensor cores. Row strides
// (elements) default to heads * d for q / out and kv_heads * d for k / v; a sample's rows
// are contiguous (sample stride = rows * stride). qk_tf32: q and k already hold values on
// the tf32 grid (read in place instead of repacked).
void launch_attention_gemm(const float* q, const float* k, const float* v, float* out, int64_t N, int64_t Sq,
                           int64_t Skv, int heads, int kv_heads, int64_t d, bool causal, int64_t q_ld = 0,
                           int64_t kv_ld = 0, int64_t o_ld = 0, bool qk_tf32 = false);
void op_geglu(const float*, float*, int64_t, int64_t);
void op_swiglu(const float*, const float*, float*, int64_t);
void op_unary(float*, int64_t, int);  // 0 silu, 1 gelu (erf), 2 quick_gelu, 3 tanh
void op_add(float*, const float*, int64_t);
void op_affine(float*, float, float, int64_t);
void op_mul_rows(float*, const float*, int64_t, int64_t);
void op_add_rows_scaled(float*, const float*, const float*, int64_t, int64_t);
void op_add_channel_bias(float*, const float*, int64_t, int64_t, int64_t);
void op_add_bias_rows(float*, int64_t, int64_t, int64_t, const float*);
void op_upsample2x(const float*, float*, int64_t, int64_t, int64_t);
void op_concat_channels(const float*, const float*, float*, int64_t, int64_t, int64_t, int64_t);
void op_nchw_to_nlc(const float*, float*, int64_t, int64_t, int64_t);
void op_nlc_to_nchw(const float*, float*, int64_t, int64_t, int64_t);
void op_patchify(const float*, float*, int64_t, int64_t, int64_t, int);
void op_unpatchify(const float*, float*, int64_t, int64_t, int64_t, int);
void op_im2col(const float*, float*, int64_t, int64_t, int64_t, int64_t, int64_t, int64_t, int, int, int64_t, int64_t,
               int64_t, int64_t);
void set_last_error(const std::string& s);

// ---- tensor-parallel communicator (comm.cu) ----
struct Comm;
constexpr int kMaxTpRanks = 8;
// A device buffer of the same size on every rank of a communicator, with every peer's
// copy mapped into this process (peer[rank] == local).
struct SymBuf {
  void* local = nullptr;
  void* peer[kMaxTpRanks] = {};
  size_t bytes = 0;
};
void comm_allreduce_sum(Comm* c, float* buf, size_t n);
int comm_world(const Comm* c);
int comm_rank(const Comm* c);
void comm_barrier(Comm* c);
void comm_barrier_nccl_sync(Comm* c);
void comm_allgather(Comm* c, const void* send, void* recv, size_t bytes);
void comm_sym_alloc(Comm* c, SymBuf& b, size_t bytes);
void comm_sym_free(Comm* c, SymBuf& b);

// Caching allocator (runtime.cu).
void* pool_malloc(size_t bytes);
void pool_free(void* p);

// Packed-operand cache (operand_cache.cu, opt-in): tf32-rounded GEMM weights and conv
// weight slabs kept across calls, dropped when their source is freed or overwritten through
// this library.
bool operand_cache_on();
void operand_cache_enable(bool on);
int64_t operand_cache_entries();
void operand_cache_invalidate(const void* p, size_t bytes);
// B [rows, cols] (ld) rounded to tf32 with row pitch ldo; packed on the first call.
const float* cached_tf32_rows(const float* B, int64_t rows, int64_t cols, int64_t ld, int64_t ldo);
// Conv weights [Cout, Cin, taps] as [Cout, taps, cq] tf32; packed on the first call.
const float* cached_conv_weight(const float* w, int64_t Cout, int64_t Cin, int64_t taps, int64_t cq);

// GEMM front-ends with argument checks (ops_api.cu).
void gemm_nt_bf16_impl(int64_t M, int64_t N, int64_t K, const float* A, int64_t lda, const uint16_t* B, int64_t ldb,
                       float* C, int64_t ldc, const float* bias, bool acc);
// b_constant: B is a caller's weight buffer that the opt-in operand cache may keep packed
// (the C-ABI entry only; internal callers pass activations or scratch as B).
void gemm_nt_f32_impl(int64_t M, int64_t N, int64_t K, const float* A, int64_t lda, const float* B, int64_t ldb,
                      float* C, int64_t ldc, const float* bias, bool acc, bool b_constant = false);
void gemm_bf16_scatter_impl(int64_t M, int64_t N, int64_t K, const void* A, int64_t lda, bool a_bf16, const uint16_t* B,
                            int64_t ldb, const float* bias, const ScatterOut& so);
void gemm_bf16_qkv_rope_impl(int64_t M, int64_t K, const void* A, int64_t lda, bool a_bf16, const uint16_t* B,
                             int64_t ldb, const float* bias, const QkvRope& r);
void gemm_bf16_epilogue_impl(int64_t M, int64_t N, int64_t K, const void* A, int64_t lda, bool a_bf16,
                             const uint16_t* B, int64_t ldb, void* Y, int64_t ldy, bool y_bf16, const float* bias,
                             int epi);

// DiT glue kernels (dit_ops.cu).
void dit_rms_mod_bf16(const float* x, uint16_t* h, int64_t rows, int D, const float* gamma, const float* scale,
                      float eps);
void dit_post_norm_residual(float* x, const float* a, int64_t rows, int D, const float* gamma, const float* g,
                            float eps);
// Tensor-parallel post-norm of rows [row0, row0 + rows): sums the world partial slots,
// updates x, and (nh > 0) stores the next GEMM's bf16 input row into nh buffers.
// x += dt * (out (+ cfg (out - neg) when neg != null)) over n values.
void dit_flow_step(float* x, const float* out, const float* neg, float cfg, float dt, int64_t n);
void dit_post_norm_mod_bcast(const float* slots, int64_t slot_rows, int world, int64_t row0, int64_t rows, float* x,
                             int D, const float* gamma2, const float* g, const float* gamma_n, const float* scale_n,
                             uint16_t* const* hdst, int nh, float eps);
void dit_adaln_split(float* mod, int D);
void dit_timestep_embed(float* out, int F, float tt);
void dit_layer_norm_mod(const float* x, float* y, int64_t rows, int D, const float* scale, float eps);
void dit_fill_rows(float* y, const float* src, int64_t r0, int64_t r1, int D);
void dit_interleave_rows16(const void* a, const void* b, void* out, int64_t rows, int64_t cols, int esize);

// Attention (attention.cu).
void launch_attention(const float* q, const float* k, const float* v, float* out, int64_t N, int64_t Sq, int64_t Skv,
                      int heads, int kv_heads, int64_t d, bool causal);
// Tensor-core attention on fp16 operands laid out [N, S, heads, dp] (dp = 64 or 128,
// zero padded); out rows are out_row elements apart, samples out_batch apart; out is
// fp32 or bf16.
void launch_attention_f16(const void* q, const void* k, const void* v, void* out, long long out_row,
                          long long out_batch, bool out_bf16, int64_t N, int64_t Sq, int64_t Skv, int heads,
                          int kv_heads, int64_t d, int64_t dp, bool causal);
// fp32 [rows, H*d] -> fp16 [rows, H, dp], zero padded.
void launch_pack_heads_f16(const float* x, void* y, int64_t rows, int H, int64_t d, int64_t dp);
// Selects the tensor-core attention (true, default) or the exact fp32 kernel.
void set_attention_tc(bool on);

}  // namespace sdb
