/* sdb200.h - C ABI of the B200 (sm_100a) backend for StableDiffusion-cpp's dense
 * contraction path.
 *
 * Every entry point takes plain device pointers, sizes in elements and leading
 * dimensions in elements, exactly like the reference backend API
 * (src/backend_cuda.h, namespace sd::cuda); the comment above each declaration names
 * the reference function it replaces as "backend_cuda.h:<line>". The same shared
 * library also exports the reference's C++ symbols (sd::cuda::gemm_nt_bf16, ...) with
 * identical signatures, so the reference's `make CUDA=1` link line can take
 * libsdb200.so in place of build/backend_cuda.o; those C++ wrappers call the functions
 * below and throw std::runtime_error(message) on a non-zero status, as the reference
 * does (backend_cuda.cu:41-48).
 *
 * Conventions
 *   - Row-major; C[M,N] = A[M,K] * B[N,K]^T (+ bias[N]) (+ C when accumulate != 0).
 *   - M <= 0 or N <= 0 is a no-op (backend_cuda.cu:455, :464).
 *   - bf16 values are uint16_t bit patterns: the top 16 bits of an IEEE float
 *     (tensor.h:43-45, :137-142).
 *   - Every op is enqueued on the current device's stream (sdb200_set_stream; default
 *     the legacy default stream) and returns without synchronising, except
 *     sdb200_download and sdb200_synchronize.
 *   - Return value: 0 on success, otherwise an SDB200_ERR_* code; the message of the
 *     last failure on the calling thread is returned by sdb200_last_error().
 *   - Thread model: one host thread (or process) per GPU. Calls for one device must
 *     not run concurrently from several threads on the same stream's workspace.
 */
#ifndef SDB200_H
#define SDB200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define SDB200_ABI_VERSION 1

#define SDB200_OK 0
#define SDB200_ERR_INVALID_ARG 1 /* bad size, leading dimension, alignment or null pointer */
#define SDB200_ERR_NO_DEVICE 2
#define SDB200_ERR_CUDA 3        /* a CUDA runtime call failed */
#define SDB200_ERR_DEVICE_WAIT 4 /* a kernel's bounded wait expired; see sdb200_device_error_word */
#define SDB200_ERR_OUT_OF_MEMORY 5
#define SDB200_ERR_UNSUPPORTED 6

/* ---- library / device ---------------------------------------------------------- */
int sdb200_version(void);
/* Number of kernels this library has launched in this process (all devices). */
unsigned long long sdb200_launch_count(void);
const char* sdb200_last_error(void);
/* backend_cuda.h:24 available(): 1 if a B200-class (sm_100) device is usable. */
int sdb200_available(void);
int sdb200_device_count(void);
/* backend_cuda.h:26 device_name() */
const char* sdb200_device_name(void);
/* backend_cuda.h:27 device_memory() */
size_t sdb200_device_memory(void);
/* Extension (the reference hard-wires device 0, backend_cuda.cu:64-72): selects the
 * calling thread's device. */
int sdb200_set_device(int device);
/* Extension (the reference uses the default stream only, backend_cuda.cu:10-11):
 * every later op of the current device is issued on `stream` (a cudaStream_t). */
int sdb200_set_stream(void* stream);
void* sdb200_get_stream(void);
/* Synchronises the stream, then reads the device error word that kernels set when a
 * bounded wait expires (0 = none) without clearing it. Bits: 1-16 GEMM / convolution
 * pipeline waits, 32 attention pipeline, 64 tensor-parallel barrier (a peer rank did not
 * arrive). */
int sdb200_device_error_word(int* out);

/* ---- memory (backend_cuda.h:29-36) --------------------------------------------- */
/* backend_cuda.h:30 malloc(): size-class caching allocator; NULL on failure. */
void* sdb200_malloc(size_t bytes);
/* backend_cuda.h:31 free() */
int sdb200_free(void* p);
/* backend_cuda.h:32 upload() host -> device (stream-ordered) */
int sdb200_upload(void* dst, const void* src, size_t bytes);
/* backend_cuda.h:33 download() device -> host; synchronises */
int sdb200_download(void* dst, const void* src, size_t bytes);
/* backend_cuda.h:34 copy() device -> device */
int sdb200_copy(void* dst, const void* src, size_t bytes);
/* backend_cuda.h:35 zero() */
int sdb200_zero(void* dst, size_t bytes);
/* backend_cuda.h:36 synchronize(); also reports an expired device wait as
 * SDB200_ERR_DEVICE_WAIT (and clears the error word). */
int sdb200_synchronize(void);

/* ---- GEMM (the hot path) ------------------------------------------------------- */
/* backend_cuda.h:39-40 gemm_nt_f32(): fp32 weights. Both operands are rounded to tf32
 * (nearest even) and multiplied on tcgen05 kind::tf32 with fp32 accumulation; M <= 16
 * uses an exact fp32 memory-bound kernel. */
int sdb200_gemm_nt_f32(int64_t M, int64_t N, int64_t K, const float* A, int64_t lda, const float* B, int64_t ldb,
                       float* C, int64_t ldc, const float* bias, int accumulate);
/* backend_cuda.h:42-43 gemm_nt_bf16(): bf16 weights; A is rounded to bf16 (nearest
 * even, as backend_cuda.cu:466-467 does) and multiplied on tcgen05 kind::f16 with fp32
 * accumulation in TMEM; M <= 16 uses an exact fp32-A memory-bound kernel. */
int sdb200_gemm_nt_bf16(int64_t M, int64_t N, int64_t K, const float* A, int64_t lda, const uint16_t* B,
                        int64_t ldb, float* C, int64_t ldc, const float* bias, int accumulate);
/* Extension of backend_cuda.h:42-43 for producers that already emit bf16 activations:
 * A is bf16 [M, lda]. */
int sdb200_gemm_nt_bf16a(int64_t M, int64_t N, int64_t K, const uint16_t* A, int64_t lda, const uint16_t* B,
                         int64_t ldb, float* C, int64_t ldc, const float* bias, int accumulate);

/* Extension (opt-in; the reference repacks nothing, its cuBLAS calls read fp32 weights
 * directly): keep the packed form of constant operands across calls - the tf32-rounded B of
 * gemm_nt_f32 and the [Cout, tap, Cin] slab of conv2d's stride-1 weights - instead of
 * repacking them on every call. While it is on, such an operand must not change while it
 * stays allocated, except through sdb200_upload / sdb200_copy / sdb200_zero, which drop the
 * entries they overwrite; sdb200_free drops the entries of the freed buffer. Buffers from
 * another allocator are not tracked: turn the cache off (which clears it) before freeing or
 * rewriting them. Only the C-ABI gemm_nt_f32 / conv2d calls use it. Default: off, or on when
 * the environment variable SDB200_OPERAND_CACHE=1 is set (so an unmodified caller of the
 * sd::cuda symbols can use it). Turning it off frees every entry. */
int sdb200_set_operand_cache(int enable);
/* Number of packed operands currently kept (tests). */
int64_t sdb200_operand_cache_entries(void);

/* Extension: the activation rounding of gemm_nt_bf16 on its own (the pack kernel it runs
 * before the tensor-core GEMM, backend_cuda.cu:183-188 / tensor.cpp:114-121: nearest
 * even, inf and NaN truncated). src fp32 [rows, ld] -> dst bf16 bit patterns [rows, ldo],
 * stream-ordered. Lets a caller round A once and reuse it through gemm_nt_bf16a. */
int sdb200_pack_bf16(const float* src, int64_t ld, uint16_t* dst, int64_t ldo, int64_t rows, int64_t cols);

/* No counterpart in the reference. The gemm_nt_bf16 contraction above (same kernels,
 * bit-identical results; M <= 16 takes the same exact fp32-A kernel) for callers that
 * cannot allocate device memory: hosts whose framework owns every device allocation
 * through its own pool, and loops that must never reach cudaMalloc/cudaFree (a cudaFree
 * synchronises the device). sdb200_gemm_nt_bf16 may grow a workspace and create a
 * device context (both cudaMalloc); this entry point calls no allocator. A's bf16 copy
 * goes to a fixed 32 MiB device array held by every GPU that loads the library:
 * M * round_up(K, 8) <= 16,777,216, and B must be 16-byte aligned with ldb % 8 == 0, else
 * SDB200_ERR_INVALID_ARG. The first call on a device resolves the array's address
 * (cudaGetSymbolAddress); make it before any stream capture. It runs on the stream set by
 * sdb200_set_stream when a context exists, else on the legacy default stream. All calls
 * share the array; calls that overlap on the GPU race on it. A bounded-wait expiry is
 * reported by sdb200_device_error_word / sdb200_synchronize. */
int sdb200_gemm_nt_bf16_noalloc(int64_t M, int64_t N, int64_t K, const float* A, int64_t lda, const uint16_t* B,
                                int64_t ldb, float* C, int64_t ldc, const float* bias, int accumulate);

/* Fused-epilogue GEMM (extension; the reference runs these as separate kernels after
 * the GEMM: swiglu backend_cuda.h:61, geglu :60, bias backend_cuda.cu:239-241).
 *   epi 0: Y = A B^T + bias (fp32 or bf16 Y)
 *   epi 1: SwiGLU. B rows are interleaved in blocks of 16: rows [32j, 32j+16) are gate
 *          rows, [32j+16, 32j+32) the matching up rows; Y[m, 16j+i] = silu(g) * u.
 *          Y has N/2 columns.
 *   epi 2: GEGLU with the same interleave; Y = value * gelu_erf(gate).
 * A is bf16 when a_bf16 != 0, else fp32 (rounded to bf16). y_bf16 != 0 stores Y as
 * bf16 (ldy in bf16 elements). */
int sdb200_gemm_bf16_epilogue(int64_t M, int64_t N, int64_t K, const void* A, int64_t lda, int a_bf16,
                              const uint16_t* B, int64_t ldb, void* Y, int64_t ldy, int y_bf16, const float* bias,
                              int epi);

/* Fused-QKV projection (extension; the reference runs these as separate calls for each of
 * q, k, v: linear, rms_norm_heads, rope, zimage.cpp:113-120): Y = X Wqkv^T (+ bias) with
 * Wqkv [3 Dq, K] bf16, rows q | k | v, Dq = heads * 128. Then, per 128-wide head of q and
 * of k, the RMS norm with eps times gamma (gq / gk, [128] each, or null for 1) and the
 * interleaved rotary embedding of rope(): pair (2i, 2i+1) of row m rotated by
 * cos[m % S][2i] / sin[m % S][2i] (cos, sin [S, 128]). q, k and v are stored as fp16
 * [M, Dq] (q16, k16, v16, 16-byte aligned), the attention operand layout of
 * sdb200_attention_f16 with dp = 128. X is bf16 when x_bf16 != 0, else fp32 (rounded to
 * bf16 as gemm_nt_bf16 does). */
int sdb200_gemm_bf16_qkv_rope(int64_t M, int64_t K, const void* X, int64_t ldx, int x_bf16, const uint16_t* Wqkv,
                              int64_t ldw, const float* bias, int64_t Dq, int64_t S, const float* cos, const float* sin,
                              const float* gq, const float* gk, float eps, void* q16, void* k16, void* v16);

/* The DiT block's post-norm step (extension; the reference runs these as separate calls,
 * zimage.cpp:122-126 / :131-135 and the next block's :113-115), one row per output row:
 *   a  = sum over s < world of partials[(s * slot_rows + r) * D + :]  (row-parallel parts)
 *   x[row0 + r] += gate * (rms_norm(a, eps) * gamma2)   (gate, gamma2 [D] or null for 1)
 *   h  = bf16(rms_norm(x[row0 + r], eps) * gamma_next * scale_next)   (each [D] or null)
 * h is stored at row row0 + r of each of the n_dst buffers h_dst[i] (n_dst = 0: no h; else
 * n_dst = world, the tensor-parallel ranks' copies). x and h are [*, D] with row pitch D. */
int sdb200_dit_post_norm(const float* partials, int64_t slot_rows, int world, int64_t row0, int64_t rows, float* x,
                         int64_t D, const float* gamma2, const float* gate, const float* gamma_next,
                         const float* scale_next, uint16_t* const* h_dst, int n_dst, float eps);

/* Tuning extension (no reference counterpart): forces the GEMM tile width N (64, 128,
 * 192 or 256) for later calls of this process; 0 restores the automatic choice. */
int sdb200_set_gemm_tile(int bn);
/* Tuning extension (no reference counterpart): bf16 GEMMs with 256-wide tiles and
 * implicit-GEMM convolutions with >= 256 output channels may run on pairs of SMs with
 * 256 x 256 tiles (M = 256 MMAs over a cluster of two CTAs). enable: 0 never, 1 when the
 * wave-count cost model prefers them (default), 2 whenever the shape allows. */
int sdb200_set_gemm_pair(int enable);
/* Tuning extension (no reference counterpart): stride-1 conv2d runs as an implicit GEMM
 * over an NHWC copy of the input when enable != 0 (default), as im2col + GEMM otherwise
 * (the reference's lowering, backend_cuda.cu:479-510). */
int sdb200_set_conv_implicit(int enable);

/* ---- attention ------------------------------------------------------------------- */
/* backend_cuda.h:58-59 attention(): q [N, Sq, heads*d]; k, v [N, Skv, kv_heads*d];
 * out [N, Sq, heads*d]; softmax(q k^T / sqrt(d)) v per head, query head h reads kv
 * head h / (heads / kv_heads); causal keeps keys j <= query row i. Head dims <= 128 run
 * on the flash kernel (fp16 operands), larger ones as tf32 GEMM -> softmax -> tf32 GEMM
 * in query-row chunks (the reference GPU backend's scheme on tensor cores). Skv = 0 gives
 * a zero output (the reference's empty score matrix times V); N = 0 or Sq = 0 does nothing. */
int sdb200_attention(const float* q, const float* k, const float* v, float* out, int64_t N, int64_t Sq, int64_t Skv,
                     int heads, int kv_heads, int64_t d, int causal);

/* Extension of backend_cuda.h:58-59 for producers that already emit fp16 operands:
 * q [N, Sq, heads, dp], k/v [N, Skv, kv_heads, dp] fp16 (dp = 64 for d <= 64, else 128,
 * zero padded beyond d); out [N, Sq, heads*d] fp32, or bf16 when out_bf16 != 0. Skv = 0
 * gives a zero output. */
int sdb200_attention_f16(const void* q, const void* k, const void* v, void* out, int out_bf16, int64_t N, int64_t Sq,
                         int64_t Skv, int heads, int kv_heads, int64_t d, int64_t dp, int causal);
/* fp32 x [rows, heads*d] -> fp16 y [rows, heads, dp] (zero padded, |x| > 65504 saturates). */
int sdb200_pack_heads_f16(const float* x, void* y, int64_t rows, int heads, int64_t d, int64_t dp);
/* Extension (no reference counterpart): 0 = tensor-core attention (flash kernel on fp16
 * operands for head dims <= 128, tf32 GEMMs above), 1 = exact fp32 streaming kernel.
 * Applies to later sdb200_attention calls of this process. */
int sdb200_set_attention_path(int path);

/* ---- Z-Image DiT forward (zimage.h:56 ZImageTransformer::forward) ------------------
 * The whole transformer on the device: create with the Config values of zimage.h:40-47,
 * register every weight (device pointer, dtype, shape) under its checkpoint name
 * (zimage.cpp:38-67), finalize (builds the fused QKV / interleaved w1-w3 weights the
 * model owns; the caller keeps the registered buffers alive), then call forward. x is
 * [B, C, H, W] fp32, cap [B, L, capdim] fp32, out [B, C, H, W] fp32, all on the device;
 * the B images share the timestep t (the reference forward is batch 1, zimage.cpp:140).
 * Block linears must be bf16; head dim must be 128. */
void* sdb200_zimage_create(int heads, int patch, float norm_eps, float rope_theta, float t_scale, int ax0, int ax1,
                           int ax2);
int sdb200_zimage_set_weight(void* model, const char* name, const void* dev_ptr, int is_bf16, const int64_t* shape,
                             int ndim);
int sdb200_zimage_finalize(void* model);
int sdb200_zimage_forward(void* model, const float* x, int64_t B, int64_t C, int64_t H, int64_t W, float t,
                          const float* cap, int64_t L, int64_t capdim, float* out);
void sdb200_zimage_destroy(void* model);
/* Per-kernel timing of later forwards with CUDA events on the stream (enable != 0).
 * profile_read fills out10 = {GEMM ms, GEMM FLOP, GEMM launches, attention ms, attention
 * FLOP, attention launches, forward ms, forwards, all-reduce ms, all-reduces} since the
 * last read, synchronising. */
int sdb200_zimage_profile(void* model, int enable);
int sdb200_zimage_profile_read(void* model, double* out10);
/* The same record with the memory-bound kernels (n <= 16 values): out[0..10) as above,
 * then post-norm ms, post-norm bytes, post-norm launches, adaLN GEMV ms, adaLN GEMV bytes,
 * adaLN GEMV launches; bytes are the algorithmic minimum (inputs read once, outputs
 * written once). */
int sdb200_zimage_profile_read_ex(void* model, double* out, int n);
/* Extension (the reference has no multi-GPU mode): Megatron-style tensor parallelism.
 * The caller registers this rank's shards (to_q/to_k/to_v rows and to_out columns of its
 * heads, w1/w3 rows and w2 columns of its FFN slice, row-parallel biases on rank 0 only)
 * and attaches a communicator (NULL detaches; also releases the peer mappings). Every
 * rank of the group must then call zimage_forward with the same shapes. */
int sdb200_zimage_set_tp(void* model, void* comm);
/* How the row-parallel outputs of to_out and w2 are combined (default 1):
 *   1  fused: the GEMM epilogue stores each partial row into the owner rank's memory
 *      over NVLink (CUDA IPC mappings), the owner sums them in its post-norm kernel on
 *      its share of the rows and stores the next GEMM's bf16 input row on every rank;
 *      NCCL only orders the steps (4-byte barrier) and gathers x at the end of a stage.
 *      On one GPU the same kernels run with local stores (post-norm and the next
 *      RMSNorm + modulation in one pass)
 *   0  per-block form: separate post-norm and RMSNorm kernels, and under tensor
 *      parallelism an NCCL all-reduce of the full fp32 partial outputs */
int sdb200_zimage_set_tp_mode(void* model, int mode);
/* Extension (pipeline.cpp:229-244 runs this loop on the host, one device round trip per
 * step): the flow-matching Euler sampler of the Z-Image pipeline on the device. x
 * [B, C, H, W] (device fp32) is the initial noise on entry and the denoised latent on
 * return; per step i the model runs at time 1 - sigma_i on cap (and on cap_neg when
 * cfg > 0, prediction = out + cfg (out - neg)), then x += (sigma_i - sigma_(i+1)) *
 * prediction. steps >= 1; shift is the schedule's shift (3 for Z-Image). */
int sdb200_zimage_sample(void* model, float* x, int64_t B, int64_t C, int64_t H, int64_t W, const float* cap,
                         const float* cap_neg, int64_t L, int64_t capdim, float cfg, int steps, float shift);
/* Extension (the reference loads the whole checkpoint on every process and has no
 * tensor parallelism): registers the weights of the checkpoint <dir>/<base> (found as
 * Weights::load_model finds it: <base>.safetensors, the shards of
 * <base>.safetensors.index.json, or <base>.fp16.safetensors) into device memory the
 * model owns, read as the reference reads them (safetensors.cpp:80-168; tensors of at
 * least bf16_min_numel elements kept as BF16, 1 << 20 when <= 0, smaller ones as F32).
 * With world > 1 only this rank's tensor-parallel shard of every block tensor is read
 * and uploaded (the layout sdb200_zimage_set_tp expects). Call before
 * sdb200_zimage_finalize. */
int sdb200_zimage_load(void* model, const char* dir, const char* base, int rank, int world, int64_t bf16_min_numel);
/* Host only: one tensor of a .safetensors file converted as above into dst (BF16 bit
 * patterns when *is_bf16, else F32); shape[0..*ndim) receives its shape (at most 8
 * dims). dst may be NULL to query the shape and dtype. */
int sdb200_safetensors_read(const char* path, const char* name, int keep_bf16, int64_t bf16_min_numel, void* dst,
                            int64_t dst_bytes, int64_t* shape, int* ndim, int* is_bf16);
/* Host only (extension of safetensors.cpp:80-194 / pipeline.cpp:113-115, which read the
 * whole checkpoint on every process): the tensor `name` of the checkpoint <dir>/<base>
 * exactly as sdb200_zimage_load uploads it for `rank` of `world` with `heads` attention
 * heads - the same file lookup, dtype rule and Megatron cut. *ndim = -1 when this rank
 * holds no part of it (a row-parallel bias on rank > 0) or its dtype is not read. dst may
 * be NULL to query the shape and dtype. */
int sdb200_checkpoint_read_shard(const char* dir, const char* base, const char* name, int rank, int world, int heads,
                                 int64_t bf16_min_numel, void* dst, int64_t dst_bytes, int64_t* shape, int* ndim,
                                 int* is_bf16);
/* Extension: copies the weight `name` registered in the model (sdb200_zimage_set_weight
 * or sdb200_zimage_load) to host memory dst (BF16 bit patterns when *is_bf16, else F32);
 * synchronises. dst may be NULL to query the shape and dtype. */
int sdb200_zimage_get_weight(void* model, const char* name, void* dst, int64_t dst_bytes, int64_t* shape, int* ndim,
                             int* is_bf16);
/* FlowMatchScheduler::set_timesteps (scheduler.cpp:117-127) on the host: sigmas[0..steps],
 * bit-identical to the reference's values. */
int sdb200_flow_sigmas(int steps, float shift, float* sigmas);

/* ---- the VAE decoder on the device (vae.cpp:13-51) ------------------------------- */
/* Extension (no reference counterpart): AutoencoderKL decode as one device program on the
 * implicit-GEMM convolution, with GroupNorm + SiLU, upsampling, the latent un-scaling and
 * residual adds folded into the convolutions' operand packing and epilogues.
 *   vae_create:     scaling_factor / shift_factor from the VAE's config.json
 *   vae_set_weight: fp32 device tensors under the checkpoint names ("decoder.*",
 *                   "post_quant_conv.*"); the caller keeps them alive
 *   vae_load:       or read <dir>/<base>.safetensors (or its shards) as fp32, as
 *                   Weights::load_model does for the VAE (pipeline.cpp:86)
 *   vae_finalize:   binds the layers (block counts and widths from the names, as the
 *                   VAEDecoder constructor, vae.cpp:15-32) and packs the conv weights
 *   vae_decode:     latents [N, C, h, w] (device) -> out [N, 3, h * upscale, w * upscale]
 * Returns NULL / a status code; the decoder owns its activation buffers. */
void* sdb200_vae_create(float scaling_factor, float shift_factor);
int sdb200_vae_set_weight(void* m, const char* name, const float* dev_ptr, const int64_t* shape, int ndim);
int sdb200_vae_load(void* m, const char* dir, const char* base);
int sdb200_vae_finalize(void* m);
int sdb200_vae_info(void* m, int64_t* latent_channels, int64_t* out_channels, int64_t* upscale);
int sdb200_vae_decode(void* m, const float* latents, int64_t N, int64_t C, int64_t h, int64_t w, float* out);
/* Tuning extension: CUDA-event timing of later decodes (on != 0); profile_read returns
 * conv ms, conv FLOPs, conv launches, attention ms, attention FLOPs and clears. */
int sdb200_vae_profile(void* m, int on);
int sdb200_vae_profile_read(void* m, double* out5);
void sdb200_vae_destroy(void* m);

/* ---- tensor-parallel communicator (NCCL over NVLink / NVSwitch, loaded at run time) -- */
/* Writes a 128-byte unique id (on one rank; share it with the others out of band). */
int sdb200_comm_unique_id(void* out128);
/* Joins the group as `rank` of `world` on the current device; NULL on failure. */
void* sdb200_comm_create(const void* unique_id128, int rank, int world);
/* In-place sum all-reduce of n fp32 values on the current device's stream. */
int sdb200_comm_allreduce_sum_f32(void* comm, float* buf, size_t n);
/* Extension: the stream-ordered barrier between the fused tensor-parallel kernels is a
 * flag exchange over NVLink (flags != 0, default) or a 4-byte NCCL all-reduce (0). Every
 * rank of the group sets the same. */
int sdb200_comm_set_barrier(void* comm, int flags);
/* Extension, self-test of that barrier on one device: `flags` is a device array of `world`
 * uint32 words standing for every rank's flag words at once. The kernel stores `epoch` into
 * word `rank` and waits until every word is >= epoch. A word that never gets there makes
 * the wait run out after its 2 s bound: the device error word then holds bit 64 and the
 * next sdb200_synchronize returns SDB200_ERR_DEVICE_WAIT. Stream-ordered. */
int sdb200_comm_barrier_selftest(uint32_t* flags, int world, int rank, uint32_t epoch);
void sdb200_comm_destroy(void* comm);

/* ---- layers (backend_cuda.h:45-61) ---------------------------------------------- */
/* backend_cuda.h:46-47 conv2d(): x NCHW [N, Cin, H, W], w [Cout, Cin, kh, kw], out NCHW
 * [N, Cout, Ho, Wo], tf32 tensor cores. Stride 1 runs as an implicit GEMM over an NHWC
 * copy of x (workspace), or for Cout <= 8 as a direct fp32 kernel over the same copy;
 * other strides as im2col + GEMM. */
int sdb200_conv2d(const float* x, int64_t N, int64_t Cin, int64_t H, int64_t W, const float* w, int64_t Cout,
                  int64_t kh, int64_t kw, const float* bias, int stride, int pad, float* out, int64_t Ho, int64_t Wo);
/* Extension (no reference counterpart): the implicit-GEMM convolution on operands already
 * in its layouts, for callers that keep activations channels-last.
 *   conv_pack_input:  x NCHW [N, C, HW] -> xh NHWC [N, HW, cp], tf32-rounded, cp % 4 == 0,
 *                     zero in channels C..cp-1
 *   conv_pack_weight: w [Cout, Cin, taps] -> wp [Cout, taps, cq], tf32-rounded,
 *                     cq = round_up(Cin, 32), zero past Cin
 *   conv2d_nhwc:      out NCHW = conv(xh, wp) (+bias[Cout]) (+res, same layout as out),
 *                     stride 1, zero padding pad; xh and wp 16-byte aligned. */
int sdb200_conv_pack_input(const float* x, float* xh, int64_t N, int64_t C, int64_t HW, int64_t cp);
int sdb200_conv_pack_weight(const float* w, float* wp, int64_t Cout, int64_t Cin, int64_t taps, int64_t cq);
int sdb200_conv2d_nhwc(const float* xh, int64_t N, int64_t Cin, int64_t cp, int64_t H, int64_t W, const float* wp,
                       int64_t cq, int64_t Cout, int64_t kh, int64_t kw, int pad, const float* bias, const float* res,
                       float* out, int64_t Ho, int64_t Wo);
/* backend_cuda.h:48-49 group_norm(): split statistics (chunk mean and squared deviations
 * combined in double per group), then y = x * a[c] + b[c]. */
int sdb200_group_norm(const float* x, float* y, int64_t N, int64_t C, int64_t HW, int groups, const float* gamma,
                      const float* beta, float eps);
/* backend_cuda.h:50 layer_norm() */
int sdb200_layer_norm(const float* x, float* y, int64_t rows, int64_t C, const float* gamma, const float* beta,
                      float eps);
/* backend_cuda.h:51 rms_norm() */
int sdb200_rms_norm(const float* x, float* y, int64_t rows, int64_t C, const float* gamma, float eps);
/* backend_cuda.h:52 rms_norm_heads() (in place) */
int sdb200_rms_norm_heads(float* x, int64_t groups, int64_t dim, const float* gamma, float eps);
/* backend_cuda.h:54-55 rope() (in place): x [N, S, inner]; cos/sin [S, dim] */
int sdb200_rope(float* x, int64_t N, int64_t S, int64_t inner, int64_t dim, const float* cos, const float* sin,
                int interleaved);
/* backend_cuda.h:56 softmax_rows() (in place) */
int sdb200_softmax_rows(float* x, int64_t rows, int64_t cols, float scale, int causal);
/* backend_cuda.h:60 geglu(): x [rows, 2D] -> y [rows, D] */
int sdb200_geglu(const float* x, float* y, int64_t rows, int64_t D);
/* backend_cuda.h:61 swiglu() */
int sdb200_swiglu(const float* gate, const float* up, float* y, int64_t n);

/* ---- elementwise / shape (backend_cuda.h:64-80) --------------------------------- */
int sdb200_silu(float* x, int64_t n);                       /* backend_cuda.h:64 */
int sdb200_tanh(float* x, int64_t n);                       /* backend_cuda.h:65 */
int sdb200_gelu(float* x, int64_t n);                       /* backend_cuda.h:66 */
int sdb200_quick_gelu(float* x, int64_t n);                 /* backend_cuda.h:67 */
int sdb200_add(float* a, const float* b, int64_t n);        /* backend_cuda.h:68 */
int sdb200_scale(float* x, float s, int64_t n);             /* backend_cuda.h:69 */
int sdb200_affine(float* x, float a, float b, int64_t n);   /* backend_cuda.h:70 */
int sdb200_mul_rows(float* x, const float* v, int64_t rows, int64_t dim);                      /* backend_cuda.h:71 */
int sdb200_add_rows_scaled(float* x, const float* y, const float* g, int64_t rows, int64_t dim); /* backend_cuda.h:72 */
int sdb200_add_channel_bias(float* x, const float* b, int64_t N, int64_t C, int64_t HW);        /* backend_cuda.h:73 */
int sdb200_upsample_nearest2x(const float* x, float* y, int64_t NC, int64_t H, int64_t W);      /* backend_cuda.h:74 */
int sdb200_concat_channels(const float* a, const float* b, float* y, int64_t N, int64_t Ca, int64_t Cb,
                           int64_t HW);                                                          /* backend_cuda.h:75 */
int sdb200_nchw_to_nlc(const float* x, float* y, int64_t N, int64_t C, int64_t HW);            /* backend_cuda.h:76 */
int sdb200_nlc_to_nchw(const float* x, float* y, int64_t N, int64_t C, int64_t HW);            /* backend_cuda.h:77 */
int sdb200_patchify(const float* x, float* y, int64_t C, int64_t H, int64_t W, int p);         /* backend_cuda.h:79 */
int sdb200_unpatchify(const float* x, float* y, int64_t C, int64_t H, int64_t W, int p);       /* backend_cuda.h:80 */

#ifdef __cplusplus
}
#endif

#endif /* SDB200_H */
