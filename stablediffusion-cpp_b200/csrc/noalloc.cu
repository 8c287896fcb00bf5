// noalloc.cu - sdb200_gemm_nt_bf16_noalloc: the bf16-weight GEMM of sdb200_gemm_nt_bf16
// (same kernels, bit-identical results) for callers that cannot allocate device memory.
//
// Who needs it: a host framework that owns every device allocation through its own pool
// and rejects allocations made behind its back, and loops that must never reach a
// cudaMalloc or cudaFree (cudaFree synchronises the whole device, so freeing a grown
// workspace stalls every stream). sdb200_gemm_nt_bf16 may allocate on any call: it grows
// a per-device workspace for the bf16 copy of A on demand, and its first call on a device
// creates a device context whose error word is cudaMalloc'ed. This entry point does
// neither.
//
// How: the bf16 copy of A lives in a file-scope device array of fixed size, g_noalloc_a
// (16 Mi bf16 elements = 32 MiB). Every GPU that loads this library's module holds that
// array until the process exits. Its device address is obtained once per device with
// cudaGetSymbolAddress, with that device current, during the first call made on the
// device; that first call should come before any stream capture. Host code never passes
// the array's name itself to a kernel: on the host it is only a stand-in symbol, not a
// device address.
//
// Stream: the call is issued on the stream given to sdb200_set_stream for this device
// when a library context exists, otherwise on the legacy default stream.
//
// Limits and sharing:
//   * M * round_up(K, 8) must not exceed 16,777,216 (e.g. 4096 x 3840); larger problems
//     are rejected with SDB200_ERR_INVALID_ARG before any GPU work.
//   * B (the bf16 weights) is read in place by TMA, so it must be 16-byte aligned with ldb
//     a multiple of 8 (there is no scratch to repack it); otherwise rejected.
//   * M <= 16 runs the exact fp32-A kernel of sdb200_gemm_nt_bf16 (A read in place, no
//     scratch used), as that entry point does.
//   * Every call on a device shares the one array and leaves its contents behind.
//     Nothing in it has to start at zero: each call overwrites the rows and columns it
//     reads (the kernel's tensor map ends at column K). Calls that may overlap on the GPU
//     (different streams, or different host threads on one device) race on the array;
//     issue them on one stream or serialise them.
//   * A bounded-wait expiry inside the kernel is recorded in a status word of this file,
//     g_noalloc_err; sdb200_device_error_word reads it and sdb200_synchronize reports and
//     clears it, together with the library context's own word.
#include <algorithm>
#include <atomic>
#include <mutex>
#include <string>

#include "internal.h"
#include "ptx.cuh"
#include "sdb200.h"

namespace sdb {
namespace {

constexpr size_t kNoAllocScratchElems = (size_t)16 << 20;  // bf16 elements (32 MiB)
constexpr int kNoAllocMaxDevices = 64;

static __device__ __align__(256) uint16_t g_noalloc_a[kNoAllocScratchElems];
static __device__ int g_noalloc_err;

struct NoAllocDevice {
  std::atomic<bool> ready{false};  // release-stored after the fields below are filled
  uint16_t* scratch = nullptr;     // device address of g_noalloc_a on this device
  int* err = nullptr;              // device address of g_noalloc_err on this device
  int num_sms = 0;
};
NoAllocDevice g_noalloc_dev[kNoAllocMaxDevices];
std::mutex g_noalloc_mutex;

// Once per device, with that device current: resolve the arrays' device addresses.
NoAllocDevice& noalloc_setup(int dev) {
  NoAllocDevice& d = g_noalloc_dev[dev];
  if (d.ready.load(std::memory_order_acquire)) return d;
  std::lock_guard<std::mutex> lk(g_noalloc_mutex);
  if (d.ready.load(std::memory_order_relaxed)) return d;
  int major = 0;
  check_cuda(cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev), "cudaDeviceGetAttribute");
  if (major != 10) fail(kErrUnsupported, "gemm_nt_bf16_noalloc: device is not sm_100");
  check_cuda(cudaDeviceGetAttribute(&d.num_sms, cudaDevAttrMultiProcessorCount, dev), "cudaDeviceGetAttribute");
  void* p = nullptr;
  check_cuda(cudaGetSymbolAddress(&p, g_noalloc_a), "cudaGetSymbolAddress(g_noalloc_a)");
  d.scratch = static_cast<uint16_t*>(p);
  p = nullptr;
  check_cuda(cudaGetSymbolAddress(&p, g_noalloc_err), "cudaGetSymbolAddress(g_noalloc_err)");
  d.err = static_cast<int*>(p);
  d.ready.store(true, std::memory_order_release);
  return d;
}

// A fp32 [M, K] (lda) -> bf16 [M, ldo] with the reference's rounding (RNE, inf/NaN
// truncated), written into the fixed scratch.
__global__ void k_noalloc_pack(const float* __restrict__ A, int64_t lda, uint16_t* __restrict__ dst, int64_t ldo,
                               int64_t M, int64_t K) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < M * K; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / K, c = i - r * K;
    dst[r * ldo + c] = f32_to_bf16_rne(A[r * lda + c]);
  }
}

// C[m, n] = bias[n] (or += when accumulate): the K == 0 case.
__global__ void k_noalloc_bias(float* __restrict__ C, int64_t ldc, int64_t M, int64_t N,
                               const float* __restrict__ bias, int acc) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < M * N; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / N, c = i - r * N;
    const float b = bias ? bias[c] : 0.0f;
    C[r * ldc + c] = acc ? C[r * ldc + c] + b : b;
  }
}

void require(bool ok, const std::string& what) {
  if (!ok) fail(kErrInvalidArg, "gemm_nt_bf16_noalloc: " + what);
}

void gemm_noalloc(int64_t M, int64_t N, int64_t K, const float* A, int64_t lda, const uint16_t* B, int64_t ldb,
                  float* C, int64_t ldc, const float* bias, bool acc) {
  if (M <= 0 || N <= 0) return;  // no-op, as the reference (backend_cuda.cu:464)
  require(M < ((int64_t)1 << 31) && N < ((int64_t)1 << 31) && K < ((int64_t)1 << 31), "dimension >= 2^31");
  require(K >= 0, "K < 0");
  require(C != nullptr, "null pointer C");
  require(ldc >= N, "ldc < N");
  require((reinterpret_cast<uintptr_t>(C) & 3) == 0, "C not 4-byte aligned");
  const int64_t Kp = (K + 7) / 8 * 8;
  const bool skinny = K > 0 && skinny_shape(M, K);
  if (K > 0) {
    require(A != nullptr && B != nullptr, "null pointer A or B");
    require(lda >= K && ldb >= K, "lda or ldb < K");
    if (!skinny) {
      require((reinterpret_cast<uintptr_t>(B) & 15) == 0 && ldb % 8 == 0,
              "B must be 16-byte aligned with ldb a multiple of 8 (read in place; no scratch to repack it)");
      require((size_t)M * (size_t)Kp <= kNoAllocScratchElems,
              "M * round_up(K, 8) = " + std::to_string(M * Kp) + " exceeds the fixed scratch of " +
                  std::to_string(kNoAllocScratchElems) + " bf16 elements");
    }
  }
  int dev = 0;
  check_cuda(cudaGetDevice(&dev), "cudaGetDevice");
  require(dev >= 0 && dev < kNoAllocMaxDevices, "device ordinal out of range");
  NoAllocDevice& d = noalloc_setup(dev);
  DeviceContext* c = ctx_if_created(dev);  // never creates one (that would allocate)
  cudaStream_t stream = c ? c->stream : nullptr;
  const unsigned blocks = (unsigned)std::max<int64_t>(1, std::min<int64_t>((M * std::max<int64_t>(K, N) + 255) / 256,
                                                                            (int64_t)d.num_sms * 16));
  if (K == 0) {
    k_noalloc_bias<<<blocks, 256, 0, stream>>>(C, ldc, M, N, bias, acc ? 1 : 0);
    check_launch("gemm_nt_bf16_noalloc bias");
    return;
  }
  if (skinny) return launch_gemm_skinny_on(M, N, K, A, lda, B, ldb, true, C, ldc, bias, acc, d.num_sms, stream);
  k_noalloc_pack<<<blocks, 256, 0, stream>>>(A, lda, d.scratch, Kp, M, K);
  check_launch("gemm_nt_bf16_noalloc pack");
  GemmCall g{};
  g.M = M;
  g.N = N;
  g.K = K;
  g.A = d.scratch;
  g.lda = Kp;
  g.B = B;
  g.ldb = ldb;
  g.C = C;
  g.ldc = ldc;
  g.bias = bias;
  g.accumulate = acc;
  g.tf32 = false;
  g.epi = Epi::kStore;
  g.out_bf16 = false;
  g.bn = 0;
  launch_gemm_tc_explicit(g, d.num_sms, stream, d.err, dev);
}

}  // namespace

int noalloc_error_word(int dev, bool clear) {
  if (dev < 0 || dev >= kNoAllocMaxDevices) return 0;
  NoAllocDevice& d = g_noalloc_dev[dev];
  if (!d.ready.load(std::memory_order_acquire)) return 0;  // the entry point never ran on dev
  int w = 0;
  check_cuda(cudaMemcpy(&w, d.err, sizeof(int), cudaMemcpyDeviceToHost), "read no-alloc error word");
  if (w && clear) check_cuda(cudaMemset(d.err, 0, sizeof(int)), "clear no-alloc error word");
  return w;
}

}  // namespace sdb

extern "C" int sdb200_gemm_nt_bf16_noalloc(int64_t M, int64_t N, int64_t K, const float* A, int64_t lda,
                                           const uint16_t* B, int64_t ldb, float* C, int64_t ldc, const float* bias,
                                           int accumulate) {
  try {
    sdb::gemm_noalloc(M, N, K, A, lda, B, ldb, C, ldc, bias, accumulate != 0);
    return sdb::kOk;
  } catch (const sdb::Error& e) {
    sdb::set_last_error(e.msg);
    return e.code;
  } catch (const std::exception& e) {
    sdb::set_last_error(e.what());
    return sdb::kErrCuda;
  }
}
