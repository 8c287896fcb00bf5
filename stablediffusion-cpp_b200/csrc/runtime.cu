// runtime.cu - device contexts, the caching allocator, the operand workspace, tensor
// map encoding, error translation, and the memory half of the C ABI (sdb200.h).
//
// The reference backend hard-wires device 0 and the default stream
// (backend_cuda.cu:50-89). Here every host thread works on its current device
// (sdb200_set_device) and each device has one context: its SM count, the stream its
// ops are issued on (default: the legacy default stream, as in the reference), a
// device error word that kernels OR into when a bounded wait expires, and a packing
// workspace. This is what lets one process per GPU (torch.distributed / NCCL) or one
// thread per GPU drive several B200s through the same API.
#include <cudaTypedefs.h>

#include <algorithm>
#include <atomic>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <mutex>
#include <string>
#include <unordered_map>
#include <vector>

#include "internal.h"
#include "sdb200.h"

namespace sdb {

namespace {
thread_local std::string g_last_error;
constexpr int kMaxDevices = 64;
DeviceContext g_ctx[kMaxDevices];
std::mutex g_ctx_mutex;
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
}  // namespace

void fail(int code, const std::string& msg) { throw Error{code, msg}; }

void check_cuda(cudaError_t e, const char* what) {
  if (e != cudaSuccess) {
    cudaGetLastError();
    fail(e == cudaErrorMemoryAllocation ? kErrOutOfMemory : kErrCuda,
         std::string("CUDA error in ") + what + ": " + cudaGetErrorString(e));
  }
}
// Every kernel launch of the library ends in check_launch, so this counts them.
static std::atomic<unsigned long long> g_launches{0};
void check_launch(const char* what) {
  g_launches.fetch_add(1, std::memory_order_relaxed);
  check_cuda(cudaGetLastError(), what);
}
unsigned long long launch_count() { return g_launches.load(std::memory_order_relaxed); }

static void init_context(DeviceContext& c, int dev) {
  cudaDeviceProp prop;
  check_cuda(cudaGetDeviceProperties(&prop, dev), "cudaGetDeviceProperties");
  if (prop.major != 10)
    fail(kErrUnsupported, std::string("device ") + prop.name + " is not sm_100 (this library is built for sm_100a only)");
  c.num_sms = prop.multiProcessorCount;
  c.cc_major = prop.major;
  c.cc_minor = prop.minor;
  c.total_mem = prop.totalGlobalMem;
  c.name = prop.name;
  check_cuda(cudaMalloc(&c.err_word, sizeof(int)), "cudaMalloc(error word)");
  check_cuda(cudaMemset(c.err_word, 0, sizeof(int)), "cudaMemset(error word)");
  c.stream = nullptr;
  c.device = dev;
}

DeviceContext& ctx() {
  int dev = 0;
  check_cuda(cudaGetDevice(&dev), "cudaGetDevice");
  if (dev < 0 || dev >= kMaxDevices) fail(kErrUnsupported, "device ordinal out of range");
  DeviceContext& c = g_ctx[dev];
  if (!c.ready.load(std::memory_order_acquire)) {
    std::lock_guard<std::mutex> lk(g_ctx_mutex);
    if (!c.ready.load(std::memory_order_relaxed)) {
      init_context(c, dev);
      c.ready.store(true, std::memory_order_release);
    }
  }
  return c;
}

DeviceContext* ctx_if_created(int dev) {
  if (dev < 0 || dev >= kMaxDevices) return nullptr;
  return g_ctx[dev].ready.load(std::memory_order_acquire) ? &g_ctx[dev] : nullptr;
}

void* workspace(size_t bytes) {
  DeviceContext& c = ctx();
  if (bytes <= c.ws_bytes) return c.ws;
  if (c.ws) check_cuda(cudaFree(c.ws), "cudaFree(workspace)");  // synchronises: in-flight users finish first
  c.ws = nullptr;
  c.ws_bytes = 0;
  const size_t want = std::max(bytes, (size_t)64 << 20);
  check_cuda(cudaMalloc(&c.ws, want), "cudaMalloc(workspace)");
  c.ws_bytes = want;
  return c.ws;
}

void* split_workspace(size_t bytes) {
  DeviceContext& c = ctx();
  if (bytes <= c.ws_split_bytes) return c.ws_split;
  if (c.ws_split) check_cuda(cudaFree(c.ws_split), "cudaFree(split workspace)");
  c.ws_split = nullptr;
  c.ws_split_bytes = 0;
  const size_t want = std::max(bytes, (size_t)16 << 20);
  check_cuda(cudaMalloc(&c.ws_split, want), "cudaMalloc(split workspace)");
  c.ws_split_bytes = want;
  return c.ws_split;
}

// Tensor maps are pure functions of (type, rank, base address, sizes, strides, box,
// swizzle), and callers such as the reference's model code pass the same weight and pooled
// activation buffers on every step. A small cache keyed by those parameters skips the
// driver's encode on repeated calls; an address reused for a new buffer with the same
// geometry maps identically, so a hit is always valid.
namespace {
struct TmapKey {
  uint64_t base;
  uint64_t dims[5];
  uint64_t strides[4];
  uint32_t box[5];
  int32_t dtype, rank, swizzle, pad;
  bool operator==(const TmapKey& o) const { return std::memcmp(this, &o, sizeof(TmapKey)) == 0; }
};
struct TmapKeyHash {
  size_t operator()(const TmapKey& k) const {
    const unsigned char* p = reinterpret_cast<const unsigned char*>(&k);
    uint64_t h = 1469598103934665603ull;  // FNV-1a over the key's bytes
    for (size_t i = 0; i < sizeof(TmapKey); ++i) h = (h ^ p[i]) * 1099511628211ull;
    return (size_t)h;
  }
};
std::mutex g_tmap_mutex;
std::unordered_map<TmapKey, CUtensorMap, TmapKeyHash> g_tmap_cache;
constexpr size_t kTmapCacheMax = 8192;
}  // namespace

static void encode_tmap_uncached(CUtensorMap* map, CUtensorMapDataType dtype, int rank, const void* base,
                                 const uint64_t* dims, const uint64_t* strides_bytes, const uint32_t* box,
                                 CUtensorMapSwizzle swizzle);

void encode_tmap(CUtensorMap* map, CUtensorMapDataType dtype, int rank, const void* base, const uint64_t* dims,
                 const uint64_t* strides_bytes, const uint32_t* box, CUtensorMapSwizzle swizzle) {
  if (rank < 1 || rank > 5) fail(kErrInvalidArg, "tensor map rank must be 1..5");
  TmapKey key;
  std::memset(&key, 0, sizeof key);
  key.base = reinterpret_cast<uint64_t>(base);
  for (int i = 0; i < rank; ++i) {
    key.dims[i] = dims[i];
    key.box[i] = box[i];
  }
  for (int i = 0; i < rank - 1; ++i) key.strides[i] = strides_bytes[i];
  key.dtype = (int32_t)dtype;
  key.rank = rank;
  key.swizzle = (int32_t)swizzle;
  {
    std::lock_guard<std::mutex> lk(g_tmap_mutex);
    const auto it = g_tmap_cache.find(key);
    if (it != g_tmap_cache.end()) {
      *map = it->second;
      return;
    }
  }
  encode_tmap_uncached(map, dtype, rank, base, dims, strides_bytes, box, swizzle);
  std::lock_guard<std::mutex> lk(g_tmap_mutex);
  if (g_tmap_cache.size() >= kTmapCacheMax) g_tmap_cache.clear();
  g_tmap_cache.emplace(key, *map);
}

static void encode_tmap_uncached(CUtensorMap* map, CUtensorMapDataType dtype, int rank, const void* base,
                                 const uint64_t* dims, const uint64_t* strides_bytes, const uint32_t* box,
                                 CUtensorMapSwizzle swizzle) {
  if (!g_encode) {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    check_cuda(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q),
               "cudaGetDriverEntryPoint(cuTensorMapEncodeTiled)");
    if (!fn || q != cudaDriverEntryPointSuccess) fail(kErrCuda, "cuTensorMapEncodeTiled not available");
    g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  }
  cuuint64_t gdim[5];
  cuuint64_t gstr[4];
  cuuint32_t bx[5], es[5];
  for (int i = 0; i < rank; ++i) {
    gdim[i] = dims[i];
    bx[i] = box[i];
    es[i] = 1;
  }
  for (int i = 0; i < rank - 1; ++i) gstr[i] = strides_bytes[i];
  const CUresult r = g_encode(map, dtype, (cuuint32_t)rank, const_cast<void*>(base), gdim, gstr, bx, es,
                              CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    char buf[256];
    std::snprintf(buf, sizeof buf, "cuTensorMapEncodeTiled failed (%d): rank %d dims %llu x %llu stride %llu", (int)r,
                  rank, (unsigned long long)dims[0], (unsigned long long)(rank > 1 ? dims[1] : 0),
                  (unsigned long long)(rank > 1 ? strides_bytes[0] : 0));
    fail(kErrInvalidArg, buf);
  }
}

// ---------------------------------------------------------------------------------
// Caching allocator: the contract of the reference's cuda::malloc / cuda::free
// (backend_cuda.cu:105-166) - size classes of 1/8 power-of-two steps, idle blocks
// kept per device up to a cap, cache dropped and the allocation retried on OOM.
// ---------------------------------------------------------------------------------
namespace {
struct Pool {
  std::mutex m;
  std::map<void*, size_t> live;
  std::map<size_t, std::vector<void*>> idle;
  size_t idle_bytes = 0;
};
Pool g_pool[kMaxDevices];
constexpr size_t kMaxIdle = (size_t)8 << 30;

size_t size_class(size_t bytes) {
  bytes = std::max<size_t>(bytes, 512);
  size_t p = 512;
  while (p < bytes) p <<= 1;
  const size_t step = std::max<size_t>(512, p / 8);
  return (bytes + step - 1) / step * step;
}
void release_idle(Pool& pl) {
  for (auto& kv : pl.idle)
    for (void* q : kv.second) cudaFree(q);
  pl.idle.clear();
  pl.idle_bytes = 0;
}
}  // namespace

void* pool_malloc(size_t bytes) {
  if (bytes == 0) return nullptr;
  const int dev = ctx().device;
  Pool& pl = g_pool[dev];
  const size_t cls = size_class(bytes);
  std::lock_guard<std::mutex> lk(pl.m);
  auto it = pl.idle.find(cls);
  if (it != pl.idle.end() && !it->second.empty()) {
    void* p = it->second.back();
    it->second.pop_back();
    pl.idle_bytes -= cls;
    pl.live[p] = cls;
    return p;
  }
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, cls);
  if (e == cudaErrorMemoryAllocation) {
    cudaGetLastError();
    release_idle(pl);
    e = cudaMalloc(&p, cls);
  }
  check_cuda(e, "cudaMalloc");
  pl.live[p] = cls;
  return p;
}

void pool_free(void* p) {
  if (!p) return;
  const int dev = ctx().device;
  Pool& pl = g_pool[dev];
  std::unique_lock<std::mutex> lk(pl.m);
  auto it = pl.live.find(p);
  if (it == pl.live.end()) fail(kErrInvalidArg, "free: pointer not allocated by this library on the current device");
  const size_t cls = it->second;
  pl.live.erase(it);
  if (pl.idle_bytes + cls > kMaxIdle) {
    check_cuda(cudaFree(p), "cudaFree");
  } else {
    pl.idle[cls].push_back(p);
    pl.idle_bytes += cls;
  }
  lk.unlock();
  operand_cache_invalidate(p, cls);  // packed copies of this buffer's contents are stale now
}

}  // namespace sdb

// ===================================================================================
// C ABI: memory, devices, errors
// ===================================================================================
using namespace sdb;

namespace sdb {
void set_last_error(const std::string& s) { g_last_error = s; }
}  // namespace sdb

#define SDB_GUARD(body)                               \
  try {                                               \
    body;                                             \
    return kOk;                                       \
  } catch (const sdb::Error& e) {                     \
    sdb::set_last_error(e.msg);                       \
    return e.code;                                    \
  } catch (const std::exception& e) {                 \
    sdb::set_last_error(e.what());                    \
    return kErrCuda;                                  \
  }

extern "C" {

const char* sdb200_last_error(void) { return g_last_error.c_str(); }

int sdb200_version(void) { return SDB200_ABI_VERSION; }

unsigned long long sdb200_launch_count(void) { return sdb::launch_count(); }

int sdb200_available(void) {
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess || n < 1) {
    cudaGetLastError();
    return 0;
  }
  try {
    ctx();
  } catch (const sdb::Error& e) {
    g_last_error = e.msg;
    return 0;
  }
  return 1;
}

int sdb200_device_count(void) {
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  return n;
}

const char* sdb200_device_name(void) {
  if (!sdb200_available()) return "";
  return ctx().name.c_str();
}

size_t sdb200_device_memory(void) {
  if (!sdb200_available()) return 0;
  return ctx().total_mem;
}

int sdb200_set_device(int device) {
  SDB_GUARD({
    check_cuda(cudaSetDevice(device), "cudaSetDevice");
    ctx();
  })
}

int sdb200_set_stream(void* stream) { SDB_GUARD({ ctx().stream = reinterpret_cast<cudaStream_t>(stream); }) }

void* sdb200_get_stream(void) {
  try {
    return reinterpret_cast<void*>(ctx().stream);
  } catch (...) {
    return nullptr;
  }
}

void* sdb200_malloc(size_t bytes) {
  try {
    return pool_malloc(bytes);
  } catch (const sdb::Error& e) {
    g_last_error = e.msg;
    return nullptr;
  }
}

int sdb200_free(void* p) { SDB_GUARD({ pool_free(p); }) }

int sdb200_upload(void* dst, const void* src, size_t bytes) {
  SDB_GUARD({
    if (bytes == 0) return kOk;
    if (!dst || !src) fail(kErrInvalidArg, "upload: null pointer");
    operand_cache_invalidate(dst, bytes);
    check_cuda(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, ctx().stream), "upload");
  })
}

int sdb200_download(void* dst, const void* src, size_t bytes) {
  SDB_GUARD({
    if (bytes == 0) return kOk;
    if (!dst || !src) fail(kErrInvalidArg, "download: null pointer");
    check_cuda(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, ctx().stream), "download");
    check_cuda(cudaStreamSynchronize(ctx().stream), "download sync");
  })
}

int sdb200_copy(void* dst, const void* src, size_t bytes) {
  SDB_GUARD({
    if (bytes == 0) return kOk;
    if (!dst || !src) fail(kErrInvalidArg, "copy: null pointer");
    operand_cache_invalidate(dst, bytes);
    check_cuda(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToDevice, ctx().stream), "copy");
  })
}

int sdb200_zero(void* dst, size_t bytes) {
  SDB_GUARD({
    if (bytes == 0) return kOk;
    if (!dst) fail(kErrInvalidArg, "zero: null pointer");
    operand_cache_invalidate(dst, bytes);
    check_cuda(cudaMemsetAsync(dst, 0, bytes, ctx().stream), "zero");
  })
}

int sdb200_synchronize(void) {
  SDB_GUARD({
    DeviceContext& c = ctx();
    check_cuda(cudaStreamSynchronize(c.stream), "synchronize");
    int w = 0;
    check_cuda(cudaMemcpy(&w, c.err_word, sizeof(int), cudaMemcpyDeviceToHost), "read error word");
    if (w) check_cuda(cudaMemset(c.err_word, 0, sizeof(int)), "clear error word");
    w |= noalloc_error_word(c.device, true);
    if (w) {
      char buf[128];
      std::snprintf(buf, sizeof buf, "a kernel's bounded wait expired (device error word 0x%x)", w);
      fail(kErrDeviceWait, buf);
    }
  })
}

int sdb200_device_error_word(int* out) {
  SDB_GUARD({
    if (!out) fail(kErrInvalidArg, "null output");
    DeviceContext& c = ctx();
    check_cuda(cudaStreamSynchronize(c.stream), "synchronize");
    check_cuda(cudaMemcpy(out, c.err_word, sizeof(int), cudaMemcpyDeviceToHost), "read error word");
    *out |= noalloc_error_word(c.device, false);
  })
}

}  // extern "C"
