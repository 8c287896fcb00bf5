// comm.cu - the tensor-parallel collective of the DiT: a sum all-reduce over NVLink /
// NVSwitch through NCCL, one communicator per tensor-parallel group, one process (or
// thread) per GPU. The reference has no collective at all (single device,
// backend_cuda.cu:64-72); this is the exchange step of Megatron-style row-parallel
// projections (to_out and w2 of each block).
//
// NCCL is loaded at run time (dlopen "libnccl.so.2"): the library itself keeps no
// link-time dependency on it, and in a process where PyTorch already loaded its NCCL
// the same copy is reused. Only the NCCL C API is called (no torch types cross here).
//
// Symmetric buffers (SymBuf): every rank allocates the same size with cudaMalloc and
// maps every peer's allocation through CUDA IPC (handles exchanged with one NCCL
// all-gather), so kernels can store straight into a peer's memory over NVLink. The
// fused tensor-parallel path uses them: the row-parallel GEMMs scatter their partial
// tiles into the owner rank's slots from the epilogue, and the post-norm kernel
// broadcasts the next GEMM's bf16 input rows. comm_barrier orders those kernels across
// ranks; kernels that store to peers end with a system-scope fence. The barrier is a flag
// exchange through a symmetric buffer (k_flag_barrier: each rank stores its epoch into
// every peer's flag word with a system-scope release, then waits, bounded, until every
// peer's epoch has arrived in its own), a few microseconds where a 4-byte NCCL all-reduce
// takes tens; the all-reduce form stays selectable (sdb200_comm_set_barrier).
#include <dlfcn.h>
#include <nccl.h>

#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "internal.h"
#include "ptx.cuh"
#include "sdb200.h"

namespace sdb {
namespace {

struct NcclApi {
  bool loaded = false;
  ncclResult_t (*GetUniqueId)(ncclUniqueId*) = nullptr;
  ncclResult_t (*CommInitRank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*AllReduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                            cudaStream_t) = nullptr;
  ncclResult_t (*AllGather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
  ncclResult_t (*CommAbort)(ncclComm_t) = nullptr;
  const char* (*GetErrorString)(ncclResult_t) = nullptr;
};
NcclApi g_nccl;
std::mutex g_nccl_mutex;

NcclApi& nccl() {
  std::lock_guard<std::mutex> lk(g_nccl_mutex);
  if (g_nccl.loaded) return g_nccl;
  void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
  if (!h) fail(kErrUnsupported, std::string("NCCL not available: ") + dlerror());
  auto sym = [&](const char* n) {
    void* f = dlsym(h, n);
    if (!f) fail(kErrUnsupported, std::string("NCCL symbol missing: ") + n);
    return f;
  };
  g_nccl.GetUniqueId = reinterpret_cast<decltype(g_nccl.GetUniqueId)>(sym("ncclGetUniqueId"));
  g_nccl.CommInitRank = reinterpret_cast<decltype(g_nccl.CommInitRank)>(sym("ncclCommInitRank"));
  g_nccl.AllReduce = reinterpret_cast<decltype(g_nccl.AllReduce)>(sym("ncclAllReduce"));
  g_nccl.AllGather = reinterpret_cast<decltype(g_nccl.AllGather)>(sym("ncclAllGather"));
  g_nccl.CommDestroy = reinterpret_cast<decltype(g_nccl.CommDestroy)>(sym("ncclCommDestroy"));
  g_nccl.CommAbort = reinterpret_cast<decltype(g_nccl.CommAbort)>(sym("ncclCommAbort"));
  g_nccl.GetErrorString = reinterpret_cast<decltype(g_nccl.GetErrorString)>(sym("ncclGetErrorString"));
  g_nccl.loaded = true;
  return g_nccl;
}

void check_nccl(ncclResult_t r, const char* what) {
  if (r != ncclSuccess) fail(kErrCuda, std::string(what) + ": " + nccl().GetErrorString(r));
}

}  // namespace

struct Comm {
  ncclComm_t comm = nullptr;
  int rank = 0, world = 1, device = -1;
  float* bar = nullptr;     // device word of the all-reduce barrier
  uint8_t* hbuf = nullptr;  // device staging of the IPC handle exchange (world x 64 bytes)
  SymBuf flags;             // uint32 per peer: the last barrier epoch that peer reached
  uint32_t epoch = 0;
  bool flag_barrier = true;
};

namespace {
struct FlagPtrs {
  uint32_t* p[kMaxTpRanks];
};
// One warp: lane i < world stores this rank's epoch into peer i's flag word `rank`
// (release, system scope: the stores of earlier kernels on this stream, fenced system-wide
// by those kernels, are visible to the peer first), then waits until peer i's epoch is in
// this rank's flag word i (acquire, system scope). Bounded: after kWaitLimitNs it records
// kErrTpBarrier and returns.
__global__ void k_flag_barrier(FlagPtrs peers, const uint32_t* mine, int rank, int world, uint32_t epoch, int* err) {
  const int i = threadIdx.x;
  if (i >= world) return;
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(peers.p[i] + rank), "r"(epoch) : "memory");
  const uint64_t t0 = globaltimer_ns();
  for (;;) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(mine + i) : "memory");
    if ((int32_t)(v - epoch) >= 0) break;
    if (globaltimer_ns() - t0 > kWaitLimitNs) {
      atomicOr(err, kErrTpBarrier);
      break;
    }
  }
}
}  // namespace

// Sum all-reduce of n fp32 values in place on the calling context's stream.
void comm_allreduce_sum(Comm* c, float* buf, size_t n) {
  if (!c || c->world <= 1 || n == 0) return;
  check_nccl(nccl().AllReduce(buf, buf, n, ncclFloat32, ncclSum, c->comm, ctx().stream), "ncclAllReduce");
}
int comm_world(const Comm* c) { return c ? c->world : 1; }
int comm_rank(const Comm* c) { return c ? c->rank : 0; }

// Stream-ordered barrier: completes on every rank only after all ranks reached it, so
// work after it sees what every rank's earlier kernels stored into its memory.
void comm_barrier(Comm* c) {
  if (!c || c->world <= 1) return;
  if (c->flag_barrier && c->flags.local) {
    FlagPtrs fp{};
    for (int r = 0; r < c->world; ++r) fp.p[r] = static_cast<uint32_t*>(c->flags.peer[r]);
    ++c->epoch;
    k_flag_barrier<<<1, 32, 0, ctx().stream>>>(fp, static_cast<const uint32_t*>(c->flags.local), c->rank, c->world,
                                               c->epoch, ctx().err_word);
    check_launch("flag_barrier");
    return;
  }
  check_nccl(nccl().AllReduce(c->bar, c->bar, 1, ncclFloat32, ncclSum, c->comm, ctx().stream), "ncclAllReduce(barrier)");
}

// The all-reduce barrier followed by a stream synchronize (set-up only).
void comm_barrier_nccl_sync(Comm* c) {
  if (!c || c->world <= 1) return;
  check_nccl(nccl().AllReduce(c->bar, c->bar, 1, ncclFloat32, ncclSum, c->comm, ctx().stream), "ncclAllReduce(barrier)");
  check_cuda(cudaStreamSynchronize(ctx().stream), "comm: set-up barrier");
}

// recv[r * bytes ...] = rank r's send (in place when send == recv + rank * bytes).
void comm_allgather(Comm* c, const void* send, void* recv, size_t bytes) {
  if (!c || c->world <= 1 || bytes == 0) return;
  check_nccl(nccl().AllGather(send, recv, bytes, ncclInt8, c->comm, ctx().stream), "ncclAllGather");
}

// Collective: every rank calls with the same size. Frees a previous allocation of b.
void comm_sym_alloc(Comm* c, SymBuf& b, size_t bytes) {
  comm_sym_free(c, b);
  const int w = comm_world(c);
  if (w > kMaxTpRanks) fail(kErrUnsupported, "symmetric buffers: at most 8 ranks");
  check_cuda(cudaMalloc(&b.local, bytes), "cudaMalloc(symmetric)");
  b.bytes = bytes;
  b.peer[comm_rank(c)] = b.local;
  if (w <= 1) return;
  cudaIpcMemHandle_t mine;
  check_cuda(cudaIpcGetMemHandle(&mine, b.local), "cudaIpcGetMemHandle");
  static_assert(sizeof(cudaIpcMemHandle_t) == 64, "IPC handle size");
  check_cuda(cudaMemcpyAsync(c->hbuf + (size_t)c->rank * 64, &mine, 64, cudaMemcpyHostToDevice, ctx().stream),
             "symmetric: handle upload");
  comm_allgather(c, c->hbuf + (size_t)c->rank * 64, c->hbuf, 64);
  std::vector<cudaIpcMemHandle_t> all((size_t)w);
  check_cuda(cudaMemcpyAsync(all.data(), c->hbuf, (size_t)w * 64, cudaMemcpyDeviceToHost, ctx().stream),
             "symmetric: handle download");
  check_cuda(cudaStreamSynchronize(ctx().stream), "symmetric: handle exchange");
  for (int r = 0; r < w; ++r) {
    if (r == c->rank) continue;
    void* p = nullptr;
    check_cuda(cudaIpcOpenMemHandle(&p, all[(size_t)r], cudaIpcMemLazyEnablePeerAccess), "cudaIpcOpenMemHandle");
    b.peer[r] = p;
  }
}

// Not collective. Callers free only between forwards: every store a peer makes into
// this buffer happens before that peer enters the forward's last collective, which this
// rank has completed once its stream is drained here.
void comm_sym_free(Comm* c, SymBuf& b) {
  (void)c;
  if (!b.local) return;
  cudaStreamSynchronize(ctx().stream);
  for (int r = 0; r < kMaxTpRanks; ++r)
    if (b.peer[r] && b.peer[r] != b.local) cudaIpcCloseMemHandle(b.peer[r]);
  cudaFree(b.local);
  b = SymBuf{};
}

}  // namespace sdb

using sdb::Comm;

extern "C" {

int sdb200_comm_unique_id(void* out) {
  try {
    if (!out) sdb::fail(sdb::kErrInvalidArg, "comm_unique_id: null output");
    ncclUniqueId id;
    sdb::check_nccl(sdb::nccl().GetUniqueId(&id), "ncclGetUniqueId");
    std::memcpy(out, &id, sizeof(id));
    return sdb::kOk;
  } catch (const sdb::Error& e) {
    sdb::set_last_error(e.msg);
    return e.code;
  }
}

void* sdb200_comm_create(const void* unique_id, int rank, int world) {
  try {
    if (!unique_id || world < 1 || rank < 0 || rank >= world) sdb::fail(sdb::kErrInvalidArg, "comm_create: bad args");
    Comm* c = new Comm();
    c->rank = rank;
    c->world = world;
    c->device = sdb::ctx().device;
    if (world > 1) {
      ncclUniqueId id;
      std::memcpy(&id, unique_id, sizeof(id));
      try {
        sdb::check_nccl(sdb::nccl().CommInitRank(&c->comm, world, id, rank), "ncclCommInitRank");
        sdb::check_cuda(cudaMalloc(&c->bar, 256), "comm: barrier word");
        sdb::check_cuda(cudaMemset(c->bar, 0, 256), "comm: barrier word");
        sdb::check_cuda(cudaMalloc(&c->hbuf, (size_t)world * 64), "comm: handle staging");
        // The flag words start at zero on every rank before any peer can reach them: the
        // handle exchange inside comm_sym_alloc follows the memset on every rank's stream.
        sdb::comm_sym_alloc(c, c->flags, 256);
        sdb::check_cuda(cudaMemsetAsync(c->flags.local, 0, 256, sdb::ctx().stream), "comm: flag words");
        sdb::comm_barrier_nccl_sync(c);
      } catch (...) {
        sdb::comm_sym_free(c, c->flags);
        if (c->comm) sdb::nccl().CommDestroy(c->comm);
        cudaFree(c->bar);
        cudaFree(c->hbuf);
        delete c;
        throw;
      }
    }
    return c;
  } catch (const sdb::Error& e) {
    sdb::set_last_error(e.msg);
    return nullptr;
  }
}

int sdb200_comm_allreduce_sum_f32(void* comm, float* buf, size_t n) {
  try {
    if (!comm || (!buf && n)) sdb::fail(sdb::kErrInvalidArg, "comm_allreduce: null pointer");
    sdb::comm_allreduce_sum(static_cast<Comm*>(comm), buf, n);
    return sdb::kOk;
  } catch (const sdb::Error& e) {
    sdb::set_last_error(e.msg);
    return e.code;
  }
}

int sdb200_comm_barrier_selftest(uint32_t* flags, int world, int rank, uint32_t epoch) {
  try {
    if (!flags || world < 1 || world > sdb::kMaxTpRanks || rank < 0 || rank >= world)
      sdb::fail(sdb::kErrInvalidArg, "comm_barrier_selftest: bad flag array, world or rank");
    if ((reinterpret_cast<uintptr_t>(flags) & 3) != 0) sdb::fail(sdb::kErrInvalidArg, "comm_barrier_selftest: unaligned");
    sdb::FlagPtrs fp{};
    for (int r = 0; r < world; ++r) fp.p[r] = flags;  // every peer's flag array is this one
    sdb::k_flag_barrier<<<1, 32, 0, sdb::ctx().stream>>>(fp, flags, rank, world, epoch, sdb::ctx().err_word);
    sdb::check_launch("flag_barrier_selftest");
    return sdb::kOk;
  } catch (const sdb::Error& e) {
    sdb::set_last_error(e.msg);
    return e.code;
  }
}

int sdb200_comm_set_barrier(void* comm, int flags) {
  try {
    if (!comm) sdb::fail(sdb::kErrInvalidArg, "comm_set_barrier: null communicator");
    static_cast<Comm*>(comm)->flag_barrier = flags != 0;
    return sdb::kOk;
  } catch (const sdb::Error& e) {
    sdb::set_last_error(e.msg);
    return e.code;
  }
}

void sdb200_comm_destroy(void* comm) {
  Comm* c = static_cast<Comm*>(comm);
  if (!c) return;
  try {
    sdb::comm_sym_free(c, c->flags);
  } catch (...) {
  }
  if (c->comm) {
    try {
      sdb::nccl().CommDestroy(c->comm);
    } catch (...) {
    }
  }
  cudaFree(c->bar);
  cudaFree(c->hbuf);
  delete c;
}

}  // extern "C"
