// Collectives behind the C ABI (fpb_comm_*): the NCCL plumbing of the
// N-split dense layers (all-gather of each rank's output columns) and of the
// expert-parallel MoE layer (all-to-all dispatch and combine, MAX all-reduce
// of the activation amax), callable from a host language that has no
// torch.distributed.
//
// NCCL is opened at run time (dlopen of libnccl.so.2), not linked: a process
// that already loaded NCCL (e.g. through torch) gets that same library, so
// both share one NCCL; a process that never communicates needs none.
// nccl.h supplies only the types.
#include <dlfcn.h>
#include <nccl.h>

#include <cstring>
#include <mutex>

#include "common.cuh"

struct fpb_comm {
  ncclComm_t nccl = nullptr;
  int nranks = 0;
  int rank = 0;
  int device = 0;
};

namespace fpb {
namespace {

struct NcclApi {
  bool ok = false;
  ncclResult_t (*get_unique_id)(ncclUniqueId *) = nullptr;
  ncclResult_t (*init_rank)(ncclComm_t *, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*destroy)(ncclComm_t) = nullptr;
  ncclResult_t (*abort)(ncclComm_t) = nullptr;
  ncclResult_t (*async_error)(ncclComm_t, ncclResult_t *) = nullptr;
  const char *(*error_string)(ncclResult_t) = nullptr;
  ncclResult_t (*version)(int *) = nullptr;
  ncclResult_t (*all_gather)(const void *, void *, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*all_reduce)(const void *, void *, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                             cudaStream_t) = nullptr;
  ncclResult_t (*send)(const void *, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*recv)(void *, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*group_start)() = nullptr;
  ncclResult_t (*group_end)() = nullptr;
};

template <typename F>
bool bind(void *lib, const char *name, F *out) {
  *out = reinterpret_cast<F>(dlsym(lib, name));
  return *out != nullptr;
}

const NcclApi &nccl() {
  static NcclApi api;
  static std::once_flag once;
  std::call_once(once, [] {
    void *lib = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!lib) lib = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
    if (!lib) return;
    api.ok = bind(lib, "ncclGetUniqueId", &api.get_unique_id) && bind(lib, "ncclCommInitRank", &api.init_rank) &&
             bind(lib, "ncclCommDestroy", &api.destroy) && bind(lib, "ncclCommAbort", &api.abort) &&
             bind(lib, "ncclCommGetAsyncError", &api.async_error) &&
             bind(lib, "ncclGetErrorString", &api.error_string) && bind(lib, "ncclGetVersion", &api.version) &&
             bind(lib, "ncclAllGather", &api.all_gather) && bind(lib, "ncclAllReduce", &api.all_reduce) &&
             bind(lib, "ncclSend", &api.send) && bind(lib, "ncclRecv", &api.recv) &&
             bind(lib, "ncclGroupStart", &api.group_start) && bind(lib, "ncclGroupEnd", &api.group_end);
  });
  return api;
}

int nccl_fail(ncclResult_t r, const char *what) {
  const NcclApi &api = nccl();
  return fail(FPB_ERR_COMM, "%s: NCCL error %d (%s)", what, (int)r, api.error_string ? api.error_string(r) : "?");
}

#define FPB_NCCL_TRY(expr, what)                   \
  do {                                             \
    ncclResult_t fpb_r_ = (expr);                  \
    if (fpb_r_ != ncclSuccess) return nccl_fail(fpb_r_, what); \
  } while (0)

int need_api(const char *fn) {
  if (!nccl().ok) return fail(FPB_ERR_COMM, "%s: NCCL (libnccl.so.2) could not be loaded", fn);
  return FPB_OK;
}

bool dtype_of(int dtype, ncclDataType_t *t, size_t *esize) {
  switch (dtype) {
    case FPB_F32: *t = ncclFloat32; *esize = 4; return true;
    case FPB_BF16: *t = ncclBfloat16; *esize = 2; return true;
    case FPB_COMM_U32: *t = ncclUint32; *esize = 4; return true;
    case FPB_COMM_I32: *t = ncclInt32; *esize = 4; return true;
    case FPB_COMM_BYTES: *t = ncclUint8; *esize = 1; return true;
    default: return false;
  }
}

// Runs `body` with the communicator's device current, restoring the caller's.
template <typename Body>
int on_device(const fpb_comm *c, Body body) {
  int prev = -1;
  cudaGetDevice(&prev);
  if (prev != c->device) {
    cudaError_t e = cudaSetDevice(c->device);
    if (e != cudaSuccess) return cuda_fail(e, "cudaSetDevice(communicator device)");
  }
  int st = body();
  if (prev >= 0 && prev != c->device) cudaSetDevice(prev);
  return st;
}

}  // namespace
}  // namespace fpb

using namespace fpb;

extern "C" int fpb_comm_available(void) { return nccl().ok ? 1 : 0; }

extern "C" int fpb_comm_version(int *version) {
  if (!version) return fail(FPB_ERR_INVALID_ARGUMENT, "fpb_comm_version: null pointer");
  if (int st = need_api("fpb_comm_version")) return st;
  FPB_NCCL_TRY(nccl().version(version), "ncclGetVersion");
  return FPB_OK;
}

extern "C" int fpb_comm_unique_id(uint8_t id[FPB_COMM_ID_BYTES]) {
  if (!id) return fail(FPB_ERR_INVALID_ARGUMENT, "fpb_comm_unique_id: null pointer");
  if (int st = need_api("fpb_comm_unique_id")) return st;
  static_assert(sizeof(ncclUniqueId) == FPB_COMM_ID_BYTES, "NCCL unique id size");
  ncclUniqueId u;
  FPB_NCCL_TRY(nccl().get_unique_id(&u), "ncclGetUniqueId");
  std::memcpy(id, &u, sizeof(u));
  return FPB_OK;
}

extern "C" int fpb_comm_init(const uint8_t id[FPB_COMM_ID_BYTES], int nranks, int rank, int device,
                             fpb_comm **out) {
  if (!id || !out) return fail(FPB_ERR_INVALID_ARGUMENT, "fpb_comm_init: null pointer");
  *out = nullptr;
  if (nranks < 1 || rank < 0 || rank >= nranks)
    return fail(FPB_ERR_INVALID_ARGUMENT, "fpb_comm_init: rank %d of %d", rank, nranks);
  if (int st = need_api("fpb_comm_init")) return st;
  fpb_comm *c = new fpb_comm();
  c->nranks = nranks;
  c->rank = rank;
  c->device = device;
  ncclUniqueId u;
  std::memcpy(&u, id, sizeof(u));
  int st = on_device(c, [&]() -> int {
    FPB_NCCL_TRY(nccl().init_rank(&c->nccl, nranks, u, rank), "ncclCommInitRank");
    return FPB_OK;
  });
  if (st) {
    delete c;
    return st;
  }
  *out = c;
  return FPB_OK;
}

extern "C" int fpb_comm_destroy(fpb_comm *c) {
  if (!c) return FPB_OK;
  int st = FPB_OK;
  if (c->nccl) st = on_device(c, [&]() -> int {
    FPB_NCCL_TRY(nccl().destroy(c->nccl), "ncclCommDestroy");
    return FPB_OK;
  });
  delete c;
  return st;
}

extern "C" int fpb_comm_abort(fpb_comm *c) {
  if (!c) return FPB_OK;
  int st = FPB_OK;
  if (c->nccl) st = on_device(c, [&]() -> int {
    FPB_NCCL_TRY(nccl().abort(c->nccl), "ncclCommAbort");
    return FPB_OK;
  });
  delete c;
  return st;
}

extern "C" int fpb_comm_status(const fpb_comm *c) {
  if (!c || !c->nccl) return fail(FPB_ERR_INVALID_ARGUMENT, "fpb_comm_status: null communicator");
  ncclResult_t r = ncclSuccess;
  FPB_NCCL_TRY(nccl().async_error(c->nccl, &r), "ncclCommGetAsyncError");
  if (r != ncclSuccess && r != ncclInProgress) return nccl_fail(r, "communicator");
  return FPB_OK;
}

extern "C" int fpb_comm_size(const fpb_comm *c, int *nranks, int *rank) {
  if (!c || !nranks || !rank) return fail(FPB_ERR_INVALID_ARGUMENT, "fpb_comm_size: null pointer");
  *nranks = c->nranks;
  *rank = c->rank;
  return FPB_OK;
}

extern "C" int fpb_comm_all_gather(fpb_comm *c, const void *send, void *recv, size_t count, int dtype,
                                   void *stream) {
  if (!c || !c->nccl || !send || !recv)
    return fail(FPB_ERR_INVALID_ARGUMENT, "fpb_comm_all_gather: null pointer");
  ncclDataType_t t;
  size_t es;
  if (!dtype_of(dtype, &t, &es)) return fail(FPB_ERR_INVALID_ARGUMENT, "fpb_comm_all_gather: dtype %d", dtype);
  return on_device(c, [&]() -> int {
    FPB_NCCL_TRY(nccl().all_gather(send, recv, count, t, c->nccl, as_stream(stream)), "ncclAllGather");
    return FPB_OK;
  });
}

extern "C" int fpb_comm_all_reduce(fpb_comm *c, const void *send, void *recv, size_t count, int dtype, int op,
                                   void *stream) {
  if (!c || !c->nccl || !send || !recv)
    return fail(FPB_ERR_INVALID_ARGUMENT, "fpb_comm_all_reduce: null pointer");
  ncclDataType_t t;
  size_t es;
  if (!dtype_of(dtype, &t, &es)) return fail(FPB_ERR_INVALID_ARGUMENT, "fpb_comm_all_reduce: dtype %d", dtype);
  ncclRedOp_t r;
  switch (op) {
    case FPB_COMM_SUM: r = ncclSum; break;
    case FPB_COMM_MAX: r = ncclMax; break;
    default: return fail(FPB_ERR_INVALID_ARGUMENT, "fpb_comm_all_reduce: op %d", op);
  }
  return on_device(c, [&]() -> int {
    FPB_NCCL_TRY(nccl().all_reduce(send, recv, count, t, r, c->nccl, as_stream(stream)), "ncclAllReduce");
    return FPB_OK;
  });
}

extern "C" int fpb_comm_all_to_all(fpb_comm *c, const void *send, const size_t *send_counts,
                                   const size_t *send_offsets, void *recv, const size_t *recv_counts,
                                   const size_t *recv_offsets, int dtype, void *stream) {
  if (!c || !c->nccl || !send_counts || !send_offsets || !recv_counts || !recv_offsets)
    return fail(FPB_ERR_INVALID_ARGUMENT, "fpb_comm_all_to_all: null pointer");
  ncclDataType_t t;
  size_t es;
  if (!dtype_of(dtype, &t, &es)) return fail(FPB_ERR_INVALID_ARGUMENT, "fpb_comm_all_to_all: dtype %d", dtype);
  for (int p = 0; p < c->nranks; ++p)
    if ((send_counts[p] && !send) || (recv_counts[p] && !recv))
      return fail(FPB_ERR_INVALID_ARGUMENT, "fpb_comm_all_to_all: null buffer with a non-zero count");
  const NcclApi &api = nccl();
  return on_device(c, [&]() -> int {
    cudaStream_t s = as_stream(stream);
    FPB_NCCL_TRY(api.group_start(), "ncclGroupStart");
    ncclResult_t first = ncclSuccess;
    for (int p = 0; p < c->nranks && first == ncclSuccess; ++p) {
      if (send_counts[p])
        first = api.send(static_cast<const char *>(send) + send_offsets[p] * es, send_counts[p], t, p, c->nccl, s);
      if (first == ncclSuccess && recv_counts[p])
        first = api.recv(static_cast<char *>(recv) + recv_offsets[p] * es, recv_counts[p], t, p, c->nccl, s);
    }
    ncclResult_t end = api.group_end();
    if (first != ncclSuccess) return nccl_fail(first, "ncclSend/ncclRecv");
    if (end != ncclSuccess) return nccl_fail(end, "ncclGroupEnd");
    return FPB_OK;
  });
}

// ---- peer memory (CUDA IPC) ----------------------------------------------------------------
// Buffers that other processes (one per GPU) map into their address space,
// so that a kernel writes another GPU's buffer with plain stores over NVLink:
// the expert-parallel layer's receive buffers.  An IPC handle names a whole
// cudaMalloc allocation, so these buffers are allocated here, one allocation
// each.
extern "C" int fpb_ipc_alloc(size_t bytes, void **ptr) {
  if (!ptr || bytes == 0) return fail(FPB_ERR_INVALID_ARGUMENT, "fpb_ipc_alloc: null pointer or zero size");
  *ptr = nullptr;
  FPB_CUDA_TRY(cudaMalloc(ptr, bytes));
  return FPB_OK;
}

extern "C" int fpb_ipc_free(void *ptr) {
  if (ptr) FPB_CUDA_TRY(cudaFree(ptr));
  return FPB_OK;
}

extern "C" int fpb_ipc_get_handle(const void *ptr, uint8_t handle[FPB_IPC_HANDLE_BYTES]) {
  static_assert(sizeof(cudaIpcMemHandle_t) == FPB_IPC_HANDLE_BYTES, "IPC handle size");
  if (!ptr || !handle) return fail(FPB_ERR_INVALID_ARGUMENT, "fpb_ipc_get_handle: null pointer");
  cudaIpcMemHandle_t h;
  FPB_CUDA_TRY(cudaIpcGetMemHandle(&h, const_cast<void *>(ptr)));
  std::memcpy(handle, &h, sizeof h);
  return FPB_OK;
}

extern "C" int fpb_ipc_open(const uint8_t handle[FPB_IPC_HANDLE_BYTES], void **ptr) {
  if (!handle || !ptr) return fail(FPB_ERR_INVALID_ARGUMENT, "fpb_ipc_open: null pointer");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof h);
  *ptr = nullptr;
  FPB_CUDA_TRY(cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess));
  return FPB_OK;
}

extern "C" int fpb_ipc_close(void *ptr) {
  if (ptr) FPB_CUDA_TRY(cudaIpcCloseMemHandle(ptr));
  return FPB_OK;
}

// ---- barrier over peer memory ----------------------------------------------------------------
// One warp: lane r < nranks stores this barrier's epoch into rank r's flag
// word for this rank (a system-scope release store over NVLink), then waits
// until rank r's epoch has arrived in this rank's own flag word r (acquire
// loads).  The release orders every store this rank made before the barrier
// (the peer stores of the kernels before it, which end with a system-scope
// fence) before the flag, so a rank that has seen every flag sees every
// rank's stores.  A flag already past the epoch counts: a faster rank may
// announce the next barrier first.  The epoch is a device counter, so a CUDA
// graph replays the barrier with new epochs.  Every wait ends after
// `timeout_ns` of global time with device error 601 (fpb_device_error) and
// the kernel returns: a rank that never arrives cannot hang the others.
namespace fpb {
namespace {

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// With `value` (all-reduce MAX of one uint32 word): before its flag, lane r
// also stores *value into rank r's slot for this rank; the slots alternate
// between two banks by epoch parity (a rank that is already one barrier
// ahead writes the other bank), and after the waits the lanes take the
// maximum of this rank's slots.
constexpr int kBarrierSlots = 32;  // words [32, 96) of the flag buffer: two banks of 32

__global__ void peer_barrier_kernel(uint32_t *counter, const uint32_t *flags, uint32_t *const *peer_flags, int nranks,
                                    int rank, unsigned long long timeout_ns, int *error, uint32_t *value) {
  pdl_enter();
  const int t = threadIdx.x;
  const uint32_t epoch = *counter + 1;
  const int bank = kBarrierSlots + (int)(epoch & 1u) * kBarrierSlots;
  if (t < nranks) {
    uint32_t *dst = peer_flags[t] + rank;
    if (value) peer_flags[t][bank + rank] = *value;
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(dst), "r"(epoch) : "memory");
    const uint64_t start = global_ns();
    bool arrived = false;
    while (true) {
      uint32_t v;
      asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(flags + t) : "memory");
      if ((int)(v - epoch) >= 0) {
        arrived = true;
        break;
      }
      if (global_ns() - start > timeout_ns) break;
    }
    if (!arrived && error) atomicCAS(error, 0, 601);
  }
  __syncwarp();
  if (value) {
    uint32_t m = t < nranks ? *reinterpret_cast<const volatile uint32_t *>(flags + bank + t) : 0u;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = max(m, __shfl_xor_sync(0xffffffffu, m, o));
    __syncwarp();
    if (t == 0) *value = m;
  }
  if (t == 0) *counter = epoch;
}

}  // namespace
}  // namespace fpb

static int peer_barrier_impl(uint32_t *counter, const uint32_t *flags, uint32_t *const *peer_flags, int nranks,
                             int rank, int timeout_ms, uint32_t *value, void *stream) {
  if (!counter || !flags || !peer_flags) return fail(FPB_ERR_INVALID_ARGUMENT, "fpb_peer_barrier: null pointer");
  if (nranks < 1 || nranks > 32 || rank < 0 || rank >= nranks || timeout_ms < 1)
    return fail(FPB_ERR_INVALID_ARGUMENT, "fpb_peer_barrier: nranks %d rank %d timeout %d ms", nranks, rank,
                timeout_ms);
  cudaError_t e = launch_pdl(fpb::peer_barrier_kernel, 1, 32, 0, fpb::as_stream(stream), counter, flags, peer_flags,
                              nranks, rank, (unsigned long long)timeout_ms * 1000000ull, fpb::device_error_ptr(),
                              value);
  if (e != cudaSuccess) return cuda_fail(e, "peer_barrier_kernel");
  FPB_LAUNCH_CHECK("peer_barrier_kernel");
  return FPB_OK;
}

extern "C" int fpb_peer_barrier(uint32_t *counter, const uint32_t *flags, uint32_t *const *peer_flags, int nranks,
                                int rank, int timeout_ms, void *stream) {
  return peer_barrier_impl(counter, flags, peer_flags, nranks, rank, timeout_ms, nullptr, stream);
}

extern "C" int fpb_peer_all_reduce_max(uint32_t *counter, const uint32_t *flags, uint32_t *const *peer_flags,
                                       int nranks, int rank, uint32_t *value, int timeout_ms, void *stream) {
  if (!value) return fail(FPB_ERR_INVALID_ARGUMENT, "fpb_peer_all_reduce_max: null value");
  return peer_barrier_impl(counter, flags, peer_flags, nranks, rank, timeout_ms, value, stream);
}
