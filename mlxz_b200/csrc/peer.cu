// Peer memory for the all-gather of head-sharded decode outputs: CUDA IPC
// export / open of device buffers between the processes of one node (one
// process per GPU), and the bounded wait on the signal words that the peers'
// decode launches publish (mz_paged_append_decode_allgather).
//
// Protocol, per launch with epoch e (the same sequence of epochs on every
// rank, starting at 1): rank s's decode kernel stores its output rows into
// every rank's gathered buffer, then its last block stores e into signal word s
// of every peer with a system-scope release.  mz_peer_wait on rank r then
// acquires signal words s != r until each holds e or later (wrap-safe), so
// work queued after it on r's stream sees every peer's rows.  A word that
// does not reach e within the time limit sets MZ_DEVERR_TIMEOUT in the
// caller's error word and the wait returns: nothing blocks beyond the limit.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <cstring>
#include <mutex>

#include "common.cuh"

namespace mz {
namespace {

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t *addr) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(addr) : "memory");
  return v;
}

// One thread per source rank; each polls its word until it reaches `epoch`
// or the time limit passes (checked every 64 polls).
__global__ void peer_wait_kernel(const uint32_t *sig, int n_ranks, int rank, uint32_t epoch,
                                 uint64_t timeout_ns, int32_t *err) {
  const int r = threadIdx.x;
  if (r >= n_ranks || r == rank) return;
  uint64_t t0 = 0;
  for (uint32_t it = 0;; ++it) {
    if (static_cast<int32_t>(ld_acquire_sys(sig + r) - epoch) >= 0) return;
    if ((it & 63u) == 63u) {
      const uint64_t now = global_timer_ns();
      if (t0 == 0) {
        t0 = now;
      } else if (now - t0 > timeout_ns) {
        dev_error(err, MZ_DEVERR_TIMEOUT);
        return;
      }
      __nanosleep(256);
    }
  }
}

using GetRangeFn = CUresult (*)(CUdeviceptr *, size_t *, CUdeviceptr);

GetRangeFn get_range_fn() {
  static GetRangeFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, []() {
    void *f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuMemGetAddressRange", &f, 12000, cudaEnableDefault,
                                         &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<GetRangeFn>(f);
  });
  return fn;
}

}  // namespace
}  // namespace mz

using namespace mz;

static_assert(sizeof(cudaIpcMemHandle_t) == MZ_IPC_HANDLE_BYTES, "IPC handle size");

extern "C" int mz_ipc_export(const void *ptr, void *handle, uint64_t *offset) {
  if (!ptr || !handle || !offset) return fail(MZ_ERR_INVALID_ARG, "mz_ipc_export: null argument");
  auto range = get_range_fn();
  if (!range) return fail(MZ_ERR_CUDA, "mz_ipc_export: cuMemGetAddressRange is unavailable");
  CUdeviceptr base = 0;
  size_t size = 0;
  CUresult r = range(&base, &size, reinterpret_cast<CUdeviceptr>(ptr));
  if (r != CUDA_SUCCESS)
    return fail(MZ_ERR_INVALID_ARG, "mz_ipc_export: %p is not device memory (%d)", ptr, (int)r);
  cudaIpcMemHandle_t h;
  cudaError_t e = cudaIpcGetMemHandle(&h, const_cast<void *>(ptr));
  if (e != cudaSuccess) return cuda_fail(e, "mz_ipc_export: cudaIpcGetMemHandle");
  std::memcpy(handle, &h, sizeof(h));
  *offset = static_cast<uint64_t>(reinterpret_cast<CUdeviceptr>(ptr) - base);
  return MZ_OK;
}

extern "C" int mz_ipc_open(const void *handle, uint64_t offset, void **base, void **ptr) {
  if (!handle || !base || !ptr) return fail(MZ_ERR_INVALID_ARG, "mz_ipc_open: null argument");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  void *b = nullptr;
  cudaError_t e = cudaIpcOpenMemHandle(&b, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return cuda_fail(e, "mz_ipc_open: cudaIpcOpenMemHandle");
  *base = b;
  *ptr = static_cast<uint8_t *>(b) + offset;
  return MZ_OK;
}

extern "C" int mz_ipc_close(void *base) {
  if (!base) return fail(MZ_ERR_INVALID_ARG, "mz_ipc_close: null base");
  cudaError_t e = cudaIpcCloseMemHandle(base);
  if (e != cudaSuccess) return cuda_fail(e, "mz_ipc_close: cudaIpcCloseMemHandle");
  return MZ_OK;
}

extern "C" int mz_peer_wait(const int32_t *signal, int32_t n_ranks, int32_t rank, uint32_t epoch,
                            uint64_t timeout_ns, int32_t *dev_err, mz_stream_t stream) {
  if (n_ranks < 1 || n_ranks > MZ_MAX_RANKS || rank < 0 || rank >= n_ranks)
    return fail(MZ_ERR_INVALID_ARG, "mz_peer_wait: n_ranks %d / rank %d out of range", n_ranks,
                rank);
  if (epoch == 0) return fail(MZ_ERR_INVALID_ARG, "mz_peer_wait: epoch must be nonzero");
  if (timeout_ns == 0 || timeout_ns > 60ull * 1000000000ull)
    return fail(MZ_ERR_INVALID_ARG, "mz_peer_wait: timeout must be in (0, 60 s]");
  if (n_ranks == 1) return MZ_OK;
  if (!signal || !aligned(signal, 4))
    return fail(MZ_ERR_INVALID_ARG, "mz_peer_wait: signal is null or misaligned");
  peer_wait_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(
      reinterpret_cast<const uint32_t *>(signal), n_ranks, rank, epoch, timeout_ns, dev_err);
  MZ_CHECK_LAUNCH("mz_peer_wait");
  return MZ_OK;
}
