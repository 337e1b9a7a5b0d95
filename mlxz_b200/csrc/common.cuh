// Shared helpers for the mlxz_b200 kernels: error plumbing, device queries,
// and the inline-PTX wrappers (mbarrier, bulk tensor copies, ldmatrix, mma).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <mutex>

#include "../../include/mlxz_b200.h"

namespace mz {

// Records a formatted message as the calling thread's last error and returns
// `code`, so call sites read `return fail(MZ_ERR_INVALID_ARG, "...")`.
int fail(int code, const char *fmt, ...);
// Maps a CUDA error to MZ_ERR_CUDA with the call that produced it.
int cuda_fail(cudaError_t e, const char *what);
// Element size of an mz_dtype, 0 for an unknown value.
int dtype_bytes(int dtype);
// Current device and its SM count (cached per device).
int current_device();
int sm_count(int device);

constexpr int kMaxDevices = 64;

// One-time set-up per device, e.g. a kernel's shared-memory opt-in: function
// attributes belong to each device's context, so a process that drives
// several GPUs needs them set on every device it launches on.  The set-up
// runs on the current device the first time device_once sees it; its status
// (and an int it produces, such as an occupancy) is kept for that device.
struct DeviceOnce {
  std::once_flag flag[kMaxDevices];
  cudaError_t err[kMaxDevices] = {};
  int value[kMaxDevices] = {};
};

template <class F>
int device_once(DeviceOnce &o, F &&setup, int *value, const char *what) {
  const int d = current_device();
  if (d < 0 || d >= kMaxDevices) return fail(MZ_ERR_CUDA, "%s: no usable current device", what);
  std::call_once(o.flag[d], [&]() { o.err[d] = setup(&o.value[d]); });
  if (o.err[d] != cudaSuccess) return cuda_fail(o.err[d], what);
  if (value) *value = o.value[d];
  return MZ_OK;
}

// Dynamic shared-memory opt-in of kernel `k` on the current device (once).
template <class KernelPtr>
int smem_optin(KernelPtr k, int smem_bytes, DeviceOnce &o, const char *what) {
  return device_once(
      o, [&](int *) { return cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_bytes); },
      nullptr, what);
}

inline bool aligned(const void *p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

#define MZ_CHECK_LAUNCH(what)                                   \
  do {                                                          \
    cudaError_t e_ = cudaGetLastError();                        \
    if (e_ != cudaSuccess) return ::mz::cuda_fail(e_, what);    \
  } while (0)

// ---------------------------------------------------------------------------
// Device-side helpers.
// ---------------------------------------------------------------------------

__device__ __forceinline__ void dev_error(int32_t *err, int bit) {
  if (err) atomicOr(err, bit);
}

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t global_timer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// mbarrier primitives (shared::cta).  One arrival (the issuing lane) plus the
// transaction bytes of the bulk copies completes a phase.
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t phase) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(phase)
      : "memory");
  return ok != 0;
}

// Bounded wait: polls the barrier phase and gives up after `timeout_ns` of
// wall time (checked every 256 polls).  Returns false on timeout.
__device__ __forceinline__ bool mbar_wait_bounded(uint32_t bar, uint32_t phase,
                                                  uint64_t timeout_ns) {
  uint64_t t0 = 0;
  for (uint32_t it = 1;; ++it) {
    if (mbar_try_wait(bar, phase)) return true;
    if ((it & 255u) == 0u) {
      uint64_t now = global_timer_ns();
      if (t0 == 0) {
        t0 = now;
      } else if (now - t0 > timeout_ns) {
        return false;
      }
    }
  }
}

// Orders this thread's generic-proxy shared-memory accesses before later
// async-proxy (bulk copy) accesses to the same buffers.
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// 2-D bulk tensor copy global -> shared (no multicast), completion counted on
// the mbarrier.  `tmap` is the generic address of a __grid_constant__ map.
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const void *tmap, int x, int y,
                                            uint32_t bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(x), "r"(y), "r"(bar), "l"(policy)
      : "memory");
}

// 1-D bulk copy global -> shared (no multicast), completion counted on the
// mbarrier.  Both addresses 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_load(uint32_t dst, const void *src, uint32_t bytes,
                                          uint32_t bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1], %2, [%3], %4;" ::"r"(dst),
      "l"(src), "r"(bytes), "r"(bar), "l"(policy)
      : "memory");
}

__device__ __forceinline__ uint64_t l2_policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}

__device__ __forceinline__ uint64_t l2_policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t &r0, uint32_t &r1, uint32_t &r2,
                                        uint32_t &r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_trans(uint32_t addr, uint32_t &r0, uint32_t &r1,
                                              uint32_t &r2, uint32_t &r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

// D(16x8 f32) += A(16x16) * B(16x8), A row-major, B column-major.
template <bool BF16>
__device__ __forceinline__ void mma_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                          uint32_t b1) {
  if constexpr (BF16) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, "
        "{%4, %5, %6, %7}, {%8, %9}, {%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  } else {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, "
        "{%4, %5, %6, %7}, {%8, %9}, {%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  }
}

// Transpose an 8x8 matrix of 16-bit elements held one row-pair per lane in
// mma C-fragment order (lane l holds row l/4, columns 2(l%4), 2(l%4)+1).
__device__ __forceinline__ uint32_t movmatrix_trans(uint32_t x) {
  uint32_t y;
  asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(y) : "r"(x));
  return y;
}

// 2^x with the hardware approximation (ex2.approx, flush-to-zero); 2^-inf = 0.
__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Pack two floats into one 32-bit register of 16-bit elements (lo in bits 0-15).
template <bool BF16>
__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  if constexpr (BF16) {
    __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t *>(&v);
  } else {
    __half2 v = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t *>(&v);
  }
}
// Round x to the 16-bit type and return the rounded value as float.
template <bool BF16>
__device__ __forceinline__ float round16(float x) {
  if constexpr (BF16) {
    return __bfloat162float(__float2bfloat16_rn(x));
  } else {
    return __half2float(__float2half_rn(x));
  }
}

}  // namespace mz
