// Shared helpers for the libsvx kernels (sm_100a): error reporting, bf16 conversions, bounded waits.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>
#include <atomic>
#include <mutex>
#include <string>
#include <utility>

#include "svx.h"

namespace svx {

// Per-host-thread error text behind svx_last_error().
void set_error(const std::string& text);
int fail(int status, const std::string& text);

#define SVX_CHECK_CUDA(expr)                                                                \
  do {                                                                                      \
    cudaError_t _e = (expr);                                                                \
    if (_e != cudaSuccess)                                                                  \
      return ::svx::fail(SVX_ERR_CUDA, std::string(#expr) + ": " + cudaGetErrorString(_e)); \
  } while (0)

#define SVX_REQUIRE(cond, text)                                   \
  do {                                                            \
    if (!(cond)) return ::svx::fail(SVX_ERR_INVALID, (text));     \
  } while (0)

// Launch error of the kernel just enqueued (configuration errors only; no host sync).
int launch_status(const char* what);

// A value set up once per device: a kernel's dynamic shared-memory opt-in (cudaFuncSetAttribute) belongs to the
// device's primary context, and occupancy, SM counts and symbol addresses are per device. `get` runs
// configure(device, &value) on the first call made with each device current (under a lock, so first calls from
// several host threads configure a device once) and returns the stored value afterwards. The values live for the
// process: after cudaDeviceReset, or once the primary context has been released and created again, they are stale,
// so the library does not support either while it is loaded.
constexpr int kMaxDevices = 64;

template <typename T>
class PerDevice {
 public:
  template <typename F>
  int get(T* value, F&& configure) {
    int device = 0;
    SVX_CHECK_CUDA(cudaGetDevice(&device));
    if (device < 0 || device >= kMaxDevices) return fail(SVX_ERR_INVALID, "device index beyond the per-device tables");
    if (!ready_[device].load(std::memory_order_acquire)) {
      std::lock_guard<std::mutex> lock(mutex_);
      if (!ready_[device].load(std::memory_order_relaxed)) {
        T v{};
        const int rc = configure(device, &v);
        if (rc) return rc;
        values_[device] = v;
        ready_[device].store(true, std::memory_order_release);
      }
    }
    *value = values_[device];
    return SVX_OK;
  }

 private:
  std::mutex mutex_;
  std::atomic<bool> ready_[kMaxDevices] = {};
  T values_[kMaxDevices] = {};
};

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

// Launch with programmatic stream serialization (the kernel must call grid_dependency_wait before dependent reads).
template <typename... Exp, typename... Act>
inline int launch_dependent(const char* what, void (*kernel)(Exp...), dim3 grid, dim3 block, size_t smem,
                            cudaStream_t stream, Act&&... args) {
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, std::forward<Act>(args)...);
  if (e != cudaSuccess) {
    (void)cudaGetLastError();
    return fail(SVX_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
  }
  return launch_status(what);
}

__device__ __forceinline__ float bf16_to_f32(uint16_t v) { return __uint_as_float(uint32_t(v) << 16); }

// Round-to-nearest-even fp32 -> bf16 (NaN stays NaN), the conversion torch uses for bf16 tensors.
__device__ __forceinline__ uint16_t f32_to_bf16(float f) { return __bfloat16_as_ushort(__float2bfloat16_rn(f)); }
__device__ __forceinline__ float round_bf16(float f) { return bf16_to_f32(f32_to_bf16(f)); }

template <typename T> __device__ __forceinline__ float load_as_f32(const T* p);
template <> __device__ __forceinline__ float load_as_f32<float>(const float* p) { return *p; }
template <> __device__ __forceinline__ float load_as_f32<uint16_t>(const uint16_t* p) { return bf16_to_f32(*p); }

// Bounded spin: an mbarrier wait gives up after this many nanoseconds of %globaltimer and the kernel reports
// SVX_STATUS_WAIT_TIMEOUT (try_wait may suspend for a system-dependent time per poll, so polls are not counted).
constexpr uint64_t kWaitNanoseconds = 2000000000ull;

__device__ __forceinline__ uint64_t global_timer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count));
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return done != 0;
}

// Wait for the phase with the given parity; false after kWaitNanoseconds (the caller records the timeout).
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t start = global_timer_ns();
  while (!mbar_try_wait(bar, parity))
    if (global_timer_ns() - start > kWaitNanoseconds) return false;
  return true;
}

// Programmatic dependent launch. Kernels of the forward signal grid_launch_dependents() on entry, so the next
// kernel of the stream (launched with launch_dependent) may be scheduled onto SMs as they free up and run its
// prologue; every such kernel calls grid_dependency_wait() before its first read of memory an earlier kernel wrote.
__device__ __forceinline__ void grid_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void grid_dependency_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

__device__ __forceinline__ int warp_id() { return threadIdx.x >> 5; }
__device__ __forceinline__ int lane_id() { return threadIdx.x & 31; }

}  // namespace svx
