// Shared helpers for the pyre_b200 CUDA sources (sm_100a only).
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>
#include <string>

#include "../../include/pyre_b200.h"

namespace pyre {

// Records msg as the calling thread's last error and returns code.
int set_error(int code, const std::string& msg);
// Maps a CUDA error to PYRE_ECUDA with context; cudaSuccess -> PYRE_OK.
int cuda_status(cudaError_t e, const char* what);
// Number of SMs of the current device (cached per device).
int sm_count();
// Raises a kernel's dynamic shared-memory limit once per (kernel, device).
int set_smem_limit(const void* kernel, int bytes);

#define PYRE_CHECK_ARG(cond, msg)                                   \
  do {                                                              \
    if (!(cond)) return ::pyre::set_error(PYRE_EINVAL, (msg));      \
  } while (0)

#define PYRE_CUDA_TRY(call)                                         \
  do {                                                              \
    cudaError_t _e = (call);                                        \
    if (_e != cudaSuccess) return ::pyre::cuda_status(_e, #call);   \
  } while (0)

// Launch-error check after a <<<>>> launch.
#define PYRE_LAUNCH_CHECK(what)                                     \
  do {                                                              \
    cudaError_t _e = cudaGetLastError();                            \
    if (_e != cudaSuccess) return ::pyre::cuda_status(_e, what);    \
  } while (0)

// ---- programmatic dependent launch ----------------------------------------------------
// A kernel launched with launch_pdl may start while the previous kernel of its stream is still
// running. Before pdl_wait() it may only read data no earlier kernel is still writing (weights,
// its own scratch) and write nothing another kernel reads; pdl_wait() returns once the previous
// kernel has finished and its writes are visible (at once when launched without the
// attribute). pdl_trigger() lets the next kernel start; every kernel here calls it only after
// its own pdl_wait(), so at most two kernels of a stream overlap.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// Whether launch_pdl sets the attribute: on unless the environment sets PYRE_PDL=0 (read once;
// the kernels are the same either way, pdl_wait() then returns at once).
bool pdl_enabled();

template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                       Args&&... args) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr{};
  attr.id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr.val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = &attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<Args&&>(args)...);
}

// ---- element loads ------------------------------------------------------------------

__device__ __forceinline__ float to_f32(float v) { return v; }
__device__ __forceinline__ float to_f32(__nv_bfloat16 v) { return __bfloat162float(v); }
__device__ __forceinline__ float to_f32(__half v) { return __half2float(v); }

// Read-only, streaming (no L1 allocation) 16-byte load for weights read exactly once.
__device__ __forceinline__ int4 ld_stream16(const void* p) {
  int4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.s32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

__device__ __forceinline__ int2 ld_stream8(const void* p) {
  int2 r;
  asm volatile("ld.global.nc.L1::no_allocate.v2.s32 {%0,%1}, [%2];"
               : "=r"(r.x), "=r"(r.y)
               : "l"(p));
  return r;
}

// Exact int8 -> f32 for the 4 signed bytes of w: each byte b becomes the float with
// bits 0x4B0000uu (= 2^23 + u) where u = b ^ 0x80 = b + 128, minus (2^23 + 128).
// One byte-permute and one add per element; both steps are exact.
__device__ __forceinline__ void s8x4_to_f32(uint32_t w, float (&f)[4]) {
  const uint32_t u = w ^ 0x80808080u;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    f[i] = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7540u + i)) - 8388736.0f;
  }
}

// ---- memory-model helpers for peer (NVLink) flags ----------------------------------

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void st_release_gpu(uint32_t* p, uint32_t v) {
  asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Spins until *flag == want or timeout_ns elapses. Returns true on success.
__device__ __forceinline__ bool wait_flag_eq(const uint32_t* flag, uint32_t want,
                                             uint64_t timeout_ns) {
  if (ld_acquire_sys(flag) == want) return true;
  const uint64_t t0 = globaltimer_ns();
  while (true) {
    if (ld_acquire_sys(flag) == want) return true;
    if (globaltimer_ns() - t0 > timeout_ns) return false;
    __nanosleep(32);
  }
}

}  // namespace pyre
