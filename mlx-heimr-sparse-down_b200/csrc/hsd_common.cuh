// Shared helpers of libhsd: status handling, dtype conversion, small PTX wrappers.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include "hsd.h"

namespace hsd {

// Records `code` and a printf-style message as this host thread's last error and
// returns `code` (host only; defined in hsd_api.cu).
int set_error(int code, const char* fmt, ...);

// HSD_ERR_CUDA with the runtime's message when `e` is not cudaSuccess, else HSD_OK.
inline int check_cuda(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return HSD_OK;
  return set_error(HSD_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

// The launch's own error (a bad configuration), without synchronising.
inline int check_launch(const char* what) { return check_cuda(cudaGetLastError(), what); }

inline bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

// ---- device-side conversion of the supported element types to / from fp32
template <typename T> __device__ __forceinline__ float to_f32(T v);
template <> __device__ __forceinline__ float to_f32<float>(float v) { return v; }
template <> __device__ __forceinline__ float to_f32<__half>(__half v) { return __half2float(v); }
template <> __device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 v) {
  return __bfloat162float(v);
}
template <typename T> __device__ __forceinline__ T from_f32(float v);
template <> __device__ __forceinline__ float from_f32<float>(float v) { return v; }
template <> __device__ __forceinline__ __half from_f32<__half>(float v) { return __float2half_rn(v); }
template <> __device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float v) {
  return __float2bfloat16_rn(v);
}

// 16-bit storage type (bf16 or f16) bits -> fp32
template <typename T> __device__ __forceinline__ float bits16_to_f32(uint16_t b);
template <> __device__ __forceinline__ float bits16_to_f32<__nv_bfloat16>(uint16_t b) {
  return __uint_as_float(static_cast<uint32_t>(b) << 16);
}
template <> __device__ __forceinline__ float bits16_to_f32<__half>(uint16_t b) {
  return __half2float(__ushort_as_half(b));
}

// ---- async copies (sm_80+ LDGSTS; 16-byte pieces, L2-only caching of the source)
__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
  const uint32_t s = static_cast<uint32_t>(__cvta_generic_to_shared(smem));
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(s), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;\n" ::: "memory"); }

// Programmatic dependent launch. A kernel launched through launch_pdl may start while the
// previous kernel of its stream is still running (once every block of that kernel has
// executed pdl_launch_dependents or finished); it must execute pdl_wait -- which returns
// when the previous kernel has finished and its memory is visible -- before it reads memory
// that earlier kernels write or writes memory that they read. Work on inputs no kernel of
// the step writes (weights) may come before the wait. Both are no-ops without a dependency.
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                              Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

// Streaming 16-byte global load that does not allocate in L1.
__device__ __forceinline__ uint4 ldg_nc_v4(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

}  // namespace hsd

// Per-translation-unit device status word: the first device-side error code wins.
#define HSD_DEFINE_STATUS(name)                                                      \
  __device__ int hsd_status_word_##name = 0;                                         \
  __device__ __forceinline__ void hsd_flag_##name(int code) {                        \
    atomicCAS(&hsd_status_word_##name, 0, code);                                     \
  }                                                                                  \
  int hsd_read_status_##name(int* out, cudaStream_t st) {                            \
    int v = 0, z = 0;                                                                \
    cudaError_t e = cudaMemcpyFromSymbolAsync(&v, hsd_status_word_##name, sizeof(int), 0, \
                                              cudaMemcpyDeviceToHost, st);           \
    if (e == cudaSuccess)                                                            \
      e = cudaMemcpyToSymbolAsync(hsd_status_word_##name, &z, sizeof(int), 0,        \
                                  cudaMemcpyHostToDevice, st);                       \
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);                             \
    *out = v;                                                                        \
    return hsd::check_cuda(e, "hsd_device_status(" #name ")");                       \
  }
