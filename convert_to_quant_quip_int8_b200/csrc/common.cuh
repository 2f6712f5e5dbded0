// Shared host/device helpers for libqi8: status codes, error recording,
// element conversions and the device status word used by bounded waits.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include "../../include/qi8.h"

namespace qi8 {

// ---------------------------------------------------------------- errors
// Records a formatted message for qi8_last_error() and returns `code`.
int fail(int code, const char* fmt, ...);
// Maps a CUDA runtime error to QI8_ECUDA (with the CUDA message) or QI8_OK.
int check_cuda(cudaError_t e, const char* what);
// Device status word (one per device) written by in-kernel bounded waits.
unsigned int* device_status_ptr();
// Number of SMs of the current device (cached).
int sm_count();
// True when the current device is sm_100 (B200 family).
bool device_ok();

#define QI8_REQUIRE(cond, code, ...) \
  do { if (!(cond)) return ::qi8::fail((code), __VA_ARGS__); } while (0)
#define QI8_CUDA(expr) \
  do { int _rc = ::qi8::check_cuda((expr), #expr); if (_rc) return _rc; } while (0)

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
inline int elem_size(int dtype) {
  switch (dtype) {
    case QI8_BF16: case QI8_F16: return 2;
    case QI8_F32: case QI8_I32: return 4;
    case QI8_I8: return 1;
    default: return 0;
  }
}

// Status bits set by bounded waits that expired.
enum : unsigned int {
  ST_GEMM_PRODUCER = 1u << 0,
  ST_GEMM_MMA = 1u << 1,
  ST_GEMM_EPILOGUE = 1u << 2,
  ST_GEMM_DRAIN = 1u << 3,
  ST_PEER_BARRIER = 1u << 4,
};

// ---------------------------------------------------------- conversions
template <typename T> struct Elem;
template <> struct Elem<float> {
  static __device__ __forceinline__ float load(const float* p) { return *p; }
  static __device__ __forceinline__ float to_f32(float v) { return v; }
  static __device__ __forceinline__ float from_f32(float v) { return v; }
};
template <> struct Elem<__nv_bfloat16> {
  static __device__ __forceinline__ float to_f32(__nv_bfloat16 v) { return __bfloat162float(v); }
  static __device__ __forceinline__ __nv_bfloat16 from_f32(float v) { return __float2bfloat16_rn(v); }
};
template <> struct Elem<__half> {
  static __device__ __forceinline__ float to_f32(__half v) { return __half2float(v); }
  static __device__ __forceinline__ __half from_f32(float v) { return __float2half_rn(v); }
};

__device__ __forceinline__ float load_as_f32(const void* base, int dtype, int64_t i) {
  if (dtype == QI8_F32) return static_cast<const float*>(base)[i];
  if (dtype == QI8_BF16) return __bfloat162float(static_cast<const __nv_bfloat16*>(base)[i]);
  return __half2float(static_cast<const __half*>(base)[i]);
}

__device__ __forceinline__ void store_from_f32(void* base, int dtype, int64_t i, float v) {
  if (dtype == QI8_F32) static_cast<float*>(base)[i] = v;
  else if (dtype == QI8_BF16) static_cast<__nv_bfloat16*>(base)[i] = __float2bfloat16_rn(v);
  else static_cast<__half*>(base)[i] = __float2half_rn(v);
}

// Round-half-even fp32 -> int8 with clamp [lo, hi]  (torch round_().clamp_())
__device__ __forceinline__ int8_t rint_clamp(float v, float lo, float hi) {
  float r = rintf(v);
  r = fminf(fmaxf(r, lo), hi);
  return static_cast<int8_t>(static_cast<int>(r));
}

// Truncating fp32 -> int8 conversion with saturation, NaN -> 0 (PTX
// cvt.rzi semantics used by the Triton kernels' .to(int8)).
__device__ __forceinline__ int8_t trunc_sat(float v) {
  int i = __float2int_rz(v);  // NaN -> 0, saturates to int32
  i = i < -128 ? -128 : (i > 127 ? 127 : i);
  return static_cast<int8_t>(i);
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// ------------------------------------------- programmatic dependent launch
// With QI8_PDL=1 the kernels of the inference path are launched with
// programmatic stream serialization: a kernel may be scheduled while the
// previous kernel on the stream is still finishing, runs its prologue
// (barrier init, TMEM allocation, descriptor prefetch), and waits in
// pdl_wait() -- before its first global-memory access -- until that kernel
// has completed and its writes are visible.  Without the launch attribute
// both are no-ops.  Off by default: on the Flux-shaped stack (one CUDA graph
// of 456 launches) it measured 34.1 ms per forward against 32.9 ms without.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
// Lets the next kernel on the stream be scheduled (it still waits in pdl_wait).
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// True when QI8_PDL is set to a value other than 0 (read once per process).
bool pdl_enabled();

// Launches kern<<<grid, block, smem, st>>>(args...) with programmatic stream
// serialization when pdl_enabled().
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, Args&&... args) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...);
}

// Exact-erf GELU on an fp32 value (torch F.gelu default formula).
__device__ __forceinline__ float gelu_erf(float x) {
  return 0.5f * x * (1.0f + erff(x * 0.70710678118654752440f));
}

}  // namespace qi8
