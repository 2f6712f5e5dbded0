// Activation chaining of the block-wise int8 layout: GELU applied to an int8
// activation with per-(row, 128-block) scales, requantized in the same format
// (the reference's int8_gelu, comfy/int8_kernels.py:1122-1312, used by the
// BlockWiseINT8Layout aten.gelu handler, comfy/quant_ops.py:435-448).
//
// One warp per (row, block) of 128 elements, four per lane (one 32-bit load
// and store), grid-stride over all blocks.  The arithmetic follows the
// reference kernel step by step:
//   v = fp32(q) * s
//   e = erf(v / fp32(1.41421356237))      evaluated in double, rounded to fp32
//   g = (v * 0.5) * (1 + e)
//   scale = max(amax(|g|) / 127, 1e-8)     per (row, block)
//   q' = trunc(clamp(g / scale, -127, 127))
// The reference's erf is the correctly rounded fp32 value (its kernels are
// pinned by the Triton interpreter, which evaluates erf in double and rounds),
// which CUDA's double erf reproduces after rounding except when the double
// result lies within a few double ulps of an fp32 rounding boundary.
#include <cstdint>

#include "common.cuh"

namespace qi8 {
namespace {

constexpr int GELU_WARPS = 8;

__global__ void __launch_bounds__(GELU_WARPS * 32)
int8_gelu_kernel(const int8_t* __restrict__ q, const float* __restrict__ s, int64_t rows, int nb,
                 int8_t* __restrict__ q_out, float* __restrict__ s_out) {
  const int lane = threadIdx.x & 31;
  const int64_t n_blocks = rows * nb;
  const int64_t warp0 = (int64_t)blockIdx.x * GELU_WARPS + (threadIdx.x >> 5);
  const int64_t stride = (int64_t)gridDim.x * GELU_WARPS;
  for (int64_t b = warp0; b < n_blocks; b += stride) {
    // block b = (row, column block) in row-major order: elements [b * 128, b * 128 + 128)
    const uint32_t word = __ldg(reinterpret_cast<const uint32_t*>(q + b * 128) + lane);
    const float sc = __ldg(s + b);
    float g[4];
    float amax = 0.0f;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int qi = (int)(int8_t)((word >> (8 * i)) & 0xFFu);
      const float v = __fmul_rn((float)qi, sc);
      const float e = (float)erf((double)__fdiv_rn(v, 1.41421356237f));
      g[i] = __fmul_rn(__fmul_rn(v, 0.5f), __fadd_rn(1.0f, e));
      amax = fmaxf(amax, fabsf(g[i]));
    }
    amax = warp_max(amax);
    const float scale = fmaxf(__fdiv_rn(amax, 127.0f), 1e-8f);
    uint32_t out = 0;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int qo = __float2int_rz(fminf(fmaxf(__fdiv_rn(g[i], scale), -127.0f), 127.0f));
      out |= (uint32_t)(qo & 0xFF) << (8 * i);
    }
    reinterpret_cast<uint32_t*>(q_out + b * 128)[lane] = out;
    if (lane == 0) s_out[b] = scale;
  }
}

}  // namespace
}  // namespace qi8

using namespace qi8;

extern "C" int qi8_int8_gelu(const int8_t* q, const float* scale, int64_t rows, int64_t n, int block, int8_t* q_out,
                             float* scale_out, void* stream) {
  QI8_REQUIRE(device_ok(), QI8_EUNSUPPORTED, "no sm_100 device current");
  QI8_REQUIRE(q && scale && q_out && scale_out, QI8_EINVAL, "null pointer");
  QI8_REQUIRE(block == 128, QI8_ESHAPE, "block_size %d: the int8 GELU uses 128-element blocks", block);
  QI8_REQUIRE(rows >= 0 && n > 0 && n % block == 0, QI8_ESHAPE,
              "Last dimension must be divisible by block_size=%d, got %lld", block, (long long)n);
  QI8_REQUIRE((reinterpret_cast<uintptr_t>(q) & 3) == 0 && (reinterpret_cast<uintptr_t>(q_out) & 3) == 0, QI8_EALIGN,
              "int8 tensors must be 4-byte aligned");
  if (rows == 0) return QI8_OK;
  const int64_t n_blocks = rows * (n / block);
  int64_t grid = (n_blocks + GELU_WARPS - 1) / GELU_WARPS;
  const int64_t cap = (int64_t)(sm_count() > 0 ? sm_count() : 148) * 16;
  if (grid > cap) grid = cap;
  int8_gelu_kernel<<<(unsigned)grid, GELU_WARPS * 32, 0, static_cast<cudaStream_t>(stream)>>>(
      q, scale, rows, (int)(n / block), q_out, scale_out);
  return check_cuda(cudaGetLastError(), "int8_gelu_kernel launch");
}
