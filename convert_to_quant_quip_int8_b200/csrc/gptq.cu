// GPTQ / LDLQ error-feedback quantization of one column block (the
// reference's gptq_quant_block_kernel, comfy/gptq_kernels.py:11-85, used by
// its GPTQ converter and by the QuIP converter's LDLQ loop,
// converters/gptq_int8.py:137 and converters/quip_int8.py:861-864).
//
// Rows are independent; inside a row the B columns are processed in order:
//   s   = max(|scale|, 1e-12)                 (scalar, or the row's scale)
//   q_j = clamp(rint(w_j / s), -127, 127)     (the reference's floor/fraction
//                                              test is round-half-even)
//   d   = max(|Hinv[j, j]|, 1e-12)
//   e_j = (w_j - q_j * s) / d
//   w_k = w_k - e_j * Hinv[j, k]   for k > j
// every operation separately rounded in fp32.  W is updated in place (column
// j keeps the value it was quantized from), Q and Err receive q and e.
//
// Layout: one lane per row; a warp's 32 rows of the block sit transposed in
// shared memory ([B][33], bank-conflict-free column access), the Hinv block
// ([B][B], row j read as a broadcast) is shared by the CTA's warps.
#include <cstdint>

#include "common.cuh"

namespace qi8 {
namespace {

constexpr int GPTQ_WARPS = 2;
constexpr int GPTQ_MAX_B = 128;

__global__ void __launch_bounds__(GPTQ_WARPS * 32)
gptq_block_kernel(float* __restrict__ W, int64_t M, int B, int64_t ld_w, const float* __restrict__ hinv, int64_t ld_h,
                  const float* __restrict__ scale, int scalar, int8_t* __restrict__ q_out, int64_t ld_q,
                  float* __restrict__ err_out, int64_t ld_e) {
  extern __shared__ float sm[];
  float* H = sm;                          // [B][B]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float* wt = sm + B * B + warp * B * 33;  // [B][33]: wt[j * 33 + r] = W[row0 + r, j]
  for (int i = threadIdx.x; i < B * B; i += blockDim.x) H[i] = hinv[(int64_t)(i / B) * ld_h + (i % B)];
  const int64_t row0 = ((int64_t)blockIdx.x * GPTQ_WARPS + warp) * 32;
  for (int r = 0; r < 32; ++r) {
    const int64_t row = row0 + r;
    for (int j = lane; j < B; j += 32) wt[j * 33 + r] = row < M ? W[row * ld_w + j] : 0.0f;
  }
  __syncthreads();
  const int64_t row = row0 + lane;
  const bool ok = row < M;
  float s = scalar ? scale[0] : (ok ? scale[row] : 1.0f);
  s = fmaxf(fabsf(s), 1e-12f);
  for (int j = 0; j < B; ++j) {
    const float w = wt[j * 33 + lane];
    const float q = fminf(fmaxf(rintf(__fdiv_rn(w, s)), -127.0f), 127.0f);
    const float d = fmaxf(fabsf(H[j * B + j]), 1e-12f);
    const float e = __fdiv_rn(__fsub_rn(w, __fmul_rn(q, s)), d);
    if (ok) {
      q_out[row * ld_q + j] = (int8_t)(int)q;
      err_out[row * ld_e + j] = e;
    }
    const float* hj = H + j * B;
    for (int k = j + 1; k < B; ++k) wt[k * 33 + lane] = __fsub_rn(wt[k * 33 + lane], __fmul_rn(e, hj[k]));
  }
  __syncwarp();
  for (int r = 0; r < 32; ++r) {
    const int64_t rr = row0 + r;
    if (rr >= M) break;
    for (int j = lane; j < B; j += 32) W[rr * ld_w + j] = wt[j * 33 + r];
  }
}

}  // namespace
}  // namespace qi8

using namespace qi8;

extern "C" int qi8_gptq_quant_block(float* W, int64_t M, int64_t B, int64_t ld_w, const float* hinv, int64_t ld_h,
                                    const float* scale, int scale_is_scalar, int8_t* q_out, int64_t ld_q,
                                    float* err_out, int64_t ld_e, void* stream) {
  QI8_REQUIRE(device_ok(), QI8_EUNSUPPORTED, "no sm_100 device current");
  QI8_REQUIRE(W && hinv && scale && q_out && err_out, QI8_EINVAL, "null pointer");
  QI8_REQUIRE(M >= 0 && B >= 1 && B <= GPTQ_MAX_B, QI8_ESHAPE, "block of %lld columns (1..%d supported)",
              (long long)B, GPTQ_MAX_B);
  QI8_REQUIRE(ld_w >= B && ld_h >= B && ld_q >= B && ld_e >= B, QI8_ESHAPE, "row strides must be >= B");
  if (M == 0) return QI8_OK;
  const size_t smem = sizeof(float) * ((size_t)B * B + (size_t)GPTQ_WARPS * B * 33);
  if (smem > 48 * 1024)
    QI8_CUDA(cudaFuncSetAttribute(gptq_block_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  const int64_t grid = (M + 32 * GPTQ_WARPS - 1) / (32 * GPTQ_WARPS);
  gptq_block_kernel<<<(unsigned)grid, GPTQ_WARPS * 32, smem, static_cast<cudaStream_t>(stream)>>>(
      W, M, (int)B, ld_w, hinv, ld_h, scale, scale_is_scalar, q_out, ld_q, err_out, ld_e);
  return check_cuda(cudaGetLastError(), "gptq_block_kernel launch");
}
