// In-CTA fast Walsh-Hadamard transform of one row of n = 2^L fp32 values.
//
// Bit-exactness contract: each butterfly is one IEEE fp32 add or subtract,
// (lo, hi) -> (lo + hi, lo - hi) with lo the lower index, and the stages run
// in ascending stride order h = 1, 2, 4, ..., n/2 -- the order of the
// reference's CPU core (utils/hadamard.py:131-150) and of its Triton
// per-stage kernels (comfy/hadamard_kernels.py:211-237, 301-310).  Because
// every stage is exact-order elementwise, the result is identical bit for bit
// whichever thread performs which butterfly.
//
// Mapping: P = n/E threads each hold E consecutive elements ("contiguous
// mapping": thread t owns t*E .. t*E+E-1).  Strides < E run in registers,
// strides E .. 16E across lanes with shuffles.  Rows wider than one warp are
// re-distributed through shared memory so thread t owns t + P*e; the
// remaining strides (>= 32E >= P) again run in registers; a second exchange
// restores the contiguous mapping.
#pragma once

#include "common.cuh"

namespace qi8 {

template <int L> struct RotCfg {
  static constexpr int N = 1 << L;
  static constexpr int Q = (L <= 5) ? 0 : (L == 6 ? 1 : (L == 7 ? 2 : (L <= 11 ? 3 : (L <= 13 ? 4 : 5))));
  static constexpr int E = 1 << Q;          // elements per thread
  static constexpr int P = N / E;           // threads holding data
  static constexpr int THREADS = P < 32 ? 32 : P;
  static constexpr bool MULTIWARP = P > 32;
  static constexpr int B0 = 5 + 2 * Q - L;  // first register stage after the exchange
  static_assert(!MULTIWARP || (L <= 2 * Q + 5), "post-exchange strides must be in registers");
  static constexpr size_t SMEM = MULTIWARP ? sizeof(float) * N : 0;
};

// Transforms the row held in v (contiguous mapping, un-normalized).
// All THREADS threads of the CTA must call it; threads t >= P hold zeros.
// buf: shared float[N] (unused for single-warp rows).
template <int L>
__device__ __forceinline__ void fwht_row(float (&v)[RotCfg<L>::E], float* buf) {
  using C = RotCfg<L>;
  constexpr int E = C::E, P = C::P, Q = C::Q;
  const int t = threadIdx.x;
  const int lane = t & 31;

#pragma unroll
  for (int h = 1; h < E; h <<= 1) {
#pragma unroll
    for (int e = 0; e < E; ++e) {
      if (!(e & h)) {
        const float lo = v[e], hi = v[e + h];
        v[e] = lo + hi;
        v[e + h] = lo - hi;
      }
    }
  }
#pragma unroll
  for (int m = 1; m < 32 && m < P; m <<= 1) {
    const bool upper = (lane & m) != 0;
#pragma unroll
    for (int e = 0; e < E; ++e) {
      const float p = __shfl_xor_sync(0xffffffffu, v[e], m);
      v[e] = upper ? (p - v[e]) : (v[e] + p);
    }
  }
  if constexpr (C::MULTIWARP) {
    const int c0 = t * E;
#pragma unroll
    for (int e = 0; e < E; ++e) buf[c0 + e] = v[e];
    __syncthreads();
#pragma unroll
    for (int e = 0; e < E; ++e) v[e] = buf[t + P * e];
#pragma unroll
    for (int b = C::B0; b < Q; ++b) {
      const int s = 1 << b;
#pragma unroll
      for (int e = 0; e < E; ++e) {
        if (!(e & s)) {
          const float lo = v[e], hi = v[e + s];
          v[e] = lo + hi;
          v[e + s] = lo - hi;
        }
      }
    }
#pragma unroll
    for (int e = 0; e < E; ++e) buf[t + P * e] = v[e];
    __syncthreads();
#pragma unroll
    for (int e = 0; e < E; ++e) v[e] = buf[c0 + e];
  }
}

// Block-wide max over blockDim.x threads (multiple of 32); every thread gets it.
__device__ __forceinline__ float block_max(float v, float* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  v = warp_max(v);
  __syncthreads();  // red may still be read by a previous call
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float r = lane < nw ? red[lane] : 0.0f;
  return warp_max(r);
}

inline int log2_exact(int64_t n) {
  if (n <= 0 || (n & (n - 1))) return -1;
  int l = 0;
  while ((int64_t(1) << l) < n) ++l;
  return l;
}

}  // namespace qi8
