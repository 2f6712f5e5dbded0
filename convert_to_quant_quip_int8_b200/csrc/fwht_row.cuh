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

// ------------------------------------------- phased row FWHT (2^9..2^14)
// One row of n = 2^L fp32 values held by P = n/16 threads, 16 elements per
// thread whose indices differ only in a 4-bit window; the window moves up by
// 4 bits per phase (0, 4, 8, ..., and L-4 last) and the data moves between
// phases through an XOR-swizzled shared buffer (bank-conflict free).  Stages
// stay in ascending bit order.  A thread's phase-k writes go exactly to the
// addresses it read in phase k-1, so one buffer serves all phases.
namespace rowfwht {

// The swizzle is linear over XOR, so for an index base ^ off (disjoint bits)
// phys = swz(base) ^ swz(off): a per-thread base and a compile-time offset.
__host__ __device__ constexpr int swz(int i) {
  return i ^ (((i >> 5) & 7) << 2) ^ (((i >> 8) & 1) << 4);
}
// index of element e (window bits) of thread t for the window starting at
// bit w is wbase(t, w) | (e << w)
__device__ __forceinline__ int wbase(int t, int w) { return (t & ((1 << w) - 1)) | ((t >> w) << (w + 4)); }
template <int L>
__host__ __device__ constexpr int nwin() { return (L + 3) / 4; }
template <int L>
__host__ __device__ constexpr int wstart(int k) { return k < nwin<L>() - 1 ? 4 * k : L - 4; }

// butterflies of index bits [4k, min(4k + 4, L)) on the window of phase k;
// strides >= 2 run as packed fp32 pairs (sum, and difference as
// fma(hi, -1, lo): both single-rounded, identical to the scalar ops)
template <int L, int K>
__device__ __forceinline__ void stages(float (&v)[16]) {
  constexpr int w = wstart<L>(K);
  constexpr int hi = (4 * K + 4 < L) ? 4 * K + 4 : L;
#pragma unroll
  for (int bit = 4 * K; bit < hi; ++bit) {
    const int s = 1 << (bit - w);
    if (s == 1) {
#pragma unroll
      for (int e = 0; e < 16; e += 2) {
        const float lo = v[e], hi_v = v[e + 1];
        v[e] = lo + hi_v;
        v[e + 1] = lo - hi_v;
      }
    } else {
#pragma unroll
      for (int e = 0; e < 16; e += 2) {
        if (!(e & s)) {
          const float2 lo = make_float2(v[e], v[e + 1]);
          const float2 hv = make_float2(v[e + s], v[e + s + 1]);
          const float2 sm = __fadd2_rn(lo, hv);
          const float2 df = __ffma2_rn(hv, make_float2(-1.0f, -1.0f), lo);
          v[e] = sm.x;
          v[e + 1] = sm.y;
          v[e + s] = df.x;
          v[e + s + 1] = df.y;
        }
      }
    }
  }
}

template <int L, int K>
__device__ __forceinline__ void phase(float (&v)[16], float* buf, int t) {
  if constexpr (K < nwin<L>()) {
    constexpr int wp = wstart<L>(K - 1), w = wstart<L>(K);
    if constexpr (K == 1) {
      const int sb = swz(t * 16);
#pragma unroll
      for (int j = 0; j < 4; ++j)
        *reinterpret_cast<float4*>(buf + (sb ^ swz(4 * j))) = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
    } else {
      const int sb = swz(wbase(t, wp));
#pragma unroll
      for (int e = 0; e < 16; ++e) buf[sb ^ swz(e << wp)] = v[e];
    }
    __syncthreads();
    const int sb = swz(wbase(t, w));
#pragma unroll
    for (int e = 0; e < 16; ++e) v[e] = buf[sb ^ swz(e << w)];
    stages<L, K>(v);
    phase<L, K + 1>(v, buf, t);
  }
}

}  // namespace rowfwht

inline int log2_exact(int64_t n) {
  if (n <= 0 || (n & (n - 1))) return -1;
  int l = 0;
  while ((int64_t(1) << l) < n) ++l;
  return l;
}

}  // namespace qi8
