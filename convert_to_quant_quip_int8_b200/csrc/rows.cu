// Row kernels of the QuIP W8A8 path (HBM-bound):
//   * qi8_quant_rows       -- per-token / per-128-block int8 quantization
//   * qi8_rotate_quant_rows (K1) -- sign + FWHT + quantization, one pass
//   * qi8_fwht_rows        -- sign + FWHT (+ sign) to fp32
//   * qi8_unrotate_rows    (K3) -- FWHT + sign + slice + bias -> bf16/f16/f32
//   * qi8_dequant, qi8_quant_weight -- layout (de)quantizers
//
// One CTA per row.  The FWHT core (fwht_row.cuh) reproduces the reference's
// butterfly order bit for bit; the normalization is one fp32 multiply by
// float(1/sqrt(n)) (utils/hadamard.py:155-157).  Quantization follows the
// reference rule selected by the mode (see qi8.h).
#include <cstdint>
#include <cmath>

#include <type_traits>

#include "common.cuh"
#include "fwht_row.cuh"

namespace qi8 {
namespace {

// ------------------------------------------------------------------ loads
template <typename T> __device__ __forceinline__ float to_f32(T v);
template <> __device__ __forceinline__ float to_f32<float>(float v) { return v; }
template <> __device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }
template <> __device__ __forceinline__ float to_f32<__half>(__half v) { return __half2float(v); }

// Loads E consecutive elements starting at column c0 of a row (zero beyond n).
template <typename T, int E>
__device__ __forceinline__ void load_run(const T* __restrict__ row, int c0, int n, bool vec, float (&v)[E]) {
  constexpr int BYTES = E * (int)sizeof(T);
  if constexpr (BYTES >= 16 && BYTES % 16 == 0) {
    if (vec && c0 + E <= n) {
      const uint4* p = reinterpret_cast<const uint4*>(row + c0);
#pragma unroll
      for (int k = 0; k < BYTES / 16; ++k) {
        uint4 u = __ldg(p + k);
        const T* tv = reinterpret_cast<const T*>(&u);
#pragma unroll
        for (int j = 0; j < 16 / (int)sizeof(T); ++j) v[k * (16 / sizeof(T)) + j] = to_f32<T>(tv[j]);
      }
      return;
    }
  }
#pragma unroll
  for (int e = 0; e < E; ++e) {
    int c = c0 + e;
    v[e] = c < n ? to_f32<T>(row[c]) : 0.0f;
  }
}

// Stores E int8 values to dst (dst aligned to E bytes when E is 4/8/16/32).
template <int E>
__device__ __forceinline__ void store_i8_run(int8_t* dst, const int8_t (&q)[E]) {
  if constexpr (E % 16 == 0) {
#pragma unroll
    for (int k = 0; k < E / 16; ++k) reinterpret_cast<uint4*>(dst)[k] = reinterpret_cast<const uint4*>(q)[k];
  } else if constexpr (E == 8) {
    *reinterpret_cast<uint2*>(dst) = *reinterpret_cast<const uint2*>(q);
  } else if constexpr (E == 4) {
    *reinterpret_cast<uint32_t*>(dst) = *reinterpret_cast<const uint32_t*>(q);
  } else {
#pragma unroll
    for (int e = 0; e < E; ++e) dst[e] = q[e];
  }
}

// ================================================== non-rotated row quant
struct QArgs {
  const void* x;
  int64_t ld_x;
  int n;
  int8_t* q;
  int64_t ld_q;
  float* scale;
  int vec;  // x rows 16B aligned and q rows 8B aligned
};

constexpr int QR_THREADS = 256;

// Exact-erf GELU of an element as torch computes it on a T tensor: fp32 math,
// result rounded to T.
template <typename T>
__device__ __forceinline__ float gelu_in_dtype(float v) {
  const float g = gelu_erf(v);
  if constexpr (sizeof(T) == 2) return to_f32<T>(Elem<T>::from_f32(g));
  return g;
}

template <typename T, int CPT, int MODE, bool GELU>
__global__ void __launch_bounds__(QR_THREADS) quant_rows_kernel(QArgs a) {
  __shared__ float red[32];
  const int t = threadIdx.x;
  const int64_t row = blockIdx.x;
  const T* xr = static_cast<const T*>(a.x) + row * a.ld_x;
  int8_t* qr = a.q + row * a.ld_q;
  const int nc = a.n >> 3;  // chunks of 8
  float v[CPT][8];
  float local = 0.0f;
#pragma unroll
  for (int r = 0; r < CPT; ++r) {
    int c = r * QR_THREADS + t;
    if (c < nc) {
      load_run<T, 8>(xr, c * 8, a.n, a.vec != 0, v[r]);
      if constexpr (GELU) {
#pragma unroll
        for (int e = 0; e < 8; ++e) v[r][e] = gelu_in_dtype<T>(v[r][e]);
      }
    } else {
#pragma unroll
      for (int e = 0; e < 8; ++e) v[r][e] = 0.0f;
    }
#pragma unroll
    for (int e = 0; e < 8; ++e) local = fmaxf(local, fabsf(v[r][e]));
  }
  if constexpr (MODE == QI8_Q_TOKEN) {
    const float amax = block_max(local, red);
    const float s = fmaxf(__fdiv_rn(amax, 127.0f), 1e-30f);
    const float rcp = __frcp_rn(s);
#pragma unroll
    for (int r = 0; r < CPT; ++r) {
      int c = r * QR_THREADS + t;
      if (c < nc) {
        int8_t q8[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) q8[e] = rint_clamp(__fmul_rn(v[r][e], rcp), -128.0f, 127.0f);
        if (a.vec) store_i8_run<8>(qr + c * 8, q8);
        else
#pragma unroll
          for (int e = 0; e < 8; ++e) qr[c * 8 + e] = q8[e];
      }
    }
    if (t == 0) a.scale[row] = s;
  } else {
    // 128-element blocks = 16 consecutive chunks = 16 consecutive lanes
    const int nb = a.n >> 7;
#pragma unroll
    for (int r = 0; r < CPT; ++r) {
      int c = r * QR_THREADS + t;
      float m = 0.0f;
#pragma unroll
      for (int e = 0; e < 8; ++e) m = fmaxf(m, fabsf(v[r][e]));
#pragma unroll
      for (int o = 1; o < 16; o <<= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
      const float s = __fdiv_rn(m, 127.0f);
      if (c < nc) {
        int8_t q8[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) q8[e] = trunc_sat(__fdiv_rn(v[r][e], s));
        if (a.vec) store_i8_run<8>(qr + c * 8, q8);
        else
#pragma unroll
          for (int e = 0; e < 8; ++e) qr[c * 8 + e] = q8[e];
        if ((t & 15) == 0) a.scale[row * nb + (c >> 4)] = s;
      }
    }
  }
}

// Scalar fallback for rows whose width is not a multiple of 8 (TOKEN) or
// whose pointers are not vector aligned; reads the row twice.
template <typename T, bool GELU>
__global__ void __launch_bounds__(QR_THREADS) quant_rows_scalar_kernel(QArgs a) {
  __shared__ float red[32];
  const int64_t row = blockIdx.x;
  const T* xr = static_cast<const T*>(a.x) + row * a.ld_x;
  int8_t* qr = a.q + row * a.ld_q;
  auto val = [&](int c) {
    const float v = to_f32<T>(xr[c]);
    if constexpr (GELU) return gelu_in_dtype<T>(v);
    return v;
  };
  float local = 0.0f;
  for (int c = threadIdx.x; c < a.n; c += blockDim.x) local = fmaxf(local, fabsf(val(c)));
  const float amax = block_max(local, red);
  const float s = fmaxf(__fdiv_rn(amax, 127.0f), 1e-30f);
  const float rcp = __frcp_rn(s);
  for (int c = threadIdx.x; c < a.n; c += blockDim.x)
    qr[c] = rint_clamp(__fmul_rn(val(c), rcp), -128.0f, 127.0f);
  if (threadIdx.x == 0) a.scale[row] = s;
}

// ================================================ rotated rows (FWHT) core
enum RotOut { RO_Q_TOKEN = 0, RO_Q_BLOCK = 1, RO_F32 = 2, RO_UNROT = 3 };

struct RotArgs {
  const void* x;
  int64_t ld_x;
  int n_in;
  const float* pre_sign;
  const float* post_sign;
  float norm;
  int do_norm;
  int vec;
  // RO_Q_*: q [rows, N] (16B-aligned rows), scale [rows] or [rows, N/128]
  int8_t* q;
  float* scale;
  // RO_F32: f_out [rows, N]
  float* f_out;
  // RO_UNROT
  const void* bias;
  int bias_dtype;
  int n_out;
  void* out;
  int out_dtype;
  int64_t ld_out;
};

template <int L, typename T, int OUT>
__global__ void __launch_bounds__(RotCfg<L>::THREADS) rotate_rows_kernel(RotArgs a) {
  using C = RotCfg<L>;
  constexpr int N = C::N, E = C::E, P = C::P;
  extern __shared__ float4 dyn_smem[];
  float* buf = reinterpret_cast<float*>(dyn_smem);
  __shared__ float red[32];

  const int t = threadIdx.x;
  const int64_t row = blockIdx.x;
  const bool active = t < P;
  const T* xr = static_cast<const T*>(a.x) + row * a.ld_x;

  float v[E];
  const int c0 = t * E;
  if (active) {
    load_run<T, E>(xr, c0, a.n_in, a.vec != 0, v);
    if (a.pre_sign) {
#pragma unroll
      for (int e = 0; e < E; ++e) v[e] = __fmul_rn(v[e], __ldg(a.pre_sign + c0 + e));
    }
  } else {
#pragma unroll
    for (int e = 0; e < E; ++e) v[e] = 0.0f;
  }

  fwht_row<L>(v, buf);

  if (a.do_norm) {
#pragma unroll
    for (int e = 0; e < E; ++e) v[e] = __fmul_rn(v[e], a.norm);
  }

  if constexpr (OUT == RO_Q_TOKEN) {
    float local = 0.0f;
#pragma unroll
    for (int e = 0; e < E; ++e) local = fmaxf(local, fabsf(v[e]));
    const float amax = block_max(local, red);
    const float s = fmaxf(__fdiv_rn(amax, 127.0f), 1e-30f);
    const float rcp = __frcp_rn(s);
    if (active) {
      int8_t q8[E];
#pragma unroll
      for (int e = 0; e < E; ++e) q8[e] = rint_clamp(__fmul_rn(v[e], rcp), -128.0f, 127.0f);
      store_i8_run<E>(a.q + row * N + c0, q8);
    }
    if (t == 0) a.scale[row] = s;
  } else if constexpr (OUT == RO_Q_BLOCK) {
    static_assert(E >= 4 || N < 128, "block mode needs >= 4 elements per thread");
    constexpr int G = (128 / E) < 32 ? (128 / E) : 32;  // lanes per 128-block
    float m = 0.0f;
#pragma unroll
    for (int e = 0; e < E; ++e) m = fmaxf(m, fabsf(v[e]));
#pragma unroll
    for (int o = 1; o < G; o <<= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    const float s = __fdiv_rn(m, 127.0f);
    if (active) {
      int8_t q8[E];
#pragma unroll
      for (int e = 0; e < E; ++e) q8[e] = trunc_sat(__fdiv_rn(v[e], s));
      store_i8_run<E>(a.q + row * N + c0, q8);
      if ((t % G) == 0) a.scale[row * (N / 128) + c0 / 128] = s;
    }
  } else if constexpr (OUT == RO_F32) {
    if (active) {
      if (a.post_sign) {
#pragma unroll
        for (int e = 0; e < E; ++e) v[e] = __fmul_rn(v[e], __ldg(a.post_sign + c0 + e));
      }
      float* dst = a.f_out + row * N + c0;
      if constexpr (E % 4 == 0) {
#pragma unroll
        for (int k = 0; k < E / 4; ++k)
          reinterpret_cast<float4*>(dst)[k] = make_float4(v[4 * k], v[4 * k + 1], v[4 * k + 2], v[4 * k + 3]);
      } else {
#pragma unroll
        for (int e = 0; e < E; ++e) dst[e] = v[e];
      }
    }
  } else {  // RO_UNROT
    if (active) {
#pragma unroll
      for (int e = 0; e < E; ++e) {
        const int c = c0 + e;
        if (c < a.n_out) {
          float y = v[e];
          if (a.post_sign) y = __fmul_rn(y, __ldg(a.post_sign + c));
          if (a.bias) y = __fadd_rn(y, load_as_f32(a.bias, a.bias_dtype, c));
          store_from_f32(a.out, a.out_dtype, row * a.ld_out + c, y);
        }
      }
    }
  }
}

// ============================================ phased row FWHT (2^9..2^14)
// One row of n = 2^L fp32 values per CTA of P = n/16 threads (persistent
// over rows).  Each thread holds 16 elements whose indices differ only in a
// 4-bit window of the index; the window moves up by 4 bits per phase
// (0, 4, 8, ..., and L-4 last), and the data moves between phases through
// shared memory.  Stages run in ascending bit (stride) order, so results are
// bit-identical to the single-row kernel above.  The shared-memory layout
// swaps 16-byte chunks (chunk ^= row bits 5..7 ^ index bit 8 << 2), which
// makes every phase's accesses bank-conflict free, including the 128-bit
// writes of the first phase.  Per-token quantization stores 16 contiguous
// bytes per thread after a byte-wide transpose.
namespace rot2 {

// the phased-transform helpers (swz, wbase, nwin, wstart, stages, phase) are
// shared with the converter's row pass: fwht_row.cuh, namespace rowfwht
using namespace rowfwht;

// two row buffers, used by alternate rows (no barrier between rows)
template <int L>
constexpr int smem_bytes() { return 2 * (1 << L) * 4; }

template <int L, typename T, int OUT>
__global__ void __launch_bounds__(1 << (L - 4), 1024 >> (L - 4)) rot2_kernel(RotArgs a, int64_t rows) {
  constexpr int N = 1 << L, P = N / 16, NW = nwin<L>(), WL = wstart<L>(NW - 1);
  extern __shared__ float4 dyn_smem[];
  float* bufs = reinterpret_cast<float*>(dyn_smem);
  __shared__ float red[2][32];
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  const int c0 = t * 16;
  // the next row's 16 raw elements are loaded while this row is transformed
  // (rows whose width is a multiple of 16 and whose pointers allow vectors)
  constexpr int NR = 16 * (int)sizeof(T) / 16;
  const bool pre = a.vec != 0 && (a.n_in & 15) == 0;
  const bool mine = c0 < a.n_in;
  uint4 raw[NR];
  auto fetch = [&](int64_t r) {
#pragma unroll
    for (int k = 0; k < NR; ++k) raw[k] = make_uint4(0, 0, 0, 0);
    if (r < rows && mine) {
      const uint4* p = reinterpret_cast<const uint4*>(static_cast<const T*>(a.x) + r * a.ld_x + c0);
#pragma unroll
      for (int k = 0; k < NR; ++k) raw[k] = __ldg(p + k);
    }
  };
  if (pre) fetch(blockIdx.x);
  // the signs are per column: this thread's 16 are loaded once for all its rows
  float sg[16];
  if (a.pre_sign) {
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const float4 s4 = __ldg(reinterpret_cast<const float4*>(a.pre_sign + c0) + q);
      sg[4 * q] = s4.x; sg[4 * q + 1] = s4.y; sg[4 * q + 2] = s4.z; sg[4 * q + 3] = s4.w;
    }
  }
  // For even L the normalization 1/sqrt(n) = 2^(-L/2) scales exactly, so in
  // the per-token path it is folded into the amax and the reciprocal:
  // rint(fl(fl(v * 2^-k) * rcp)) == rint(fl(v * (rcp * 2^-k))) and
  // amax(fl(v * 2^-k)) == amax(v) * 2^-k, barring subnormal intermediates,
  // which the row's amax test below sends to the unfolded path.
  constexpr bool POW2_NORM = (L % 2) == 0;
  int it = 0;
  for (int64_t row = blockIdx.x; row < rows; row += gridDim.x, ++it) {
    // a row's first write to its buffer follows the first barrier of the
    // previous row, which every thread passes only after finishing the row
    // before it -- the last reader of this buffer
    float* buf = bufs + (it & 1) * N;
    const T* xr = static_cast<const T*>(a.x) + row * a.ld_x;
    float v[16];
    if (pre) {
      const T* tv = reinterpret_cast<const T*>(raw);
#pragma unroll
      for (int e = 0; e < 16; ++e) v[e] = to_f32<T>(tv[e]);
      fetch(row + gridDim.x);
    } else {
      load_run<T, 16>(xr, c0, a.n_in, a.vec != 0, v);
    }
    if (a.pre_sign) {
#pragma unroll
      for (int e = 0; e < 16; ++e) v[e] = __fmul_rn(v[e], sg[e]);
    }
    stages<L, 0>(v);
    phase<L, 1>(v, buf, t);
    const bool fold = OUT == RO_Q_TOKEN && POW2_NORM && a.do_norm;
    if (a.do_norm && !fold) {
#pragma unroll
      for (int e = 0; e < 16; ++e) v[e] = __fmul_rn(v[e], a.norm);
    }
    if constexpr (OUT == RO_Q_TOKEN) {
      float m = 0.0f;
#pragma unroll
      for (int e = 0; e < 16; ++e) m = fmaxf(m, fabsf(v[e]));
      m = warp_max(m);
      if (lane == 0) red[it & 1][warp] = m;
      __syncthreads();
      float amax = red[it & 1][0];
#pragma unroll 1
      for (int w = 1; w < P / 32; ++w) amax = fmaxf(amax, red[it & 1][w]);
      float nrm = 1.0f;
      if (fold) {
        amax = __fmul_rn(amax, a.norm);
        // 2^-100 <= amax <= 2^100: a subnormal fl(v * 2^-k) quantizes to 0 on
        // both paths and rcp * 2^-k stays normal
        if (amax >= 7.8886091e-31f && amax <= 1.2676506e30f) {
          nrm = a.norm;
        } else {
#pragma unroll
          for (int e = 0; e < 16; ++e) v[e] = __fmul_rn(v[e], a.norm);
        }
      }
      const float s = fmaxf(__fdiv_rn(amax, 127.0f), 1e-30f);
      const float rcp = __fmul_rn(__frcp_rn(s), nrm);
      // one byte per element in the last window's mapping: a warp writes 32
      // consecutive bytes per element index
      int8_t* qrow = a.q + row * N + wbase(t, WL);
#pragma unroll
      for (int e = 0; e < 16; ++e) {
        // rint(fl(v * rcp)) in [-127, 127]: low byte of fl(fl(v * rcp) + 1.5 * 2^23)
        const float r = __fadd_rn(__fmul_rn(v[e], rcp), 12582912.0f);
        qrow[e << WL] = (int8_t)(__float_as_uint(r) & 0xFF);
      }
      if (t == 0) a.scale[row] = s;
    } else if constexpr (OUT == RO_F32) {
      float* dst = a.f_out + row * N;
#pragma unroll
      for (int e = 0; e < 16; ++e) {
        const int i = wbase(t, WL) + (e << WL);
        float y = v[e];
        if (a.post_sign) y = __fmul_rn(y, __ldg(a.post_sign + i));
        dst[i] = y;
      }
    } else {  // RO_UNROT
#pragma unroll
      for (int e = 0; e < 16; ++e) {
        const int i = wbase(t, WL) + (e << WL);
        if (i < a.n_out) {
          float y = v[e];
          if (a.post_sign) y = __fmul_rn(y, __ldg(a.post_sign + i));
          if (a.bias) y = __fadd_rn(y, load_as_f32(a.bias, a.bias_dtype, i));
          store_from_f32(a.out, a.out_dtype, row * a.ld_out + i, y);
        }
      }
    }
  }
}

template <int L, typename T, int OUT>
int launch(const RotArgs& a, int64_t rows, cudaStream_t st) {
  constexpr int P = 1 << (L - 4);
  constexpr int SMEM = smem_bytes<L>();
  auto kern = rot2_kernel<L, T, OUT>;
  static int per_sm = 0;
  if (per_sm == 0) {
    if (SMEM > 48 * 1024) QI8_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM));
    int b = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&b, kern, P, SMEM) != cudaSuccess || b < 1) b = 1;
    per_sm = b;
  }
  const int64_t cap = (int64_t)(sm_count() > 0 ? sm_count() : 148) * per_sm;
  const unsigned grid = (unsigned)(rows < cap ? rows : cap);
  kern<<<grid, P, SMEM, st>>>(a, rows);
  return check_cuda(cudaGetLastError(), "rot2_kernel launch");
}

}  // namespace rot2

// ============================== two-phase row FWHT, n = 4096 (K1 per-token)
// 64 threads per row, 64 elements per thread, so the 12 butterfly stages
// take two register phases and one trip through shared memory:
//   phase 0: thread t holds the contiguous run 64t .. 64t+63 and runs the
//            stages of index bits 0-5;
//   phase 1: thread t holds t + 64j (j = 0..63) and runs bits 6-11.
// Stages stay in ascending bit order (the bit-exactness contract of
// fwht_row.cuh).  The exchange buffer pads each 64-float run to 68 floats,
// phys(i) = 68 (i >> 6) + (i & 63): the phase-0 128-bit stores (thread t at
// 68t + 4q, eight threads per wavefront on banks 4(t + q) mod 32) and the
// phase-1 loads (a warp at 68j + t) are bank-conflict free, and every
// address is a per-thread base plus an immediate.  The quantized bytes go
// out in the phase-1 mapping: one byte store per element, a warp writing 32
// consecutive bytes per store.  The quantization multiply and rounding add
// stay scalar __fmul_rn/__fadd_rn: a packed f32x2 pair was contracted into
// one FFMA2 (single rounding), which moves round-half-even ties.
//
// Signs: a ±1 sign flips the sign bit of the 16-bit input exactly, so each
// thread keeps its 64 signs as two bit masks (built once) and XORs them into
// the raw words -- no per-row sign loads.  Bit p of mask h is the sign of
// element 32h + 2p, bit 16 + p that of element 32h + 2p + 1, so the masks
// of word i (elements 2i, 2i + 1) are (mask << (15 - p)) & 0x80008000 with
// p = i % 16.  A sign vector with any entry other than ±1 takes the
// multiply path instead (decided per CTA).
namespace rot64 {

constexpr int L = 12, N = 1 << L, E = 64, P = N / E, PAD = 68;
constexpr int SMEM = P * PAD * 4;

// butterflies of the six bits of the in-thread index e (stride 1 .. 32):
// stride 1 pairs sit in one register pair and run as scalar add/sub; the
// others run on packed pairs (sum, and difference as fma(hi, -1, lo), both
// single-rounded and identical to the scalar ops)
__device__ __forceinline__ void stages64(float (&v)[E]) {
#pragma unroll
  for (int e = 0; e < E; e += 2) {
    const float lo = v[e], hi = v[e + 1];
    v[e] = lo + hi;
    v[e + 1] = lo - hi;
  }
#pragma unroll
  for (int s = 2; s < E; s <<= 1) {
#pragma unroll
    for (int e = 0; e < E; e += 2) {
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

// Per-token int8 of sign(x) FWHT: 16-bit inputs whose width is a multiple
// of 64 with 16-byte aligned rows (the launcher checks), persistent CTAs of
// one row at a time; the next row's 128 input bytes per thread are loaded
// while this row is transformed.
template <typename T>
__global__ void __launch_bounds__(P, 8) rot64_quant_kernel(RotArgs a, int64_t rows) {
  static_assert(sizeof(T) == 2, "16-bit inputs");
  extern __shared__ float4 dyn_smem[];
  float* buf = reinterpret_cast<float*>(dyn_smem);
  __shared__ float red[P / 32];
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  const int c0 = t * E;
  const bool mine = c0 < a.n_in;
  uint4 raw[8];
  auto fetch = [&](int64_t r) {
    if (r < rows && mine) {
      const uint4* p = reinterpret_cast<const uint4*>(static_cast<const T*>(a.x) + r * a.ld_x + c0);
#pragma unroll
      for (int k = 0; k < 8; ++k) raw[k] = __ldg(p + k);
    } else {
#pragma unroll
      for (int k = 0; k < 8; ++k) raw[k] = make_uint4(0, 0, 0, 0);
    }
  };
  // this thread's signs as bit masks; ±1 everywhere in the CTA or not
  uint32_t smask[2] = {0u, 0u};
  bool pm1 = true;
  if (a.pre_sign && mine) {
    const float4* sg4 = reinterpret_cast<const float4*>(a.pre_sign + c0);
#pragma unroll
    for (int q = 0; q < E / 4; ++q) {
      const float4 s4 = __ldg(sg4 + q);
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int e = 4 * q + u;
        const float f = u == 0 ? s4.x : (u == 1 ? s4.y : (u == 2 ? s4.z : s4.w));
        pm1 = pm1 && (f == 1.0f || f == -1.0f);
        if (f < 0.0f) smask[e >> 5] |= 1u << (((e & 31) >> 1) + 16 * (e & 1));
      }
    }
  }
  const bool xor_signs = __syncthreads_and(pm1) != 0;
  fetch(blockIdx.x);
  float* wrow = buf + t * PAD;  // phase-0 stores
  const float* rcol = buf + t;  // phase-1 loads
  for (int64_t row = blockIdx.x; row < rows; row += gridDim.x) {
    float v[E];
    {
      if (a.pre_sign && xor_signs) {
        // recomputed per row: hoisted out of the loop, the 32 word masks
        // would hold 32 registers
        asm volatile("" : "+r"(smask[0]), "+r"(smask[1]));
        // word i = 4k + c of the row's 32 input words
        auto flip = [&](int i) { return (smask[i >> 4] << (15 - (i & 15))) & 0x80008000u; };
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          raw[k].x ^= flip(4 * k);
          raw[k].y ^= flip(4 * k + 1);
          raw[k].z ^= flip(4 * k + 2);
          raw[k].w ^= flip(4 * k + 3);
        }
      }
      const T* tv = reinterpret_cast<const T*>(raw);
#pragma unroll
      for (int e = 0; e < E; ++e) v[e] = Elem<T>::to_f32(tv[e]);
    }
    fetch(row + gridDim.x);
    if (a.pre_sign && !xor_signs && mine) {
#pragma unroll
      for (int e = 0; e < E; ++e) v[e] = __fmul_rn(v[e], __ldg(a.pre_sign + c0 + e));
    }
    stages64(v);
#pragma unroll
    for (int q = 0; q < E / 4; ++q)
      *reinterpret_cast<float4*>(wrow + 4 * q) = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
    __syncthreads();
#pragma unroll
    for (int j = 0; j < E; ++j) v[j] = rcol[PAD * j];
    stages64(v);
    float m = 0.0f;
#pragma unroll
    for (int e = 0; e < E; ++e) m = fmaxf(m, fabsf(v[e]));
    m = warp_max(m);
    if (lane == 0) red[warp] = m;
    // also orders this row's phase-1 loads before the next row's stores
    __syncthreads();
    float amax = red[0];
#pragma unroll
    for (int w = 1; w < P / 32; ++w) amax = fmaxf(amax, red[w]);
    // 1/sqrt(4096) = 2^-6 scales exactly: folded into the amax and the
    // reciprocal, rint(fl(fl(v * 2^-6) * rcp)) == rint(fl(v * (rcp * 2^-6)))
    // barring subnormal intermediates, which the range test sends to the
    // unfolded path
    float nrm = 1.0f;
    if (a.do_norm) {
      amax = __fmul_rn(amax, a.norm);
      if (amax >= 7.8886091e-31f && amax <= 1.2676506e30f) {
        nrm = a.norm;
      } else {
#pragma unroll
        for (int e = 0; e < E; ++e) v[e] = __fmul_rn(v[e], a.norm);
      }
    }
    const float s = fmaxf(__fdiv_rn(amax, 127.0f), 1e-30f);
    const float rcp = __fmul_rn(__frcp_rn(s), nrm);
    int8_t* qrow = a.q + row * N + t;
#pragma unroll
    for (int j = 0; j < E; ++j) {
      // rint(fl(v * rcp)) in [-127, 127]: low byte of fl(fl(v * rcp) + 1.5 * 2^23)
      const float r = __fadd_rn(__fmul_rn(v[j], rcp), 12582912.0f);
      qrow[P * j] = (int8_t)(__float_as_uint(r) & 0xFF);
    }
    if (t == 0) a.scale[row] = s;
  }
}

// true when the two-phase kernel takes these arguments: 16-bit rows whose
// width is a multiple of 64, and enough rows that each persistent CTA
// walks about two (with one row per CTA its prologue -- sign masks, the
// unprefetched first row -- is not amortized: 512 rows measured 12.3 us
// against 10.2 us for the phased kernel; 4096 rows 25.4 against 29.7 us)
template <typename T>
bool usable(const RotArgs& a, int64_t rows) {
  return sizeof(T) == 2 && a.vec != 0 && (a.n_in % E) == 0 && rows >= 2048 &&
         (!a.pre_sign || (reinterpret_cast<uintptr_t>(a.pre_sign) & 15) == 0);
}

template <typename T>
int launch(const RotArgs& a, int64_t rows, cudaStream_t st) {
  auto kern = rot64_quant_kernel<T>;
  static int per_sm = 0;
  if (per_sm == 0) {
    int b = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&b, kern, P, SMEM) != cudaSuccess || b < 1) b = 1;
    per_sm = b;
  }
  const int64_t cap = (int64_t)(sm_count() > 0 ? sm_count() : 148) * per_sm;
  const unsigned grid = (unsigned)(rows < cap ? rows : cap);
  kern<<<grid, P, SMEM, st>>>(a, rows);
  return check_cuda(cudaGetLastError(), "rot64_quant_kernel launch");
}

}  // namespace rot64

template <int L, typename T, int OUT>
int launch_rotate_L(const RotArgs& a, int64_t rows, cudaStream_t st) {
  // per-token K1 of 16-bit rows at n = 4096: the two-phase kernel
  if constexpr (L == rot64::L && OUT == RO_Q_TOKEN && sizeof(T) == 2) {
    if (rot64::usable<T>(a, rows)) return rot64::launch<T>(a, rows, st);
  }
  // rows of 2^9 .. 2^14: the phased kernel (vector loads of the pre-signs
  // need them 16-byte aligned); block-128 quantization stays below
  if constexpr (L >= 9 && L <= 14 && OUT != RO_Q_BLOCK) {
    if (!a.pre_sign || (reinterpret_cast<uintptr_t>(a.pre_sign) & 15) == 0) return rot2::launch<L, T, OUT>(a, rows, st);
  }
  using C = RotCfg<L>;
  auto kern = rotate_rows_kernel<L, T, OUT>;
  if (C::SMEM > 48 * 1024) {
    QI8_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)C::SMEM));
  }
  kern<<<(unsigned)rows, C::THREADS, C::SMEM, st>>>(a);
  return check_cuda(cudaGetLastError(), "rotate_rows_kernel launch");
}

template <typename T, int OUT>
int launch_rotate(int L, const RotArgs& a, int64_t rows, cudaStream_t st) {
  switch (L) {
#define QI8_CASE(l) case l: return launch_rotate_L<l, T, OUT>(a, rows, st);
    QI8_CASE(1) QI8_CASE(2) QI8_CASE(3) QI8_CASE(4) QI8_CASE(5) QI8_CASE(6) QI8_CASE(7)
    QI8_CASE(8) QI8_CASE(9) QI8_CASE(10) QI8_CASE(11) QI8_CASE(12) QI8_CASE(13) QI8_CASE(14)
    QI8_CASE(15)
#undef QI8_CASE
    default: return fail(QI8_ESHAPE, "n_pad = 2^%d out of range [2, 32768]", L);
  }
}

template <int OUT>
int launch_rotate_dtype(int x_dtype, int L, const RotArgs& a, int64_t rows, cudaStream_t st) {
  switch (x_dtype) {
    case QI8_BF16: return launch_rotate<__nv_bfloat16, OUT>(L, a, rows, st);
    case QI8_F16: return launch_rotate<__half, OUT>(L, a, rows, st);
    case QI8_F32: return launch_rotate<float, OUT>(L, a, rows, st);
    default: return fail(QI8_EDTYPE, "input dtype %d not in {bf16, f16, f32}", x_dtype);
  }
}

// ================================================================ dequant
__global__ void dequant_kernel(const int8_t* __restrict__ q, int64_t rows, int64_t n,
                               const float* __restrict__ scale, int kind, int block, void* out,
                               int out_dtype) {
  const int64_t total = rows * n;
  const int64_t nb = block > 0 ? (n + block - 1) / block : 1;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / n, c = i - r * n;
    float s;
    switch (kind) {
      case QI8_S_SCALAR: s = scale[0]; break;
      case QI8_S_ROW: s = scale[r]; break;
      case QI8_S_ROW_KBLOCK: s = scale[r * nb + c / block]; break;
      default: s = scale[(r / block) * nb + c / block]; break;  // TILE128
    }
    store_from_f32(out, out_dtype, i, __fmul_rn((float)q[i], s));
  }
}

// ====================================================== weight quantizers
template <typename T>
__global__ void absmax_kernel(const T* __restrict__ w, int64_t total, unsigned int* __restrict__ out) {
  float m = 0.0f;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x)
    m = fmaxf(m, fabsf(to_f32<T>(w[i])));
  m = warp_max(m);
  if ((threadIdx.x & 31) == 0) atomicMax(out, __float_as_uint(m));  // m >= 0: uint order == float order
}

template <typename T>
__global__ void quant_tensorwise_kernel(const T* __restrict__ w, int64_t total,
                                        const unsigned int* __restrict__ amax_bits,
                                        int8_t* __restrict__ q, float* __restrict__ scale_out) {
  const float amax = __uint_as_float(*amax_bits);
  const float s = fmaxf(__fdiv_rn(amax, 127.0f), 1e-30f);
  const float rcp = __frcp_rn(s);
  if (blockIdx.x == 0 && threadIdx.x == 0) scale_out[0] = s;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x)
    q[i] = rint_clamp(__fmul_rn(to_f32<T>(w[i]), rcp), -128.0f, 127.0f);
}

// Triton weight_quant semantics: one CTA per 128x128 tile.
template <typename T>
__global__ void __launch_bounds__(256) quant_tile128_kernel(const T* __restrict__ w, int64_t rows, int64_t n,
                                                           int8_t* __restrict__ q, float* __restrict__ scale) {
  __shared__ float red[32];
  const int64_t tr = blockIdx.y, tc = blockIdx.x;
  const int64_t nbc = (n + 127) / 128;
  float v[64];
  float local = 0.0f;
#pragma unroll
  for (int k = 0; k < 64; ++k) {
    const int idx = k * 256 + threadIdx.x;
    const int64_t r = tr * 128 + idx / 128, c = tc * 128 + idx % 128;
    v[k] = (r < rows && c < n) ? to_f32<T>(w[r * n + c]) : 0.0f;
    local = fmaxf(local, fabsf(v[k]));
  }
  const float amax = block_max(local, red);
  const float s = fmaxf(__fdiv_rn(amax, 127.0f), 1e-8f);
#pragma unroll
  for (int k = 0; k < 64; ++k) {
    const int idx = k * 256 + threadIdx.x;
    const int64_t r = tr * 128 + idx / 128, c = tc * 128 + idx % 128;
    if (r < rows && c < n) q[r * n + c] = trunc_sat(__fdiv_rn(v[k], s));
  }
  if (threadIdx.x == 0) scale[tr * nbc + tc] = s;
}

// ============================================ per-token quant, warps per row
// The per-token path of the activation quantizer for 16-byte aligned rows:
// W warps share one row (W in {1,2,4,8}, 8/W rows per 256-thread block),
// every lane keeps CPL raw 16-byte chunks in registers so that all of a
// row's loads are in flight at once, and the block loops over row groups
// (persistent grid).  GELU rounds to T in place, so both passes read the
// packed values.  Quantization is q = rint(v * rcp) with s = max(amax/127,
// 1e-30) and rcp = 1/s (both correctly rounded, as the row kernel above):
// |v * rcp| <= 127 * (1 + 3 ulp) rounds into [-127, 127], so the clamp is a
// no-op and rint is done by adding 1.5 * 2^23 in fp32 (round to nearest
// even), leaving the int8 in the low byte of the sum.
namespace tok {

template <typename T> struct Pack;
template <> struct Pack<__nv_bfloat16> {
  static constexpr int EPC = 8;  // elements per 16-byte chunk
  __device__ static __forceinline__ float2 f2(uint32_t w) {
    return make_float2(__uint_as_float(w << 16), __uint_as_float(w & 0xFFFF0000u));
  }
  __device__ static __forceinline__ uint32_t from_f2(float lo, float hi) {
    __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&h);
  }
  __device__ static __forceinline__ uint32_t absmax2(uint32_t m, uint32_t w) {
    __nv_bfloat162 a = *reinterpret_cast<__nv_bfloat162*>(&m), b = *reinterpret_cast<__nv_bfloat162*>(&w);
    __nv_bfloat162 r = __hmax2(a, __habs2(b));
    return *reinterpret_cast<uint32_t*>(&r);
  }
  __device__ static __forceinline__ float fold(uint32_t m) { float2 f = f2(m); return fmaxf(f.x, f.y); }
};
template <> struct Pack<__half> {
  static constexpr int EPC = 8;
  __device__ static __forceinline__ float2 f2(uint32_t w) {
    return __half22float2(*reinterpret_cast<__half2*>(&w));
  }
  __device__ static __forceinline__ uint32_t from_f2(float lo, float hi) {
    __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&h);
  }
  __device__ static __forceinline__ uint32_t absmax2(uint32_t m, uint32_t w) {
    __half2 a = *reinterpret_cast<__half2*>(&m), b = *reinterpret_cast<__half2*>(&w);
    __half2 r = __hmax2(a, __habs2(b));
    return *reinterpret_cast<uint32_t*>(&r);
  }
  __device__ static __forceinline__ float fold(uint32_t m) { float2 f = f2(m); return fmaxf(f.x, f.y); }
};
template <> struct Pack<float> {
  static constexpr int EPC = 4;
  // one fp32 per word; pairs of words form the float2 operands
};

__device__ __forceinline__ uint32_t bytes4(float2 a, float2 b) {
  const uint32_t lo = __byte_perm(__float_as_uint(a.x), __float_as_uint(a.y), 0x0040);
  const uint32_t hi = __byte_perm(__float_as_uint(b.x), __float_as_uint(b.y), 0x0040);
  return __byte_perm(lo, hi, 0x5410);
}

constexpr float RINT_MAGIC = 12582912.0f;  // 1.5 * 2^23

// rint(fl(v * rcp)) + 1.5 * 2^23 for two values: separately rounded scalar
// multiply and add (__fmul_rn / __fadd_rn are never merged into an fma).
__device__ __forceinline__ float2 magic_q(float2 v, float rcp) {
  return make_float2(__fadd_rn(__fmul_rn(v.x, rcp), RINT_MAGIC), __fadd_rn(__fmul_rn(v.y, rcp), RINT_MAGIC));
}

// GELU of a pair of T values, rounded to T: gelu_erf on each,
// (0.5 x) * (1 + erf(x / sqrt 2)) with separately rounded products and sum.
template <typename T>
__device__ __forceinline__ uint32_t gelu2(uint32_t w) {
  const float2 f = Pack<T>::f2(w);
  const float2 tt = __fmul2_rn(f, make_float2(0.70710678118654752440f, 0.70710678118654752440f));
  const float2 e = make_float2(erff(tt.x), erff(tt.y));
  const float2 g = __fmul2_rn(__fmul2_rn(f, make_float2(0.5f, 0.5f)), __fadd2_rn(make_float2(1.0f, 1.0f), e));
  return Pack<T>::from_f2(g.x, g.y);
}

// GELU table for bf16 inputs: a bf16 value has 7 mantissa bits, so the
// binades 2^-16 <= |x| < 16 hold 2 x 20 x 128 values.  Each CTA fills the
// table with gelu2 itself, so a lookup returns exactly what gelu2 computes;
// inputs outside the range (zeros, tiny, |x| >= 16, inf/nan) take gelu2.
constexpr int GT_ELO = 127 - 16, GT_NE = 20;
constexpr uint32_t GT_HALF = GT_NE * 128, GT_BASE = GT_ELO * 128;

__device__ __forceinline__ void gelu_table_fill(uint32_t* tab) {
  for (uint32_t i = threadIdx.x; i < GT_HALF; i += blockDim.x) {  // word i = entries 2i, 2i+1
    const uint32_t k = 2 * i, s = k >= GT_HALF ? 1u : 0u, r = k - s * GT_HALF;
    const uint32_t b0 = (s << 15) | (GT_BASE + r);
    tab[i] = gelu2<__nv_bfloat16>(b0 | ((b0 + 1) << 16));
  }
}

__device__ __forceinline__ uint32_t gelu2_lut(uint32_t w, const uint16_t* tab) {
  const uint32_t t0 = (w & 0x7FFFu) - GT_BASE, t1 = ((w >> 16) & 0x7FFFu) - GT_BASE;
  if (t0 < GT_HALF && t1 < GT_HALF) {
    const uint32_t lo = tab[t0 + ((w & 0x8000u) ? GT_HALF : 0u)];
    const uint32_t hi = tab[t1 + ((w & 0x80000000u) ? GT_HALF : 0u)];
    return lo | (hi << 16);
  }
  return gelu2<__nv_bfloat16>(w);
}

template <typename T, int CPL, bool GELU>
__global__ void __launch_bounds__(256, 3) token_rows_kernel(QArgs a, int rows, int W) {
  __shared__ float red[2][8];
  constexpr int EPC = Pack<T>::EPC;
  constexpr bool LUT = GELU && std::is_same<T, __nv_bfloat16>::value;
  __shared__ uint32_t gtab_w[LUT ? GT_HALF : 1];
  if constexpr (LUT) {
    gelu_table_fill(gtab_w);
    __syncthreads();
  }
  const uint16_t* gtab = reinterpret_cast<const uint16_t*>(gtab_w);
  pdl_wait();
  pdl_launch_dependents();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int rpb = 8 / W, wr = warp % W, rsub = warp / W;
  const int nc = a.n / EPC;
  const int groups = (rows + rpb - 1) / rpb;
  int it = 0;
  for (int g = blockIdx.x; g < groups; g += gridDim.x, ++it) {
    const int row = g * rpb + rsub;
    const bool live = row < rows;
    const uint4* xr = reinterpret_cast<const uint4*>(static_cast<const T*>(a.x) + (int64_t)row * a.ld_x);
    uint4 x[CPL];
#pragma unroll
    for (int i = 0; i < CPL; ++i) {
      const int c = (i * W + wr) * 32 + lane;
      x[i] = (live && c < nc) ? __ldcs(xr + c) : make_uint4(0, 0, 0, 0);
    }
    float amax;
    if constexpr (sizeof(T) == 2) {
      uint32_t m = 0;
#pragma unroll
      for (int i = 0; i < CPL; ++i) {
        uint32_t* w = reinterpret_cast<uint32_t*>(&x[i]);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          if constexpr (LUT) w[j] = gelu2_lut(w[j], gtab);
          else if constexpr (GELU) w[j] = gelu2<T>(w[j]);
          m = Pack<T>::absmax2(m, w[j]);
        }
      }
      amax = Pack<T>::fold(m);
    } else {
      amax = 0.0f;
#pragma unroll
      for (int i = 0; i < CPL; ++i) {
        float* f = reinterpret_cast<float*>(&x[i]);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          if constexpr (GELU) f[j] = gelu_erf(f[j]);
          amax = fmaxf(amax, fabsf(f[j]));
        }
      }
    }
    amax = warp_max(amax);
    if (W > 1) {
      if (lane == 0) red[it & 1][warp] = amax;
      __syncthreads();
      amax = red[it & 1][rsub * W];
      for (int k = 1; k < W; ++k) amax = fmaxf(amax, red[it & 1][rsub * W + k]);
    }
    if (!live) continue;
    const float s = fmaxf(__fdiv_rn(amax, 127.0f), 1e-30f);
    const float rcp = __frcp_rn(s);
    int8_t* qr = a.q + (int64_t)row * a.ld_q;
#pragma unroll
    for (int i = 0; i < CPL; ++i) {
      const int c = (i * W + wr) * 32 + lane;
      if (c < nc) {
        const uint32_t* w = reinterpret_cast<const uint32_t*>(&x[i]);
        if constexpr (sizeof(T) == 2) {
          float2 f[4];
#pragma unroll
          for (int j = 0; j < 4; ++j) f[j] = magic_q(Pack<T>::f2(w[j]), rcp);
          *reinterpret_cast<uint2*>(qr + (int64_t)c * EPC) = make_uint2(bytes4(f[0], f[1]), bytes4(f[2], f[3]));
        } else {
          const float2 f0 = magic_q(make_float2(__uint_as_float(w[0]), __uint_as_float(w[1])), rcp);
          const float2 f1 = magic_q(make_float2(__uint_as_float(w[2]), __uint_as_float(w[3])), rcp);
          *reinterpret_cast<uint32_t*>(qr + (int64_t)c * EPC) = bytes4(f0, f1);
        }
      }
    }
    if (wr == 0 && lane == 0) a.scale[row] = s;
  }
}

// (W, CPL) for a row of nc chunks: the fewest warps whose lanes hold the row
// in at most 12 chunks each; 0 if the row is too wide.
inline void choose_shape(int nc, int& W, int& cpl) {
  static const int allowed[] = {1, 2, 3, 4, 6, 8, 12};
  for (W = 1; W <= 8; W *= 2) {
    const int need = (nc + 32 * W - 1) / (32 * W);
    if (need <= 12) {
      for (int c : allowed)
        if (c >= need) { cpl = c; return; }
    }
  }
  W = 0; cpl = 0;
}

template <typename T, int CPL, bool GELU>
int launch_cpl(const QArgs& a, int rows, int W, cudaStream_t st) {
  static int per_sm = 0;
  if (per_sm == 0) {
    int b = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&b, token_rows_kernel<T, CPL, GELU>, 256, 0) != cudaSuccess || b < 1)
      b = 1;
    per_sm = b;
  }
  const int rpb = 8 / W;
  const int64_t groups = (rows + rpb - 1) / rpb;
  const int64_t cap = (int64_t)sm_count() * per_sm;
  const unsigned grid = (unsigned)(groups < cap ? groups : (cap > 0 ? cap : 1));
  return check_cuda(launch_pdl(token_rows_kernel<T, CPL, GELU>, dim3(grid), dim3(256), 0, st, a, rows, W),
                    "token_rows_kernel launch");
}

// Returns -1 when the row shape is outside this path (caller falls back).
template <typename T, bool GELU>
int launch(const QArgs& a, int64_t rows, cudaStream_t st) {
  constexpr int EPC = Pack<T>::EPC;
  if (!a.vec || a.n % EPC != 0 || rows >= (int64_t(1) << 31) || (a.ld_x * (int64_t)sizeof(T)) % 16 != 0 ||
      a.ld_q % EPC != 0)
    return -1;
  int W, cpl;
  choose_shape(a.n / EPC, W, cpl);
  const int r = (int)rows;
  switch (cpl) {
    case 1: return launch_cpl<T, 1, GELU>(a, r, W, st);
    case 2: return launch_cpl<T, 2, GELU>(a, r, W, st);
    case 3: return launch_cpl<T, 3, GELU>(a, r, W, st);
    case 4: return launch_cpl<T, 4, GELU>(a, r, W, st);
    case 6: return launch_cpl<T, 6, GELU>(a, r, W, st);
    case 8: return launch_cpl<T, 8, GELU>(a, r, W, st);
    case 12: return launch_cpl<T, 12, GELU>(a, r, W, st);
    default: return -1;
  }
}

}  // namespace tok

template <typename T, int MODE, bool GELU>
int launch_quant_rows_T(const QArgs& a, int64_t rows, cudaStream_t st) {
  if constexpr (MODE == QI8_Q_TOKEN) {
    const int rc = tok::launch<T, GELU>(a, rows, st);
    if (rc >= 0) return rc;
  }
  const int nc = (a.n + 7) / 8;
  const int cpt = (nc + QR_THREADS - 1) / QR_THREADS;
  if (a.n % 8 != 0 || !a.vec) {
    if (MODE != QI8_Q_TOKEN) return fail(QI8_EALIGN, "block quantization needs 16-byte aligned rows");
    quant_rows_scalar_kernel<T, GELU><<<(unsigned)rows, QR_THREADS, 0, st>>>(a);
    return check_cuda(cudaGetLastError(), "quant_rows_scalar_kernel launch");
  }
  switch (cpt) {
#define QI8_CPT(c) case c: quant_rows_kernel<T, c, MODE, GELU><<<(unsigned)rows, QR_THREADS, 0, st>>>(a); break;
    QI8_CPT(1) QI8_CPT(2)
    case 3: QI8_CPT(4)
    case 5: case 6: case 7: QI8_CPT(8)
    case 9: case 10: case 11: case 12: case 13: case 14: case 15: QI8_CPT(16)
#undef QI8_CPT
    default:
      if (MODE != QI8_Q_TOKEN) return fail(QI8_ESHAPE, "row width %d > 32768", a.n);
      quant_rows_scalar_kernel<T, GELU><<<(unsigned)rows, QR_THREADS, 0, st>>>(a);
  }
  return check_cuda(cudaGetLastError(), "quant_rows_kernel launch");
}

template <int MODE, bool GELU>
int launch_quant_rows(int dtype, const QArgs& a, int64_t rows, cudaStream_t st) {
  switch (dtype) {
    case QI8_BF16: return launch_quant_rows_T<__nv_bfloat16, MODE, GELU>(a, rows, st);
    case QI8_F16: return launch_quant_rows_T<__half, MODE, GELU>(a, rows, st);
    case QI8_F32: return launch_quant_rows_T<float, MODE, GELU>(a, rows, st);
    default: return fail(QI8_EDTYPE, "input dtype %d not in {bf16, f16, f32}", dtype);
  }
}

int grid_for(int64_t total, int threads) {
  int64_t b = (total + threads - 1) / threads;
  int64_t cap = (int64_t)sm_count() * 8;
  if (cap <= 0) cap = 1184;
  return (int)(b < 1 ? 1 : (b > cap ? cap : b));
}

}  // namespace
}  // namespace qi8

using namespace qi8;

extern "C" {

int qi8_quant_rows(const void* x, int x_dtype, int64_t rows, int64_t n, int64_t ld_x, int mode,
                   int block, int8_t* q_out, int64_t ld_q, float* scale_out, void* stream) {
  QI8_REQUIRE(device_ok(), QI8_EUNSUPPORTED, "no sm_100 device current");
  QI8_REQUIRE(x && q_out && scale_out, QI8_EINVAL, "null pointer");
  QI8_REQUIRE(rows >= 0 && n > 0 && ld_x >= n && ld_q >= n, QI8_ESHAPE, "bad sizes rows=%lld n=%lld",
              (long long)rows, (long long)n);
  QI8_REQUIRE(n <= (1 << 30) && rows < (int64_t(1) << 31), QI8_ESHAPE, "sizes too large");
  if (rows == 0) return QI8_OK;
  const int es = elem_size(x_dtype);
  QI8_REQUIRE(es == 2 || x_dtype == QI8_F32, QI8_EDTYPE, "input dtype %d not in {bf16, f16, f32}", x_dtype);
  QArgs a{x, ld_x, (int)n, q_out, ld_q, scale_out, 0};
  a.vec = aligned16(x) && (ld_x * es) % 16 == 0 && (reinterpret_cast<uintptr_t>(q_out) & 7) == 0 && ld_q % 8 == 0;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const bool gelu = (mode & QI8_Q_GELU) != 0;
  mode &= ~QI8_Q_GELU;
  if (mode == QI8_Q_TOKEN)
    return gelu ? launch_quant_rows<QI8_Q_TOKEN, true>(x_dtype, a, rows, st)
                : launch_quant_rows<QI8_Q_TOKEN, false>(x_dtype, a, rows, st);
  if (mode == QI8_Q_BLOCK) {
    QI8_REQUIRE(block == 128, QI8_ESHAPE, "block size must be 128 (got %d)", block);
    QI8_REQUIRE(n % 128 == 0, QI8_ESHAPE, "Last dimension size must be divisible by block_size (block_size=128)");
    return gelu ? launch_quant_rows<QI8_Q_BLOCK, true>(x_dtype, a, rows, st)
                : launch_quant_rows<QI8_Q_BLOCK, false>(x_dtype, a, rows, st);
  }
  return fail(QI8_EINVAL, "unknown quantization mode %d", mode);
}

int qi8_rotate_quant_rows(const void* x, int x_dtype, int64_t rows, int64_t n, int64_t ld_x,
                          int64_t n_pad, const float* sign, int normalize, int mode, int8_t* q_out,
                          float* scale_out, void* stream) {
  QI8_REQUIRE(device_ok(), QI8_EUNSUPPORTED, "no sm_100 device current");
  QI8_REQUIRE(x && q_out && scale_out, QI8_EINVAL, "null pointer");
  const int L = log2_exact(n_pad);
  QI8_REQUIRE(L >= 1 && L <= 15, QI8_ESHAPE, "Hadamard size must be a power of 2 in [2, 32768], got %lld",
              (long long)n_pad);
  QI8_REQUIRE(n > 0 && n <= n_pad && ld_x >= n && rows >= 0 && rows < (int64_t(1) << 31), QI8_ESHAPE,
              "bad sizes rows=%lld n=%lld n_pad=%lld", (long long)rows, (long long)n, (long long)n_pad);
  QI8_REQUIRE(aligned16(q_out), QI8_EALIGN, "q_out must be 16-byte aligned");
  if (rows == 0) return QI8_OK;
  const int es = elem_size(x_dtype);
  RotArgs a{};
  a.x = x; a.ld_x = ld_x; a.n_in = (int)n; a.pre_sign = sign; a.post_sign = nullptr;
  a.norm = (float)(1.0 / std::sqrt((double)n_pad)); a.do_norm = normalize != 0;
  a.vec = aligned16(x) && (ld_x * es) % 16 == 0;
  a.q = q_out; a.scale = scale_out;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (mode == QI8_Q_TOKEN) return launch_rotate_dtype<RO_Q_TOKEN>(x_dtype, L, a, rows, st);
  if (mode == QI8_Q_BLOCK) {
    QI8_REQUIRE(n_pad >= 128, QI8_ESHAPE, "block mode needs n_pad >= 128");
    return launch_rotate_dtype<RO_Q_BLOCK>(x_dtype, L, a, rows, st);
  }
  return fail(QI8_EINVAL, "unknown quantization mode %d", mode);
}

int qi8_fwht_rows(const void* x, int x_dtype, int64_t rows, int64_t n, int64_t ld_x, int64_t n_pad,
                  const float* pre_sign, const float* post_sign, int normalize, float* out,
                  void* stream) {
  QI8_REQUIRE(device_ok(), QI8_EUNSUPPORTED, "no sm_100 device current");
  QI8_REQUIRE(x && out, QI8_EINVAL, "null pointer");
  const int L = log2_exact(n_pad);
  QI8_REQUIRE(L >= 1 && L <= 15, QI8_ESHAPE, "Hadamard size must be a power of 2 in [2, 32768], got %lld",
              (long long)n_pad);
  QI8_REQUIRE(n > 0 && n <= n_pad && ld_x >= n && rows >= 0 && rows < (int64_t(1) << 31), QI8_ESHAPE,
              "bad sizes");
  QI8_REQUIRE(aligned16(out), QI8_EALIGN, "out must be 16-byte aligned");
  if (rows == 0) return QI8_OK;
  const int es = elem_size(x_dtype);
  RotArgs a{};
  a.x = x; a.ld_x = ld_x; a.n_in = (int)n; a.pre_sign = pre_sign; a.post_sign = post_sign;
  a.norm = (float)(1.0 / std::sqrt((double)n_pad)); a.do_norm = normalize != 0;
  a.vec = aligned16(x) && (ld_x * es) % 16 == 0;
  a.f_out = out;
  return launch_rotate_dtype<RO_F32>(x_dtype, L, a, rows, static_cast<cudaStream_t>(stream));
}

int qi8_unrotate_rows(const float* y_had, int64_t rows, int64_t n_pad, const float* sign_u,
                      const void* bias, int bias_dtype, int64_t n_out, void* out, int out_dtype,
                      int64_t ld_out, void* stream) {
  QI8_REQUIRE(device_ok(), QI8_EUNSUPPORTED, "no sm_100 device current");
  QI8_REQUIRE(y_had && out, QI8_EINVAL, "null pointer");
  const int L = log2_exact(n_pad);
  QI8_REQUIRE(L >= 1 && L <= 15, QI8_ESHAPE, "Hadamard size must be a power of 2 in [2, 32768], got %lld",
              (long long)n_pad);
  QI8_REQUIRE(n_out > 0 && n_out <= n_pad && ld_out >= n_out && rows >= 0, QI8_ESHAPE, "bad sizes");
  QI8_REQUIRE(out_dtype == QI8_BF16 || out_dtype == QI8_F16 || out_dtype == QI8_F32, QI8_EDTYPE,
              "out dtype %d", out_dtype);
  QI8_REQUIRE(!bias || bias_dtype == QI8_BF16 || bias_dtype == QI8_F16 || bias_dtype == QI8_F32, QI8_EDTYPE,
              "bias dtype %d", bias_dtype);
  if (rows == 0) return QI8_OK;
  RotArgs a{};
  a.x = y_had; a.ld_x = n_pad; a.n_in = (int)n_pad; a.pre_sign = nullptr; a.post_sign = sign_u;
  a.norm = (float)(1.0 / std::sqrt((double)n_pad)); a.do_norm = 1;
  a.vec = aligned16(y_had);
  a.bias = bias; a.bias_dtype = bias_dtype; a.n_out = (int)n_out; a.out = out; a.out_dtype = out_dtype;
  a.ld_out = ld_out;
  return launch_rotate<float, RO_UNROT>(L, a, rows, static_cast<cudaStream_t>(stream));
}

int qi8_dequant(const int8_t* q, int64_t rows, int64_t n, const float* scale, int scale_kind, int block,
                void* out, int out_dtype, void* stream) {
  QI8_REQUIRE(device_ok(), QI8_EUNSUPPORTED, "no sm_100 device current");
  QI8_REQUIRE(q && scale && out, QI8_EINVAL, "null pointer");
  QI8_REQUIRE(rows >= 0 && n > 0, QI8_ESHAPE, "bad sizes");
  QI8_REQUIRE(out_dtype == QI8_BF16 || out_dtype == QI8_F16 || out_dtype == QI8_F32, QI8_EDTYPE,
              "out dtype %d", out_dtype);
  QI8_REQUIRE(scale_kind >= QI8_S_SCALAR && scale_kind <= QI8_S_TILE128, QI8_EINVAL, "scale kind %d",
              scale_kind);
  if ((scale_kind == QI8_S_ROW_KBLOCK || scale_kind == QI8_S_TILE128))
    QI8_REQUIRE(block > 0 && n % block == 0, QI8_ESHAPE, "n %% block != 0");
  if (rows == 0) return QI8_OK;
  const int64_t total = rows * n;
  dequant_kernel<<<grid_for(total, 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      q, rows, n, scale, scale_kind, block, out, out_dtype);
  return check_cuda(cudaGetLastError(), "dequant_kernel launch");
}

int qi8_quant_weight(const void* w, int w_dtype, int64_t rows, int64_t n, int scale_kind, int8_t* q_out,
                     float* scale_out, void* workspace, int64_t workspace_bytes, void* stream) {
  QI8_REQUIRE(device_ok(), QI8_EUNSUPPORTED, "no sm_100 device current");
  QI8_REQUIRE(w && q_out && scale_out, QI8_EINVAL, "null pointer");
  QI8_REQUIRE(rows > 0 && n > 0, QI8_ESHAPE, "bad sizes");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int64_t total = rows * n;
  if (scale_kind == QI8_S_ROW) return qi8_quant_rows(w, w_dtype, rows, n, n, QI8_Q_TOKEN, 0, q_out, n, scale_out, stream);
  if (scale_kind == QI8_S_SCALAR) {
    QI8_REQUIRE(workspace && workspace_bytes >= 4, QI8_EINVAL, "tensorwise quantization needs a 4-byte workspace");
    unsigned int* ws = static_cast<unsigned int*>(workspace);
    QI8_CUDA(cudaMemsetAsync(ws, 0, 4, st));
    const int g = grid_for(total, 256);
    switch (w_dtype) {
      case QI8_BF16:
        absmax_kernel<__nv_bfloat16><<<g, 256, 0, st>>>(static_cast<const __nv_bfloat16*>(w), total, ws);
        quant_tensorwise_kernel<__nv_bfloat16><<<g, 256, 0, st>>>(static_cast<const __nv_bfloat16*>(w), total, ws, q_out, scale_out);
        break;
      case QI8_F16:
        absmax_kernel<__half><<<g, 256, 0, st>>>(static_cast<const __half*>(w), total, ws);
        quant_tensorwise_kernel<__half><<<g, 256, 0, st>>>(static_cast<const __half*>(w), total, ws, q_out, scale_out);
        break;
      case QI8_F32:
        absmax_kernel<float><<<g, 256, 0, st>>>(static_cast<const float*>(w), total, ws);
        quant_tensorwise_kernel<float><<<g, 256, 0, st>>>(static_cast<const float*>(w), total, ws, q_out, scale_out);
        break;
      default: return fail(QI8_EDTYPE, "weight dtype %d", w_dtype);
    }
    return check_cuda(cudaGetLastError(), "tensorwise quant launch");
  }
  if (scale_kind == QI8_S_TILE128) {
    QI8_REQUIRE(rows % 128 == 0 && n % 128 == 0, QI8_ESHAPE,
                "Dimensions must be divisible by block_size=128, got shape (%lld, %lld)", (long long)rows, (long long)n);
    dim3 grid((unsigned)(n / 128), (unsigned)(rows / 128));
    switch (w_dtype) {
      case QI8_BF16: quant_tile128_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>(static_cast<const __nv_bfloat16*>(w), rows, n, q_out, scale_out); break;
      case QI8_F16: quant_tile128_kernel<__half><<<grid, 256, 0, st>>>(static_cast<const __half*>(w), rows, n, q_out, scale_out); break;
      case QI8_F32: quant_tile128_kernel<float><<<grid, 256, 0, st>>>(static_cast<const float*>(w), rows, n, q_out, scale_out); break;
      default: return fail(QI8_EDTYPE, "weight dtype %d", w_dtype);
    }
    return check_cuda(cudaGetLastError(), "quant_tile128_kernel launch");
  }
  return fail(QI8_EINVAL, "scale kind %d not supported for weight quantization", scale_kind);
}

}  // extern "C"
