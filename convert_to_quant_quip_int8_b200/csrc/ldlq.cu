// QuIP with the reference's default options: diagonal rescaling, random
// permutation, damping, act-order, the fp64 factorization of the Hessian and
// the blocked lazy LDLQ loop (converters/quip_int8.py:244-352, 1031-1345).
//
// Device work here, host work (O(N) vectors) in the Python converter:
//   qi8_col_sumsq      (W**2).sum(dim=0) in torch's CPU summation order       :266
//   qi8_scale2d        W * D, (H * Dinv_j) * Dinv_i, W / D                    :280-285, :303
//   qi8_ldlq_prepare   column gather of W' (dead columns zeroed), row scale,
//                      the damped, permuted Hessian reversed for the factorization
//                                                                           :336-340, 1105-1146, 1272-1274
//   qi8_hinv_upper     U = upper Cholesky factor of H^-1 (fp64 -> fp32)      :1195-1199
//   qi8_ldlq           the LDLQ pass: 128-column blocks, 16-column lazy batches,
//                      fp32 trailing updates                                 :813-945, 638-672
//   qi8_ldlq_finish    undo act-order + random permutation, dequantize Q * s  :1348-1365, 1452, 1467-1474
//
// Hessian factorization.  The reference computes chol(H) -> cholesky_inverse
// -> chol(., upper=True) in fp64.  U (H^-1 = U^T U, U upper, positive
// diagonal) is unique, and with J the index reversal U = J L2^-1 J where
// L2 = chol(J H J): a recursive Cholesky that carries the inverse along
// (halves split until 64-wide leaves, every off-diagonal step an h x h x h
// fp64 GEMM on the tensor cores), 2/3 N^3 flops, half of the reference's.  The factorization reads the lower
// triangle of the damped Hessian, as LAPACK's potrf does in the reference;
// the rotated Hessian is not bit-symmetric (the two 1-D transforms of each
// entry pair round in different orders).
//
// LDLQ summation order: each dot product of the error feedback (16-long in
// a batch, 128-long across blocks) is accumulated by fmaf in index order
// from zero and then subtracted, fp32.  The reference's CPU path uses fp32
// BLAS (a different order of the same sums); its CUDA path runs the
// cross-block updates under bf16 autocast.
#include <cstdint>
#include <cmath>
#include "common.cuh"

namespace qi8 {
namespace {

// ----------------------------------------------------------------------------
// column sum of squares, torch CPU order
// ----------------------------------------------------------------------------

__device__ __forceinline__ int ceil_log2_i64(int64_t x) {
  return x <= 2 ? 1 : 64 - __clzll((unsigned long long)(x - 1));
}

// Four-level cascade over `size` terms (torch's multi_row_sum for one lane);
// term t is v(t).
template <class F>
__device__ __forceinline__ float cascade_sum(int64_t size, F v) {
  const int lp = max(4, ceil_log2_i64(size) / 4);
  const int64_t step = (int64_t)1 << lp, mask = step - 1;
  float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
  int64_t i = 0;
  while (i + step <= size) {
    for (int64_t j = 0; j < step; ++j, ++i) a0 = __fadd_rn(a0, v(i));
    a1 = __fadd_rn(a1, a0);
    a0 = 0.f;
    if ((i & (mask << lp)) == 0) {
      a2 = __fadd_rn(a2, a1);
      a1 = 0.f;
      if ((i & (mask << (2 * lp))) == 0) {
        a3 = __fadd_rn(a3, a2);
        a2 = 0.f;
      }
    }
  }
  for (; i < size; ++i) a0 = __fadd_rn(a0, v(i));
  a0 = __fadd_rn(a0, a1);
  a0 = __fadd_rn(a0, a2);
  return __fadd_rn(a0, a3);
}

// One thread per column.  Columns < nv: cascade over the M rows; columns >=
// nv: torch's row_sum (the column as [M/4, 4], a cascade per lane over M/4
// terms, the M % 4 left-over rows into lane 0, then lane0 += lane1 + ...).
__global__ void col_sumsq_kernel(const void* __restrict__ w, int dtype, int64_t M, int64_t N, int64_t ld,
                                 int64_t nv, float* __restrict__ out) {
  const int64_t col = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (col >= N) return;
  auto sq = [&](int64_t r) {
    const float f = load_as_f32(w, dtype, r * ld + col);
    return __fmul_rn(f, f);
  };
  float s;
  if (col < nv) {
    s = cascade_sum(M, sq);
  } else {
    const int64_t si = M / 4;
    float lane[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) lane[k] = si ? cascade_sum(si, [&](int64_t t) { return sq(4 * t + k); }) : 0.f;
    for (int64_t r = 4 * si; r < M; ++r) lane[0] = __fadd_rn(lane[0], sq(r));
    s = __fadd_rn(__fadd_rn(__fadd_rn(lane[0], lane[1]), lane[2]), lane[3]);
  }
  out[col] = s;
}

// out[i, j] = divide ? x[i, j] / col[j] : (x[i, j] * col[j]) * row[i]
// (row may be null; x null is the identity matrix).
__global__ void scale2d_kernel(const void* __restrict__ x, int dtype, int64_t M, int64_t N, int64_t ld,
                               const float* __restrict__ row, const float* __restrict__ col, int divide,
                               float* __restrict__ out, int64_t ld_out) {
  const int64_t total = M * N;
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x) {
    const int64_t i = e / N, j = e - i * N;
    const float v = x ? load_as_f32(x, dtype, i * ld + j) : (i == j ? 1.f : 0.f);
    float r;
    if (divide) {
      r = __fdiv_rn(v, col[j]);
    } else {
      r = col ? __fmul_rn(v, col[j]) : v;
      if (row) r = __fmul_rn(r, row[i]);
    }
    out[i * ld_out + j] = r;
  }
}

// One CTA per row of W': stage the row in shared memory, gather columns
// cols[j] (zero where dead[j]), write the row of W_p, and the row scale
// max(amax / 127, 1e-12).
__global__ void __launch_bounds__(256) ldlq_gather_w_kernel(const float* __restrict__ wrot, int64_t N,
                                                           const int* __restrict__ cols,
                                                           const uint8_t* __restrict__ dead, float* __restrict__ wp,
                                                           float* __restrict__ scale) {
  extern __shared__ float srow[];
  __shared__ float red[8];
  const int64_t r = blockIdx.x;
  const float4* src = reinterpret_cast<const float4*>(wrot + r * N);
  for (int64_t i = threadIdx.x; i < N / 4; i += blockDim.x) reinterpret_cast<float4*>(srow)[i] = src[i];
  for (int64_t i = (N / 4) * 4 + threadIdx.x; i < N; i += blockDim.x) srow[i] = wrot[r * N + i];
  __syncthreads();
  float amax = 0.f;
  for (int64_t j = threadIdx.x; j < N; j += blockDim.x) {
    const float v = dead[j] ? 0.f : srow[cols[j]];
    wp[r * N + j] = v;
    amax = fmaxf(amax, fabsf(v));
  }
  amax = warp_max(amax);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = amax;
  __syncthreads();
  if (threadIdx.x == 0) {
    float m = red[0];
    for (int k = 1; k < (int)(blockDim.x >> 5); ++k) m = fmaxf(m, red[k]);
    scale[r] = fmaxf(__fdiv_rn(m, 127.0f), 1e-12f);
  }
}

// Hrev[i, j] (fp64, lower triangle, zeros above) = Hs[N-1-i, N-1-j] where Hs
// is the damped, permuted Hessian symmetrized from its lower triangle:
//   Hs[a, b] = a == b ? diag[a] : H'[cols[max(a,b)], cols[min(a,b)]].
// For i > j that is H'[cols[N-1-j], cols[N-1-i]].  64x64 output tiles; the
// tile's 64 source rows are read whole-row-coalesced through shared memory
// in 64-column slices of the gathered index list.
constexpr int HT = 64;
__global__ void __launch_bounds__(256) ldlq_gather_h_kernel(const float* __restrict__ hrot, int64_t N,
                                                           const int* __restrict__ cols,
                                                           const float* __restrict__ diag,
                                                           double* __restrict__ hrev) {
  __shared__ float tile[HT][HT + 1];  // tile[jj][ii] = H'[cols[N-1-j], cols[N-1-i]]
  const int64_t i0 = (int64_t)blockIdx.y * HT, j0 = (int64_t)blockIdx.x * HT;
  const int tid = threadIdx.x;
  if (j0 > i0) {  // strictly upper tile: zeros
    for (int e = tid; e < HT * HT; e += 256) hrev[(i0 + e / HT) * N + j0 + e % HT] = 0.0;
    return;
  }
  // each warp fills 8 source rows; lane l reads the gathered columns l, l+32
  const int warp = tid >> 5, lane = tid & 31;
  for (int jj = warp; jj < HT; jj += 8) {
    const int64_t src = cols[N - 1 - (j0 + jj)];
    const float* hr = hrot + src * N;
    for (int ii = lane; ii < HT; ii += 32) tile[jj][ii] = hr[cols[N - 1 - (i0 + ii)]];
  }
  __syncthreads();
  for (int e = tid; e < HT * HT; e += 256) {
    const int ii = e / HT, jj = e % HT;
    const int64_t i = i0 + ii, j = j0 + jj;
    double v;
    if (i == j) v = (double)diag[N - 1 - i];
    else if (i > j) v = (double)tile[jj][ii];
    else v = 0.0;
    hrev[i * N + j] = v;
  }
}

// Small N (< 64): one CTA, plain loops.
__global__ void ldlq_gather_h_small_kernel(const float* __restrict__ hrot, int64_t N, const int* __restrict__ cols,
                                           const float* __restrict__ diag, double* __restrict__ hrev) {
  for (int64_t e = threadIdx.x; e < N * N; e += blockDim.x) {
    const int64_t i = e / N, j = e % N;
    double v = 0.0;
    if (i == j) v = (double)diag[N - 1 - i];
    else if (i > j) v = (double)hrot[(int64_t)cols[N - 1 - j] * N + cols[N - 1 - i]];
    hrev[e] = v;
  }
}

// One CTA per row: deq[r, cols[j]] = Q[r, j] * scale[r] and/or
// qs[r, cols[j]] = Q[r, j], scattered through shared memory so the stores
// stay row-contiguous.
__global__ void __launch_bounds__(256) ldlq_scatter_kernel(const int8_t* __restrict__ q, int64_t N,
                                                          const float* __restrict__ scale,
                                                          const int* __restrict__ cols, float* __restrict__ deq,
                                                          int8_t* __restrict__ qs) {
  extern __shared__ float sdeq[];
  int8_t* sq = reinterpret_cast<int8_t*>(sdeq + N);
  const int64_t r = blockIdx.x;
  const float s = scale[r];
  for (int64_t j = threadIdx.x; j < N; j += blockDim.x) {
    const int8_t v = q[r * N + j];
    const int c = cols[j];
    sdeq[c] = __fmul_rn((float)v, s);
    sq[c] = v;
  }
  __syncthreads();
  if (deq)
    for (int64_t j = threadIdx.x; j < N; j += blockDim.x) deq[r * N + j] = sdeq[j];
  if (qs)
    for (int64_t j = threadIdx.x; j < N; j += blockDim.x) qs[r * N + j] = sq[j];
}

// Hinv[i, j] = i <= j ? float(X[N-1-i, N-1-j]) : 0   (U = J X J, X = L2^-1)
__global__ void hinv_out_kernel(const double* __restrict__ x, int64_t N, float* __restrict__ hinv) {
  const int64_t total = N * N;
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x) {
    const int64_t i = e / N, j = e - i * N;
    hinv[e] = i <= j ? (float)x[(N - 1 - i) * N + (N - 1 - j)] : 0.f;
  }
}

__global__ void eye_kernel(int64_t N, float* __restrict__ out) {
  const int64_t total = N * N;
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x)
    out[e] = (e / N == e % N) ? 1.f : 0.f;
}

// ----------------------------------------------------------------------------
// fp64 factorization
// ----------------------------------------------------------------------------

// Cholesky of one nb x nb diagonal block (nb <= 64, lower triangle of A at
// ld), then its inverse, written back over the block (zeros above the
// diagonal).  A non-positive or non-finite pivot records its global index + 1
// in *info (first failure wins) and continues with pivot 1.
//
// Factorization: one barrier per column.  At step j every thread reads the
// (final) column j of the working matrix a, takes the pivot d = sqrt(a_jj)
// itself, writes its entries of L[:, j] = a[:, j] * (1 / d) into l (a separate
// array, so no thread overwrites what another still reads) and applies its
// share of the rank-1 update to the trailing lower triangle of a.  Inverse:
// one warp per column c solves L x = e_c right-looking with the diagonal
// reciprocals precomputed; lane holds rows lane and lane + 32.
constexpr int PB = 64;
__global__ void __launch_bounds__(256) potf2_inv_kernel(double* A, int64_t ld, int nb, int64_t base, int* info) {
  extern __shared__ double psm[];
  double (*a)[PB + 1] = reinterpret_cast<double (*)[PB + 1]>(psm);
  double (*l)[PB + 1] = reinterpret_cast<double (*)[PB + 1]>(psm + PB * (PB + 1));
  double* rd = psm + 2 * PB * (PB + 1);  // reciprocals of L's diagonal
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  for (int e = tid; e < nb * nb; e += 256) {
    const int i = e / nb, j = e % nb;
    a[i][j] = j <= i ? A[(int64_t)i * ld + j] : 0.0;
  }
  __syncthreads();
  for (int j = 0; j < nb; ++j) {
    double d = a[j][j];
    const bool bad = !(d > 0.0) || !isfinite(d);
    if (bad) d = 1.0;
    if (bad && tid == 0) atomicCAS(info, 0, (int)(base + j + 1));
    d = sqrt(d);
    const double r = 1.0 / d;
    const int m = nb - j;  // rows j..nb-1 of column j
    for (int i = tid; i < m; i += 256) l[j + i][j] = i == 0 ? d : a[j + i][j] * r;
    const int t = m - 1;   // trailing rows / columns j+1..nb-1
    for (int e = tid; e < t * t; e += 256) {
      const int ii = e / t, ll = e % t;
      if (ll <= ii) {
        const double li = a[j + 1 + ii][j] * r, lj = a[j + 1 + ll][j] * r;
        a[j + 1 + ii][j + 1 + ll] = fma(-li, lj, a[j + 1 + ii][j + 1 + ll]);
      }
    }
    __syncthreads();
  }
  for (int i = tid; i < nb; i += 256) rd[i] = 1.0 / l[i][i];
  __syncthreads();
  const unsigned full = 0xffffffffu;
  for (int c = warp; c < nb; c += 8) {
    double x0 = lane == c ? 1.0 : 0.0, x1 = lane + 32 == c ? 1.0 : 0.0;
    for (int t = c; t < nb; ++t) {
      double xt = t < 32 ? __shfl_sync(full, x0, t) : __shfl_sync(full, x1, t - 32);
      xt *= rd[t];
      if (lane == t) x0 = xt;
      if (lane + 32 == t) x1 = xt;
      if (lane > t && lane < nb) x0 = fma(-l[lane][t], xt, x0);
      if (lane + 32 > t && lane + 32 < nb) x1 = fma(-l[lane + 32][t], xt, x1);
    }
    if (lane < nb) A[(int64_t)lane * ld + c] = lane >= c ? x0 : 0.0;
    if (lane + 32 < nb) A[(int64_t)(lane + 32) * ld + c] = lane + 32 >= c ? x1 : 0.0;
  }
}

// C = alpha * A @ op(B) (+ C when accumulate), fp64, 64x64 tiles, batched
// over blockIdx.z.  op(B)[k, n] = transB ? B[n, k] : B[k, n].  Triangular
// operands restrict the k range per tile: triA (A lower) k < m0 + 64;
// triB (B lower as stored) k >= n0 without transB, k < n0 + 64 with it.
// lowerC skips tiles strictly above the diagonal and leaves the strict upper
// triangle of diagonal tiles untouched.  M, N multiples of 64, the k range a
// multiple of 16; every offset fits in 32 bits (N <= 32768).  C must not
// alias A or B.
struct DGemm {
  const double* A;
  const double* B;
  double* C;
  int64_t lda, ldb, ldc, sA, sB, sC;
  int M, N, K, transB, triA, triB, lowerC, accumulate;
  double alpha;
};

// The GEMM on the fp64 tensor cores (mma.sync m8n8k4 f64; tcgen05 has no
// fp64 kind): 64x64 tiles, 4 warps of 32x32 (4x4 fragments of 8x8), 16-deep
// k chunks double-buffered through registers.  A is staged row-major [m][20] (k inner), B
// row-major [n][20] with transB and k-major [k][68] without; the strides
// make the fragment reads (8 rows x 4 k per warp) and the coalesced stores
// free of bank conflicts.
template <bool TRANSB>
__global__ void __launch_bounds__(128, 3) dgemm_mma_kernel(DGemm g) {
  const int m0 = blockIdx.y * 64, n0 = blockIdx.x * 64;
  if (g.lowerC && m0 + 64 <= n0) return;
  const double* __restrict__ A = g.A + (int64_t)blockIdx.z * g.sA;
  const double* __restrict__ B = g.B + (int64_t)blockIdx.z * g.sB;
  double* C = g.C + (int64_t)blockIdx.z * g.sC;
  const int lda = (int)g.lda, ldb = (int)g.ldb, ldc = (int)g.ldc;
  int k0 = 0, k1 = g.K;
  if (g.triA) k1 = min(k1, m0 + 64);
  if (g.triB) {
    if (TRANSB) k1 = min(k1, n0 + 64);
    else k0 = n0;
  }
  constexpr int SA = 20;                 // [64][SA]
  constexpr int SBK = TRANSB ? 20 : 68;  // transB: [64 n][20]; else [16 k][68]
  constexpr int BSZ = TRANSB ? 64 * 20 : 16 * 68;
  __shared__ __align__(16) double As[2][64 * SA];
  __shared__ __align__(16) double Bs[2][BSZ];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int wm = (warp >> 1) * 32, wn = (warp & 1) * 32;
  // loads: 64 x 16 doubles per operand, 8 per thread
  const int lk = tid & 15, lr = tid >> 4;  // k-contiguous: rows lr + 8 r
  const int bn = tid & 63, bk = tid >> 6;  // n-contiguous: k rows bk + 2 r
  double ra[8], rb[8];
  auto gload = [&](int kb) {
#pragma unroll
    for (int r = 0; r < 8; ++r) ra[r] = A[(m0 + lr + 8 * r) * lda + kb + lk];
#pragma unroll
    for (int r = 0; r < 8; ++r) {
      if (TRANSB) rb[r] = B[(n0 + lr + 8 * r) * ldb + kb + lk];
      else rb[r] = B[(kb + bk + 2 * r) * ldb + n0 + bn];
    }
  };
  auto sstore = [&](int buf) {
#pragma unroll
    for (int r = 0; r < 8; ++r) As[buf][(lr + 8 * r) * SA + lk] = ra[r];
#pragma unroll
    for (int r = 0; r < 8; ++r) {
      if (TRANSB) Bs[buf][(lr + 8 * r) * SBK + lk] = rb[r];
      else Bs[buf][(bk + 2 * r) * SBK + bn] = rb[r];
    }
  };
  double acc[4][4][2];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j][0] = acc[i][j][1] = 0.0;
  if (k0 < k1) {
    gload(k0);
    sstore(0);
  }
  __syncthreads();
  const int fr = lane >> 2, fk = lane & 3;  // fragment row / k of this lane
  int buf = 0;
  for (int kb = k0; kb < k1; kb += 16) {
    const bool more = kb + 16 < k1;
    if (more) gload(kb + 16);
#pragma unroll
    for (int kk = 0; kk < 16; kk += 4) {
      double af[4], bf[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) af[i] = As[buf][(wm + i * 8 + fr) * SA + kk + fk];
#pragma unroll
      for (int j = 0; j < 4; ++j)
        bf[j] = TRANSB ? Bs[buf][(wn + j * 8 + fr) * SBK + kk + fk] : Bs[buf][(kk + fk) * SBK + wn + j * 8 + fr];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j)
          asm volatile("mma.sync.aligned.m8n8k4.row.col.f64.f64.f64.f64 {%0,%1}, {%2}, {%3}, {%0,%1};"
                       : "+d"(acc[i][j][0]), "+d"(acc[i][j][1])
                       : "d"(af[i]), "d"(bf[j]));
    }
    if (more) sstore(buf ^ 1);
    __syncthreads();
    buf ^= 1;
  }
  // accumulator fragment: row fr, columns 2 fk + {0, 1} of each 8x8 tile
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int row = m0 + wm + i * 8 + fr;
    double* c = C + row * ldc;
#pragma unroll
    for (int j = 0; j < 4; ++j)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int col = n0 + wn + j * 8 + 2 * fk + e;
        if (g.lowerC && col > row) continue;
        c[col] = g.accumulate ? fma(g.alpha, acc[i][j][e], c[col]) : g.alpha * acc[i][j][e];
      }
  }
}

int dgemm(const DGemm& g, int batch, cudaStream_t st) {
  dim3 grid((unsigned)(g.N / 64), (unsigned)(g.M / 64), (unsigned)batch);
  if (g.transB) dgemm_mma_kernel<true><<<grid, 128, 0, st>>>(g);
  else dgemm_mma_kernel<false><<<grid, 128, 0, st>>>(g);
  return check_cuda(cudaGetLastError(), "dgemm_mma_kernel launch");
}

// ----------------------------------------------------------------------------
// fp32 LDLQ
// ----------------------------------------------------------------------------

constexpr int LB = 128;    // LDLQ column block (the reference's block_size)
constexpr int LBATCH = 16; // lazy batch (_quantize_block_lazy BATCH)

// One 128-column block for 128 rows per CTA (one thread per row).  The
// block's columns sit transposed in shared memory ([c][129]), the Hinv block
// [Bw][Bw] is read as broadcasts.  Per batch of 16 columns: q = clamp(rint(w
// / s), +-127), err = (w - q * s) / max(Hinv_jj, 1e-12), then every later
// column of the block: acc = sum_k err_k * Hinv[k, c] (fmaf from zero, k in
// order), w_c = w_c - acc.  Writes Q and the block's errors.
__global__ void __launch_bounds__(LB) ldlq_block_kernel(const float* __restrict__ wp, int64_t ld, int64_t M,
                                                       int64_t i1, int bw, const float* __restrict__ hinv,
                                                       const float* __restrict__ scale, int8_t* __restrict__ q,
                                                       float* __restrict__ err) {
  extern __shared__ float lsm[];
  float* wt = lsm;                 // [bw][129]
  float* hb = lsm + bw * (LB + 1); // [bw][bw]
  const int r = threadIdx.x;
  const int64_t row0 = (int64_t)blockIdx.x * LB;
  for (int e = r; e < LB * bw; e += LB) {
    const int rr = e / bw, c = e % bw;
    wt[c * (LB + 1) + rr] = row0 + rr < M ? wp[(row0 + rr) * ld + i1 + c] : 0.f;
  }
  for (int e = r; e < bw * bw; e += LB) hb[e] = hinv[(i1 + e / bw) * ld + i1 + e % bw];
  __syncthreads();
  const int64_t row = row0 + r;
  const bool ok = row < M;
  const float s = ok ? scale[row] : 1.f;
  float* wr = wt + r;
  for (int b0 = 0; b0 < bw; b0 += LBATCH) {
    const int nb = min(LBATCH, bw - b0);
    float e[LBATCH];
    int8_t qv[LBATCH];
#pragma unroll
    for (int k = 0; k < LBATCH; ++k) {
      if (k < nb) {
        const int c = b0 + k;
        const float w = wr[c * (LB + 1)];
        const float qq = fminf(fmaxf(rintf(__fdiv_rn(w, s)), -127.f), 127.f);
        const float d = fmaxf(hb[c * bw + c], 1e-12f);
        e[k] = __fdiv_rn(__fsub_rn(w, __fmul_rn(qq, s)), d);
        qv[k] = (int8_t)(int)qq;
      } else {
        e[k] = 0.f;
        qv[k] = 0;
      }
    }
    if (ok) {
      int8_t* qo = q + row * ld + i1 + b0;
      float* eo = err + row * bw + b0;
      if (nb == LBATCH) {
        uint32_t pk[4];
#pragma unroll
        for (int t = 0; t < 4; ++t)
          pk[t] = (uint32_t)(uint8_t)qv[4 * t] | ((uint32_t)(uint8_t)qv[4 * t + 1] << 8) |
                  ((uint32_t)(uint8_t)qv[4 * t + 2] << 16) | ((uint32_t)(uint8_t)qv[4 * t + 3] << 24);
        *reinterpret_cast<uint4*>(qo) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
#pragma unroll
        for (int t = 0; t < 4; ++t)
          *reinterpret_cast<float4*>(eo + 4 * t) = make_float4(e[4 * t], e[4 * t + 1], e[4 * t + 2], e[4 * t + 3]);
      } else {
#pragma unroll
        for (int k = 0; k < LBATCH; ++k)
          if (k < nb) {
            qo[k] = qv[k];
            eo[k] = e[k];
          }
      }
    }
    for (int c = b0 + nb; c < bw; ++c) {
      float acc = 0.f;
      const float* hc = hb + b0 * bw + c;
#pragma unroll
      for (int k = 0; k < LBATCH; ++k)
        if (k < nb) acc = __fmaf_rn(e[k], hc[k * bw], acc);
      wr[c * (LB + 1)] = __fsub_rn(wr[c * (LB + 1)], acc);
    }
  }
}

// W[:, i2:i2+R] -= Err @ Hinv[i1:i1+K, i2:i2+R]: fp32, 128x128 output
// tiles, 8x8 per thread, k = 0..K-1 accumulated by fmaf in order from zero,
// then one subtraction per element.  K a multiple of 16 (<= 128, the row
// stride of err), R a multiple of 8.
__global__ void __launch_bounds__(256) ldlq_trail_kernel(float* __restrict__ w, int64_t ld, int64_t M, int64_t R,
                                                        int K, const float* __restrict__ err,
                                                        const float* __restrict__ h) {
  __shared__ __align__(16) float Es[16][LB + 4];  // Es[k][m]
  __shared__ __align__(16) float Hs[16][LB + 4];  // Hs[k][n]
  const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
  const int64_t m0 = (int64_t)blockIdx.y * LB, n0 = (int64_t)blockIdx.x * LB;
  float acc[8][8];
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[i][j] = 0.f;
  for (int kb = 0; kb < K; kb += 16) {
#pragma unroll
    for (int t = 0; t < 2; ++t) {
      const int e = tid + 256 * t, m = e >> 2, kq = (e & 3) * 4;
      float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
      if (m0 + m < M) v = *reinterpret_cast<const float4*>(err + (m0 + m) * K + kb + kq);
      Es[kq][m] = v.x;
      Es[kq + 1][m] = v.y;
      Es[kq + 2][m] = v.z;
      Es[kq + 3][m] = v.w;
    }
#pragma unroll
    for (int t = 0; t < 2; ++t) {
      const int e = tid + 256 * t, k = e >> 5, nq = (e & 31) * 4;
      float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
      if (n0 + nq < R) v = *reinterpret_cast<const float4*>(h + (int64_t)(kb + k) * ld + n0 + nq);
      *reinterpret_cast<float4*>(&Hs[k][nq]) = v;
    }
    __syncthreads();
#pragma unroll
    for (int k = 0; k < 16; ++k) {
      const float4 a0 = *reinterpret_cast<const float4*>(&Es[k][ty * 8]);
      const float4 a1 = *reinterpret_cast<const float4*>(&Es[k][ty * 8 + 4]);
      const float4 b0 = *reinterpret_cast<const float4*>(&Hs[k][tx * 8]);
      const float4 b1 = *reinterpret_cast<const float4*>(&Hs[k][tx * 8 + 4]);
      const float av[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
      const float bv[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[i][j] = __fmaf_rn(av[i], bv[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int64_t m = m0 + ty * 8 + i;
    if (m >= M || n0 + tx * 8 >= R) break;
    float* wr = w + m * ld + n0 + tx * 8;
    float4 v0 = *reinterpret_cast<float4*>(wr), v1 = *reinterpret_cast<float4*>(wr + 4);
    v0.x = __fsub_rn(v0.x, acc[i][0]);
    v0.y = __fsub_rn(v0.y, acc[i][1]);
    v0.z = __fsub_rn(v0.z, acc[i][2]);
    v0.w = __fsub_rn(v0.w, acc[i][3]);
    v1.x = __fsub_rn(v1.x, acc[i][4]);
    v1.y = __fsub_rn(v1.y, acc[i][5]);
    v1.z = __fsub_rn(v1.z, acc[i][6]);
    v1.w = __fsub_rn(v1.w, acc[i][7]);
    *reinterpret_cast<float4*>(wr) = v0;
    *reinterpret_cast<float4*>(wr + 4) = v1;
  }
}

}  // namespace
}  // namespace qi8

using namespace qi8;

namespace {
int set_smem(const void* fn, size_t bytes) {
  if (bytes > 48 * 1024)
    return check_cuda(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes),
                      "cudaFuncSetAttribute");
  return QI8_OK;
}
unsigned grid_for(int64_t total, int threads) {
  const int64_t g = (total + threads - 1) / threads;
  return (unsigned)(g < 148 * 16 ? (g < 1 ? 1 : g) : 148 * 16);
}
bool pow2(int64_t n) { return n > 0 && (n & (n - 1)) == 0; }
}  // namespace

extern "C" int qi8_col_sumsq(const void* w, int w_dtype, int64_t M, int64_t N, int64_t ld_w, float* out,
                             void* stream) {
  QI8_REQUIRE(device_ok(), QI8_EUNSUPPORTED, "no sm_100 device current");
  QI8_REQUIRE(w && out, QI8_EINVAL, "null pointer");
  QI8_REQUIRE(elem_size(w_dtype) > 0, QI8_EDTYPE, "w dtype must be bf16, f16 or f32");
  QI8_REQUIRE(M >= 1 && N >= 1 && ld_w >= N, QI8_ESHAPE, "bad shape");
  const int64_t nv = N >= 8 ? (N / 32) * 32 : (N / 4) * 4;
  col_sumsq_kernel<<<(unsigned)((N + 127) / 128), 128, 0, static_cast<cudaStream_t>(stream)>>>(w, w_dtype, M, N,
                                                                                              ld_w, nv, out);
  return check_cuda(cudaGetLastError(), "col_sumsq_kernel launch");
}

extern "C" int qi8_scale2d(const void* x, int x_dtype, int64_t M, int64_t N, int64_t ld_x, const float* row_scale,
                           const float* col_scale, int divide, float* out, int64_t ld_out, void* stream) {
  QI8_REQUIRE(device_ok(), QI8_EUNSUPPORTED, "no sm_100 device current");
  QI8_REQUIRE(out && (!divide || col_scale), QI8_EINVAL, "null pointer");
  QI8_REQUIRE(!x || elem_size(x_dtype) > 0, QI8_EDTYPE, "x dtype must be bf16, f16 or f32");
  QI8_REQUIRE(M >= 0 && N >= 0 && (!x || ld_x >= N) && ld_out >= N, QI8_ESHAPE, "bad shape");
  QI8_REQUIRE(x || M == N, QI8_ESHAPE, "the identity (x = NULL) must be square");
  if (M == 0 || N == 0) return QI8_OK;
  scale2d_kernel<<<grid_for(M * N, 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      x, x_dtype, M, N, ld_x, row_scale, col_scale, divide, out, ld_out);
  return check_cuda(cudaGetLastError(), "scale2d_kernel launch");
}

extern "C" int qi8_ldlq_prepare(const float* w_rot, const float* h_rot, int64_t M, int64_t N, const int32_t* cols,
                                const uint8_t* dead, const float* diag, float* w_out, float* scale_out,
                                double* h_rev, void* stream) {
  QI8_REQUIRE(device_ok(), QI8_EUNSUPPORTED, "no sm_100 device current");
  QI8_REQUIRE(w_rot && h_rot && cols && dead && diag && w_out && scale_out && h_rev, QI8_EINVAL, "null pointer");
  QI8_REQUIRE(M >= 1 && pow2(N) && N <= 32768, QI8_ESHAPE, "N must be a power of two <= 32768");
  QI8_REQUIRE(aligned16(w_rot), QI8_EALIGN, "w_rot must be 16-byte aligned");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const size_t smem = (size_t)N * sizeof(float);
  int rc = set_smem((const void*)ldlq_gather_w_kernel, smem);
  if (rc != QI8_OK) return rc;
  ldlq_gather_w_kernel<<<(unsigned)M, 256, smem, st>>>(w_rot, N, cols, dead, w_out, scale_out);
  rc = check_cuda(cudaGetLastError(), "ldlq_gather_w_kernel launch");
  if (rc != QI8_OK) return rc;
  if (N >= HT) {
    dim3 grid((unsigned)(N / HT), (unsigned)(N / HT));
    ldlq_gather_h_kernel<<<grid, 256, 0, st>>>(h_rot, N, cols, diag, h_rev);
  } else {
    ldlq_gather_h_small_kernel<<<1, 256, 0, st>>>(h_rot, N, cols, diag, h_rev);
  }
  return check_cuda(cudaGetLastError(), "ldlq_gather_h_kernel launch");
}

namespace {
// Recursive Cholesky with the inverse carried along: for the n x n diagonal
// block at A + off (N + 1) (lower triangle on entry), on exit the block holds
// X = chol(block)^-1 (lower, zeros above).  With h = n / 2:
//   X11 = chol_inv(A11); L21 = A21 X11^T (into t1[level]); A22 -= L21 L21^T;
//   X22 = chol_inv(A22); X21 = -(X22 L21) X11 (through t3).
// Every GEMM is h x h x h with the triangular operand's zero tiles skipped;
// the 64-wide leaves are factored and inverted by potf2_inv_kernel.
constexpr size_t POTF2_SMEM = sizeof(double) * (2 * PB * (PB + 1) + PB);

struct HinvCtx {
  double* A;
  int64_t N;
  double* t1[16];
  double* t3;
  int* info;
  cudaStream_t st;
};

int chol_inv(const HinvCtx& c, int64_t off, int64_t n, int level) {
  const int64_t N = c.N;
  double* A11 = c.A + off * (N + 1);
  if (n <= PB) {
    potf2_inv_kernel<<<1, 256, POTF2_SMEM, c.st>>>(A11, N, (int)n, off, c.info);
    return check_cuda(cudaGetLastError(), "potf2_inv_kernel launch");
  }
  const int64_t h = n / 2;
  double* A21 = A11 + h * N;
  double* A22 = A11 + h * (N + 1);
  double* T1 = c.t1[level];
  int rc = chol_inv(c, off, h, level + 1);
  if (rc != QI8_OK) return rc;
  DGemm a{};  // L21 = A21 @ X11^T
  a.A = A21; a.lda = N; a.B = A11; a.ldb = N; a.transB = 1; a.triB = 1;
  a.C = T1; a.ldc = h; a.M = a.N = a.K = (int)h; a.alpha = 1.0;
  if ((rc = dgemm(a, 1, c.st)) != QI8_OK) return rc;
  DGemm b{};  // A22 -= L21 @ L21^T (lower tiles)
  b.A = T1; b.lda = h; b.B = T1; b.ldb = h; b.transB = 1; b.lowerC = 1; b.accumulate = 1;
  b.C = A22; b.ldc = N; b.M = b.N = b.K = (int)h; b.alpha = -1.0;
  if ((rc = dgemm(b, 1, c.st)) != QI8_OK) return rc;
  if ((rc = chol_inv(c, off + h, h, level + 1)) != QI8_OK) return rc;
  DGemm d{};  // T3 = X22 @ L21
  d.A = A22; d.lda = N; d.triA = 1; d.B = T1; d.ldb = h;
  d.C = c.t3; d.ldc = h; d.M = d.N = d.K = (int)h; d.alpha = 1.0;
  if ((rc = dgemm(d, 1, c.st)) != QI8_OK) return rc;
  DGemm e{};  // X21 = -(T3 @ X11)
  e.A = c.t3; e.lda = h; e.B = A11; e.ldb = N; e.triB = 1;
  e.C = A21; e.ldc = N; e.M = e.N = e.K = (int)h; e.alpha = -1.0;
  return dgemm(e, 1, c.st);
}
}  // namespace

extern "C" int64_t qi8_hinv_workspace_bytes(int64_t N) {
  if (N < 1) return -1;
  int64_t elems = 0;
  for (int64_t h = N / 2; h >= PB; h /= 2) elems += h * h;  // t1 per level
  elems += (N / 2 >= PB) ? (N / 2) * (N / 2) : 0;             // t3
  return elems * (int64_t)sizeof(double) + 256 * 16;
}

extern "C" int qi8_hinv_upper(double* h_rev, int64_t N, float* hinv_out, int* info, void* workspace,
                              int64_t workspace_bytes, void* stream) {
  QI8_REQUIRE(device_ok(), QI8_EUNSUPPORTED, "no sm_100 device current");
  QI8_REQUIRE(h_rev && hinv_out && info && workspace, QI8_EINVAL, "null pointer");
  QI8_REQUIRE(pow2(N) && N <= 32768, QI8_ESHAPE, "N must be a power of two <= 32768");
  QI8_REQUIRE(workspace_bytes >= qi8_hinv_workspace_bytes(N), QI8_ESHAPE, "workspace too small");
  QI8_REQUIRE(aligned16(workspace) && aligned16(h_rev), QI8_EALIGN, "h_rev and workspace must be 16-byte aligned");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int rc = check_cuda(cudaMemsetAsync(info, 0, sizeof(int), st), "cudaMemsetAsync");
  if (rc != QI8_OK) return rc;
  rc = set_smem((const void*)potf2_inv_kernel, POTF2_SMEM);
  if (rc != QI8_OK) return rc;
  HinvCtx c{};
  c.A = h_rev;
  c.N = N;
  c.info = info;
  c.st = st;
  char* p = static_cast<char*>(workspace);
  int level = 0;
  for (int64_t h = N / 2; h >= PB; h /= 2, ++level) {
    c.t1[level] = reinterpret_cast<double*>(p);
    p += ((h * h * (int64_t)sizeof(double) + 255) / 256) * 256;
  }
  c.t3 = reinterpret_cast<double*>(p);
  if ((rc = chol_inv(c, 0, N, 0)) != QI8_OK) return rc;
  hinv_out_kernel<<<grid_for(N * N, 256), 256, 0, st>>>(h_rev, N, hinv_out);
  return check_cuda(cudaGetLastError(), "hinv_out_kernel launch");
}

extern "C" int qi8_eye_f32(float* out, int64_t N, void* stream) {
  QI8_REQUIRE(device_ok(), QI8_EUNSUPPORTED, "no sm_100 device current");
  QI8_REQUIRE(out, QI8_EINVAL, "null pointer");
  QI8_REQUIRE(N >= 1, QI8_ESHAPE, "bad shape");
  eye_kernel<<<grid_for(N * N, 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(N, out);
  return check_cuda(cudaGetLastError(), "eye_kernel launch");
}

extern "C" int64_t qi8_ldlq_workspace_bytes(int64_t M, int64_t N, int block) {
  if (M < 1 || N < 1 || block < 1) return -1;
  return M * (N < block ? N : block) * (int64_t)sizeof(float) + 256;
}

extern "C" int qi8_ldlq(float* w, int64_t M, int64_t N, const float* hinv, const float* scale, int block,
                        int8_t* q_out, void* workspace, int64_t workspace_bytes, void* stream) {
  QI8_REQUIRE(device_ok(), QI8_EUNSUPPORTED, "no sm_100 device current");
  QI8_REQUIRE(w && hinv && scale && q_out && workspace, QI8_EINVAL, "null pointer");
  QI8_REQUIRE(pow2(N) && N <= 32768 && M >= 1, QI8_ESHAPE, "N must be a power of two <= 32768");
  QI8_REQUIRE(block >= 16 && block <= LB && block % 16 == 0, QI8_ESHAPE, "block must be 16..128, a multiple of 16");
  QI8_REQUIRE(workspace_bytes >= qi8_ldlq_workspace_bytes(M, N, block), QI8_ESHAPE, "workspace too small");
  QI8_REQUIRE(aligned16(w) && aligned16(hinv) && aligned16(q_out) && aligned16(workspace), QI8_EALIGN,
              "w, hinv, q_out and workspace must be 16-byte aligned");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  float* err = static_cast<float*>(workspace);
  const size_t smax = sizeof(float) * ((size_t)LB * (LB + 1) + (size_t)LB * LB);
  int rc = set_smem((const void*)ldlq_block_kernel, smax);
  if (rc != QI8_OK) return rc;
  for (int64_t i1 = 0; i1 < N; i1 += block) {
    const int bw = (int)(N - i1 < block ? N - i1 : block);
    const size_t smem = sizeof(float) * ((size_t)bw * (LB + 1) + (size_t)bw * bw);
    ldlq_block_kernel<<<(unsigned)((M + LB - 1) / LB), LB, smem, st>>>(w, N, M, i1, bw, hinv, scale, q_out, err);
    if ((rc = check_cuda(cudaGetLastError(), "ldlq_block_kernel launch")) != QI8_OK) return rc;
    const int64_t i2 = i1 + bw, R = N - i2;
    if (R <= 0) break;
    dim3 grid((unsigned)((R + LB - 1) / LB), (unsigned)((M + LB - 1) / LB));
    ldlq_trail_kernel<<<grid, 256, 0, st>>>(w + i2, N, M, R, bw, err, hinv + i1 * N + i2);
    if ((rc = check_cuda(cudaGetLastError(), "ldlq_trail_kernel launch")) != QI8_OK) return rc;
  }
  return QI8_OK;
}

extern "C" int qi8_ldlq_finish(const int8_t* q, int64_t M, int64_t N, const float* scale, const int32_t* cols,
                               float* deq_out, int8_t* q_out, void* stream) {
  QI8_REQUIRE(device_ok(), QI8_EUNSUPPORTED, "no sm_100 device current");
  QI8_REQUIRE(q && scale && cols && (deq_out || q_out), QI8_EINVAL, "null pointer");
  QI8_REQUIRE(M >= 1 && pow2(N) && N <= 32768, QI8_ESHAPE, "N must be a power of two <= 32768");
  const size_t smem = (size_t)N * (sizeof(float) + 1);
  int rc = set_smem((const void*)ldlq_scatter_kernel, smem);
  if (rc != QI8_OK) return rc;
  ldlq_scatter_kernel<<<(unsigned)M, 256, smem, static_cast<cudaStream_t>(stream)>>>(q, N, scale, cols, deq_out,
                                                                                     q_out);
  return check_cuda(cudaGetLastError(), "ldlq_scatter_kernel launch");
}
