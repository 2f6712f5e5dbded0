// K4: offline QuIP Hadamard conversion of one weight matrix on the GPU.
//
// Reference (converters/quip_int8.py, identity Hessian):
//   W' = FHT_N(FHT_M(pad(W) * s_u * s_v^T))                        :539-551
//   s' = clamp(rowamax(W') / 127, 1e-12); Q' = clamp(round(W'/s'), +-127)  :1272-1274, 655
//   W_d = slice(FHT_M(FHT_N(Q' * s')) * s_u * s_v)                   :1452, 1489-1506
//   requant of W_d with per-row / global / per-(row, K-block) scales :1614-1669
// FHT_* is the normalized 1-D transform along one dimension; the M-direction
// (down the columns) runs first on the way in and last on the way out, as
// in the reference, because fp32 rounding depends on that order.
//
// GPU plan (fp32 workspace X = [M_pad, N_pad]):
//   col_fwht (1-2 passes): bf16/f32 W -> signs -> M-direction stages -> X
//   quip_row:  one CTA per row: FHT_N, RTN to int8, dequant, FHT_N -> X
//   col_fwht (1-2 passes): M-direction stages -> signs -> slice -> W_d
//   requant_{row,block,global}: W_d -> int8 + scales
// A column pass holds up to 512 rows x 32 columns in shared memory and
// performs the butterfly stages of a contiguous range of row-index bits;
// ranges run in ascending order, so the stage order equals the reference's.
#include <atomic>
#include <cmath>
#include <cstdint>

#include "common.cuh"
#include "fwht_row.cuh"

namespace qi8 {
namespace {

constexpr int COL_STRIP = 32;
constexpr int COL_THREADS = 256;
constexpr int COL_MAX_BITS = 9;

struct ColArgs {
  const void* w;  // first forward pass: source weight [M, N]
  int w_dtype;
  int64_t M, N, M_pad, N_pad;
  float* x;  // workspace [M_pad, N_pad]
  const float* s_u;
  const float* s_v;
  int b0, rbits;  // this pass transforms row-index bits [b0, b0 + rbits)
  float norm;     // last pass: multiply by norm (FINAL_MUL) or divide by it (FINAL_DIV)
  int64_t ld_x;   // row stride of x (columns j < N_pad are transformed)
  float* dst;  // inverse last pass: W_d destination [M, N] with row stride ld_dst
  int64_t ld_dst;
};

enum { FINAL_NONE = 0, FINAL_MUL = 1, FINAL_DIV = 2 };

// One round of the column transform: the RB butterfly stages of strides
// 2^s .. 2^(s+RB-1) (in rows of the strip) on groups of 2^RB rows held in
// registers, one column per lane.  Stages run in ascending stride order, as
// in the reference's FWHT, so every element sees the same operations.
template <int RB>
__device__ __forceinline__ void col_round(float* tile, int R, int s, int warp, int nw, int lane) {
  constexpr int G = 1 << RB;
  const int groups = R >> RB;
  const int lo_mask = (1 << s) - 1;
  for (int g = warp; g < groups; g += nw) {
    const int base = (g & lo_mask) | ((g >> s) << (s + RB));
    float v[G];
#pragma unroll
    for (int j = 0; j < G; ++j) v[j] = tile[(base | (j << s)) * COL_STRIP + lane];
#pragma unroll
    for (int b = 0; b < RB; ++b) {
#pragma unroll
      for (int j = 0; j < G; ++j) {
        if (j & (1 << b)) continue;
        const float x = v[j], y = v[j | (1 << b)];
        v[j] = x + y;
        v[j | (1 << b)] = x - y;
      }
    }
#pragma unroll
    for (int j = 0; j < G; ++j) tile[(base | (j << s)) * COL_STRIP + lane] = v[j];
  }
}

// Column (M-direction) FWHT over row-index bits [b0, b0 + rbits) of X: a CTA
// holds a strip of R = 2^rbits rows (stride 2^b0 apart) x 32 columns in shared
// memory (bank = lane, conflict-free), runs the stages in rounds of up to
// four bits in registers, and writes the strip back.  Loads and stores are
// 128-byte row segments per warp.
template <bool LOAD_W, int FINAL, bool SIGN_OUT>
__global__ void __launch_bounds__(COL_THREADS) col_fwht_kernel(ColArgs a) {
  extern __shared__ float tile[];  // [R][COL_STRIP]
  const int R = 1 << a.rbits;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nw = blockDim.x >> 5;
  const int64_t j = (int64_t)blockIdx.x * COL_STRIP + lane;
  const bool col_ok = j < a.N_pad;
  const int64_t lo_count = int64_t(1) << a.b0;
  const int64_t lo = blockIdx.y % lo_count, hi = blockIdx.y / lo_count;
  const int64_t hi_base = lo + (hi << (a.b0 + a.rbits));

  float sv = 1.0f;
  if constexpr (LOAD_W) sv = (col_ok && j < a.N_pad) ? __ldg(a.s_v + j) : 0.0f;
#pragma unroll 16
  for (int k = warp; k < R; k += nw) {
    const int64_t i = hi_base + ((int64_t)k << a.b0);
    float v = 0.0f;
    if (col_ok) {
      if constexpr (LOAD_W) {
        v = (i < a.M && j < a.N) ? load_as_f32(a.w, a.w_dtype, i * a.N + j) : 0.0f;
        v = __fmul_rn(v, __ldg(a.s_u + i));
        v = __fmul_rn(v, sv);
      } else {
        v = a.x[i * a.ld_x + j];
      }
    }
    tile[k * COL_STRIP + lane] = v;
  }
  __syncthreads();
  for (int s = 0; s < a.rbits; s += 4) {
    switch (a.rbits - s >= 4 ? 4 : a.rbits - s) {
      case 4: col_round<4>(tile, R, s, warp, nw, lane); break;
      case 3: col_round<3>(tile, R, s, warp, nw, lane); break;
      case 2: col_round<2>(tile, R, s, warp, nw, lane); break;
      default: col_round<1>(tile, R, s, warp, nw, lane); break;
    }
    __syncthreads();
  }
#pragma unroll 16
  for (int k = warp; k < R; k += nw) {
    const int64_t i = hi_base + ((int64_t)k << a.b0);
    float v = tile[k * COL_STRIP + lane];
    if constexpr (FINAL == FINAL_MUL) v = __fmul_rn(v, a.norm);
    if constexpr (FINAL == FINAL_DIV) v = __fdiv_rn(v, a.norm);
    if constexpr (SIGN_OUT) {
      if (i < a.M && j < a.N) {
        v = __fmul_rn(v, __ldg(a.s_u + i));
        v = __fmul_rn(v, __ldg(a.s_v + j));
        a.dst[i * a.ld_dst + j] = v;
      }
    } else {
      if (col_ok) a.x[i * a.ld_x + j] = v;
    }
  }
}

struct RowArgs {
  float* x;
  int64_t ld_x;
  float norm;
  int8_t* q_rot;  // optional [M_pad, N_pad]
  float* s_rot;   // optional [M_pad]
};

template <int L>
__global__ void __launch_bounds__(RotCfg<L>::THREADS) quip_row_kernel(RowArgs a) {
  using C = RotCfg<L>;
  constexpr int E = C::E, P = C::P;
  extern __shared__ float4 dyn_smem[];
  float* buf = reinterpret_cast<float*>(dyn_smem);
  __shared__ float red[32];
  const int t = threadIdx.x;
  const bool active = t < P;
  const int64_t row = blockIdx.x;
  float* xr = a.x + row * a.ld_x;
  const int c0 = t * E;
  float v[E];
#pragma unroll
  for (int e = 0; e < E; ++e) v[e] = active ? xr[c0 + e] : 0.0f;

  fwht_row<L>(v, buf);
  float local = 0.0f;
#pragma unroll
  for (int e = 0; e < E; ++e) {
    v[e] = __fmul_rn(v[e], a.norm);
    local = fmaxf(local, fabsf(v[e]));
  }
  const float amax = block_max(local, red);
  const float s = fmaxf(__fdiv_rn(amax, 127.0f), 1e-12f);
  int8_t q[E];
#pragma unroll
  for (int e = 0; e < E; ++e) q[e] = rint_clamp(__fdiv_rn(v[e], s), -127.0f, 127.0f);
  if (a.q_rot && active) {
#pragma unroll
    for (int e = 0; e < E; ++e) a.q_rot[row * C::N + c0 + e] = q[e];
  }
  if (a.s_rot && t == 0) a.s_rot[row] = s;
#pragma unroll
  for (int e = 0; e < E; ++e) v[e] = __fmul_rn((float)q[e], s);
  fwht_row<L>(v, buf);
  if (active) {
#pragma unroll
    for (int e = 0; e < E; ++e) xr[c0 + e] = __fmul_rn(v[e], a.norm);
  }
}

// Row pass for rows of 2^9..2^14 on the phased transform (16 elements per
// thread, see fwht_row.cuh): forward FWHT, x norm, row amax, division RTN
// (+-127), dequantize, one exchange back to the contiguous mapping, inverse
// FWHT, x norm.  The same operations in the same order as quip_row_kernel.
template <int L>
__global__ void __launch_bounds__(1 << (L - 4)) quip_row_phased_kernel(RowArgs a) {
  using namespace rowfwht;
  constexpr int N = 1 << L, NW = nwin<L>(), WL = wstart<L>(NW - 1);
  extern __shared__ float4 dyn_smem[];
  float* buf = reinterpret_cast<float*>(dyn_smem);
  __shared__ float red[32];
  const int t = threadIdx.x;
  const int64_t row = blockIdx.x;
  float* xr = a.x + row * a.ld_x;
  float v[16];
  // contiguous mapping: this thread holds elements t*16 .. t*16 + 15
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const float4 f = reinterpret_cast<const float4*>(xr + t * 16)[q];
    v[4 * q] = f.x; v[4 * q + 1] = f.y; v[4 * q + 2] = f.z; v[4 * q + 3] = f.w;
  }
  stages<L, 0>(v);
  phase<L, 1>(v, buf, t);
  // last-window mapping: element e is index ib + (e << WL)
  const int ib = wbase(t, WL);
  float local = 0.0f;
#pragma unroll
  for (int e = 0; e < 16; ++e) {
    v[e] = __fmul_rn(v[e], a.norm);
    local = fmaxf(local, fabsf(v[e]));
  }
  const float amax = block_max(local, red);
  const float s = fmaxf(__fdiv_rn(amax, 127.0f), 1e-12f);
#pragma unroll
  for (int e = 0; e < 16; ++e) {
    const int8_t q = rint_clamp(__fdiv_rn(v[e], s), -127.0f, 127.0f);
    if (a.q_rot) a.q_rot[row * N + ib + (e << WL)] = q;
    v[e] = __fmul_rn((float)q, s);
  }
  if (a.s_rot && t == 0) a.s_rot[row] = s;
  // back to the contiguous mapping (block_max above ordered every read of the
  // last phase before these writes; each address is written by its reader)
  {
    const int sb = swz(ib);
#pragma unroll
    for (int e = 0; e < 16; ++e) buf[sb ^ swz(e << WL)] = v[e];
    __syncthreads();
    const int sc = swz(t * 16);
#pragma unroll
    for (int e = 0; e < 16; ++e) v[e] = buf[sc ^ swz(e)];
  }
  stages<L, 0>(v);
  phase<L, 1>(v, buf, t);
#pragma unroll
  for (int e = 0; e < 16; ++e) xr[ib + (e << WL)] = __fmul_rn(v[e], a.norm);
}

template <int L>
int launch_row_L(const RowArgs& a, int64_t rows, cudaStream_t st) {
  if constexpr (L >= 9 && L <= 14) {
    auto pk = quip_row_phased_kernel<L>;
    constexpr int SM = (1 << L) * 4;
    if (SM > 48 * 1024) QI8_CUDA(cudaFuncSetAttribute(pk, cudaFuncAttributeMaxDynamicSharedMemorySize, SM));
    pk<<<(unsigned)rows, 1 << (L - 4), SM, st>>>(a);
    return check_cuda(cudaGetLastError(), "quip_row_phased_kernel launch");
  }
  using C = RotCfg<L>;
  auto kern = quip_row_kernel<L>;
  if (C::SMEM > 48 * 1024)
    QI8_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)C::SMEM));
  kern<<<(unsigned)rows, C::THREADS, C::SMEM, st>>>(a);
  return check_cuda(cudaGetLastError(), "quip_row_kernel launch");
}

int launch_row(int L, const RowArgs& a, int64_t rows, cudaStream_t st) {
  switch (L) {
#define QI8_CASE(l) case l: return launch_row_L<l>(a, rows, st);
    QI8_CASE(0) QI8_CASE(1) QI8_CASE(2) QI8_CASE(3) QI8_CASE(4) QI8_CASE(5) QI8_CASE(6) QI8_CASE(7)
    QI8_CASE(8) QI8_CASE(9) QI8_CASE(10) QI8_CASE(11) QI8_CASE(12) QI8_CASE(13) QI8_CASE(14)
    QI8_CASE(15)
#undef QI8_CASE
    default: return fail(QI8_ESHAPE, "row length 2^%d out of range", L);
  }
}

// ------------------------------------------------------------- requant
struct ReqArgs {
  const void* w;
  int w_dtype;
  int64_t ld_w, M, N;
  int8_t* q;
  float* scale;
  int block;
  const unsigned int* gmax;
};

__global__ void __launch_bounds__(256) requant_row_kernel(ReqArgs a) {
  __shared__ float red[32];
  const int64_t row = blockIdx.x;
  const int64_t r0 = row * a.ld_w;
  float local = 0.0f;
  for (int64_t c = threadIdx.x; c < a.N; c += blockDim.x) local = fmaxf(local, fabsf(load_as_f32(a.w, a.w_dtype, r0 + c)));
  const float amax = block_max(local, red);
  const float s = fmaxf(__fdiv_rn(amax, 127.0f), 1e-12f);
  for (int64_t c = threadIdx.x; c < a.N; c += blockDim.x)
    a.q[row * a.N + c] = rint_clamp(__fdiv_rn(load_as_f32(a.w, a.w_dtype, r0 + c), s), -127.0f, 127.0f);
  if (threadIdx.x == 0) a.scale[row] = s;
}

__global__ void __launch_bounds__(256) requant_block_kernel(ReqArgs a) {
  const int64_t row = blockIdx.x;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int per = a.block / 32;  // 1, 2 or 4
  const int64_t nb = a.N / a.block;
  const int64_t r0 = row * a.ld_w;
  for (int64_t b = warp; b < nb; b += 8) {
    float v[4];
    float m = 0.0f;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      v[k] = k < per ? load_as_f32(a.w, a.w_dtype, r0 + b * a.block + k * 32 + lane) : 0.0f;
      m = fmaxf(m, fabsf(v[k]));
    }
    m = warp_max(m);
    const float s = fmaxf(__fdiv_rn(m, 127.0f), 1e-12f);
#pragma unroll
    for (int k = 0; k < 4; ++k)
      if (k < per) a.q[row * a.N + b * a.block + k * 32 + lane] = rint_clamp(__fdiv_rn(v[k], s), -127.0f, 127.0f);
    if (lane == 0) a.scale[row * nb + b] = s;
  }
}

__global__ void absmax_rows_kernel(ReqArgs a, unsigned int* __restrict__ out) {
  float m = 0.0f;
  const int64_t total = a.M * a.N;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / a.N, c = i - r * a.N;
    m = fmaxf(m, fabsf(load_as_f32(a.w, a.w_dtype, r * a.ld_w + c)));
  }
  m = warp_max(m);
  if ((threadIdx.x & 31) == 0) atomicMax(out, __float_as_uint(m));
}

__global__ void requant_global_kernel(ReqArgs a) {
  const float s = fmaxf(__fdiv_rn(__uint_as_float(*a.gmax), 127.0f), 1e-12f);
  if (blockIdx.x == 0 && threadIdx.x == 0) a.scale[0] = s;
  const int64_t total = a.M * a.N;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / a.N, c = i - r * a.N;
    a.q[i] = rint_clamp(__fdiv_rn(load_as_f32(a.w, a.w_dtype, r * a.ld_w + c), s), -127.0f, 127.0f);
  }
}

int launch_requant(ReqArgs qa, int requant, cudaStream_t st) {
  if (requant == QI8_REQ_BLOCK && qa.N % qa.block != 0) requant = QI8_REQ_ROW;
  if (requant == QI8_REQ_ROW) {
    requant_row_kernel<<<(unsigned)qa.M, 256, 0, st>>>(qa);
  } else if (requant == QI8_REQ_BLOCK) {
    requant_block_kernel<<<(unsigned)qa.M, 256, 0, st>>>(qa);
  } else {
    unsigned int* gword = const_cast<unsigned int*>(qa.gmax);
    QI8_CUDA(cudaMemsetAsync(gword, 0, 4, st));
    const int sms = sm_count() > 0 ? sm_count() : 148;
    absmax_rows_kernel<<<sms * 4, 256, 0, st>>>(qa, gword);
    requant_global_kernel<<<sms * 4, 256, 0, st>>>(qa);
  }
  return check_cuda(cudaGetLastError(), "requant launch");
}

int64_t next_pow2(int64_t n) {
  int64_t p = 1;
  while (p < n) p <<= 1;
  return p;
}

// Runs the M-direction transform over X in passes of <= COL_MAX_BITS bits.
// forward: the first pass loads W (signs, zero padding); backward: the last
// pass applies the signs and writes the sliced result to dst.  `final`
// selects the normalization of the last pass.
int col_passes(bool forward, const ColArgs& base, cudaStream_t st, int final = FINAL_MUL) {
  const int L = log2_exact(base.M_pad);
  // one pass up to COL_MAX_BITS bits, otherwise two balanced passes
  const int first_bits = L <= COL_MAX_BITS ? L : (L + 1) / 2;
  int b0 = 0;
  while (b0 < L || (L == 0 && b0 == 0)) {
    const int rb = b0 == 0 ? first_bits : (L - b0);
    ColArgs a = base;
    a.b0 = b0;
    a.rbits = rb;
    const bool first = (b0 == 0), last = (b0 + rb == L);
    const size_t smem = sizeof(float) * COL_STRIP * ((size_t)1 << rb);
    dim3 grid((unsigned)((base.N_pad + COL_STRIP - 1) / COL_STRIP), (unsigned)(base.M_pad >> rb));
    void (*kern)(ColArgs) = col_fwht_kernel<false, FINAL_NONE, false>;
    if (forward == true && base.w != nullptr) {
      if (first && last) kern = col_fwht_kernel<true, FINAL_MUL, false>;
      else if (first) kern = col_fwht_kernel<true, FINAL_NONE, false>;
      else if (last) kern = col_fwht_kernel<false, FINAL_MUL, false>;
    } else if (forward) {  // in-place transform of x (no signs)
      if (last) {
        if (final == FINAL_MUL) kern = col_fwht_kernel<false, FINAL_MUL, false>;
        else if (final == FINAL_DIV) kern = col_fwht_kernel<false, FINAL_DIV, false>;
      }
    } else if (last) {
      kern = col_fwht_kernel<false, FINAL_MUL, true>;
    }
    if (smem > 48 * 1024) QI8_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    // enough warps for the radix-16 rounds of a strip: R / 16 groups, at most COL_THREADS / 32 warps
    const int warps = rb >= 7 ? COL_THREADS / 32 : (rb >= 4 ? (1 << (rb - 4)) : 1);
    kern<<<grid, warps * 32, smem, st>>>(a);
    QI8_CUDA(cudaGetLastError());
    if (L == 0) break;
    b0 += rb;
  }
  return QI8_OK;
}

// ------------------------------------------- converter without allocation
// Scratch of qi8_quip_convert_noalloc: one fp32 plane of at most
// NOALLOC_MAX_ELEMS = 2^24 padded elements (a 4096 x 4096 weight) plus the
// 256-byte tail the global requant uses -- 64 MiB + 256 B that every device
// which loads this library keeps until the process exits.
constexpr int64_t NOALLOC_MAX_ELEMS = int64_t(1) << 24;
constexpr int64_t NOALLOC_BYTES = NOALLOC_MAX_ELEMS * 4 + 256;
static __device__ __align__(256) unsigned char g_noalloc_scratch[NOALLOC_BYTES];

// Device address of g_noalloc_scratch, looked up once per device with that
// device current (host code only sees a stand-in for the symbol).  Host
// threads may make their first call on a device concurrently, so the cache
// entries are atomics; every thread that misses stores the same address.
// The cached address is not refreshed after cudaDeviceReset.
std::atomic<void*> g_noalloc_ptr[64];

int noalloc_scratch(void** out) {
  int dev = 0;
  QI8_CUDA(cudaGetDevice(&dev));
  QI8_REQUIRE(dev >= 0 && dev < 64, QI8_EUNSUPPORTED, "device ordinal %d out of range", dev);
  void* p = g_noalloc_ptr[dev].load(std::memory_order_acquire);
  if (!p) {
    QI8_CUDA(cudaGetSymbolAddress(&p, g_noalloc_scratch));
    g_noalloc_ptr[dev].store(p, std::memory_order_release);
  }
  *out = p;
  return QI8_OK;
}

}  // namespace
}  // namespace qi8

using namespace qi8;

extern "C" {

int qi8_fwht_cols(float* x, int64_t rows, int64_t cols, int64_t ld, int final_mode, float factor, void* stream) {
  QI8_REQUIRE(device_ok(), QI8_EUNSUPPORTED, "no sm_100 device current");
  QI8_REQUIRE(x, QI8_EINVAL, "null pointer");
  const int L = log2_exact(rows);
  QI8_REQUIRE(L >= 0 && L <= 15, QI8_ESHAPE, "Second-to-last dimension must be a power of 2 <= 32768, got %lld",
              (long long)rows);
  QI8_REQUIRE(cols > 0 && ld >= cols, QI8_ESHAPE, "bad sizes");
  QI8_REQUIRE(final_mode >= FINAL_NONE && final_mode <= FINAL_DIV, QI8_EINVAL, "final mode %d", final_mode);
  ColArgs ca{};
  ca.w = nullptr; ca.M = rows; ca.N = cols; ca.M_pad = rows; ca.N_pad = cols; ca.x = x; ca.ld_x = ld;
  ca.norm = factor;
  return col_passes(true, ca, static_cast<cudaStream_t>(stream), final_mode);
}

int64_t qi8_quip_workspace_bytes(int64_t M, int64_t N) {
  if (M <= 0 || N <= 0) return 0;
  return next_pow2(M) * next_pow2(N) * 4 + 256;
}

int qi8_quip_convert(const void* w, int w_dtype, int64_t M, int64_t N, const float* s_u, const float* s_v,
                     int store_transformed, int requant, int block, int8_t* q_out, float* scale_out,
                     float* dequant_out, void* workspace, int64_t workspace_bytes, void* stream) {
  QI8_REQUIRE(device_ok(), QI8_EUNSUPPORTED, "no sm_100 device current");
  QI8_REQUIRE(w && s_u && s_v && q_out && scale_out && workspace, QI8_EINVAL, "null pointer");
  QI8_REQUIRE(M > 0 && N > 0, QI8_ESHAPE, "bad sizes M=%lld N=%lld", (long long)M, (long long)N);
  QI8_REQUIRE(w_dtype == QI8_BF16 || w_dtype == QI8_F16 || w_dtype == QI8_F32, QI8_EDTYPE, "weight dtype %d", w_dtype);
  const int64_t M_pad = next_pow2(M), N_pad = next_pow2(N);
  QI8_REQUIRE(M_pad <= 32768 && N_pad <= 32768, QI8_ESHAPE, "padded size %lldx%lld exceeds 32768",
              (long long)M_pad, (long long)N_pad);
  QI8_REQUIRE(workspace_bytes >= qi8_quip_workspace_bytes(M, N), QI8_EINVAL, "workspace too small (%lld < %lld)",
              (long long)workspace_bytes, (long long)qi8_quip_workspace_bytes(M, N));
  QI8_REQUIRE((reinterpret_cast<uintptr_t>(workspace) & 255) == 0, QI8_EALIGN, "workspace must be 256-byte aligned");
  QI8_REQUIRE(requant == QI8_REQ_ROW || requant == QI8_REQ_GLOBAL || requant == QI8_REQ_BLOCK, QI8_EINVAL,
              "requant scheme %d", requant);
  if (requant == QI8_REQ_BLOCK && !store_transformed)
    QI8_REQUIRE(block == 32 || block == 64 || block == 128, QI8_ESHAPE, "block size %d not in {32, 64, 128}", block);
  cudaStream_t st = static_cast<cudaStream_t>(stream);

  float* X = static_cast<float*>(workspace);
  unsigned int* gword = reinterpret_cast<unsigned int*>(static_cast<char*>(workspace) + M_pad * N_pad * 4);

  ColArgs ca{};
  ca.w = w; ca.w_dtype = w_dtype; ca.M = M; ca.N = N; ca.M_pad = M_pad; ca.N_pad = N_pad; ca.x = X;
  ca.ld_x = N_pad;
  ca.s_u = s_u; ca.s_v = s_v;
  ca.norm = (float)(1.0 / std::sqrt((double)M_pad));
  float* wd = dequant_out ? dequant_out : X;
  const int64_t ld_wd = dequant_out ? N : N_pad;
  ca.dst = wd; ca.ld_dst = ld_wd;

  int rc = col_passes(true, ca, st);
  if (rc) return rc;
  RowArgs ra{X, N_pad, (float)(1.0 / std::sqrt((double)N_pad)), store_transformed ? q_out : nullptr,
             store_transformed ? scale_out : nullptr};
  rc = launch_row(log2_exact(N_pad), ra, M_pad, st);
  if (rc) return rc;
  rc = col_passes(false, ca, st);
  if (rc) return rc;
  if (store_transformed) return QI8_OK;

  return launch_requant(ReqArgs{wd, QI8_F32, ld_wd, M, N, q_out, scale_out, block, gword}, requant, st);
}

int qi8_quip_convert_noalloc(const void* w, int w_dtype, int64_t M, int64_t N, const float* s_u, const float* s_v,
                             int store_transformed, int requant, int block, int8_t* q_out, float* scale_out,
                             float* dequant_out, void* stream) {
  QI8_REQUIRE(M > 0 && N > 0, QI8_ESHAPE, "bad sizes M=%lld N=%lld", (long long)M, (long long)N);
  const int64_t padded = next_pow2(M) * next_pow2(N);
  QI8_REQUIRE(padded <= NOALLOC_MAX_ELEMS, QI8_ESHAPE,
              "qi8_quip_convert_noalloc: padded weight %lld x %lld = %lld elements exceeds the built-in scratch of "
              "%lld elements (64 MiB); use qi8_quip_convert with a caller workspace",
              (long long)next_pow2(M), (long long)next_pow2(N), (long long)padded, (long long)NOALLOC_MAX_ELEMS);
  QI8_REQUIRE(device_ok(), QI8_EUNSUPPORTED, "no sm_100 device current");
  void* scratch = nullptr;
  int rc = noalloc_scratch(&scratch);
  if (rc) return rc;
  // Every cell of the fp32 plane the call reads is written earlier in the
  // same call, and the 4-byte global-amax word is zeroed before use, so the
  // previous call's contents never leak into this one.
  return qi8_quip_convert(w, w_dtype, M, N, s_u, s_v, store_transformed, requant, block, q_out, scale_out,
                          dequant_out, scratch, NOALLOC_BYTES, stream);
}

int qi8_weight_rotate2d(const void* w, int w_dtype, int64_t M, int64_t N, int64_t M_pad, int64_t N_pad,
                        const float* s_u, const float* s_v, int inverse, float* out, void* workspace,
                        int64_t workspace_bytes, void* stream) {
  QI8_REQUIRE(device_ok(), QI8_EUNSUPPORTED, "no sm_100 device current");
  QI8_REQUIRE(w && s_u && s_v && out, QI8_EINVAL, "null pointer");
  QI8_REQUIRE(w_dtype == QI8_BF16 || w_dtype == QI8_F16 || w_dtype == QI8_F32, QI8_EDTYPE, "weight dtype %d", w_dtype);
  const int LM = log2_exact(M_pad), LN = log2_exact(N_pad);
  QI8_REQUIRE(LM >= 0 && LM <= 15 && LN >= 1 && LN <= 15, QI8_ESHAPE,
              "padded sizes must be powers of two (rows <= 32768, 2 <= cols <= 32768), got %lld x %lld",
              (long long)M_pad, (long long)N_pad);
  QI8_REQUIRE(M > 0 && N > 0 && M <= M_pad && N <= N_pad, QI8_ESHAPE, "bad sizes M=%lld N=%lld (padded %lld x %lld)",
              (long long)M, (long long)N, (long long)M_pad, (long long)N_pad);
  QI8_REQUIRE(aligned16(out), QI8_EALIGN, "out must be 16-byte aligned");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  ColArgs ca{};
  ca.w_dtype = w_dtype; ca.M = M; ca.N = N; ca.M_pad = M_pad; ca.N_pad = N_pad;
  ca.s_u = s_u; ca.s_v = s_v;
  ca.norm = (float)(1.0 / std::sqrt((double)M_pad));
  if (!inverse) {
    // out [M_pad, N_pad] = FHT_N(FHT_M(pad(W) * s_u * s_v^T)): the column
    // passes load W with the signs, then one in-place FWHT per row
    ca.w = w; ca.x = out; ca.ld_x = N_pad;
    int rc = col_passes(true, ca, st);
    if (rc) return rc;
    return qi8_fwht_rows(out, QI8_F32, M_pad, N_pad, N_pad, N_pad, nullptr, nullptr, 1, out, stream);
  }
  // out [M, N] = slice(FHT_M(FHT_N(W')) * s_u * s_v^T) for W' [M_pad, N_pad]:
  // row FWHTs into the workspace, then the column passes apply the signs and slice
  QI8_REQUIRE(workspace && workspace_bytes >= M_pad * N_pad * 4, QI8_EINVAL,
              "inverse rotation needs an fp32 workspace of M_pad * N_pad elements");
  QI8_REQUIRE(aligned16(workspace), QI8_EALIGN, "workspace must be 16-byte aligned");
  float* X = static_cast<float*>(workspace);
  int rc = qi8_fwht_rows(w, w_dtype, M_pad, N_pad, N_pad, N_pad, nullptr, nullptr, 1, X, stream);
  if (rc) return rc;
  ca.w = nullptr; ca.x = X; ca.ld_x = N_pad; ca.dst = out; ca.ld_dst = N;
  return col_passes(false, ca, st);
}

int qi8_requant_weight(const void* w, int w_dtype, int64_t M, int64_t N, int64_t ld_w, int requant, int block,
                       int8_t* q_out, float* scale_out, void* workspace, int64_t workspace_bytes, void* stream) {
  QI8_REQUIRE(device_ok(), QI8_EUNSUPPORTED, "no sm_100 device current");
  QI8_REQUIRE(w && q_out && scale_out, QI8_EINVAL, "null pointer");
  QI8_REQUIRE(M > 0 && N > 0 && ld_w >= N, QI8_ESHAPE, "bad sizes");
  QI8_REQUIRE(w_dtype == QI8_BF16 || w_dtype == QI8_F16 || w_dtype == QI8_F32, QI8_EDTYPE, "weight dtype %d", w_dtype);
  QI8_REQUIRE(requant == QI8_REQ_ROW || requant == QI8_REQ_GLOBAL || requant == QI8_REQ_BLOCK, QI8_EINVAL,
              "requant scheme %d", requant);
  if (requant == QI8_REQ_BLOCK)
    QI8_REQUIRE(block == 32 || block == 64 || block == 128, QI8_ESHAPE, "block size %d not in {32, 64, 128}", block);
  if (requant == QI8_REQ_GLOBAL)
    QI8_REQUIRE(workspace && workspace_bytes >= 4, QI8_EINVAL, "global requant needs a 4-byte workspace");
  return launch_requant(ReqArgs{w, w_dtype, ld_w, M, N, q_out, scale_out, block, static_cast<unsigned int*>(workspace)},
                        requant, static_cast<cudaStream_t>(stream));
}

}  // extern "C"
