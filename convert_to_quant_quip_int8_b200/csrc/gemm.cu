// K2: int8 x int8 GEMM on the sm_100a 5th-generation tensor cores.
//
//   D[M,N] = A[M,K] . B[N,K]^T   (both operands K-major, exactly the
//   checkpoint layout of the reference's weights, so no per-call transpose
//   copy as in comfy/quant_ops.py:471)
//
// One persistent CTA per SM, warp-specialized:
//   warp 8      TMA producer: 128x128 (A) and 256x128 (B) int8 tiles, 128-byte
//               swizzle, 4-stage mbarrier ring (48 KB / stage)
//   warp 9      TMEM allocator + single-thread tcgen05.mma.kind::i8 issuer
//               (M=128, N=256, K=32 per instruction, s32 accumulators)
//   warps 0..7  epilogue: tcgen05.ld from TMEM (warp w reads lane quadrant
//               w%4, column half w/4), scaling, bias, activation, store
// TMEM holds two 128x256 s32 accumulator buffers (all 512 columns), so the
// MMA of the next accumulation unit overlaps the epilogue of the current one.
//
// Accumulation units:
//   * plain epilogue (tensor / row / no scales): one unit per output tile,
//     exact int32 over all of K (mm_8bit / optimized_linear semantics);
//   * block-scaled epilogue (per-128-K-block scales): one unit per K block;
//     the epilogue promotes each block's int32 partial to fp32 and
//     accumulates acc += p * sa * sb in registers (int8_gemm semantics,
//     comfy/int8_kernels.py:468-480).  The int32 -> fp32 conversion uses the
//     exact 1.5*2^23 bias trick (|p| <= 128*128*128 < 2^22) so it costs one
//     integer add and one packed fp32 add instead of a low-throughput I2F.
//
// Every mbarrier wait is bounded (globaltimer); on expiry the waiting role
// sets a bit in the device status word and an abort flag in shared memory,
// all roles leave their loops, in-flight TMA copies and MMAs are waited for
// (again bounded) and TMEM is freed before the CTA exits.
#include <cuda.h>
#include <cstdint>

#include "common.cuh"

namespace qi8 {
namespace {

constexpr int BM = 128, BN = 256, BK = 128;
constexpr int STAGES = 4;
constexpr int A_BYTES = BM * BK;
constexpr int B_BYTES = BN * BK;
constexpr int NUM_EPI_WARPS = 8;
constexpr int PRODUCER_WARP = 8;
constexpr int MMA_WARP = 9;
constexpr int THREADS = 32 * 10;
constexpr uint32_t TMEM_COLS = 512;
constexpr int SCALE_BYTES = NUM_EPI_WARPS * 128 * 4;
constexpr int NUM_BARS = 2 * STAGES + 4 + 1;  // full, empty, tfull[2], tempty[2], drain
constexpr int SMEM_BYTES = 1024 /*align slack*/ + STAGES * (A_BYTES + B_BYTES) + SCALE_BYTES + NUM_BARS * 8 + 16;
constexpr uint64_t WAIT_LIMIT_NS = 2000000000ull;  // 2 s per wait
constexpr uint64_t DRAIN_LIMIT_NS = 200000000ull;  // 0.2 s when cleaning up

// Block-scaled mode keeps every TMEM accumulator pre-loaded with the int32
// bit pattern of 1.5*2^23 and always accumulates onto it: after the K block,
// the bits read back are exactly the fp32 value 1.5*2^23 + partial (partial
// magnitude <= 128*128*128 < 2^22), so one fp32 subtract recovers it.
constexpr uint32_t MAGIC_BITS = 0x4B400000u;
constexpr float MAGIC_F = 12582912.0f;

// instruction descriptor: D s32, A/B signed int8, both K-major, N=256, M=128
constexpr uint32_t IDESC = (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(BN >> 3) << 17) |
                           ((uint32_t)(BM >> 4) << 24);

struct GemmArgs {
  int M, N, K, KB;
  int m_tiles, n_tiles, num_tiles;
  const float* a_scale;
  int a_kind;
  const float* b_scale;
  int b_kind;
  const void* bias;
  int bias_dtype;
  void* out;
  int out_dtype;
  int64_t ld_out;
  int act;
  unsigned int* status;
};

// ------------------------------------------------------------- PTX glue
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ uint32_t mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok;
}
__device__ __forceinline__ uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
// Bounded wait: true when the phase completed; false on expiry or when
// another role of this CTA already gave up.
__device__ __noinline__ bool mbar_wait(uint32_t bar, uint32_t parity, volatile int* abort_flag,
                                       unsigned int* status, unsigned int bit, uint64_t limit) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer();
  while (true) {
#pragma unroll 1
    for (int i = 0; i < 32; ++i)
      if (mbar_try_wait(bar, parity)) return true;
    if (*abort_flag) return false;
    if (globaltimer() - t0 > limit) {
      *abort_flag = 1;
      if (status) atomicOr(status, bit);
      return false;
    }
  }
}

// Bounded wait used while cleaning up after an abort (ignores the flag).
__device__ __noinline__ void drain_wait(uint32_t bar, uint32_t parity) {
  const uint64_t t0 = globaltimer();
  while (!mbar_try_wait(bar, parity))
    if (globaltimer() - t0 > DRAIN_LIMIT_NS) return;
}

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int x, int y, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar)
      : "memory");
}
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void tc_mma_i8(uint32_t d, uint64_t a, uint64_t b, uint32_t accum) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d),
      "l"(a), "l"(b), "r"(IDESC), "r"(accum)
      : "memory");
}
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
// Writes the same 32-bit value v into 16 consecutive columns of this warp's lanes.
__device__ __forceinline__ void tmem_fill16(uint32_t taddr, uint32_t v) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1};" ::"r"(taddr),
      "r"(v)
      : "memory");
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// Shared-memory matrix descriptor: K-major operand, 128-byte swizzle, rows of
// 128 bytes, 8-row core groups 1024 bytes apart (SBO), sm_100 version bit.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
  uint64_t d = (uint64_t)((saddr & 0x3FFFFu) >> 4);
  d |= (uint64_t)1 << 16;             // leading byte offset (unused for swizzled K-major)
  d |= (uint64_t)(1024 >> 4) << 32;   // stride byte offset
  d |= (uint64_t)1 << 46;             // descriptor version
  d |= (uint64_t)2 << 61;             // SWIZZLE_128B
  return d;
}

// ------------------------------------------------------------ epilogue
__device__ __forceinline__ float finish_value(float y, int n, const GemmArgs& p) {
  if (p.bias) y = __fadd_rn(y, load_as_f32(p.bias, p.bias_dtype, n));
  if (p.act == QI8_ACT_GELU) {
    if (p.out_dtype == QI8_BF16) y = __bfloat162float(__float2bfloat16_rn(y));
    else if (p.out_dtype == QI8_F16) y = __half2float(__float2half_rn(y));
    y = gelu_erf(y);
  }
  return y;
}

// Stores 32 consecutive fp32 results of row m starting at column n0.
__device__ __forceinline__ void store_row32(const GemmArgs& p, int m, int n0, const float (&y)[32]) {
  const int64_t off = (int64_t)m * p.ld_out + n0;
  const bool full = (n0 + 32 <= p.N);
  if (p.out_dtype == QI8_BF16) {
    __nv_bfloat16* o = static_cast<__nv_bfloat16*>(p.out) + off;
    if (full) {
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        uint4 u;
        __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&u);
#pragma unroll
        for (int j = 0; j < 4; ++j) h[j] = __floats2bfloat162_rn(y[8 * k + 2 * j], y[8 * k + 2 * j + 1]);
        reinterpret_cast<uint4*>(o)[k] = u;
      }
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (n0 + j < p.N) o[j] = __float2bfloat16_rn(y[j]);
    }
  } else if (p.out_dtype == QI8_F16) {
    __half* o = static_cast<__half*>(p.out) + off;
    if (full) {
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        uint4 u;
        __half2* h = reinterpret_cast<__half2*>(&u);
#pragma unroll
        for (int j = 0; j < 4; ++j) h[j] = __floats2half2_rn(y[8 * k + 2 * j], y[8 * k + 2 * j + 1]);
        reinterpret_cast<uint4*>(o)[k] = u;
      }
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (n0 + j < p.N) o[j] = __float2half_rn(y[j]);
    }
  } else {
    float* o = static_cast<float*>(p.out) + off;
    if (full) {
#pragma unroll
      for (int k = 0; k < 8; ++k)
        reinterpret_cast<float4*>(o)[k] = make_float4(y[4 * k], y[4 * k + 1], y[4 * k + 2], y[4 * k + 3]);
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (n0 + j < p.N) o[j] = y[j];
    }
  }
}

// Stores 8 consecutive fp32 results of row m starting at column n0 (n0 % 8 == 0).
__device__ __forceinline__ void store_row8(const GemmArgs& p, int m, int n0, const float (&y)[8]) {
  const int64_t off = (int64_t)m * p.ld_out + n0;
  const bool full = (n0 + 8 <= p.N);
  if (p.out_dtype == QI8_BF16) {
    __nv_bfloat16* o = static_cast<__nv_bfloat16*>(p.out) + off;
    if (full) {
      uint4 u;
      __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&u);
#pragma unroll
      for (int j = 0; j < 4; ++j) h[j] = __floats2bfloat162_rn(y[2 * j], y[2 * j + 1]);
      *reinterpret_cast<uint4*>(o) = u;
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j)
        if (n0 + j < p.N) o[j] = __float2bfloat16_rn(y[j]);
    }
  } else if (p.out_dtype == QI8_F16) {
    __half* o = static_cast<__half*>(p.out) + off;
    if (full) {
      uint4 u;
      __half2* h = reinterpret_cast<__half2*>(&u);
#pragma unroll
      for (int j = 0; j < 4; ++j) h[j] = __floats2half2_rn(y[2 * j], y[2 * j + 1]);
      *reinterpret_cast<uint4*>(o) = u;
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j)
        if (n0 + j < p.N) o[j] = __float2half_rn(y[j]);
    }
  } else {
    float* o = static_cast<float*>(p.out) + off;
    if (full) {
      reinterpret_cast<float4*>(o)[0] = make_float4(y[0], y[1], y[2], y[3]);
      reinterpret_cast<float4*>(o)[1] = make_float4(y[4], y[5], y[6], y[7]);
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j)
        if (n0 + j < p.N) o[j] = y[j];
    }
  }
}

__device__ __forceinline__ void store_row32_i32(const GemmArgs& p, int m, int n0, const uint32_t (&r)[32]) {
  int32_t* o = static_cast<int32_t*>(p.out) + (int64_t)m * p.ld_out + n0;
  if (n0 + 32 <= p.N) {
#pragma unroll
    for (int k = 0; k < 8; ++k) reinterpret_cast<uint4*>(o)[k] = make_uint4(r[4 * k], r[4 * k + 1], r[4 * k + 2], r[4 * k + 3]);
  } else {
#pragma unroll
    for (int j = 0; j < 32; ++j)
      if (n0 + j < p.N) o[j] = (int32_t)r[j];
  }
}

__device__ __forceinline__ float row_scale(const float* s, int kind, int m) {
  if (kind == QI8_S_ROW) return __ldg(s + m);
  if (kind == QI8_S_SCALAR) return __ldg(s);
  return 1.0f;
}

template <bool PROMOTE>
__global__ void __launch_bounds__(THREADS, 1)
    gemm_i8_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const GemmArgs p) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* sb = smem_raw + (base - raw);
  const uint32_t sA = base;
  const uint32_t sB = base + STAGES * A_BYTES;
  float* sscale = reinterpret_cast<float*>(sb + STAGES * (A_BYTES + B_BYTES));
  uint64_t* bars = reinterpret_cast<uint64_t*>(sb + STAGES * (A_BYTES + B_BYTES) + SCALE_BYTES);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + NUM_BARS);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  auto full_bar = [&](int s) { return smem_u32(bars + s); };
  auto empty_bar = [&](int s) { return smem_u32(bars + STAGES + s); };
  auto tfull_bar = [&](int b) { return smem_u32(bars + 2 * STAGES + b); };
  auto tempty_bar = [&](int b) { return smem_u32(bars + 2 * STAGES + 2 + b); };
  const uint32_t drain_bar = smem_u32(bars + 2 * STAGES + 4);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(tfull_bar(b), 1);
      mbar_init(tempty_bar(b), NUM_EPI_WARPS);
    }
    mbar_init(drain_bar, 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == MMA_WARP) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  if (warp == PRODUCER_WARP && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const int KB = p.KB;
  if constexpr (PROMOTE) {
    if (warp < NUM_EPI_WARPS) {
      // pre-bias both accumulator buffers (this warp's lanes and columns)
      const uint32_t lb = (uint32_t)((warp & 3) * 32) << 16;
#pragma unroll
      for (int b = 0; b < 2; ++b)
#pragma unroll
        for (int c = 0; c < 8; ++c) tmem_fill16(tmem_base + lb + (uint32_t)(b * BN + (warp >> 2) * 128 + c * 16), MAGIC_BITS);
      tmem_wait_st();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
  }

  if (warp == PRODUCER_WARP) {
    if (lane == 0) {
      int s = 0;
      uint32_t ph = 0;
      uint32_t issued = 0, issued_ph = 0;  // per-stage: load in flight, and its phase
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < p.num_tiles; tile += gridDim.x) {
        const int m0 = (tile % p.m_tiles) * BM;
        const int n0 = (tile / p.m_tiles) * BN;
        for (int kb = 0; kb < KB; ++kb) {
          if (!mbar_wait(empty_bar(s), ph ^ 1u, abort_flag, p.status, ST_GEMM_PRODUCER, WAIT_LIMIT_NS)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(full_bar(s), A_BYTES + B_BYTES);
          tma_load_2d(sA + s * A_BYTES, &tmA, kb * BK, m0, full_bar(s));
          tma_load_2d(sB + s * B_BYTES, &tmB, kb * BK, n0, full_bar(s));
          issued |= 1u << s;
          issued_ph = (issued_ph & ~(1u << s)) | (ph << s);
          if (++s == STAGES) {
            s = 0;
            ph ^= 1u;
          }
        }
      }
      if (!ok) {
        // let copies already in flight land before the CTA exits
        for (int t = 0; t < STAGES; ++t)
          if (issued & (1u << t)) drain_wait(full_bar(t), (issued_ph >> t) & 1u);
      }
    }
  } else if (warp == MMA_WARP) {
    if (lane == 0) {
      int s = 0;
      uint32_t ph = 0;
      int au = 0;
      bool ok = true;
      const int n_units = PROMOTE ? KB : 1;
      for (int tile = blockIdx.x; ok && tile < p.num_tiles; tile += gridDim.x) {
        for (int u = 0; ok && u < n_units; ++u, ++au) {
          const int buf = au & 1;
          if (!mbar_wait(tempty_bar(buf), ((au >> 1) & 1) ^ 1u, abort_flag, p.status, ST_GEMM_MMA, WAIT_LIMIT_NS)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t d = tmem_base + (uint32_t)(buf * BN);
          const int kb0 = PROMOTE ? u : 0, kb1 = PROMOTE ? u + 1 : KB;
          for (int kb = kb0; kb < kb1; ++kb) {
            if (!mbar_wait(full_bar(s), ph, abort_flag, p.status, ST_GEMM_MMA, WAIT_LIMIT_NS)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint64_t da = sw128_desc(sA + s * A_BYTES);
            const uint64_t db = sw128_desc(sB + s * B_BYTES);
#pragma unroll
            for (int k = 0; k < BK / 32; ++k)
              tc_mma_i8(d, da + (uint64_t)(2 * k), db + (uint64_t)(2 * k),
                        (PROMOTE || kb > kb0 || k > 0) ? 1u : 0u);
            tc_commit(empty_bar(s));
            if (++s == STAGES) {
              s = 0;
              ph ^= 1u;
            }
          }
          if (ok) tc_commit(tfull_bar(buf));
        }
      }
      // all MMAs issued by this thread complete before TMEM is released
      tc_commit(drain_bar);
      if (ok) mbar_wait(drain_bar, 0, abort_flag, p.status, ST_GEMM_DRAIN, WAIT_LIMIT_NS);
      else drain_wait(drain_bar, 0);
    }
  } else {
    // ------------------------------------------------------- epilogue
    const int quad = warp & 3, half = warp >> 2;
    const uint32_t lane_base = (uint32_t)(quad * 32) << 16;
    float* my_sc = sscale + warp * 128;
    int au = 0;
    bool ok = true;
    for (int tile = blockIdx.x; ok && tile < p.num_tiles; tile += gridDim.x) {
      const int m = (tile % p.m_tiles) * BM + quad * 32 + lane;
      const int ncol0 = (tile / p.m_tiles) * BN + half * 128;
      const bool row_ok = m < p.M;
      const bool cols_ok = ncol0 < p.N;
      if constexpr (PROMOTE) {
        float2 acc[64];
#pragma unroll
        for (int i = 0; i < 64; ++i) acc[i] = make_float2(0.0f, 0.0f);
        const bool a_kb = p.a_kind == QI8_S_ROW_KBLOCK;
        const bool b_col = p.b_kind == QI8_S_ROW_KBLOCK;
        const bool b_tile = p.b_kind == QI8_S_TILE128;
        for (int kb = 0; kb < KB; ++kb, ++au) {
          const int buf = au & 1;
          float sa = 1.0f;
          if (a_kb) sa = row_ok ? __ldg(p.a_scale + (int64_t)m * KB + kb) : 0.0f;
          float sconst = sa;
          if (b_tile) sconst = __fmul_rn(sa, cols_ok ? __ldg(p.b_scale + (int64_t)(ncol0 >> 7) * KB + kb) : 0.0f);
          if (b_col) {
            __syncwarp();
#pragma unroll
            for (int c = 0; c < 4; ++c) {
              const int n = ncol0 + c * 32 + lane;
              my_sc[c * 32 + lane] = n < p.N ? __ldg(p.b_scale + (int64_t)n * KB + kb) : 0.0f;
            }
            __syncwarp();
          }
          if (!mbar_wait(tfull_bar(buf), (au >> 1) & 1, abort_flag, p.status, ST_GEMM_EPILOGUE, WAIT_LIMIT_NS)) {
            ok = false;
            break;
          }
          tc_fence_after();
#pragma unroll
          for (int c = 0; c < 8; ++c) {
            uint32_t r[16];
            const uint32_t ta = tmem_base + lane_base + (uint32_t)(buf * BN + half * 128 + c * 16);
            tmem_ld16(ta, r);
            tmem_wait_ld();
            tmem_fill16(ta, MAGIC_BITS);  // re-bias for this buffer's next K block
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              float2 f = make_float2(__uint_as_float(r[2 * j]), __uint_as_float(r[2 * j + 1]));
              f = __fadd2_rn(f, make_float2(-MAGIC_F, -MAGIC_F));
              float2 sc;
              if (b_col) {
                sc = *reinterpret_cast<const float2*>(my_sc + c * 16 + 2 * j);
                if (a_kb) sc = __fmul2_rn(sc, make_float2(sa, sa));
              } else {
                sc = make_float2(sconst, sconst);
              }
              acc[c * 8 + j] = __ffma2_rn(f, sc, acc[c * 8 + j]);
            }
          }
          tmem_wait_st();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(tempty_bar(buf));
        }
        if (!ok) break;
        if (row_ok && cols_ok) {
          const float fa = row_scale(p.a_scale, p.a_kind, m);
#pragma unroll
          for (int g = 0; g < 16; ++g) {
            const int n0 = ncol0 + g * 8;
            if (n0 < p.N) {
              float y[8];
#pragma unroll
              for (int j = 0; j < 8; ++j) {
                const int n = n0 + j < p.N ? n0 + j : p.N - 1;
                const float v = (j & 1) ? acc[g * 4 + (j >> 1)].y : acc[g * 4 + (j >> 1)].x;
                y[j] = finish_value(__fmul_rn(__fmul_rn(v, fa), row_scale(p.b_scale, p.b_kind, n)), n, p);
              }
              store_row8(p, m, n0, y);
            }
          }
        }
      } else {
        const int buf = au & 1;
        if (!mbar_wait(tfull_bar(buf), (au >> 1) & 1, abort_flag, p.status, ST_GEMM_EPILOGUE, WAIT_LIMIT_NS)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const float xs = row_ok ? row_scale(p.a_scale, p.a_kind, m) : 0.0f;
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          uint32_t r[32];
          tmem_ld32(tmem_base + lane_base + (uint32_t)(buf * BN + half * 128 + c * 32), r);
          tmem_wait_ld();
          if (c == 3) {
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(tempty_bar(buf));
          }
          const int n0 = ncol0 + c * 32;
          if (!row_ok || n0 >= p.N) continue;
          if (p.out_dtype == QI8_I32) {
            store_row32_i32(p, m, n0, r);
          } else {
            float y[32];
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              const int n = n0 + j < p.N ? n0 + j : p.N - 1;
              // optimized_linear: res.float() * (x_s * w_s) + bias  (comfy/quant_ops.py:472-473)
              const float s = __fmul_rn(xs, row_scale(p.b_scale, p.b_kind, n));
              y[j] = finish_value(__fmul_rn(__int2float_rn((int)r[j]), s), n, p);
            }
            store_row32(p, m, n0, y);
          }
        }
        ++au;
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == MMA_WARP) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(TMEM_COLS) : "memory");
  }
}

// --------------------------------------------------------------- host side
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(ptr);
  }
  return fn;
}

// K-major int8 matrix [rows, K] -> tensor map with a (128 x box_rows) box.
int make_map(CUtensorMap* map, const int8_t* ptr, int64_t rows, int64_t K, uint32_t box_rows) {
  EncodeTiledFn fn = encode_fn();
  QI8_REQUIRE(fn, QI8_ECUDA, "cuTensorMapEncodeTiled unavailable");
  cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)K};
  cuuint32_t box[2] = {(cuuint32_t)BK, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<int8_t*>(ptr), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  QI8_REQUIRE(r == CUDA_SUCCESS, QI8_ECUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return QI8_OK;
}

bool g_attr_set[2][64];

}  // namespace
}  // namespace qi8

using namespace qi8;

extern "C" int qi8_gemm_i8(const int8_t* A, const int8_t* B, int64_t M, int64_t N, int64_t K, const float* a_scale,
                           int a_kind, const float* b_scale, int b_kind, const void* bias, int bias_dtype, void* out,
                           int out_dtype, int64_t ld_out, int act, void* stream) {
  QI8_REQUIRE(device_ok(), QI8_EUNSUPPORTED, "no sm_100 device current");
  QI8_REQUIRE(A && B && out, QI8_EINVAL, "null pointer");
  QI8_REQUIRE(M >= 0 && N > 0 && K > 0 && M < (1ll << 31) && N < (1ll << 31) && K < (1ll << 31), QI8_ESHAPE,
              "bad sizes M=%lld N=%lld K=%lld", (long long)M, (long long)N, (long long)K);
  QI8_REQUIRE(K % 16 == 0, QI8_ESHAPE, "K=%lld must be a multiple of 16", (long long)K);
  QI8_REQUIRE(N % 16 == 0, QI8_ESHAPE, "N=%lld must be a multiple of 16", (long long)N);
  QI8_REQUIRE(ld_out >= N, QI8_ESHAPE, "ld_out < N");
  QI8_REQUIRE(aligned16(A) && aligned16(B) && aligned16(out), QI8_EALIGN, "A, B and out must be 16-byte aligned");
  QI8_REQUIRE(a_kind >= QI8_S_NONE && a_kind <= QI8_S_ROW_KBLOCK, QI8_EINVAL, "a_kind %d", a_kind);
  QI8_REQUIRE(b_kind >= QI8_S_NONE && b_kind <= QI8_S_TILE128, QI8_EINVAL, "b_kind %d", b_kind);
  QI8_REQUIRE((a_kind == QI8_S_NONE) == (a_scale == nullptr), QI8_EINVAL, "a_scale/a_kind mismatch");
  QI8_REQUIRE((b_kind == QI8_S_NONE) == (b_scale == nullptr), QI8_EINVAL, "b_scale/b_kind mismatch");
  QI8_REQUIRE(out_dtype == QI8_BF16 || out_dtype == QI8_F16 || out_dtype == QI8_F32 || out_dtype == QI8_I32,
              QI8_EDTYPE, "out dtype %d", out_dtype);
  QI8_REQUIRE(!bias || bias_dtype == QI8_BF16 || bias_dtype == QI8_F16 || bias_dtype == QI8_F32, QI8_EDTYPE,
              "bias dtype %d", bias_dtype);
  const int es = elem_size(out_dtype);
  QI8_REQUIRE((ld_out * es) % 16 == 0, QI8_EALIGN, "ld_out * elem_size must be a multiple of 16");
  const bool promote = a_kind == QI8_S_ROW_KBLOCK || b_kind == QI8_S_ROW_KBLOCK || b_kind == QI8_S_TILE128;
  if (promote) QI8_REQUIRE(K % 128 == 0, QI8_ESHAPE, "block scales need K %% 128 == 0 (K=%lld)", (long long)K);
  if (out_dtype == QI8_I32)
    QI8_REQUIRE(!promote && a_kind == QI8_S_NONE && b_kind == QI8_S_NONE && !bias && act == QI8_ACT_NONE,
                QI8_EINVAL, "int32 output takes no scales, bias or activation");
  QI8_REQUIRE(act == QI8_ACT_NONE || act == QI8_ACT_GELU, QI8_EINVAL, "act %d", act);
  if (M == 0) return QI8_OK;

  CUtensorMap mapA, mapB;
  int rc = make_map(&mapA, A, M, K, BM);
  if (rc) return rc;
  rc = make_map(&mapB, B, N, K, BN);
  if (rc) return rc;

  GemmArgs p{};
  p.M = (int)M; p.N = (int)N; p.K = (int)K; p.KB = (int)((K + BK - 1) / BK);
  p.m_tiles = (int)((M + BM - 1) / BM);
  p.n_tiles = (int)((N + BN - 1) / BN);
  p.num_tiles = p.m_tiles * p.n_tiles;
  p.a_scale = a_scale; p.a_kind = a_kind; p.b_scale = b_scale; p.b_kind = b_kind;
  p.bias = bias; p.bias_dtype = bias_dtype; p.out = out; p.out_dtype = out_dtype; p.ld_out = ld_out;
  p.act = act;
  p.status = device_status_ptr();

  int dev = 0;
  QI8_CUDA(cudaGetDevice(&dev));
  auto kern = promote ? gemm_i8_kernel<true> : gemm_i8_kernel<false>;
  if (dev < 64 && !g_attr_set[promote][dev]) {
    QI8_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES));
    g_attr_set[promote][dev] = true;
  }
  const int sms = sm_count() > 0 ? sm_count() : 148;
  const int grid = p.num_tiles < sms ? p.num_tiles : sms;
  kern<<<grid, THREADS, SMEM_BYTES, static_cast<cudaStream_t>(stream)>>>(mapA, mapB, p);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    cudaFuncAttributes fa{};
    cudaFuncGetAttributes(&fa, kern);
    return fail(QI8_ECUDA, "gemm_i8_kernel launch: %s (regs=%d maxThreads=%d local=%zu smem=%d grid=%d)",
                cudaGetErrorString(e), fa.numRegs, fa.maxThreadsPerBlock, fa.localSizeBytes, SMEM_BYTES, grid);
  }
  return QI8_OK;
}
