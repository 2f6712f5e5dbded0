// K2: int8 x int8 GEMM on the sm_100a 5th-generation tensor cores.
//
//   D[M,N] = A[M,K] . B[N,K]^T   (both operands K-major, exactly the
//   checkpoint layout of the reference's weights, so no per-call transpose
//   copy as in comfy/quant_ops.py:471)
//
// Two persistent, warp-specialized kernels share the roles:
//   warp 8      TMA producer (128-byte swizzle, mbarrier stage ring)
//   warp 9      TMEM allocator + single-thread tcgen05.mma.kind::i8 issuer
//   warps 0..7  epilogue: tcgen05.ld from TMEM (warp w reads lane quadrant
//               w%4, column half w/4), scaling, bias, activation, store
//   warps 10,11 only donate registers to the epilogue (block-scaled kernels)
//
// * gemm_pair_kernel (used whenever the TMEM-lane operand has more than 128
//   rows): CTA pairs of a 2-CTA cluster issue tcgen05.mma.cta_group::2 with
//   M=256, N=256, K=32; each CTA loads 128 rows of A and 128 rows of B per
//   K block (32 KB, 6-stage ring) and holds its 128 output rows in two
//   256-column TMEM buffers.  Per SM this loads a third less operand data
//   from L2 than a single-CTA 128x256 tile for the same MMA work.
// * gemm_i8_kernel: one CTA per 128x256 tile (M=128, N=256), for operands
//   of at most 128 TMEM-lane rows.
//
// Accumulation units:
//   * plain epilogue (tensor / row / no scales): one unit per output tile,
//     exact int32 over all of K (mm_8bit / optimized_linear semantics);
//   * block-scaled epilogue (per-128-K-block scales): one unit per K block;
//     the epilogue promotes each block's int32 partial to fp32 and
//     accumulates acc += p * sa * sb in registers (int8_gemm semantics,
//     comfy/int8_kernels.py:468-480): one I2F and half a packed FFMA per
//     partial (the sm_100 I2F is cheaper than the exact 1.5*2^23 integer-add
//     trick, which costs an INT add plus half a packed FADD, by 15-18 % in
//     the whole kernel); TMEM loads of the next 32 columns are in flight
//     during the math.
//
// Every mbarrier wait is bounded (globaltimer); on expiry the waiting role
// sets a bit in the device status word and an abort flag in shared memory,
// all roles leave their loops, in-flight TMA copies and MMAs are waited for
// (again bounded) and TMEM is freed before the CTA exits (the CTA pair meets
// at a cluster barrier first).
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
constexpr int THREADS = 32 * 12;  // three warpgroups; warps 10 and 11 only donate registers
// Register split of the block-scaled kernel: launched at 168 registers per
// thread (384 x 168 = 64512 <= 65536; three warps per SM sub-partition), the
// control warpgroup drops to 56 and the two epilogue warpgroups rise to 224:
// 256 x 224 + 128 x 56 == 384 x 168.  The host refuses to launch if the
// compiled kernel does not use exactly LAUNCH_REGS registers.
constexpr int LAUNCH_REGS = 168;
constexpr int EPI_REGS = 240;
constexpr int CTRL_REGS = 24;
static_assert(256 * EPI_REGS + 128 * CTRL_REGS == THREADS * LAUNCH_REGS, "register split must balance");
constexpr uint32_t TMEM_COLS = 512;
// column scales, bias, per-kb scales (fp32 x 128 per warp each) + two 32x16 bf16 transpose tiles per warp
constexpr int STAGE_SCRATCH_BYTES = 3 * NUM_EPI_WARPS * 128 * 4 + NUM_EPI_WARPS * 2 * 16 * 32 * 2;
constexpr int NUM_BARS = 2 * STAGES + 8 + 1;  // full, empty, tfull[2][2], tempty[2][2], drain
constexpr int SMEM_BYTES = 1024 /*align slack*/ + STAGES * (A_BYTES + B_BYTES) + STAGE_SCRATCH_BYTES + NUM_BARS * 8 + 16;
static_assert(SMEM_BYTES <= 232448, "shared memory");
constexpr uint64_t WAIT_LIMIT_NS = 2000000000ull;  // 2 s per wait
constexpr uint64_t DRAIN_LIMIT_NS = 200000000ull;  // 0.2 s when cleaning up


// instruction descriptor: D s32, A/B signed int8, both K-major, N=256, M=128
constexpr uint32_t IDESC = (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(BN >> 3) << 17) |
                           ((uint32_t)(BM >> 4) << 24);
// same with N = 128: the block-scaled kernel issues each K block as two column halves
constexpr uint32_t IDESC_N128 = (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(128 >> 3) << 17) |
                                ((uint32_t)(BM >> 4) << 24);

struct GemmArgs {
  int M, N, K, KB;
  int r_tiles, c_tiles, num_tiles;  // tiles over the TMEM-lane operand (128 rows) and the column operand (256 rows)
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

// Launch extensions, a separate kernel parameter so that the common
// single-output kernels keep GemmArgs unchanged.
struct GemmExt {
  // split-K (plain path of the pair kernel): tile t covers K blocks
  // [s * kb_split, (s + 1) * kb_split) of split s = t / (r_tiles * c_tiles) and
  // stores its raw int32 sums to plane s (split_stride elements apart)
  int kb_split;
  int64_t split_stride;
  // pair-tile width in output columns: 256, or 128 for a plain-scale,
  // single-output, unsplit GEMM whose 256-wide tiles would fill at most a
  // quarter of the co-resident CTA pairs (twice the tiles, each half the work)
  int pbn;
  // Output destinations, each [M, ld_out] from its own base: outs[0] == out
  // on this device; outs[1..n_outs) peer-mapped copies (column-parallel
  // gather), which receive the same tile at the same offset.
  int n_outs;
  void* outs[QI8_MAX_PEERS];
  // int8 output (out_dtype QI8_I8, non-swapped block-scaled kernels only):
  // every (row, 128-column block) of the fp32 result is requantized with
  // scale = max(amax / 127, 1e-8), q = trunc(clamp(y / scale, +-127)); the
  // scales go to q_scale [M, N / 128].  The K-block promotion then follows
  // the reference's order, acc + (fp32(p) * a_s) * b_s, in separately
  // rounded operations.
  float* q_scale;
  int exact;
};

// Calls f(base) for every output destination (static indices, so the
// parameter struct stays in the constant bank).
template <typename F>
__device__ __forceinline__ void for_each_out(const GemmExt& e, F&& f) {
#pragma unroll
  for (int d = 0; d < QI8_MAX_PEERS; ++d) {
    if (d >= e.n_outs) break;
    f(e.outs[d]);
  }
}

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
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, volatile int* abort_flag,
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
__device__ __forceinline__ void tc_mma_i8(uint32_t d, uint64_t a, uint64_t b, uint32_t accum,
                                          uint32_t idesc = IDESC) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d),
      "l"(a), "l"(b), "r"(idesc), "r"(accum)
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
// Shared-memory float2 load that stays in program order with the tcgen05
// asm statements around it (keeps scale registers from being hoisted).
__device__ __forceinline__ float2 lds_f2(const float* p) {
  float2 v;
  asm volatile("ld.shared.v2.f32 {%0, %1}, [%2];" : "=f"(v.x), "=f"(v.y) : "r"(smem_u32(p)));
  return v;
}

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
// GELU of the linear output as the reference computes it on a bf16/fp16
// tensor: the value is first rounded to the output dtype.
__device__ __forceinline__ float act_gelu(float y, int out_dtype) {
  if (out_dtype == QI8_BF16) y = __bfloat162float(__float2bfloat16_rn(y));
  else if (out_dtype == QI8_F16) y = __half2float(__float2half_rn(y));
  return gelu_erf(y);
}

// Multi-destination forms: every outs[d] receives the values.
__device__ __forceinline__ void store_row32_multi(const GemmArgs& p, const GemmExt& e, int m, int n0,
                                                  const float (&y)[32]) {
  const int64_t off = (int64_t)m * p.ld_out + n0;
  const bool full = (n0 + 32 <= p.N);
  if (p.out_dtype == QI8_BF16 || p.out_dtype == QI8_F16) {
    const bool bf = p.out_dtype == QI8_BF16;
    if (full) {
      uint4 u[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        uint32_t* w = reinterpret_cast<uint32_t*>(&u[k]);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float a = y[8 * k + 2 * j], b = y[8 * k + 2 * j + 1];
          if (bf) {
            __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
            w[j] = *reinterpret_cast<uint32_t*>(&h);
          } else {
            __half2 h = __floats2half2_rn(a, b);
            w[j] = *reinterpret_cast<uint32_t*>(&h);
          }
        }
      }
      for_each_out(e, [&](void* base) {
        uint4* o = reinterpret_cast<uint4*>(static_cast<uint16_t*>(base) + off);
#pragma unroll
        for (int k = 0; k < 4; ++k) o[k] = u[k];
      });
    } else {
      for_each_out(e, [&](void* base) {
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          if (n0 + j >= p.N) continue;
          if (bf) static_cast<__nv_bfloat16*>(base)[off + j] = __float2bfloat16_rn(y[j]);
          else static_cast<__half*>(base)[off + j] = __float2half_rn(y[j]);
        }
      });
    }
  } else {
    for_each_out(e, [&](void* base) {
      float* o = static_cast<float*>(base) + off;
      if (full) {
#pragma unroll
        for (int k = 0; k < 8; ++k)
          reinterpret_cast<float4*>(o)[k] = make_float4(y[4 * k], y[4 * k + 1], y[4 * k + 2], y[4 * k + 3]);
      } else {
#pragma unroll
        for (int j = 0; j < 32; ++j)
          if (n0 + j < p.N) o[j] = y[j];
      }
    });
  }
}

__device__ __forceinline__ void store_row8_multi(const GemmArgs& p, const GemmExt& e, int m, int n0,
                                                 const float (&y)[8]) {
  const int64_t off = (int64_t)m * p.ld_out + n0;
  const bool full = (n0 + 8 <= p.N);
  if (p.out_dtype == QI8_BF16 || p.out_dtype == QI8_F16) {
    const bool bf = p.out_dtype == QI8_BF16;
    if (full) {
      uint4 u;
      uint32_t* w = reinterpret_cast<uint32_t*>(&u);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        if (bf) {
          __nv_bfloat162 h = __floats2bfloat162_rn(y[2 * j], y[2 * j + 1]);
          w[j] = *reinterpret_cast<uint32_t*>(&h);
        } else {
          __half2 h = __floats2half2_rn(y[2 * j], y[2 * j + 1]);
          w[j] = *reinterpret_cast<uint32_t*>(&h);
        }
      }
      for_each_out(e, [&](void* base) { *reinterpret_cast<uint4*>(static_cast<uint16_t*>(base) + off) = u; });
    } else {
      for_each_out(e, [&](void* base) {
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          if (n0 + j >= p.N) continue;
          if (bf) static_cast<__nv_bfloat16*>(base)[off + j] = __float2bfloat16_rn(y[j]);
          else static_cast<__half*>(base)[off + j] = __float2half_rn(y[j]);
        }
      });
    }
  } else {
    for_each_out(e, [&](void* base) {
      float* o = static_cast<float*>(base) + off;
      if (full) {
        reinterpret_cast<float4*>(o)[0] = make_float4(y[0], y[1], y[2], y[3]);
        reinterpret_cast<float4*>(o)[1] = make_float4(y[4], y[5], y[6], y[7]);
      } else {
#pragma unroll
        for (int j = 0; j < 8; ++j)
          if (n0 + j < p.N) o[j] = y[j];
      }
    });
  }
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

// Multi-destination store of a warp's 32 rows x 32 columns (16-bit output):
// each lane packs its row into the warp's 2 KB tile (16-byte chunks XOR-
// swizzled, conflict-free), then lanes 4r..4r+3 write row r's 64 contiguous
// bytes to every destination -- wide row segments instead of one 16-byte
// piece per row, which is what NVLink stores need.  Warp-collective.
__device__ __forceinline__ void store_tile32_multi(const GemmArgs& p, const GemmExt& e, uint4* tile, int row0, int R,
                                                   int n0, const float (&y)[32], int lane) {
  const bool bf = p.out_dtype == QI8_BF16;
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    uint4 u;
    uint32_t* w = reinterpret_cast<uint32_t*>(&u);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float a = y[8 * k + 2 * j], b = y[8 * k + 2 * j + 1];
      if (bf) {
        __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
        w[j] = *reinterpret_cast<uint32_t*>(&h);
      } else {
        __half2 h = __floats2half2_rn(a, b);
        w[j] = *reinterpret_cast<uint32_t*>(&h);
      }
    }
    tile[lane * 4 + (k ^ ((lane >> 1) & 3))] = u;
  }
  __syncwarp();
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int r = 8 * i + (lane >> 2), k = lane & 3;
    const uint4 v = tile[r * 4 + (k ^ ((r >> 1) & 3))];
    if (row0 + r < R) {
      const int64_t off = (int64_t)(row0 + r) * p.ld_out + n0 + k * 8;
      for_each_out(e, [&](void* base) { *reinterpret_cast<uint4*>(static_cast<uint16_t*>(base) + off) = v; });
    }
  }
  __syncwarp();
}

template <bool MULTI>
__device__ __forceinline__ void store_row32_t(const GemmArgs& p, const GemmExt& e, int m, int n0,
                                              const float (&y)[32]) {
  if constexpr (MULTI) store_row32_multi(p, e, m, n0, y);
  else store_row32(p, m, n0, y);
}
template <bool MULTI>
__device__ __forceinline__ void store_row8_t(const GemmArgs& p, const GemmExt& e, int m, int n0, const float (&y)[8]) {
  if constexpr (MULTI) store_row8_multi(p, e, m, n0, y);
  else store_row8(p, m, n0, y);
}

__device__ __forceinline__ void store_row32_i32(const GemmArgs& p, int m, int n0, const uint32_t (&r)[32],
                                                int64_t plane = 0) {
  int32_t* o = static_cast<int32_t*>(p.out) + plane + (int64_t)m * p.ld_out + n0;  // int32: one destination
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

// Plain-scale epilogue of 32 consecutive output columns of one row
// (optimized_linear, comfy/quant_ops.py:472-474):
//   y[j] = float(acc[j]) * (frow * col[j]) + bias[j], then the optional GELU,
// every operation separately rounded.  col / bias are this warp's staged
// column scales and bias (16-byte aligned, read as vectors); the GELU runs
// as its own pass so the scale loop stays branch-free -- with the GELU test
// inside it every unrolled element carried the inlined GELU code, and that
// epilogue, not the MMAs, set the pace of short-K GEMMs.
__device__ __forceinline__ void plain_epilogue32(const uint32_t (&acc)[32], float frow, const float* col,
                                                 const float* bias, bool has_bias, int act, int out_dtype,
                                                 float (&y)[32]) {
  const float4* c4 = reinterpret_cast<const float4*>(col);
  const float4* b4 = reinterpret_cast<const float4*>(bias);
#pragma unroll
  for (int q = 0; q < 8; ++q) {
    const float4 s = c4[q];
    const float sv[4] = {s.x, s.y, s.z, s.w};
#pragma unroll
    for (int u = 0; u < 4; ++u) y[4 * q + u] = __fmul_rn(__int2float_rn((int)acc[4 * q + u]), __fmul_rn(frow, sv[u]));
    if (has_bias) {
      const float4 b = b4[q];
      const float bv[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
      for (int u = 0; u < 4; ++u) y[4 * q + u] = __fadd_rn(y[4 * q + u], bv[u]);
    }
  }
  if (act == QI8_ACT_GELU) {
#pragma unroll
    for (int j = 0; j < 32; ++j) y[j] = act_gelu(y[j], out_dtype);
  }
}

// The transposed form of plain_epilogue32 (weights on the TMEM lanes): the
// thread is output feature n with weight scale frow and bias brow, its 32
// values are tokens m0 .. m0 + 31 with the staged token scales col[j]:
//   y[j] = float(acc[j]) * (frow * col[j]) + brow, then the optional GELU;
// frow * col[j] is the same rounded product as the untransposed x_s * w_s.
__device__ __forceinline__ void swap_epilogue32(const uint32_t (&acc)[32], float frow, const float* col, float brow,
                                                bool has_bias, int act, int out_dtype, float (&y)[32]) {
  const float4* c4 = reinterpret_cast<const float4*>(col);
#pragma unroll
  for (int q = 0; q < 8; ++q) {
    const float4 s = c4[q];
    const float sv[4] = {s.x, s.y, s.z, s.w};
#pragma unroll
    for (int u = 0; u < 4; ++u) y[4 * q + u] = __fmul_rn(__int2float_rn((int)acc[4 * q + u]), __fmul_rn(frow, sv[u]));
  }
  if (has_bias) {
#pragma unroll
    for (int j = 0; j < 32; ++j) y[j] = __fadd_rn(y[j], brow);
  }
  if (act == QI8_ACT_GELU) {
#pragma unroll
    for (int j = 0; j < 32; ++j) y[j] = act_gelu(y[j], out_dtype);
  }
}

__device__ __forceinline__ uint16_t bits16(float v, int out_dtype) {
  return out_dtype == QI8_BF16 ? __bfloat16_as_ushort(__float2bfloat16_rn(v)) : __half_as_ushort(__float2half_rn(v));
}

// Stores the warp's transposed 32 x 32 tile (lane = feature nb + lane,
// y[j] = token m0 + j) as rows of the 16-bit output: each lane writes its
// column into a per-warp shared tile of 32 rows x 40 halfwords (80-byte rows:
// the column writes and the 16-byte row reads are bank-conflict free), then
// lane l stores token m0 + l's 32 features as four 16-byte stores; features
// >= N (N is a multiple of 16) and tokens >= M are skipped.
constexpr int SWAP_TILE_LD = 40;
__device__ __forceinline__ void store_tile32_swap(const GemmArgs& p, uint16_t* tile, int nb, int m0,
                                                  const float (&y)[32], int lane) {
#pragma unroll
  for (int j = 0; j < 32; ++j) tile[j * SWAP_TILE_LD + lane] = bits16(y[j], p.out_dtype);
  __syncwarp();
  const int m = m0 + lane;
  if (m < p.M) {
    const uint4* src = reinterpret_cast<const uint4*>(tile + lane * SWAP_TILE_LD);
    uint4* dst = reinterpret_cast<uint4*>(static_cast<uint16_t*>(p.out) + (int64_t)m * p.ld_out + nb);
#pragma unroll
    for (int q = 0; q < 4; ++q)
      if (nb + 8 * q + 8 <= p.N) dst[q] = src[q];
  }
  // the tile is rewritten by this warp's next chunk
  __syncwarp();
}

// Tile epilogue of the block-scaled kernels: final scales, optional GELU and
// the stores, from the WC accumulator registers of one thread.
// SWAP: thread = output feature rr, the 128 values are tokens cc0..cc0+127;
// stores go through a per-warp 16x32 bf16 transpose tile so each lane writes
// 32 contiguous bytes.  Otherwise: thread = token rr, values = features.
template <bool SWAP, bool GELU, bool MULTI, int WC = 128>
__device__ __forceinline__ void finalize_tile(const GemmArgs& p, const GemmExt& e, const float2 (&acc)[WC / 2],
                                              const float* my_col,
                                              const float* my_bias, float frow, float brow, int rr, int cc0, int cc1,
                                              int R, int C, int warp, int lane, __nv_bfloat16* sxp) {
  // accumulator column j < WC/2 is output column cc0 + j, column j >= WC/2 is cc1 + j - WC/2
  constexpr int RUN = WC / 2;
  const bool row_ok = rr < R;
  if constexpr (SWAP) {
    // two 16x32 bf16 transpose tiles per warp, used alternately, so one
    // __syncwarp per chunk orders the writes before the transposed reads and
    // the reads of chunk c before the writes of chunk c + 2
    __nv_bfloat16* tbw = sxp + warp * (2 * 16 * 32);
    const bool unit_row = p.b_kind == QI8_S_ROW_KBLOCK;  // frow == 1 exactly
    const bool has_bias = p.bias != nullptr;
#pragma unroll
    for (int c = 0; c < WC / 16; ++c) {
      const int col0 = c * 16 < RUN ? cc0 + c * 16 : cc1 + c * 16 - RUN;
      if (col0 >= C) {  // warp-uniform; keeps one __syncwarp per chunk
        __syncwarp();
        continue;
      }
      if (p.out_dtype == QI8_BF16) {
        __nv_bfloat16* tb = tbw + (c & 1) * (16 * 32);
        float cs[16];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float4 v = reinterpret_cast<const float4*>(my_col + c * 16)[q];
          cs[4 * q] = v.x; cs[4 * q + 1] = v.y; cs[4 * q + 2] = v.z; cs[4 * q + 3] = v.w;
        }
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const int col = c * 16 + j;
          const float a = (j & 1) ? acc[col >> 1].y : acc[col >> 1].x;
          float y = __fmul_rn(a, cs[j]);
          if (!unit_row) y = __fmul_rn(y, frow);
          if (has_bias) y = __fadd_rn(y, brow);
          if (GELU) y = act_gelu(y, p.out_dtype);
          tb[j * 32 + lane] = __float2bfloat16_rn(y);
        }
        __syncwarp();
        const int t = lane >> 1, h = lane & 1;
        const int tok = col0 + t;
        const int f0 = rr - lane + h * 16;  // first of the 16 features this lane stores
        if (tok < C && f0 < R) {
          const uint4* src = reinterpret_cast<const uint4*>(tb + t * 32 + h * 16);
          if constexpr (MULTI) {
            const uint4 v0 = src[0], v1 = src[1];
            for_each_out(e, [&](void* base) {
              uint4* dst = reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(base) + (int64_t)tok * p.ld_out + f0);
              dst[0] = v0;
              dst[1] = v1;
            });
          } else {
            uint4* dst =
                reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(p.out) + (int64_t)tok * p.ld_out + f0);
            dst[0] = src[0];
            dst[1] = src[1];
          }
        }
      } else if (row_ok) {
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const int col = c * 16 + j;
          const float a = (j & 1) ? acc[col >> 1].y : acc[col >> 1].x;
          float y = __fadd_rn(__fmul_rn(__fmul_rn(a, my_col[col]), frow), brow);
          if (GELU) y = act_gelu(y, p.out_dtype);
          if (col0 + j < C) {
            const int64_t o = (int64_t)(col0 + j) * p.ld_out + rr;
            if constexpr (MULTI) {
              for_each_out(e, [&](void* base) {
                if (p.out_dtype == QI8_F16) static_cast<__half*>(base)[o] = __float2half_rn(y);
                else static_cast<float*>(base)[o] = y;
              });
            } else {
              if (p.out_dtype == QI8_F16) static_cast<__half*>(p.out)[o] = __float2half_rn(y);
              else static_cast<float*>(p.out)[o] = y;
            }
          }
        }
      }
    }
  } else {
    if (!row_ok) return;
#pragma unroll
    for (int g = 0; g < WC / 8; ++g) {
      const int n0 = g * 8 < RUN ? cc0 + g * 8 : cc1 + g * 8 - RUN;
      if (n0 >= C) continue;
      const float4 c0 = reinterpret_cast<const float4*>(my_col + g * 8)[0];
      const float4 c1 = reinterpret_cast<const float4*>(my_col + g * 8)[1];
      const float4 b0 = reinterpret_cast<const float4*>(my_bias + g * 8)[0];
      const float4 b1 = reinterpret_cast<const float4*>(my_bias + g * 8)[1];
      const float cs[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
      const float bs[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
      float y[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int col = g * 8 + j;
        const float a = (j & 1) ? acc[col >> 1].y : acc[col >> 1].x;
        y[j] = __fadd_rn(__fmul_rn(__fmul_rn(a, frow), cs[j]), bs[j]);
        if (GELU) y[j] = act_gelu(y[j], p.out_dtype);
      }
      store_row8_t<MULTI>(p, e, rr, n0, y);
    }
  }
}

// Tile epilogue with int8 output (fused output requantization of the
// reference's int8_gemm_quant / int8_addmm_quant, comfy/int8_kernels.py:
// 684-917): thread = token rr, its 128 accumulator columns are the output
// columns cc0 .. cc0 + 127, i.e. exactly one 128-column quantization block.
// y = acc * frow * col_scale + bias (unit factors for block scales), then
// scale = max(amax / 127, 1e-8) and q = trunc(clamp(y / scale, -127, 127)).
__device__ __forceinline__ void finalize_tile_q8(const GemmArgs& p, const GemmExt& e, float2 (&acc)[64],
                                                 const float* my_col, const float* my_bias, float frow, int rr,
                                                 int cc0) {
  float amax = 0.0f;
#pragma unroll
  for (int i = 0; i < 64; ++i) {
    const float y0 = __fadd_rn(__fmul_rn(__fmul_rn(acc[i].x, frow), my_col[2 * i]), my_bias[2 * i]);
    const float y1 = __fadd_rn(__fmul_rn(__fmul_rn(acc[i].y, frow), my_col[2 * i + 1]), my_bias[2 * i + 1]);
    acc[i] = make_float2(y0, y1);
    amax = fmaxf(amax, fmaxf(fabsf(y0), fabsf(y1)));
  }
  const float scale = fmaxf(__fdiv_rn(amax, 127.0f), 1e-8f);
  uint4* q = reinterpret_cast<uint4*>(static_cast<int8_t*>(p.out) + (int64_t)rr * p.ld_out + cc0);
#pragma unroll
  for (int g = 0; g < 8; ++g) {
    uint32_t w[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      uint32_t word = 0;
#pragma unroll
      for (int b = 0; b < 4; b += 2) {
        const float2 y = acc[g * 8 + k * 2 + (b >> 1)];
        const int q0 = __float2int_rz(fminf(fmaxf(__fdiv_rn(y.x, scale), -127.0f), 127.0f));
        const int q1 = __float2int_rz(fminf(fmaxf(__fdiv_rn(y.y, scale), -127.0f), 127.0f));
        word |= ((uint32_t)(q0 & 0xFF) << (8 * b)) | ((uint32_t)(q1 & 0xFF) << (8 * (b + 1)));
      }
      w[k] = word;
    }
    q[g] = make_uint4(w[0], w[1], w[2], w[3]);
  }
  e.q_scale[(int64_t)rr * (p.N >> 7) + (cc0 >> 7)] = scale;
}

// SWAP: the weight tile is the MMA A operand (TMEM lanes = output features)
// and the activation tile the B operand (TMEM columns = tokens).  Used when
// the weight scale varies per (row, K block) and the activation scale does
// not, so that every epilogue thread promotes with one scalar per K block.
template <bool PROMOTE, bool SWAP, bool MULTI>
__global__ void __launch_bounds__(THREADS, 1)
    gemm_i8_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const GemmArgs p, const GemmExt e) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* sb = smem_raw + (base - raw);
  const uint32_t sA = base;
  const uint32_t sB = base + STAGES * A_BYTES;
  float* scol = reinterpret_cast<float*>(sb + STAGES * (A_BYTES + B_BYTES));  // [8 warps][128] column scales
  float* sbias = scol + NUM_EPI_WARPS * 128;                                   // [8 warps][128] bias
  float* skb = sbias + NUM_EPI_WARPS * 128;                                    // [8 warps][128] per-kb scales
  __nv_bfloat16* sxp = reinterpret_cast<__nv_bfloat16*>(skb + NUM_EPI_WARPS * 128);  // [8 warps][2][16][32] transpose
  uint64_t* bars = reinterpret_cast<uint64_t*>(sb + STAGES * (A_BYTES + B_BYTES) + STAGE_SCRATCH_BYTES);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + NUM_BARS);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  auto full_bar = [&](int s) { return smem_u32(bars + s); };
  auto empty_bar = [&](int s) { return smem_u32(bars + STAGES + s); };
  // accumulator buffer b, column half h (the plain kernel uses half 0 for the whole buffer)
  auto tfull_bar = [&](int b, int h) { return smem_u32(bars + 2 * STAGES + 2 * b + h); };
  auto tempty_bar = [&](int b, int h) { return smem_u32(bars + 2 * STAGES + 4 + 2 * b + h); };
  const uint32_t drain_bar = smem_u32(bars + 2 * STAGES + 8);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), 1);
    }
    for (int b = 0; b < 2; ++b) {
      for (int h = 0; h < 2; ++h) {
        mbar_init(tfull_bar(b, h), 1);
        mbar_init(tempty_bar(b, h), PROMOTE ? NUM_EPI_WARPS / 2 : NUM_EPI_WARPS);
      }
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
  // everything above overlaps the previous kernel on the stream; global
  // memory is touched only after it has completed
  pdl_wait();
  pdl_launch_dependents();
  const uint32_t tmem_base = *tmem_slot;
  const int KB = p.KB;
  if (warp >= NUM_EPI_WARPS) {
    // control warpgroup: producer, MMA issuer and two idle warps.  In the
    // block-scaled kernel it hands registers to the epilogue warpgroups.
    if constexpr (PROMOTE) asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(CTRL_REGS));
  if (warp == PRODUCER_WARP) {
    if (lane == 0) {
      int s = 0;
      uint32_t ph = 0;
      uint32_t issued = 0, issued_ph = 0;  // per-stage: load in flight, and its phase
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < p.num_tiles; tile += gridDim.x) {
        const int m0 = (tile % p.r_tiles) * BM;
        const int n0 = (tile / p.r_tiles) * BN;
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
          const uint32_t tpar = ((au >> 1) & 1) ^ 1u;
          if constexpr (PROMOTE) {
            // one K block, issued as two N=128 halves so each epilogue
            // warpgroup can start (and release) its half independently
            if (!mbar_wait(full_bar(s), ph, abort_flag, p.status, ST_GEMM_MMA, WAIT_LIMIT_NS)) {
              ok = false;
              break;
            }
            const uint64_t da = sw128_desc(sA + s * A_BYTES);
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              if (!mbar_wait(tempty_bar(buf, h), tpar, abort_flag, p.status, ST_GEMM_MMA, WAIT_LIMIT_NS)) {
                ok = false;
                break;
              }
              tc_fence_after();
              const uint32_t d = tmem_base + (uint32_t)(buf * BN + h * 128);
              const uint64_t db = sw128_desc(sB + s * B_BYTES + h * (128 * BK));
#pragma unroll
              for (int k = 0; k < BK / 32; ++k)
                tc_mma_i8(d, da + (uint64_t)(2 * k), db + (uint64_t)(2 * k), k > 0 ? 1u : 0u, IDESC_N128);
              tc_commit(tfull_bar(buf, h));
            }
            if (!ok) break;
            tc_commit(empty_bar(s));
            if (++s == STAGES) {
              s = 0;
              ph ^= 1u;
            }
          } else {
            if (!mbar_wait(tempty_bar(buf, 0), tpar, abort_flag, p.status, ST_GEMM_MMA, WAIT_LIMIT_NS)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t d = tmem_base + (uint32_t)(buf * BN);
            for (int kb = 0; kb < KB; ++kb) {
              if (!mbar_wait(full_bar(s), ph, abort_flag, p.status, ST_GEMM_MMA, WAIT_LIMIT_NS)) {
                ok = false;
                break;
              }
              tc_fence_after();
              const uint64_t da = sw128_desc(sA + s * A_BYTES);
              const uint64_t db = sw128_desc(sB + s * B_BYTES);
#pragma unroll
              for (int k = 0; k < BK / 32; ++k)
                tc_mma_i8(d, da + (uint64_t)(2 * k), db + (uint64_t)(2 * k), (kb > 0 || k > 0) ? 1u : 0u);
              tc_commit(empty_bar(s));
              if (++s == STAGES) {
                s = 0;
                ph ^= 1u;
              }
            }
            if (ok) tc_commit(tfull_bar(buf, 0));
          }
        }
      }
      // all MMAs issued by this thread complete before TMEM is released
      tc_commit(drain_bar);
      if (ok) mbar_wait(drain_bar, 0, abort_flag, p.status, ST_GEMM_DRAIN, WAIT_LIMIT_NS);
      else drain_wait(drain_bar, 0);
    }
  }
  } else {
    // ------------------------------------------------------- epilogue
    if constexpr (PROMOTE) asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(EPI_REGS));
    const int quad = warp & 3, half = warp >> 2;
    const uint32_t lane_base = (uint32_t)(quad * 32) << 16;
    float* my_col = scol + warp * 128;
    float* my_bias = sbias + warp * 128;
    float* my_kb = skb + warp * 128;
    const int R = SWAP ? p.N : p.M;  // rows on TMEM lanes
    const int C = SWAP ? p.M : p.N;  // rows on TMEM columns
    int au = 0;
    bool ok = true;
    for (int tile = blockIdx.x; ok && tile < p.num_tiles; tile += gridDim.x) {
      const int rr = (tile % p.r_tiles) * BM + quad * 32 + lane;  // this thread's row (m, or n when SWAP)
      const int cc0 = (tile / p.r_tiles) * BN + half * 128;       // first column of this warp
      const bool row_ok = rr < R;
      const bool cols_ok = cc0 < C;
      // per-column factors of this warp's 128 columns (coalesced, once per tile):
      // weight scale and bias per output feature, or (SWAP) activation scale per token
      __syncwarp();
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const int cc = cc0 + c * 32 + lane;
        if constexpr (SWAP) {
          my_col[c * 32 + lane] = cc < C ? row_scale(p.a_scale, p.a_kind, cc) : 0.0f;
        } else {
          my_col[c * 32 + lane] = cc < C ? row_scale(p.b_scale, p.b_kind, cc) : 0.0f;
          my_bias[c * 32 + lane] = (p.bias && cc < C) ? load_as_f32(p.bias, p.bias_dtype, cc) : 0.0f;
        }
      }
      __syncwarp();
      // this thread's final row factor (and bias when the row is an output feature)
      float frow = 1.0f, brow = 0.0f;
      if (row_ok) {
        if constexpr (SWAP) {
          frow = row_scale(p.b_scale, p.b_kind, rr);
          if (p.bias) brow = load_as_f32(p.bias, p.bias_dtype, rr);
        } else {
          frow = row_scale(p.a_scale, p.a_kind, rr);
        }
      }
      if constexpr (PROMOTE) {
        float2 acc[64];
#pragma unroll
        for (int i = 0; i < 64; ++i) acc[i] = make_float2(0.0f, 0.0f);
        // K-block scale: one scalar per thread, except a per-column weight
        // scale combined with per-(row, K block) activation scales
        const bool a_kb = !SWAP && p.a_kind == QI8_S_ROW_KBLOCK;
        const bool b_col = !SWAP && p.b_kind == QI8_S_ROW_KBLOCK;
        const bool b_tile = p.b_kind == QI8_S_TILE128;
        const bool exact = !SWAP && e.exact;
        // the K-block scales of blocks kb and kb + 1, loaded two blocks ahead
        auto ld_s = [&](int k) -> float {
          if (k >= KB) return 0.0f;
          if constexpr (SWAP) return row_ok ? __ldg(p.b_scale + (int64_t)rr * KB + k) : 0.0f;
          return a_kb ? (row_ok ? __ldg(p.a_scale + (int64_t)rr * KB + k) : 0.0f) : 1.0f;
        };
        auto ld_b = [&](int k) -> float {
          if (!b_tile || SWAP) return 1.0f;
          return (cols_ok && k < KB) ? __ldg(p.b_scale + (int64_t)(cc0 >> 7) * KB + k) : 0.0f;
        };
        auto ld_c = [&](int k, int c) -> float {
          const int n = cc0 + c * 32 + lane;
          return (b_col && n < p.N && k < KB) ? __ldg(p.b_scale + (int64_t)n * KB + k) : 0.0f;
        };
        float ps1 = ld_s(0), ps2 = ld_s(1), pb1 = ld_b(0), pb2 = ld_b(1), pc1[4], pc2[4];
#pragma unroll
        for (int c = 0; c < 4; ++c) { pc1[c] = ld_c(0, c); pc2[c] = ld_c(1, c); }
        for (int kb = 0; kb < KB; ++kb, ++au) {
          const int buf = au & 1;
          float sk = 1.0f, ska = 1.0f, skb = 1.0f;
          if constexpr (SWAP) {
            sk = ps1;
          } else {
            sk = ska = ps1;
            skb = pb1;
            if (b_tile) sk = __fmul_rn(sk, skb);
            if (b_col) {
              __syncwarp();
#pragma unroll
              for (int c = 0; c < 4; ++c) {
                my_kb[c * 32 + lane] = pc1[c];
                pc1[c] = pc2[c];
                pc2[c] = ld_c(kb + 2, c);
              }
              __syncwarp();
            }
          }
          ps1 = ps2; ps2 = ld_s(kb + 2);
          pb1 = pb2; pb2 = ld_b(kb + 2);
          const float2 sk2 = make_float2(sk, sk);
          if (!mbar_wait(tfull_bar(buf, half), (au >> 1) & 1, abort_flag, p.status, ST_GEMM_EPILOGUE, WAIT_LIMIT_NS)) {
            ok = false;
            break;
          }
          tc_fence_after();
          // 4 chunks of 32 columns; the load of chunk c+1 is in flight while
          // chunk c is promoted (tcgen05.wait::ld waits for all earlier loads)
          {
            const uint32_t ta = tmem_base + lane_base + (uint32_t)(buf * BN + half * 128);
            uint32_t rb[2][32];
            tmem_ld32(ta, rb[0]);
#pragma unroll
            for (int c = 0; c < 4; ++c) {
              tmem_wait_ld();
              if (c < 3) tmem_ld32(ta + (c + 1) * 32, rb[(c + 1) & 1]);
              if (c == 3) {
                // every column of this buffer half is in registers: release it
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(tempty_bar(buf, half));
              }
              if (exact) {
                // the reference's order: acc + (fp32(p) * a_s) * b_s, each rounded
#pragma unroll
                for (int j = 0; j < 16; ++j) {
                  const int col = c * 32 + 2 * j;
                  const float b0 = b_col ? my_kb[col] : skb, b1 = b_col ? my_kb[col + 1] : skb;
                  const float f0 = __int2float_rn((int)rb[c & 1][2 * j]), f1 = __int2float_rn((int)rb[c & 1][2 * j + 1]);
                  acc[col >> 1].x = __fadd_rn(acc[col >> 1].x, __fmul_rn(__fmul_rn(f0, ska), b0));
                  acc[col >> 1].y = __fadd_rn(acc[col >> 1].y, __fmul_rn(__fmul_rn(f1, ska), b1));
                }
              } else if (!SWAP && b_col) {
                // per-column weight scales of this K block (shared memory)
#pragma unroll
                for (int j = 0; j < 16; ++j) {
                  const int col = c * 32 + 2 * j;
                  const float2 f = make_float2(__int2float_rn((int)rb[c & 1][2 * j]),
                                               __int2float_rn((int)rb[c & 1][2 * j + 1]));
                  acc[col >> 1] = __ffma2_rn(f, __fmul2_rn(lds_f2(my_kb + col), sk2), acc[col >> 1]);
                }
              } else {
                // one scale for the thread's columns in this K block
#pragma unroll
                for (int j = 0; j < 16; ++j) {
                  const int col = c * 32 + 2 * j;
                  // exact int32 -> fp32 (|p| <= 128*128*128 < 2^24)
                  const float2 f = make_float2(__int2float_rn((int)rb[c & 1][2 * j]),
                                               __int2float_rn((int)rb[c & 1][2 * j + 1]));
                  acc[col >> 1] = __ffma2_rn(f, sk2, acc[col >> 1]);
                }
              }
            }
          }
        }
        if (!ok) break;
        // ---- tile epilogue, straight from the registers (the TMEM buffer is
        // already released, so the next tile's MMAs overlap these stores)
        // SWAP transposes through shared memory with __syncwarp, so the whole
        // warp enters together; lanes whose row is out of range store nothing
        if constexpr (!SWAP && !MULTI) {
          if (p.out_dtype == QI8_I8) {
            if (cols_ok && row_ok) finalize_tile_q8(p, e, acc, my_col, my_bias, frow, rr, cc0);
            continue;
          }
        }
        if (cols_ok && (SWAP || row_ok)) {
          if (p.act == QI8_ACT_GELU)
            finalize_tile<SWAP, true, MULTI>(p, e, acc, my_col, my_bias, frow, brow, rr, cc0, cc0 + 64, R, C, warp, lane, sxp);
          else
            finalize_tile<SWAP, false, MULTI>(p, e, acc, my_col, my_bias, frow, brow, rr, cc0, cc0 + 64, R, C, warp, lane, sxp);
        }
      } else {
        const int m = rr;
        const int ncol0 = cc0;
        const float fa = frow;
        const int buf = au & 1;
        if (!mbar_wait(tfull_bar(buf, 0), (au >> 1) & 1, abort_flag, p.status, ST_GEMM_EPILOGUE, WAIT_LIMIT_NS)) {
          ok = false;
          break;
        }
        tc_fence_after();
#pragma unroll
        for (int rnd = 0; rnd < 2; ++rnd) {
          uint32_t r[2][32];
          const uint32_t ta = tmem_base + lane_base + (uint32_t)(buf * BN + half * 128 + rnd * 64);
          tmem_ld32(ta, r[0]);
          tmem_ld32(ta + 32, r[1]);
          tmem_wait_ld();
          if (rnd == 1) {
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(tempty_bar(buf, 0));
          }
#pragma unroll
          for (int c = 0; c < 2; ++c) {
            const int cc = rnd * 64 + c * 32;  // column within this warp's 128
            const int n0 = ncol0 + cc;
            if (!row_ok || n0 >= p.N) continue;
            if (p.out_dtype == QI8_I32) {
              store_row32_i32(p, m, n0, r[c]);
            } else {
              float y[32];
              plain_epilogue32(r[c], fa, my_col + cc, my_bias + cc, p.bias != nullptr, p.act, p.out_dtype, y);
              store_row32_t<MULTI>(p, e, m, n0, y);
            }
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

// ============================================== CTA-pair kernel (cta_group::2)
// Two CTAs of a cluster share each MMA: tcgen05.mma.cta_group::2 with M=256
// reads the A rows of each CTA (128 each) and the B rows of both CTAs (BNP/2
// each) from their own shared memory, and writes each CTA's 128 output rows
// into that CTA's TMEM.  Per SM this halves the B tile that has to be
// loaded and read from shared memory for the same MMA work, or (BNP = 128)
// keeps the traffic of the single-CTA 128x256 tile while giving four
// accumulator buffers instead of two.
//   * both producers load their halves; the pair's stage barrier lives in
//     the even CTA (the leader), which alone arms it with the bytes of both;
//   * the leader's warp 9 lane 0 issues the MMAs; its commits arrive on the
//     stage-empty and accumulator-full barriers of both CTAs (multicast
//     commit; no multicast loads are used anywhere);
//   * both CTAs' epilogue warps release an accumulator buffer by arriving on
//     the leader's accumulator-empty barrier (16 arrivals).
// Every wait is bounded as in the single-CTA kernel; both CTAs meet at a
// cluster barrier before the TMEM is freed and the CTAs exit.
namespace pairk {

// Pair tile: 256 TMEM-lane rows (128 per CTA) x 256 columns (each CTA loads
// 128 of the column operand's rows; the MMA reads both halves).
constexpr int PBN = 256;
constexpr int B_HALF = PBN / 2;
constexpr int P_A_BYTES = 128 * BK;
constexpr int P_B_BYTES = B_HALF * BK;
constexpr int P_STAGE_BYTES = P_A_BYTES + P_B_BYTES;  // 32 KB per CTA
constexpr int P_STAGES = 6;
constexpr int P_BUFS = 2;  // TMEM accumulator buffers of 256 columns
// M = 256 (pair), N = n: s32 accumulator, signed A and B, K-major operands
__host__ __device__ constexpr uint32_t idesc_pair(int n) {
  return (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(256 >> 4) << 24);
}
constexpr uint32_t IDESC_P256 = idesc_pair(256);
constexpr int P_NUM_BARS = 2 * P_STAGES + 2 * P_BUFS + 1;  // full, empty, tfull, tempty, drain
// column scales, bias, K-block scales; then the per-warp transpose tiles
// (the block-scaled finalize uses 2 x 16 x 32 bf16 of each warp's share,
// the transposed plain epilogue 32 x SWAP_TILE_LD halfwords)
constexpr int P_SWAP_TILE = 32 * SWAP_TILE_LD;  // halfwords per warp
static_assert(P_SWAP_TILE >= 2 * 16 * 32, "transpose tile");
constexpr int P_SCRATCH = 3 * NUM_EPI_WARPS * 128 * 4 + NUM_EPI_WARPS * P_SWAP_TILE * 2;
constexpr int P_SMEM = 1024 + P_STAGES * P_STAGE_BYTES + P_SCRATCH + P_NUM_BARS * 8 + 16;
static_assert(P_SMEM <= 232448, "shared memory");

__device__ __forceinline__ uint32_t cta_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// shared::cluster address of the same shared-memory offset in CTA `rank`
__device__ __forceinline__ uint32_t mapa(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}
// Arrive on a barrier of either CTA of the pair.  Default semantics
// (release at CTA scope): the TMEM reads it publishes are ordered by
// tcgen05.wait::ld + tcgen05.fence::before_thread_sync, and a cluster-scope
// release would also wait for this thread's outstanding global loads.
__device__ __forceinline__ void arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// TMA load into this CTA's shared memory whose completion is counted on a
// barrier of either CTA of the pair (bar is a shared::cluster address)
__device__ __forceinline__ void tma_load_pair(uint32_t dst, const CUtensorMap* map, int x, int y, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar)
      : "memory");
}
__device__ __forceinline__ void mma_pair(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t accum) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d),
      "l"(a), "l"(b), "r"(idesc), "r"(accum)
      : "memory");
}
// arrive on the barrier at offset `bar` of every CTA in `mask` once all
// earlier MMAs of this thread have completed
__device__ __forceinline__ void commit_pair(uint32_t bar, uint16_t mask) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(bar),
               "h"(mask)
               : "memory");
}

// One accumulation unit per K block (block-scaled) or per tile (plain), in
// TMEM buffer (unit % 2); each epilogue warp drains 32 lanes x 128 columns.
template <bool PROMOTE, bool SWAP, bool MULTI, bool SPLIT>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(THREADS, 1)
    gemm_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                     const GemmArgs p, const GemmExt e) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* sb = smem_raw + (base - raw);
  const uint32_t sA = base;
  const uint32_t sB = base + P_STAGES * P_A_BYTES;
  float* scol = reinterpret_cast<float*>(sb + P_STAGES * P_STAGE_BYTES);  // [8 warps][128] column scales
  float* sbias = scol + NUM_EPI_WARPS * 128;                              // [8 warps][128] bias
  float* skb = sbias + NUM_EPI_WARPS * 128;                               // [8 warps][128] per-kb scales
  __nv_bfloat16* sxp = reinterpret_cast<__nv_bfloat16*>(skb + NUM_EPI_WARPS * 128);  // [8 warps][P_SWAP_TILE] transpose tiles
  uint64_t* bars = reinterpret_cast<uint64_t*>(sb + P_STAGES * P_STAGE_BYTES + P_SCRATCH);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + P_NUM_BARS);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  auto full_bar = [&](int s) { return smem_u32(bars + s); };
  auto empty_bar = [&](int s) { return smem_u32(bars + P_STAGES + s); };
  auto tfull_bar = [&](int b) { return smem_u32(bars + 2 * P_STAGES + b); };
  auto tempty_bar = [&](int b) { return smem_u32(bars + 2 * P_STAGES + P_BUFS + b); };
  const uint32_t drain_bar = smem_u32(bars + 2 * P_STAGES + 2 * P_BUFS);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cta_rank();
  const bool leader = rank == 0;
  const int cluster = blockIdx.x >> 1, nclusters = gridDim.x >> 1;

  if (threadIdx.x == 0) {
    for (int s = 0; s < P_STAGES; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), 1);
    }
    for (int b = 0; b < P_BUFS; ++b) {
      mbar_init(tfull_bar(b), 1);
      mbar_init(tempty_bar(b), 2 * NUM_EPI_WARPS);  // every epilogue warp of both CTAs
    }
    mbar_init(drain_bar, 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == MMA_WARP) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
  }
  if (warp == PRODUCER_WARP && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  // barriers initialised and TMEM allocated in both CTAs before any peer access
  tc_fence_before();
  cluster_sync();
  tc_fence_after();
  // everything above overlaps the previous kernel on the stream; global
  // memory is touched only after it has completed
  pdl_wait();
  pdl_launch_dependents();
  const uint32_t tmem_base = *tmem_slot;
  const int KB = p.KB;
  const int r_ptiles = p.r_tiles;  // tiles of 256 rows over the TMEM-lane operand
  const int rc_tiles = p.r_tiles * p.c_tiles;
  if (warp >= NUM_EPI_WARPS) {
    if constexpr (PROMOTE) asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(CTRL_REGS));
    if (warp == PRODUCER_WARP) {
      if (lane == 0) {
        const uint32_t full0 = mapa(full_bar(0), 0);
        int s = 0;
        uint32_t ph = 0;
        bool ok = true;
        for (int tile = cluster; ok && tile < p.num_tiles; tile += nclusters) {
          int rc = tile, kb_lo = 0, kb_hi = KB;
          if constexpr (SPLIT) {
            rc = tile % rc_tiles;
            kb_lo = (tile / rc_tiles) * e.kb_split;
            kb_hi = kb_lo + e.kb_split < KB ? kb_lo + e.kb_split : KB;
          }
          // each CTA loads its 128 rows of the lane operand and half of the
          // tile's pbn columns of the column operand
          const int bh = PROMOTE ? B_HALF : e.pbn >> 1;
          const int r0 = (rc % r_ptiles) * 256 + (int)rank * 128;
          const int c0 = (rc / r_ptiles) * 2 * bh + (int)rank * bh;
          for (int kb = kb_lo; kb < kb_hi; ++kb) {
            if (!mbar_wait(empty_bar(s), ph ^ 1u, abort_flag, p.status, ST_GEMM_PRODUCER, WAIT_LIMIT_NS)) {
              ok = false;
              break;
            }
            if (leader) mbar_arrive_expect_tx(full_bar(s), 2u * (uint32_t)(P_A_BYTES + bh * BK));
            const uint32_t fb = full0 + (uint32_t)(s * 8);
            tma_load_pair(sA + s * P_A_BYTES, &tmA, kb * BK, r0, fb);
            tma_load_pair(sB + s * P_B_BYTES, &tmB, kb * BK, c0, fb);
            if (++s == P_STAGES) {
              s = 0;
              ph ^= 1u;
            }
          }
        }
      }
    } else if (warp == MMA_WARP) {
      if (leader && lane == 0) {
        int s = 0;
        uint32_t ph = 0;
        int u = 0;  // accumulation units issued (one per K block, or one per tile)
        bool ok = true;
        const int n_units = PROMOTE ? KB : 1;
        const uint32_t idesc = PROMOTE ? IDESC_P256 : idesc_pair(e.pbn);
        for (int tile = cluster; ok && tile < p.num_tiles; tile += nclusters) {
          for (int w = 0; ok && w < n_units; ++w, ++u) {
            const int buf = u & 1;
            if (!mbar_wait(tempty_bar(buf), ((u >> 1) & 1) ^ 1u, abort_flag, p.status, ST_GEMM_MMA, WAIT_LIMIT_NS)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t d = tmem_base + (uint32_t)(buf * PBN);
            int kb_n = PROMOTE ? 1 : KB;
            if constexpr (SPLIT) {
              const int kb_lo = (tile / rc_tiles) * e.kb_split;
              kb_n = kb_lo + e.kb_split < KB ? e.kb_split : KB - kb_lo;
            }
            for (int kb = 0; kb < kb_n; ++kb) {
              if (!mbar_wait(full_bar(s), ph, abort_flag, p.status, ST_GEMM_MMA, WAIT_LIMIT_NS)) {
                ok = false;
                break;
              }
              tc_fence_after();
              const uint64_t da = sw128_desc(sA + s * P_A_BYTES);
              const uint64_t db = sw128_desc(sB + s * P_B_BYTES);
#pragma unroll
              for (int k = 0; k < BK / 32; ++k)
                mma_pair(d, da + (uint64_t)(2 * k), db + (uint64_t)(2 * k), idesc, (kb > 0 || k > 0) ? 1u : 0u);
              commit_pair(empty_bar(s), 3);
              if (++s == P_STAGES) {
                s = 0;
                ph ^= 1u;
              }
            }
            if (!ok) break;
            commit_pair(tfull_bar(buf), 3);
          }
        }
        // every MMA of this thread completes before the cluster barrier below
        commit_pair(drain_bar, 1);
        if (ok) mbar_wait(drain_bar, 0, abort_flag, p.status, ST_GEMM_DRAIN, WAIT_LIMIT_NS);
        else drain_wait(drain_bar, 0);
      }
    }
  } else {
    // ------------------------------------------------------- epilogue
    if constexpr (PROMOTE) asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(EPI_REGS));
    const int quad = warp & 3, cg = warp >> 2;
    const uint32_t lane_base = (uint32_t)(quad * 32) << 16;
    float* my_col = scol + warp * 128;
    float* my_bias = sbias + warp * 128;
    float* my_kb = skb + warp * 128;
    const int R = SWAP ? p.N : p.M;
    const int C = SWAP ? p.M : p.N;
    const uint32_t tempty0 = mapa(tempty_bar(0), 0);
    int au = 0;
    bool ok = true;
    for (int tile = cluster; ok && tile < p.num_tiles; tile += nclusters) {
      int rc = tile;
      int64_t plane = 0;
      if constexpr (SPLIT) {
        rc = tile % rc_tiles;
        plane = (int64_t)(tile / rc_tiles) * e.split_stride;
      }
      const int rr = (rc % r_ptiles) * 256 + (int)rank * 128 + quad * 32 + lane;
      // this warp's pbn / 2 accumulator columns (output columns cc0 ..)
      const int half = PROMOTE ? 128 : e.pbn >> 1;
      const int c0 = (rc / r_ptiles) * 2 * half;
      const int cc0 = c0 + cg * half;
      const int cc1 = cc0 + 64;
      const bool row_ok = rr < R;
      const bool cols_ok = cc0 < C;
      __syncwarp();
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const int j = c * 32 + lane;
        const int cc = j < 64 ? cc0 + j : cc1 + j - 64;
        if constexpr (SWAP) {
          my_col[j] = cc < C ? row_scale(p.a_scale, p.a_kind, cc) : 0.0f;
        } else {
          my_col[j] = cc < C ? row_scale(p.b_scale, p.b_kind, cc) : 0.0f;
          my_bias[j] = (p.bias && cc < C) ? load_as_f32(p.bias, p.bias_dtype, cc) : 0.0f;
        }
      }
      __syncwarp();
      float frow = 1.0f, brow = 0.0f;
      if (row_ok) {
        if constexpr (SWAP) {
          frow = row_scale(p.b_scale, p.b_kind, rr);
          if (p.bias) brow = load_as_f32(p.bias, p.bias_dtype, rr);
        } else {
          frow = row_scale(p.a_scale, p.a_kind, rr);
        }
      }
      if constexpr (PROMOTE) {
        float2 acc[64];
#pragma unroll
        for (int i = 0; i < 64; ++i) acc[i] = make_float2(0.0f, 0.0f);
        const bool a_kb = !SWAP && p.a_kind == QI8_S_ROW_KBLOCK;
        const bool b_col = !SWAP && p.b_kind == QI8_S_ROW_KBLOCK;
        const bool b_tile = p.b_kind == QI8_S_TILE128;
        const bool exact = !SWAP && e.exact;
        // SWAP: this row's K-block weight scales, loaded two K blocks ahead
        const float* srow = p.b_scale + (int64_t)(row_ok ? rr : 0) * KB;
        float sk_n1 = 0.0f, sk_n2 = 0.0f;
        if constexpr (SWAP) {
          sk_n1 = row_ok ? __ldg(srow) : 0.0f;
          sk_n2 = (row_ok && KB > 1) ? __ldg(srow + 1) : 0.0f;
        }
        // Not swapped: the activation's (row, K block) scale, the weight's
        // 128-tile scale and (per-row K-block weights) this lane's four column
        // scales of K blocks kb and kb + 1, loaded two K blocks ahead like the
        // swapped path's.  Columns cc0 .. cc0 + 127 lie in one 128-tile.
        auto ld_a = [&](int k) -> float {
          if (!a_kb) return 1.0f;
          return (row_ok && k < KB) ? __ldg(p.a_scale + (int64_t)rr * KB + k) : 0.0f;
        };
        auto ld_b = [&](int k) -> float {
          if (!b_tile) return 1.0f;
          return (cc0 < C && k < KB) ? __ldg(p.b_scale + (int64_t)(cc0 >> 7) * KB + k) : 0.0f;
        };
        auto ld_c = [&](int k, int c) -> float {
          const int n = cc0 + c * 32 + lane;
          return (b_col && n < p.N && k < KB) ? __ldg(p.b_scale + (int64_t)n * KB + k) : 0.0f;
        };
        float pa1 = 1.0f, pa2 = 1.0f, pb1 = 1.0f, pb2 = 1.0f, pc1[4], pc2[4];
        if constexpr (!SWAP) {
          pa1 = ld_a(0); pa2 = ld_a(1);
          pb1 = ld_b(0); pb2 = ld_b(1);
#pragma unroll
          for (int c = 0; c < 4; ++c) { pc1[c] = ld_c(0, c); pc2[c] = ld_c(1, c); }
        }
        for (int kb = 0; kb < KB; ++kb, ++au) {
          const int buf = au & 1;
          // scale of the first and of the second 64-column run
          float sk0 = 1.0f, sk1 = 1.0f, ska = 1.0f, skb0 = 1.0f, skb1 = 1.0f;
          if constexpr (SWAP) {
            sk0 = sk1 = sk_n1;
            sk_n1 = sk_n2;
            sk_n2 = (row_ok && kb + 2 < KB) ? __ldg(srow + kb + 2) : 0.0f;
          } else {
            ska = pa1;
            skb0 = skb1 = pb1;
            sk0 = sk1 = b_tile ? __fmul_rn(ska, skb0) : ska;
            pa1 = pa2; pa2 = ld_a(kb + 2);
            pb1 = pb2; pb2 = ld_b(kb + 2);
            if (b_col) {
              __syncwarp();
#pragma unroll
              for (int c = 0; c < 4; ++c) {
                my_kb[c * 32 + lane] = pc1[c];
                pc1[c] = pc2[c];
                pc2[c] = ld_c(kb + 2, c);
              }
              __syncwarp();
            }
          }
          if (!mbar_wait(tfull_bar(buf), (au >> 1) & 1, abort_flag, p.status, ST_GEMM_EPILOGUE, WAIT_LIMIT_NS)) {
            ok = false;
            break;
          }
          tc_fence_after();
          {
            const uint32_t ta = tmem_base + lane_base + (uint32_t)(buf * PBN + cg * 128);
            uint32_t rb[2][32];
            tmem_ld32(ta, rb[0]);
#pragma unroll
            for (int c = 0; c < 4; ++c) {
              tmem_wait_ld();
              if (c < 3) tmem_ld32(ta + (c + 1) * 32, rb[(c + 1) & 1]);
              if (c == 3) {
                // every column of this warp's share is in registers: release the buffer
                tc_fence_before();
                __syncwarp();
                if (lane == 0) arrive_cluster(tempty0 + (uint32_t)(buf * 8));
              }
              const float skc = c < 2 ? sk0 : sk1;
              const float2 sk2 = make_float2(skc, skc);
              if (exact) {
                // the reference's order: acc + (fp32(p) * a_s) * b_s, each rounded
                const float skbc = c < 2 ? skb0 : skb1;
#pragma unroll
                for (int j = 0; j < 16; ++j) {
                  const int col = c * 32 + 2 * j;
                  const float b0 = b_col ? my_kb[col] : skbc, b1 = b_col ? my_kb[col + 1] : skbc;
                  const float f0 = __int2float_rn((int)rb[c & 1][2 * j]), f1 = __int2float_rn((int)rb[c & 1][2 * j + 1]);
                  acc[col >> 1].x = __fadd_rn(acc[col >> 1].x, __fmul_rn(__fmul_rn(f0, ska), b0));
                  acc[col >> 1].y = __fadd_rn(acc[col >> 1].y, __fmul_rn(__fmul_rn(f1, ska), b1));
                }
              } else if (!SWAP && b_col) {
                // per-column weight scales of this K block (shared memory)
#pragma unroll
                for (int j = 0; j < 16; ++j) {
                  const int col = c * 32 + 2 * j;
                  const float2 f = make_float2(__int2float_rn((int)rb[c & 1][2 * j]),
                                               __int2float_rn((int)rb[c & 1][2 * j + 1]));
                  acc[col >> 1] = __ffma2_rn(f, __fmul2_rn(lds_f2(my_kb + col), sk2), acc[col >> 1]);
                }
              } else {
                // one scale for the thread's columns in this K block
#pragma unroll
                for (int j = 0; j < 16; ++j) {
                  const int col = c * 32 + 2 * j;
                  // exact int32 -> fp32 (|p| <= 128*128*128 < 2^24)
                  const float2 f = make_float2(__int2float_rn((int)rb[c & 1][2 * j]),
                                               __int2float_rn((int)rb[c & 1][2 * j + 1]));
                  acc[col >> 1] = __ffma2_rn(f, sk2, acc[col >> 1]);
                }
              }
            }
          }
        }
        if (!ok) break;
        if constexpr (!SWAP && !MULTI && !SPLIT) {
          if (p.out_dtype == QI8_I8) {
            if (cols_ok && row_ok) finalize_tile_q8(p, e, acc, my_col, my_bias, frow, rr, cc0);
            continue;
          }
        }
        if (cols_ok && (SWAP || row_ok)) {
          if (p.act == QI8_ACT_GELU)
            finalize_tile<SWAP, true, MULTI>(p, e, acc, my_col, my_bias, frow, brow, rr, cc0, cc1, R, C, warp, lane, sxp);
          else
            finalize_tile<SWAP, false, MULTI>(p, e, acc, my_col, my_bias, frow, brow, rr, cc0, cc1, R, C, warp, lane, sxp);
        }
      } else {
        const int buf = au & 1;
        if (!mbar_wait(tfull_bar(buf), (au >> 1) & 1, abort_flag, p.status, ST_GEMM_EPILOGUE, WAIT_LIMIT_NS)) {
          ok = false;
          break;
        }
        tc_fence_after();
        // chunks of 32 columns, loaded two at a time: half / 32 of them
        // (4 for 256-wide tiles, 3 for 192, 2 for 128, 1 for 64)
        const int nch = half >> 5;
#pragma unroll 1
        for (int ch = 0; ch < nch; ch += 2) {
          const bool two = ch + 1 < nch;  // warp-uniform
          uint32_t r[2][32];
          const uint32_t ta = tmem_base + lane_base + (uint32_t)(buf * PBN + cg * half + ch * 32);
          tmem_ld32(ta, r[0]);
          if (two) tmem_ld32(ta + 32, r[1]);
          tmem_wait_ld();
          if (ch + 2 >= nch) {
            tc_fence_before();
            __syncwarp();
            if (lane == 0) arrive_cluster(tempty0 + (uint32_t)(buf * 8));
          }
#pragma unroll
          for (int c = 0; c < 2; ++c) {
            if (c == 1 && !two) break;
            const int cc = ch * 32 + c * 32;
            const int n0 = cc0 + cc;
            if constexpr (SWAP) {
              // weights on the lanes: rr is feature n, the 32 columns are tokens n0 ..
              if (n0 >= p.M || rr - lane >= p.N) continue;  // warp-uniform
              float y[32];
              swap_epilogue32(r[c], frow, my_col + cc, brow, p.bias != nullptr, p.act, p.out_dtype, y);
              store_tile32_swap(p, reinterpret_cast<uint16_t*>(sxp) + warp * P_SWAP_TILE, rr - lane, n0, y, lane);
              continue;
            }
            if constexpr (MULTI) {
              // peer destinations: the warp's 32 x 32 tile goes through shared
              // memory so that each store writes 64 contiguous bytes of a row
              if (n0 < p.N && n0 + 32 <= p.N && p.out_dtype != QI8_F32) {  // warp-uniform
                float y[32];
                plain_epilogue32(r[c], frow, my_col + cc, my_bias + cc, p.bias != nullptr, p.act, p.out_dtype, y);
                store_tile32_multi(p, e, reinterpret_cast<uint4*>(sxp + warp * (2 * 16 * 32)), rr - lane, R, n0,
                                   y, lane);
                continue;
              }
            }
            if (!row_ok || n0 >= p.N) continue;
            if (p.out_dtype == QI8_I32) {
              store_row32_i32(p, rr, n0, r[c], plane);
            } else {
              float y[32];
              plain_epilogue32(r[c], frow, my_col + cc, my_bias + cc, p.bias != nullptr, p.act, p.out_dtype, y);
              store_row32_t<MULTI>(p, e, rr, n0, y);
            }
          }
        }
        ++au;
      }
    }
  }

  // no CTA of the pair frees TMEM or exits while the other may still touch it
  tc_fence_before();
  cluster_sync();
  if (warp == MMA_WARP) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(TMEM_COLS) : "memory");
  }
}

}  // namespace pairk

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

bool g_attr_set[6][64];

void set_outs(GemmArgs& p, GemmExt& e, void* const* outs, int n_outs) {
  for (int d = 0; d < QI8_MAX_PEERS; ++d) e.outs[d] = d < n_outs ? outs[d] : nullptr;
  e.n_outs = n_outs;
  p.out = outs[0];
}

// Co-resident CTA pairs of the pair kernel on device `dev` (queried once;
// 0 with the error set when the kernel cannot run there).
template <bool PROMOTE, bool SWAP, bool MULTI, bool SPLIT>
int pair_max_clusters(int dev) {
  auto kern = pairk::gemm_pair_kernel<PROMOTE, SWAP, MULTI, SPLIT>;
  static int max_clusters[64];
  if (dev < 0 || dev >= 64) dev = 0;
  if (max_clusters[dev] == 0) {
    if (check_cuda(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, pairk::P_SMEM),
                   "cudaFuncSetAttribute"))
      return 0;
    if (PROMOTE) {
      cudaFuncAttributes fa{};
      if (check_cuda(cudaFuncGetAttributes(&fa, kern), "cudaFuncGetAttributes")) return 0;
      if (fa.numRegs != LAUNCH_REGS) {
        fail(QI8_EUNSUPPORTED, "block-scaled GEMM compiled with %d registers per thread, register split needs %d",
             fa.numRegs, LAUNCH_REGS);
        return 0;
      }
    }
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(2 * (sm_count() > 0 ? sm_count() / 2 : 74), 1, 1);
    cfg.blockDim = dim3(THREADS, 1, 1);
    cfg.dynamicSmemBytes = pairk::P_SMEM;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n = 0;
    if (check_cuda(cudaOccupancyMaxActiveClusters(&n, kern, &cfg), "cudaOccupancyMaxActiveClusters")) return 0;
    if (n <= 0) {
      fail(QI8_EUNSUPPORTED, "no CTA pair of the GEMM fits on the device");
      return 0;
    }
    max_clusters[dev] = n;
  }
  return max_clusters[dev];
}

// Launches the CTA-pair kernel; grid = 2 x min(tiles, co-resident clusters).
template <bool PROMOTE, bool SWAP, bool MULTI, bool SPLIT = false>
int launch_pair(const CUtensorMap& mapA, const CUtensorMap& mapB, const GemmArgs& p, const GemmExt& e, int dev,
                cudaStream_t st) {
  auto kern = pairk::gemm_pair_kernel<PROMOTE, SWAP, MULTI, SPLIT>;
  const int maxc = pair_max_clusters<PROMOTE, SWAP, MULTI, SPLIT>(dev);
  if (maxc <= 0) return QI8_EUNSUPPORTED;
  const int ncl = p.num_tiles < maxc ? p.num_tiles : maxc;
  cudaError_t err = launch_pdl(kern, dim3(2 * ncl), dim3(THREADS), pairk::P_SMEM, st, mapA, mapB, p, e);
  if (err == cudaSuccess) err = cudaGetLastError();
  if (err != cudaSuccess) {
    cudaFuncAttributes fa{};
    cudaFuncGetAttributes(&fa, kern);
    return fail(QI8_ECUDA, "gemm_pair_kernel launch: %s (regs=%d smem=%d clusters=%d)", cudaGetErrorString(err),
                fa.numRegs, pairk::P_SMEM, ncl);
  }
  return QI8_OK;
}

// Split-K reduction with the plain epilogue: acc = sum of the S int32
// planes (exact), then the same arithmetic as the GEMM's own epilogue,
// y = fl(fl(acc) * fl(x_s * w_s)) (+ bias) (GELU) -> out dtype
// (comfy/quant_ops.py:472-474).  Four consecutive columns per thread.
__global__ void splitk_finalize_kernel(const int32_t* __restrict__ ws, int S, int64_t plane, int M, int N,
                                       const float* __restrict__ a_scale, int a_kind, const float* __restrict__ b_scale,
                                       int b_kind, const void* __restrict__ bias, int bias_dtype, void* out,
                                       int out_dtype, int64_t ld_out, int act) {
  pdl_wait();
  pdl_launch_dependents();
  const int nq = N >> 2;
  const int64_t total = (int64_t)M * nq;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int m = (int)(i / nq), n = (int)(i - (int64_t)m * nq) * 4;
    const int32_t* src = ws + (int64_t)m * N + n;
    int4 a = *reinterpret_cast<const int4*>(src);
    for (int sp = 1; sp < S; ++sp) {
      const int4 b = *reinterpret_cast<const int4*>(src + sp * plane);
      a.x += b.x; a.y += b.y; a.z += b.z; a.w += b.w;
    }
    const int acc[4] = {a.x, a.y, a.z, a.w};
    const int64_t o = (int64_t)m * ld_out + n;
    if (out_dtype == QI8_I32) {
      *reinterpret_cast<int4*>(static_cast<int32_t*>(out) + o) = a;
      continue;
    }
    const float fr = row_scale(a_scale, a_kind, m);
    float y[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      y[j] = __fmul_rn(__int2float_rn(acc[j]), __fmul_rn(fr, row_scale(b_scale, b_kind, n + j)));
      if (bias) y[j] = __fadd_rn(y[j], load_as_f32(bias, bias_dtype, n + j));
    }
    if (act == QI8_ACT_GELU) {  // its own pass, as in plain_epilogue32
#pragma unroll
      for (int j = 0; j < 4; ++j) y[j] = act_gelu(y[j], out_dtype);
    }
    if (out_dtype == QI8_F32) {
      *reinterpret_cast<float4*>(static_cast<float*>(out) + o) = make_float4(y[0], y[1], y[2], y[3]);
    } else {
      uint2 u;
      if (out_dtype == QI8_BF16) {
        __nv_bfloat162 h0 = __floats2bfloat162_rn(y[0], y[1]), h1 = __floats2bfloat162_rn(y[2], y[3]);
        u = make_uint2(*reinterpret_cast<uint32_t*>(&h0), *reinterpret_cast<uint32_t*>(&h1));
      } else {
        __half2 h0 = __floats2half2_rn(y[0], y[1]), h1 = __floats2half2_rn(y[2], y[3]);
        u = make_uint2(*reinterpret_cast<uint32_t*>(&h0), *reinterpret_cast<uint32_t*>(&h1));
      }
      *reinterpret_cast<uint2*>(static_cast<uint16_t*>(out) + o) = u;
    }
  }
}

// Tile width in tokens (64 or 128) of an unsplit plain GEMM of at most 128
// tokens run with the weights on the TMEM lanes, or 0 when that does not pad
// the work (padded lanes x padded columns) by at least 10 % less than the
// single-CTA kernel's 128-row tiles.  Larger token counts stay on the lanes:
// 576 tokens as 3 x 192-token tiles measured 8 % slower than 3 x 256-row
// tiles at K = 3072, where the per-tile epilogue (here with the transposed
// store) and not the MMAs sets the tile time.
int plain_swap_width(int64_t M, int64_t N) {
  if (M <= 0 || M > BM) return 0;
  int best = 0;
  int64_t best_pad = 0;
  for (int w = 256; w >= 64; w -= 64) {
    const int64_t pad = (M + w - 1) / w * w;
    if (best == 0 || pad < best_pad) {
      best = w;
      best_pad = pad;
    }
  }
  const int64_t n_pad = (N + 255) / 256 * 256;
  const int64_t m_lanes = M <= BM ? BM : (M + 255) / 256 * 256;
  return n_pad * best_pad * 10 <= m_lanes * n_pad * 9 ? best : 0;
}

// K splits of a plain-scale GEMM on the pair kernel: only when its tiles
// fill at most half of the co-resident CTA pairs, K has >= 64 blocks
// (K >= 8192) and every split keeps >= 8 blocks.  Measured as device time
// under graph replay, splitting lost 0.5-5 us at K = 3072 and 4096 (the
// unsplit tile is ~14 us there, and the int32 planes plus the reduce cost
// more than the shorter main loop saves) and won from K = 12288 up
// (64 x 3072 x 12288: 20.6 against 40.7 us).  Returns the number of splits
// (1 = none) and the blocks per split.
int choose_splits(int64_t Rrows, int64_t Crows, int64_t K, int max_clusters, int* kb_split) {
  const int KB = (int)((K + BK - 1) / BK);
  *kb_split = KB;
  const int64_t tiles = ((Rrows + 255) / 256) * ((Crows + pairk::PBN - 1) / pairk::PBN);
  if (max_clusters <= 0 || tiles * 2 > max_clusters || KB < 64) return 1;
  int s = (int)(max_clusters / tiles);
  if (s > 8) s = 8;
  if (s > KB / 8) s = KB / 8;
  if (s < 2) return 1;
  *kb_split = (KB + s - 1) / s;
  return (KB + *kb_split - 1) / *kb_split;
}

}  // namespace
}  // namespace qi8

using namespace qi8;

namespace qi8 {
namespace {

// Validates the GEMM and launches it; every destination in outs[0..n_outs)
// receives the full [M, N] result at row stride ld_out.
int gemm_launch(const int8_t* A, const int8_t* B, int64_t M, int64_t N, int64_t K, const float* a_scale, int a_kind,
                const float* b_scale, int b_kind, const void* bias, int bias_dtype, void* const* outs, int n_outs,
                int out_dtype, int64_t ld_out, int act, void* stream, void* workspace = nullptr,
                int64_t workspace_bytes = 0, float* q_scale = nullptr) {
  QI8_REQUIRE(device_ok(), QI8_EUNSUPPORTED, "no sm_100 device current");
  QI8_REQUIRE(A && B && outs && n_outs >= 1 && n_outs <= QI8_MAX_PEERS, QI8_EINVAL, "null pointer or bad n_outs");
  for (int d = 0; d < n_outs; ++d) QI8_REQUIRE(outs[d], QI8_EINVAL, "null output pointer %d", d);
  QI8_REQUIRE(M >= 0 && N > 0 && K > 0 && M < (1ll << 31) && N < (1ll << 31) && K < (1ll << 31), QI8_ESHAPE,
              "bad sizes M=%lld N=%lld K=%lld", (long long)M, (long long)N, (long long)K);
  QI8_REQUIRE(K % 16 == 0, QI8_ESHAPE, "K=%lld must be a multiple of 16", (long long)K);
  QI8_REQUIRE(N % 16 == 0, QI8_ESHAPE, "N=%lld must be a multiple of 16", (long long)N);
  QI8_REQUIRE(ld_out >= N, QI8_ESHAPE, "ld_out < N");
  QI8_REQUIRE(aligned16(A) && aligned16(B), QI8_EALIGN, "A, B and out must be 16-byte aligned");
  for (int d = 0; d < n_outs; ++d) QI8_REQUIRE(aligned16(outs[d]), QI8_EALIGN, "A, B and out must be 16-byte aligned");
  QI8_REQUIRE(a_kind >= QI8_S_NONE && a_kind <= QI8_S_ROW_KBLOCK, QI8_EINVAL, "a_kind %d", a_kind);
  QI8_REQUIRE(b_kind >= QI8_S_NONE && b_kind <= QI8_S_TILE128, QI8_EINVAL, "b_kind %d", b_kind);
  QI8_REQUIRE((a_kind == QI8_S_NONE) == (a_scale == nullptr), QI8_EINVAL, "a_scale/a_kind mismatch");
  QI8_REQUIRE((b_kind == QI8_S_NONE) == (b_scale == nullptr), QI8_EINVAL, "b_scale/b_kind mismatch");
  QI8_REQUIRE(out_dtype == QI8_BF16 || out_dtype == QI8_F16 || out_dtype == QI8_F32 || out_dtype == QI8_I32 ||
                  (out_dtype == QI8_I8 && q_scale),
              QI8_EDTYPE, "out dtype %d", out_dtype);
  QI8_REQUIRE(!bias || bias_dtype == QI8_BF16 || bias_dtype == QI8_F16 || bias_dtype == QI8_F32, QI8_EDTYPE,
              "bias dtype %d", bias_dtype);
  const int es = elem_size(out_dtype);
  QI8_REQUIRE((ld_out * es) % 16 == 0, QI8_EALIGN, "ld_out * elem_size must be a multiple of 16");
  const bool promote = a_kind == QI8_S_ROW_KBLOCK || b_kind == QI8_S_ROW_KBLOCK || b_kind == QI8_S_TILE128;
  if (promote) QI8_REQUIRE(K % 128 == 0, QI8_ESHAPE, "block scales need K %% 128 == 0 (K=%lld)", (long long)K);
  QI8_REQUIRE(out_dtype != QI8_I32 || n_outs == 1, QI8_EINVAL, "int32 output has one destination");
  if (out_dtype == QI8_I32)
    QI8_REQUIRE(!promote && a_kind == QI8_S_NONE && b_kind == QI8_S_NONE && !bias && act == QI8_ACT_NONE,
                QI8_EINVAL, "int32 output takes no scales, bias or activation");
  QI8_REQUIRE(act == QI8_ACT_NONE || act == QI8_ACT_GELU, QI8_EINVAL, "act %d", act);
  if (out_dtype == QI8_I8) {
    // fused output requantization: block-scaled activations and weights, one destination
    QI8_REQUIRE(a_kind == QI8_S_ROW_KBLOCK && (b_kind == QI8_S_TILE128 || b_kind == QI8_S_ROW_KBLOCK), QI8_EINVAL,
                "int8 output needs per-(row, K block) activation scales and 128-block weight scales");
    QI8_REQUIRE(n_outs == 1 && act == QI8_ACT_NONE, QI8_EINVAL, "int8 output has one destination and no activation");
    QI8_REQUIRE(N % 128 == 0, QI8_ESHAPE, "N=%lld must be divisible by out_block_size=128", (long long)N);
    QI8_REQUIRE((reinterpret_cast<uintptr_t>(q_scale) & 3) == 0, QI8_EALIGN, "scale_out must be 4-byte aligned");
  }
  if (M == 0) return QI8_OK;

  int dev = 0;
  QI8_CUDA(cudaGetDevice(&dev));
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // a plain GEMM whose output tiles fill few CTA pairs splits K when the
  // caller gives a workspace and K is long, also with at most 128 rows (the
  // pair tile's rows beyond M are zero-filled by TMA and never stored)
  int S = 1, kb_split = (int)((K + BK - 1) / BK);
  if (!promote && n_outs == 1 && workspace && aligned16(workspace)) {
    S = choose_splits(M, N, K, pair_max_clusters<false, false, false, true>(dev), &kb_split);
    if (S > 1 && workspace_bytes < (int64_t)S * M * N * 4) S = 1;
  }
  // weights on TMEM lanes when their scale varies per (row, K block) and the
  // activations' does not; for an unsplit plain GEMM with 16-bit output and
  // at most 128 tokens, when the tokens pad less as a tile width (64 tokens:
  // one 64-wide tile instead of a 128-row lane tile)
  const int swap_pbn = (!promote && n_outs == 1 && S == 1 && (out_dtype == QI8_BF16 || out_dtype == QI8_F16))
                           ? plain_swap_width(M, N)
                           : 0;
  const bool swap = (promote && b_kind == QI8_S_ROW_KBLOCK && a_kind != QI8_S_ROW_KBLOCK) || swap_pbn > 0;
  const int8_t* Rop = swap ? B : A;
  const int8_t* Cop = swap ? A : B;
  const int64_t Rrows = swap ? N : M, Crows = swap ? M : N;
  if (Rrows > BM || S > 1 || swap_pbn > 0) {
    // CTA pairs: 256 rows on TMEM lanes x bnp columns per pair tile.  A
    // plain GEMM with few tiles splits K (caller workspace, long K), or
    // else, when even the 128-column tiles fill at most half of the pairs,
    // halves the tile width so that twice the pairs share the work.  The
    // narrow tiles cost more L2 traffic and epilogue per multiply-add: a
    // rule of tiles * 2 <= pairs measured slower on the linear stacks,
    // whose second stream's GEMM runs on the pairs a lone GEMM leaves idle.
    int bnp = swap_pbn > 0 ? swap_pbn : pairk::PBN;
    if (S == 1 && !promote && n_outs == 1 && swap_pbn == 0) {
      const int64_t tiles = ((Rrows + 255) / 256) * ((Crows + pairk::PBN - 1) / pairk::PBN);
      const int maxc = pair_max_clusters<false, false, false, false>(dev);
      if (maxc > 0 && tiles * 4 <= maxc) bnp = pairk::PBN / 2;
    }
    GemmArgs p{};
    p.M = (int)M; p.N = (int)N; p.K = (int)K; p.KB = (int)((K + BK - 1) / BK);
    p.r_tiles = (int)((Rrows + 255) / 256);
    p.c_tiles = (int)((Crows + bnp - 1) / bnp);
    p.num_tiles = p.r_tiles * p.c_tiles;
    p.a_scale = a_scale; p.a_kind = a_kind; p.b_scale = b_scale; p.b_kind = b_kind;
    p.bias = bias; p.bias_dtype = bias_dtype; p.out_dtype = out_dtype; p.ld_out = ld_out;
    GemmExt e{};
    set_outs(p, e, outs, n_outs);
    e.q_scale = q_scale;
    e.exact = out_dtype == QI8_I8;
    p.act = act;
    p.status = device_status_ptr();
    e.kb_split = p.KB;
    e.split_stride = 0;
    e.pbn = bnp;
    CUtensorMap mapA, mapB;
    int rc = make_map(&mapA, Rop, Rrows, K, 128);
    if (rc) return rc;
    rc = make_map(&mapB, Cop, Crows, K, bnp / 2);
    if (rc) return rc;
    {
      // few tiles: split K over more CTA pairs, int32 partial planes, then one reduce + epilogue pass
      if (S > 1) {
        GemmArgs q = p;
        GemmExt qe = e;
        qe.kb_split = kb_split;
        q.num_tiles = p.num_tiles * S;
        qe.split_stride = M * N;
        q.ld_out = N;
        q.out_dtype = QI8_I32;
        void* ws_out[1] = {workspace};
        set_outs(q, qe, ws_out, 1);
        rc = launch_pair<false, false, false, true>(mapA, mapB, q, qe, dev, st);
        if (rc) return rc;
        const int64_t work = M * (N / 4);
        int64_t blocks = (work + 255) / 256;
        const int64_t cap = (int64_t)(sm_count() > 0 ? sm_count() : 148) * 8;
        if (blocks > cap) blocks = cap;
        return check_cuda(launch_pdl(splitk_finalize_kernel, dim3((unsigned)blocks), dim3(256), 0, st,
                                     static_cast<const int32_t*>(workspace), S, M * N, (int)M, (int)N, a_scale, a_kind,
                                     b_scale, b_kind, bias, bias_dtype, outs[0], out_dtype, ld_out, act),
                          "splitk_finalize_kernel launch");
      }
    }
    if (n_outs > 1) {
      if (!promote) return launch_pair<false, false, true>(mapA, mapB, p, e, dev, st);
      if (swap) return launch_pair<true, true, true>(mapA, mapB, p, e, dev, st);
      return launch_pair<true, false, true>(mapA, mapB, p, e, dev, st);
    }
    if (!promote) {
      if (swap) return launch_pair<false, true, false>(mapA, mapB, p, e, dev, st);
      return launch_pair<false, false, false>(mapA, mapB, p, e, dev, st);
    }
    if (swap) return launch_pair<true, true, false>(mapA, mapB, p, e, dev, st);
    return launch_pair<true, false, false>(mapA, mapB, p, e, dev, st);
  }
  CUtensorMap mapA, mapB;
  int rc = make_map(&mapA, Rop, Rrows, K, BM);
  if (rc) return rc;
  rc = make_map(&mapB, Cop, Crows, K, BN);
  if (rc) return rc;

  GemmArgs p{};
  p.M = (int)M; p.N = (int)N; p.K = (int)K; p.KB = (int)((K + BK - 1) / BK);
  p.r_tiles = (int)((Rrows + BM - 1) / BM);
  p.c_tiles = (int)((Crows + BN - 1) / BN);
  p.num_tiles = p.r_tiles * p.c_tiles;
  p.a_scale = a_scale; p.a_kind = a_kind; p.b_scale = b_scale; p.b_kind = b_kind;
  p.bias = bias; p.bias_dtype = bias_dtype; p.out_dtype = out_dtype; p.ld_out = ld_out;
  GemmExt e{};
  set_outs(p, e, outs, n_outs);
  e.q_scale = q_scale;
  e.exact = out_dtype == QI8_I8;
  e.kb_split = p.KB;
  p.act = act;
  p.status = device_status_ptr();

  auto kern = n_outs > 1
                  ? (!promote ? gemm_i8_kernel<false, false, true>
                              : (swap ? gemm_i8_kernel<true, true, true> : gemm_i8_kernel<true, false, true>))
                  : (!promote ? gemm_i8_kernel<false, false, false>
                              : (swap ? gemm_i8_kernel<true, true, false> : gemm_i8_kernel<true, false, false>));
  const int variant = (!promote ? 0 : (swap ? 2 : 1)) + (n_outs > 1 ? 3 : 0);
  if (dev < 64 && !g_attr_set[variant][dev]) {
    QI8_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES));
    if (promote) {
      // the in-kernel register split assumes exactly LAUNCH_REGS registers per thread at launch
      cudaFuncAttributes fa{};
      QI8_CUDA(cudaFuncGetAttributes(&fa, kern));
      QI8_REQUIRE(fa.numRegs == LAUNCH_REGS, QI8_EUNSUPPORTED,
                  "block-scaled GEMM compiled with %d registers per thread, register split needs %d", fa.numRegs,
                  LAUNCH_REGS);
    }
    g_attr_set[variant][dev] = true;
  }
  const int sms = sm_count() > 0 ? sm_count() : 148;
  const int grid = p.num_tiles < sms ? p.num_tiles : sms;
  cudaError_t err = launch_pdl(kern, dim3(grid), dim3(THREADS), SMEM_BYTES, static_cast<cudaStream_t>(stream), mapA,
                               mapB, p, e);
  if (err == cudaSuccess) err = cudaGetLastError();
  if (err != cudaSuccess) {
    cudaFuncAttributes fa{};
    cudaFuncGetAttributes(&fa, kern);
    return fail(QI8_ECUDA, "gemm_i8_kernel launch: %s (regs=%d maxThreads=%d local=%zu smem=%d grid=%d)",
                cudaGetErrorString(err), fa.numRegs, fa.maxThreadsPerBlock, fa.localSizeBytes, SMEM_BYTES, grid);
  }
  return QI8_OK;
}

}  // namespace
}  // namespace qi8

extern "C" int qi8_gemm_i8(const int8_t* A, const int8_t* B, int64_t M, int64_t N, int64_t K, const float* a_scale,
                           int a_kind, const float* b_scale, int b_kind, const void* bias, int bias_dtype, void* out,
                           int out_dtype, int64_t ld_out, int act, void* stream) {
  void* outs[1] = {out};
  return gemm_launch(A, B, M, N, K, a_scale, a_kind, b_scale, b_kind, bias, bias_dtype, outs, 1, out_dtype, ld_out,
                     act, stream);
}

extern "C" int qi8_gemm_i8_quant(const int8_t* A, const int8_t* B, int64_t M, int64_t N, int64_t K,
                                 const float* a_scale, int a_kind, const float* b_scale, int b_kind, const void* bias,
                                 int bias_dtype, int8_t* q_out, int64_t ld_q, float* scale_out, int out_block,
                                 void* stream) {
  QI8_REQUIRE(out_block == 128, QI8_ESHAPE, "out_block_size %d: the fused requantization uses 128", out_block);
  QI8_REQUIRE(scale_out, QI8_EINVAL, "null scale_out");
  void* outs[1] = {q_out};
  return gemm_launch(A, B, M, N, K, a_scale, a_kind, b_scale, b_kind, bias, bias_dtype, outs, 1, QI8_I8, ld_q,
                     QI8_ACT_NONE, stream, nullptr, 0, scale_out);
}

extern "C" int64_t qi8_gemm_workspace_bytes(int64_t M, int64_t N, int64_t K, int a_kind, int b_kind) {
  if (!device_ok() || M <= 0 || N <= 0 || K <= 0) return 0;
  if (a_kind == QI8_S_ROW_KBLOCK || b_kind == QI8_S_ROW_KBLOCK || b_kind == QI8_S_TILE128) return 0;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 0;
  int kb_split = 0;
  const int S = choose_splits(M, N, K, pair_max_clusters<false, false, false, true>(dev), &kb_split);
  return S > 1 ? (int64_t)S * M * N * 4 : 0;
}

extern "C" int qi8_gemm_i8_ws(const int8_t* A, const int8_t* B, int64_t M, int64_t N, int64_t K, const float* a_scale,
                              int a_kind, const float* b_scale, int b_kind, const void* bias, int bias_dtype, void* out,
                              int out_dtype, int64_t ld_out, int act, void* workspace, int64_t workspace_bytes,
                              void* stream) {
  void* outs[1] = {out};
  return gemm_launch(A, B, M, N, K, a_scale, a_kind, b_scale, b_kind, bias, bias_dtype, outs, 1, out_dtype, ld_out,
                     act, stream, workspace, workspace_bytes);
}

extern "C" int qi8_gemm_i8_gather(const int8_t* A, const int8_t* B_local, int64_t M, int64_t n_loc, int64_t K,
                                  const float* a_scale, int a_kind, const float* b_scale, int b_kind, const void* bias,
                                  int bias_dtype, void* const* out_bases, int world, int rank, int out_dtype,
                                  int64_t ld_out, int act, void* stream) {
  QI8_REQUIRE(out_bases, QI8_EINVAL, "null out_bases");
  QI8_REQUIRE(world >= 1 && world <= QI8_MAX_PEERS && rank >= 0 && rank < world, QI8_EINVAL,
              "world %d / rank %d (at most %d ranks)", world, rank, QI8_MAX_PEERS);
  QI8_REQUIRE(out_dtype == QI8_BF16 || out_dtype == QI8_F16 || out_dtype == QI8_F32, QI8_EDTYPE,
              "gathered output dtype %d (bf16, f16 or f32)", out_dtype);
  QI8_REQUIRE(n_loc > 0 && ld_out >= (int64_t)world * n_loc, QI8_ESHAPE, "ld_out %lld < world * n_loc = %lld",
              (long long)ld_out, (long long)world * n_loc);
  const int64_t col_bytes = (int64_t)rank * n_loc * elem_size(out_dtype);
  // this device's own buffer first, then the peers in rank order
  void* outs[QI8_MAX_PEERS];
  int n = 0;
  outs[n++] = static_cast<char*>(out_bases[rank]) + col_bytes;
  for (int r = 0; r < world; ++r)
    if (r != rank) outs[n++] = out_bases[r] ? static_cast<char*>(out_bases[r]) + col_bytes : nullptr;
  return gemm_launch(A, B_local, M, n_loc, K, a_scale, a_kind, b_scale, b_kind, bias, bias_dtype, outs, world,
                     out_dtype, ld_out, act, stream);
}
