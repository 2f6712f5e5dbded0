/*
 * qi8.h -- C ABI of libqi8.so, the B200 (sm_100a) kernels behind the QuIP
 * W8A8 quantized-linear path of convert_to_quant (ThunderFun/
 * convert_to_quant_QuIP_INT8 v0.8.2).
 *
 * Every entry point:
 *   - takes plain device pointers, element counts and a cudaStream_t passed
 *     as void* (NULL = legacy default stream); work is stream-ordered and the
 *     call never synchronizes the host;
 *   - never allocates or frees device memory (scratch is caller-provided);
 *   - returns 0 (QI8_OK) or a negative qi8_status and records a message that
 *     qi8_last_error() returns (thread-local).
 *
 * Matrices are row-major.  "ld" arguments are row strides in elements.
 * Citations name the reference function (file:line inside the reference
 * project) whose behaviour the entry point reproduces.
 */
#ifndef QI8_H_
#define QI8_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define QI8_ABI_VERSION 1

/* Largest number of ranks (output destinations) of the column-parallel
   entry points (qi8_gemm_i8_gather, qi8_peer_barrier). */
#define QI8_MAX_PEERS 8

#if defined(__GNUC__)
#define QI8_API __attribute__((visibility("default")))
#else
#define QI8_API
#endif

/* status codes */
enum {
  QI8_OK = 0,
  QI8_EINVAL = -1,       /* null pointer / bad enum value */
  QI8_ESHAPE = -2,       /* unsupported or inconsistent sizes */
  QI8_EALIGN = -3,       /* pointer or stride misaligned for vector/TMA access */
  QI8_EDTYPE = -4,       /* unsupported dtype combination */
  QI8_ECUDA = -5,        /* a CUDA runtime/driver call failed */
  QI8_ETIMEOUT = -6,     /* a kernel's bounded wait expired (device status word) */
  QI8_EUNSUPPORTED = -7  /* no sm_100a device */
};

/* element types */
enum { QI8_BF16 = 0, QI8_F16 = 1, QI8_F32 = 2, QI8_I8 = 3, QI8_I32 = 4 };

/* activation / row quantization rules */
enum {
  /* per row: s = max(amax/127, 1e-30); q = rint(x * (1/s)) in [-128,127]
     -- quantize_int8_axiswise, utils/float_utils.py:9-37 */
  QI8_Q_TOKEN = 0,
  /* per (row, 128-block): s = amax/127; q = trunc(x / s)
     -- Triton act_quant, comfy/int8_kernels.py:72-123 */
  QI8_Q_BLOCK = 1,
  /* flag for qi8_quant_rows: apply exact-erf GELU to every element first
     (rounded to the input dtype, as torch's gelu on that tensor), then
     quantize -- the GELU between the two projections of a DiT MLP */
  QI8_Q_GELU = 0x100
};

/* GEMM scale kinds */
enum {
  QI8_S_NONE = 0,      /* scale 1 (no scale pointer)                          */
  QI8_S_SCALAR = 1,    /* one value                       (tensorwise weight) */
  QI8_S_ROW = 2,       /* one value per row of the operand (token / axis / QuIP [N,1]) */
  QI8_S_ROW_KBLOCK = 3,/* [rows, K/128]: per row per 128-wide K block
                          (comfy block act; QuIP block requant [N, K/128, 1]) */
  QI8_S_TILE128 = 4    /* [rows/128, K/128]: per 128x128 weight tile (comfy block weight) */
};

/* GEMM epilogue activation */
enum { QI8_ACT_NONE = 0, QI8_ACT_GELU = 1 };

/* weight requantization schemes (converters/quip_int8.py:1614-1669) */
enum { QI8_REQ_ROW = 0, QI8_REQ_GLOBAL = 1, QI8_REQ_BLOCK = 2 };

QI8_API int qi8_version(void);
QI8_API const char* qi8_last_error(void);
/* 1 if device `device` is an sm_100 part this library was built for, else 0. */
QI8_API int qi8_device_supported(int device);
/* Reads (and with reset!=0 clears) the device status word that bounded
   in-kernel waits set on expiry.  Returns QI8_OK, QI8_ETIMEOUT or QI8_ECUDA.
   Synchronizes the current device. */
QI8_API int qi8_device_status(int reset);

/* Row quantization without rotation.
   QI8_Q_TOKEN replaces quantize_int8_axiswise (utils/float_utils.py:9-37) as
   called by optimized_linear (comfy/quant_ops.py:469); scale_out gets [rows].
   QI8_Q_BLOCK replaces act_quant (comfy/int8_kernels.py:96-123); scale_out
   gets [rows, n/block], block must be 128 (the reference default). */
QI8_API int qi8_quant_rows(const void* x, int x_dtype, int64_t rows, int64_t n, int64_t ld_x,
                   int mode, int block, int8_t* q_out, int64_t ld_q, float* scale_out,
                   void* stream);

/* K1: fused randomized FWHT + quantization of each row:
     r = FWHT_{n_pad}(pad(x, n_pad) * sign) * (normalize ? 1/sqrt(n_pad) : 1)
   then QI8_Q_TOKEN / QI8_Q_BLOCK quantization of r.  Replaces steps 1-2 of
   quip_int8_matmul (comfy/int8_kernels.py:1424-1428, utils/hadamard.py:339-408)
   followed by quantize_int8_axiswise.  n_pad is a power of two, 2 <= n_pad <=
   32768, n <= n_pad (columns n..n_pad-1 are zero); sign may be NULL. */
QI8_API int qi8_rotate_quant_rows(const void* x, int x_dtype, int64_t rows, int64_t n, int64_t ld_x,
                          int64_t n_pad, const float* sign, int normalize, int mode,
                          int8_t* q_out, float* scale_out, void* stream);

/* FWHT of each row to fp32: out = FWHT(pad(x)*pre_sign)*norm*post_sign.
   fast_hadamard_transform (utils/hadamard.py:339-408, comfy/hadamard_kernels.py:
   244-373, 376-497); out is [rows, n_pad] with row stride n_pad; may alias x
   when x is fp32 with ld_x == n_pad == n. */
QI8_API int qi8_fwht_rows(const void* x, int x_dtype, int64_t rows, int64_t n, int64_t ld_x,
                  int64_t n_pad, const float* pre_sign, const float* post_sign,
                  int normalize, float* out, void* stream);

/* In-place FWHT down the columns of x [rows, cols] (row stride ld), rows a
   power of two <= 32768: the row-dimension half of fast_hadamard_transform_2d
   (utils/hadamard.py:467-516).  final_mode 0: un-normalized; 1: multiply by
   factor; 2: divide by factor (the 2-D transform's x / sqrt(rows*cols)). */
QI8_API int qi8_fwht_cols(float* x, int64_t rows, int64_t cols, int64_t ld, int final_mode, float factor,
                          void* stream);

/* K3: output un-rotation of a transformed-space linear:
     y = (FWHT_{n_pad}(y_had) / sqrt(n_pad) * sign_u)[:, :n_out] + bias
   (quip_int8_matmul steps 4-5, comfy/int8_kernels.py:1446-1450), written as
   out_dtype (bf16 / f16 / f32) [rows, n_out] with row stride ld_out. */
QI8_API int qi8_unrotate_rows(const float* y_had, int64_t rows, int64_t n_pad, const float* sign_u,
                      const void* bias, int bias_dtype, int64_t n_out, void* out,
                      int out_dtype, int64_t ld_out, void* stream);

/* K2: D[M,N] = A[M,K] (int8) x B[N,K]^T (int8) on tcgen05 tensor cores with a
   fused epilogue, TMA-fed, TMEM accumulators.
   - No block scale kinds: exact int32 accumulation over all of K, then
     out = acc (QI8_I32 output; scales must be NONE) or
     out = float(acc) * (sa[m] * sb[n]) + bias[n]   -> out_dtype
     exactly as optimized_linear (comfy/quant_ops.py:471-474) / mm_8bit
     (comfy/int8_matmul_kernels.py:82-110).
   - QI8_S_ROW_KBLOCK / QI8_S_TILE128 on either side: per-128-K-block
     promotion acc += float(acc_kb) * sa(m,kb) * sb(n,kb), as int8_gemm /
     int8_addmm (comfy/int8_kernels.py:335-647); row-constant scales are
     applied once at the end.
   A, B: 16-byte aligned, K % 16 == 0 (TMA row pitch); N % 16 == 0;
   block kinds need K % 128 == 0.  act: QI8_ACT_GELU applies exact-erf GELU
   to the bias-added value (bf16-rounded first when out_dtype is bf16).
   ld_out: row stride of out (>= N). */
QI8_API int qi8_gemm_i8(const int8_t* A, const int8_t* B, int64_t M, int64_t N, int64_t K,
                const float* a_scale, int a_kind, const float* b_scale, int b_kind,
                const void* bias, int bias_dtype, void* out, int out_dtype, int64_t ld_out,
                int act, void* stream);

/* Dequantize int8 rows/tiles: out = q * scale.
   scale_kind QI8_S_SCALAR / QI8_S_ROW (TensorWise / AxisWise dequantize,
   comfy/quant_ops.py:326-339), QI8_S_ROW_KBLOCK with block (act_dequant,
   comfy/int8_kernels.py:126-179), QI8_S_TILE128 (weight_dequant,
   comfy/int8_kernels.py:256-330). */
QI8_API int qi8_dequant(const int8_t* q, int64_t rows, int64_t n, const float* scale, int scale_kind,
                int block, void* out, int out_dtype, void* stream);

/* Weight quantization (no rotation).
   QI8_S_SCALAR: quantize_int8_tensorwise (utils/float_utils.py:40-66),
     needs workspace of >= 4 bytes (global absmax); scale_out [1].
   QI8_S_ROW:    quantize_int8_axiswise per row; scale_out [rows].
   QI8_S_TILE128: Triton weight_quant (comfy/int8_kernels.py:182-253):
     s = max(amax/127, 1e-8), trunc; scale_out [rows/128, n/128]. */
QI8_API int qi8_quant_weight(const void* w, int w_dtype, int64_t rows, int64_t n, int scale_kind,
                     int8_t* q_out, float* scale_out, void* workspace, int64_t workspace_bytes,
                     void* stream);

/* K4: offline QuIP Hadamard conversion of one weight W[M,N] (identity Hessian:
   the LDLQ step reduces to rotated-space RTN):
     W' = FHT_N(FHT_M(pad(W) * s_u * s_v^T)),  s' = max(rowamax(W')/127, 1e-12),
     Q' = rint(W'/s') in [-127,127],  W_d = slice(FHT_M(FHT_N(Q' s')) * s_u * s_v)
   (converters/quip_int8.py:539-551, 1272-1274, 655, 1452, 1489-1506), then
   - store_transformed != 0: q_out = Q' [M_pad, N_pad], scale_out = s' [M_pad]
     (quip_int8.py:1558-1608);
   - else requant W_d (quip_int8.py:1614-1669): QI8_REQ_ROW -> scale [M],
     QI8_REQ_GLOBAL -> scale [1], QI8_REQ_BLOCK -> scale [M, N/block]
     (falls back to QI8_REQ_ROW when N % block != 0, as the reference does);
     q_out = Q [M, N].
   dequant_out (optional, fp32 [M,N]) receives W_d.  s_u [M_pad], s_v [N_pad]
   are +-1 fp32 with M_pad = next_pow2(M), N_pad = next_pow2(N), both <= 32768.
   workspace: >= qi8_quip_workspace_bytes(M, N) bytes, 256-byte aligned. */
QI8_API int64_t qi8_quip_workspace_bytes(int64_t M, int64_t N);
QI8_API int qi8_quip_convert(const void* w, int w_dtype, int64_t M, int64_t N, const float* s_u,
                     const float* s_v, int store_transformed, int requant, int block,
                     int8_t* q_out, float* scale_out, float* dequant_out, void* workspace,
                     int64_t workspace_bytes, void* stream);

/* qi8_quip_convert without a caller workspace (no counterpart in the
   reference).  For callers that cannot allocate device memory: a host
   program binding this C ABI from a runtime that has no CUDA allocator of
   its own, or a process whose device memory is already reserved by another
   allocator (PyTorch's caching allocator holds freed blocks, so a fresh
   cudaMalloc can fail although memory is free inside its pool).  The scratch
   is a fixed 64 MiB + 256 B array inside the library, held by every device
   that loads it until exit; M_pad * N_pad must be <= 2^24 (e.g. 4096 x 4096),
   larger weights are rejected with QI8_ESHAPE.  Nothing is allocated or freed.
   The first call on a device looks up the array's device address (issue it
   before any stream capture); the address is cached for the process, so do
   not use this entry point on a device after cudaDeviceReset.  All calls share the one array: calls that
   overlap on the GPU (different streams, or threads sharing a device) race
   and must be serialized by the caller.  Arguments and results as
   qi8_quip_convert. */
QI8_API int qi8_quip_convert_noalloc(const void* w, int w_dtype, int64_t M, int64_t N, const float* s_u,
                                     const float* s_v, int store_transformed, int requant, int block,
                                     int8_t* q_out, float* scale_out, float* dequant_out, void* stream);

/* Two-sided signed Hadamard rotation of a weight, the incoherence step of
   the QuIP converter on its own (converters/quip_int8.py:523-551 forward,
   :1489-1506 inverse); each 1-D transform is normalized by float(1/sqrt(n)),
   the M direction runs first on the way in and last on the way out.
   inverse == 0: out [M_pad, N_pad] fp32 = FHT_N(FHT_M(pad(W) * s_u * s_v^T)),
                 W [M, N] bf16/f16/f32 (zero padded); workspace unused.
   inverse != 0: out [M, N] fp32 = slice(FHT_M(FHT_N(W)) * s_u * s_v^T),
                 W [M_pad, N_pad] bf16/f16/f32; workspace >= M_pad*N_pad*4 bytes.
   M_pad, N_pad: powers of two (rows <= 32768, 2 <= cols <= 32768);
   s_u [M_pad], s_v [N_pad] are +-1 fp32.  out 16-byte aligned. */
QI8_API int qi8_weight_rotate2d(const void* w, int w_dtype, int64_t M, int64_t N, int64_t M_pad, int64_t N_pad,
                                const float* s_u, const float* s_v, int inverse, float* out, void* workspace,
                                int64_t workspace_bytes, void* stream);

/* Column all-gather of a column-sharded linear (multi-GPU inference): rank
   r holds Y[:, r*n_loc:(r+1)*n_loc] as a contiguous [rows, n_loc] tile
   y_local; every rank receives Y [rows, G*n_loc] (row stride ld_out) in
   y_out.  One ncclAllGather on `stream` into scratch (>= G*rows*n_loc
   elements), then one re-layout kernel; G = ncclCommCount(nccl_comm).
   nccl_comm is an ncclComm_t created by the caller; NCCL (libnccl.so.2) is
   resolved on the first call, QI8_EUNSUPPORTED if it cannot be loaded.
   dtype: bf16 / f16 / f32 / i32 / i8.  Replaces the gather half of the
   column-parallel plan for the largest linears (the reference runs them on
   one GPU only). */
QI8_API int qi8_allgather_cols(const void* y_local, int dtype, int64_t rows, int64_t n_loc, void* y_out,
                               int64_t ld_out, void* nccl_comm, void* scratch, int64_t scratch_bytes,
                               void* stream);

/* Re-layout of an all-gather result: gathered [G, rows, n_loc] (rank-major,
   as ncclAllGather leaves it) -> Y [rows, G*n_loc] with row stride ld_out,
   Y[t, r*n_loc + j] = gathered[r, t, j].  For callers that run the
   collective themselves (e.g. torch.distributed, per token chunk).  Any
   1/2/4-byte dtype; 16-byte vector copies when every row start is 16-byte
   aligned. */
QI8_API int qi8_gather_layout(const void* gathered, int dtype, int world, int64_t rows, int64_t n_loc,
                              void* y_out, int64_t ld_out, void* stream);

/* Device workspace (bytes) with which qi8_gemm_i8_ws splits K over more CTA
   pairs for this shape: nonzero only for plain (tensor / row / none) scales
   when the output tiles fill at most half of the device's co-resident CTA
   pairs (e.g. 512 tokens x 4096 x 4096); 0 = no split.  Needs the device. */
QI8_API int64_t qi8_gemm_workspace_bytes(int64_t M, int64_t N, int64_t K, int a_kind, int b_kind);

/* qi8_gemm_i8 with a caller workspace: when workspace_bytes >=
   qi8_gemm_workspace_bytes(...) the K blocks are split over S CTA-pair tiles
   that store exact int32 partial sums into the workspace ([S, M, N]), and one
   reduce pass sums them and applies the epilogue (same arithmetic, so the
   result is identical to qi8_gemm_i8); otherwise it is qi8_gemm_i8. */
QI8_API int qi8_gemm_i8_ws(const int8_t* A, const int8_t* B, int64_t M, int64_t N, int64_t K, const float* a_scale,
                           int a_kind, const float* b_scale, int b_kind, const void* bias, int bias_dtype, void* out,
                           int out_dtype, int64_t ld_out, int act, void* workspace, int64_t workspace_bytes,
                           void* stream);

/* K2 with the output requantized in the epilogue (replaces int8_gemm_quant /
   int8_addmm_quant, comfy/int8_kernels.py:684-1089, used by the
   BlockWiseINT8Layout linear with out_quant=True, comfy/quant_ops.py:362-364).
   A [M, K] int8 with a_scale [M, K/128] (a_kind QI8_S_ROW_KBLOCK), B [N, K]
   int8 with b_scale [N/128, K/128] (QI8_S_TILE128) or [N, K/128]
   (QI8_S_ROW_KBLOCK); bias (or null) [N].  acc accumulates
   fp32(A_kb B_kb^T) * a_s * b_s in K-block order (separately rounded, as the
   reference), + bias; then per (row, 128-column block):
   scale = max(amax / 127, 1e-8), q = trunc(clamp(acc / scale, -127, 127)).
   q_out [M, ld_q] int8 (ld_q % 16 == 0), scale_out [M, N/128] fp32;
   N % 128 == 0, out_block must be 128. */
QI8_API int qi8_gemm_i8_quant(const int8_t* A, const int8_t* B, int64_t M, int64_t N, int64_t K,
                              const float* a_scale, int a_kind, const float* b_scale, int b_kind, const void* bias,
                              int bias_dtype, int8_t* q_out, int64_t ld_q, float* scale_out, int out_block,
                              void* stream);

/* Fused int8 GELU (replaces int8_gelu, comfy/int8_kernels.py:1122-1312, the
   BlockWiseINT8Layout aten.gelu handler, comfy/quant_ops.py:435-448):
   v = q * scale per (row, 128-block), g = (v * 0.5) * (1 + erf(v / 1.41421356237))
   with erf correctly rounded to fp32, then the same per-block requantization
   as qi8_gemm_i8_quant.  q, q_out [rows, n] int8 (4-byte aligned), scale and
   scale_out [rows, n/128]; n % 128 == 0, block must be 128. */
QI8_API int qi8_int8_gelu(const int8_t* q, const float* scale, int64_t rows, int64_t n, int block, int8_t* q_out,
                          float* scale_out, void* stream);

/* GPTQ / LDLQ error-feedback quantization of one column block (replaces
   gptq_quant_block_kernel / triton_gptq_quant_block, comfy/gptq_kernels.py:
   11-124, called by converters/gptq_int8.py:137 and
   converters/quip_int8.py:861-864).  W [M, B] fp32 (row stride ld_w, updated
   in place), hinv [B, B] fp32 (row stride ld_h), scale: one fp32 value when
   scale_is_scalar, else [M].  Per row, columns in order:
   q = clamp(rint(w / s), -127, 127), e = (w - q s) / max(|hinv[j,j]|, 1e-12),
   w_k -= e * hinv[j, k] for k > j (s = max(|scale|, 1e-12)), fp32, each
   operation rounded separately.  q_out [M, B] int8, err_out [M, B] fp32;
   B <= 128. */
QI8_API int qi8_gptq_quant_block(float* W, int64_t M, int64_t B, int64_t ld_w, const float* hinv, int64_t ld_h,
                                 const float* scale, int scale_is_scalar, int8_t* q_out, int64_t ld_q, float* err_out,
                                 int64_t ld_e, void* stream);

/* ---- QuIP with the reference's default options (QuIPInt8Converter.convert,
   converters/quip_int8.py:1031-1345: diagonal rescaling, random permutation,
   damping, act-order, fp64 Hessian factorization, blocked LDLQ).  The
   converter's host side computes the O(N) vectors between these steps
   (D_tilde, the permutations, the damped diagonal). */

/* out[j] = sum_i w[i, j]^2 in fp32, summed in torch's CPU order: columns in
   groups of 32 (N >= 8; groups of 4 for N < 8) by a four-level cascade over
   the rows, the remaining columns by the 4-lane row_sum (replaces
   (W ** 2).sum(dim=0), converters/quip_int8.py:266).  w [M, N] bf16 / f16 /
   f32, row stride ld_w. */
QI8_API int qi8_col_sumsq(const void* w, int w_dtype, int64_t M, int64_t N, int64_t ld_w, float* out, void* stream);

/* out[i, j] = divide ? x[i, j] / col_scale[j] : (x[i, j] * col_scale[j]) * row_scale[i]
   (row_scale may be NULL; x == NULL is the identity, M == N): the rescaling
   W * D, (H * Dinv_j) * Dinv_i and its undo W / D
   (converters/quip_int8.py:280-285, 303).  out fp32, row stride ld_out. */
QI8_API int qi8_scale2d(const void* x, int x_dtype, int64_t M, int64_t N, int64_t ld_x, const float* row_scale,
                        const float* col_scale, int divide, float* out, int64_t ld_out, void* stream);

/* LDLQ inputs in LDLQ column order (converters/quip_int8.py:336-340,
   1105-1146, 1272-1274).  w_rot [M, N] and h_rot [N, N] fp32 are the rotated
   weight and Hessian; LDLQ position j holds rotated column cols[j] (the
   random permutation composed with act-order); dead[j] != 0 zeroes that
   weight column; diag[j] is the damped diagonal at position j.  Outputs:
   w_out [M, N] fp32, scale_out [M] = max(row amax / 127, 1e-12), and h_rev
   [N, N] fp64 = J Hs J (lower triangle, zeros above), Hs being the damped
   permuted Hessian symmetrized from its lower triangle.  N a power of two
   <= 32768. */
QI8_API int qi8_ldlq_prepare(const float* w_rot, const float* h_rot, int64_t M, int64_t N, const int32_t* cols,
                             const uint8_t* dead, const float* diag, float* w_out, float* scale_out, double* h_rev,
                             void* stream);

/* hinv_out [N, N] fp32 = the upper Cholesky factor U of Hs^-1 (Hs^-1 = U^T U),
   computed in fp64 from h_rev (overwritten) as J L^-1 J with L = chol(h_rev);
   replaces chol -> cholesky_inverse -> chol(upper) (converters/quip_int8.py:
   1195-1199).  *info (device int) is 0, or 1 + the index of the first
   non-positive pivot (the reference then falls back to the identity,
   :1211-1216).  workspace >= qi8_hinv_workspace_bytes(N), 16-byte aligned. */
QI8_API int64_t qi8_hinv_workspace_bytes(int64_t N);
QI8_API int qi8_hinv_upper(double* h_rev, int64_t N, float* hinv_out, int* info, void* workspace,
                           int64_t workspace_bytes, void* stream);

/* out [N, N] fp32 = identity (the fallback Hinv of :1216). */
QI8_API int qi8_eye_f32(float* out, int64_t N, void* stream);

/* One LDLQ pass (replaces _single_ldlq_pass + _quantize_block_lazy,
   converters/quip_int8.py:813-945, 638-672): for each `block` columns
   (16..128, a multiple of 16), 16-column batches q = clamp(rint(w / s),
   -127, 127), err = (w - q s) / max(hinv_jj, 1e-12), the rest of the block
   updated by err @ hinv[batch, rest]; after the block every later column
   by Err_block @ hinv[block, later].  Every dot product is accumulated by
   fmaf in index order from zero, then subtracted (fp32).  w [M, N] fp32 is
   consumed; scale [M]; q_out [M, N] int8.  workspace >=
   qi8_ldlq_workspace_bytes(M, N, block). */
QI8_API int64_t qi8_ldlq_workspace_bytes(int64_t M, int64_t N, int block);
QI8_API int qi8_ldlq(float* w, int64_t M, int64_t N, const float* hinv, const float* scale, int block,
                     int8_t* q_out, void* workspace, int64_t workspace_bytes, void* stream);

/* Back to rotated column order (undo act-order and the random permutation,
   converters/quip_int8.py:1348-1365, 1467-1474): deq_out[i, cols[j]] =
   q[i, j] * scale[i] (fp32, :1452) and/or q_out[i, cols[j]] = q[i, j]. */
QI8_API int qi8_ldlq_finish(const int8_t* q, int64_t M, int64_t N, const float* scale, const int32_t* cols,
                            float* deq_out, int8_t* q_out, void* stream);

/* Column-parallel K2 with the output all-gather fused into the epilogue
   (multi-GPU inference, one process per GPU).  Rank `rank` of `world` holds
   weight rows [rank*n_loc, (rank+1)*n_loc) as B_local [n_loc, K] (scales and
   bias sliced the same way); out_bases[r] is rank r's output buffer Y
   [M, ld_out] (ld_out >= world*n_loc) mapped into this process
   (qi8_ipc_open; out_bases[rank] is the local buffer).  The epilogue stores
   this rank's [M, n_loc] tile at column rank*n_loc of every rank's Y with
   plain stores over NVLink, so after qi8_peer_barrier every rank holds the
   whole Y.  Scales, bias, activation and dtypes as qi8_gemm_i8 (bf16 / f16 /
   f32 output).  Replaces the GEMM + ncclAllGather + re-layout sequence of
   the column-parallel plan (the reference runs these linears on one GPU,
   comfy/quant_ops.py:461-475). */
QI8_API int qi8_gemm_i8_gather(const int8_t* A, const int8_t* B_local, int64_t M, int64_t n_loc, int64_t K,
                               const float* a_scale, int a_kind, const float* b_scale, int b_kind, const void* bias,
                               int bias_dtype, void* const* out_bases, int world, int rank, int out_dtype,
                               int64_t ld_out, int act, void* stream);

/* CUDA IPC export of the allocation holding `ptr`: handle_out receives the
   64-byte cudaIpcMemHandle_t of the allocation's base, offset_out the byte
   offset of ptr inside it. */
QI8_API int qi8_ipc_handle(const void* ptr, void* handle_out, int64_t* offset_out);
/* Maps a peer's exported allocation into this process (peer access enabled
   on demand); *ptr_out = mapped base + offset. */
QI8_API int qi8_ipc_open(const void* handle, int64_t offset, void** ptr_out);
/* Unmaps a pointer returned by qi8_ipc_open (same offset). */
QI8_API int qi8_ipc_close(void* ptr, int64_t offset);

/* Stream-ordered barrier of `world` ranks over peer memory: flags[r] points
   to rank r's QI8_MAX_PEERS + 1 uint32 flag words (zeroed by their owner
   before the first barrier), mapped into this process.  Every rank must call
   it the same number of times.  Waits at most 2 s, then sets a status bit
   (reported as QI8_ETIMEOUT by qi8_device_status) and returns. */
QI8_API int qi8_peer_barrier(uint32_t* const* flags, int world, int rank, void* stream);

/* Original-space requantization of a weight W[M,N] (row stride ld_w) with the
   QuIP requant rule (converters/quip_int8.py:1614-1669): scale =
   max(amax/127, 1e-12), q = rint(w / scale) in [-127, 127]; QI8_REQ_ROW ->
   scale [M], QI8_REQ_GLOBAL -> scale [1] (workspace >= 4 bytes),
   QI8_REQ_BLOCK -> scale [M, N/block] (per-row fallback if N % block != 0). */
QI8_API int qi8_requant_weight(const void* w, int w_dtype, int64_t M, int64_t N, int64_t ld_w, int requant,
                               int block, int8_t* q_out, float* scale_out, void* workspace,
                               int64_t workspace_bytes, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* QI8_H_ */
