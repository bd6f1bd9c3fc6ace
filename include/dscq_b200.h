/*
 * dscq_b200 -- C ABI of the B200 (sm_100a) W4A4 quantized-linear path.
 *
 * Plain pointers and sizes only. Every device pointer refers to memory on the
 * current CUDA device; `stream` is a cudaStream_t (NULL = legacy default
 * stream). All entry points are asynchronous with respect to the host unless
 * stated otherwise and return DSCQ_OK (0) or an error code; dscq_last_error()
 * returns a message for the last failure on the calling thread.
 *
 * Packed int4 layout (identical to the reference): byte j of a row holds
 * element 2j in its low nibble and 2j+1 in its high nibble, two's complement
 * (core/quantization.py:31-45, kernel/w4a4.cu:53).
 */
#ifndef DSCQ_B200_H_
#define DSCQ_B200_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* status codes */
#define DSCQ_OK 0
#define DSCQ_ERR_INVALID 1     /* bad shape, dtype, alignment or null pointer */
#define DSCQ_ERR_CUDA 2        /* CUDA runtime error (launch, query)          */
#define DSCQ_ERR_UNSUPPORTED 3 /* device is not sm_100 / unsupported size      */
#define DSCQ_ERR_RANGE 4       /* value out of range (pack_int4 codes)         */

/* element types */
#define DSCQ_BF16 0
#define DSCQ_F16 1
#define DSCQ_F32 2

/* per-row quantizer modes */
#define DSCQ_ACT_SYM 0          /* scale = absmax*clip/7, codes in [-8, 7]                  */
#define DSCQ_WEIGHT_SYM 1       /* core/quantization.py:7-11, codes in [-7, 7] + code sums   */
#define DSCQ_ACT_ASYM 2         /* kernel/w4a4.cu:20-63 (rn(x/s) + zero)                     */
#define DSCQ_ACT_ASYM_TORCH 3   /* core/quantization.py:13-21 (rn(x/s + zero))               */

/* GEMM variants (dscq_matmul `variant`) */
#define DSCQ_GEMM_AUTO 0
#define DSCQ_GEMM_SMALL_M 1     /* decode kernel for M <= 32, else the SMALL_M_TC path */
#define DSCQ_GEMM_LARGE_M 2     /* 1-CTA persistent kernel, activations on the 128-row MMA side */
#define DSCQ_GEMM_LARGE_M_DIRECT 3 /* as LARGE_M, operands loaded to registers (A/B timing) */
#define DSCQ_GEMM_LARGE_M_PAIR 4   /* 256x256 tiles on CTA pairs (cta_group::2); AUTO's choice for large M */
#define DSCQ_GEMM_SMALL_M_TC 5     /* tcgen05 with weights on the 128-row MMA side (tokens as MMA N) */
#define DSCQ_GEMM_LARGE_M_PAIR_TMEM 6 /* 256x192 tiles on CTA pairs, expanded activations in TMEM */

/* Rotate+quantize kernel choice (dscq_rowquant_variant `variant`) */
#define DSCQ_QUANT_AUTO 0
#define DSCQ_QUANT_TC 1         /* tcgen05: dense Hadamard factor on the tensor cores, WHT-64 in registers */
#define DSCQ_QUANT_LEGACY 2     /* CUDA-core kernels (register WHT, mma.sync Kronecker, general)        */

int dscq_version(void);
const char* dscq_last_error(void);

/* Reads the sticky device status word of `device` (bit 0: a bounded wait in a
 * kernel expired; bit 1: bad launch geometry). Synchronises the device.
 * `clear` != 0 resets it. */
int dscq_device_status(int device, uint32_t* status, int clear);

/* Host-side +-1 Hadamard matrix of order n (row-major, n*n int8) for the
 * orders the library constructs: 2^j, Paley I/II primes, 172. */
int dscq_hadamard(int n, int8_t* out);

/* Dense factor `a` of the Kronecker rotation H_a (x) H_(K/a) used for K. */
int dscq_rotation_split(int64_t K, int* a, int* b);

/*
 * Replaces quantize_cuda(x, clip, fused), kernel/w4a4.cu:164-187.
 * x [M, K] (bf16/f16/f32, row stride K). Asymmetric per-row codes exactly as
 * the reference kernel; outputs padded like the reference:
 *   packed [MP, KP/2] u8, scales [MP] f32, zeros [MP] i32,
 *   MP = ceil(M/8)*8, KP = ceil(K/64)*64.
 * `fused` is accepted for signature parity; both settings give the same bytes.
 */
int dscq_quantize(const void* x, int x_dtype, int64_t M, int64_t K, float clip, int fused, uint8_t* packed,
                  float* scales, int32_t* zeros, void* stream);

/*
 * General per-row quantizer with optional online rotation (no counterpart in
 * the reference, which absorbs rotations into weights: core/linear.py:22-46).
 *   rotate == 0: identity. rotate != 0: y = x (H_a (x) H_b) / sqrt(K),
 *   a from dscq_rotation_split(K) and h_a its +-1 matrix in DEVICE memory
 *   (NULL when a == 1).
 * mode: DSCQ_ACT_SYM / DSCQ_WEIGHT_SYM / DSCQ_ACT_ASYM / DSCQ_ACT_ASYM_TORCH.
 * Writes rows_out (>= M) rows; KP (even, >= K) packed columns:
 *   packed [rows_out, ld_packed >= KP/2] (may be NULL when codes is given), scales [rows_out],
 *   zeros [rows_out] (asym modes, may be NULL otherwise),
 *   row_sums [rows_out] (sum of codes over k < K, may be NULL),
 *   codes [rows_out, ld_codes >= KP] int8 (may be NULL).
 */
int dscq_rowquant(const void* x, int x_dtype, int64_t M, int64_t K, int64_t ld_x, int rotate, int rot_a,
                  const int8_t* h_a, int mode, float clip, int64_t rows_out, int64_t KP, uint8_t* packed,
                  int64_t ld_packed, float* scales, int32_t* zeros, int32_t* row_sums, int8_t* codes,
                  int64_t ld_codes, void* stream);

/*
 * dscq_rowquant with an explicit kernel choice (no counterpart in the reference):
 *   DSCQ_QUANT_AUTO   as dscq_rowquant;
 *   DSCQ_QUANT_TC     the tcgen05 rotate+quantize kernel (K = a' * 64 with 16 <= a' <= 224,
 *                     symmetric modes, bf16 input, KP == K, 16-byte aligned rows;
 *                     DSCQ_ERR_UNSUPPORTED otherwise);
 *   DSCQ_QUANT_LEGACY the CUDA-core kernels (register WHT / mma.sync Kronecker / general).
 * All choices produce codes of the same rotation; the float summation order differs.
 */
int dscq_rowquant_variant(const void* x, int x_dtype, int64_t M, int64_t K, int64_t ld_x, int rotate, int rot_a,
                          const int8_t* h_a, int mode, float clip, int64_t rows_out, int64_t KP, uint8_t* packed,
                          int64_t ld_packed, float* scales, int32_t* zeros, int32_t* row_sums, int8_t* codes,
                          int64_t ld_codes, int variant, void* stream);

/*
 * Online per-head block rotation + symmetric per-row int4 quantisation: the
 * online form of the reference's Rotation transform (core/transforms.py:51-52,
 * absorbed into the v / o weights by core/linear.py:28-37; the reference has no
 * online form). x [M, ld_x] bf16 with K = 128 * heads (heads a multiple of 4, at
 * most 64), rotated per head, y[t, 128h + e] = sum_d x[t, 128h + d] R_h[d][e],
 * then quantised per row exactly like dscq_rowquant in DSCQ_ACT_SYM /
 * DSCQ_WEIGHT_SYM mode (scale = max(absmax * clip / 7, 1e-8)). R_h is given as
 * two bf16 parts, rot_hi + rot_lo ~ R_h (lo = the bf16 rounding of R_h - hi),
 * each [heads, 128, 128] stored transposed per head: rot[h][e][d] = R_h[d][e].
 * Outputs as dscq_rowquant: packed [rows_out, KP/2] (or NULL), scales
 * [rows_out], codes [rows_out, ld_codes] (or NULL); no zero points or code
 * sums. KP must equal K; rows M .. rows_out-1 are zero rows.
 */
int dscq_rowquant_headrot(const void* x, int64_t M, int64_t K, int64_t ld_x, int heads, const void* rot_hi,
                          const void* rot_lo, int mode, float clip, int64_t rows_out, int64_t KP, uint8_t* packed,
                          int64_t ld_packed, float* scales, int8_t* codes, int64_t ld_codes, void* stream);

/*
 * Replaces matmul_cuda(a, b, sx, zx, sw, sums, bias, M, N, fused,
 * force_decode, fp32), kernel/w4a4.cu:189-225.
 *   a [>= M rows, KP/2] u8 packed activations (row stride KP/2 bytes)
 *   b [>= N rows, KP/2] u8 packed weights
 *   sx [M] f32, sw [N] f32; zx [M] i32 + sums [N] i32 for the asymmetric
 *   correction (both NULL for symmetric activations)
 *   bias [N] and residual [M, N] in out_dtype, or NULL
 *   out [M, N] out_dtype (DSCQ_BF16 / DSCQ_F16 / DSCQ_F32), or NULL
 *   raw [M, N] i32 int32 accumulators sum_k a[m,k] b[n,k], or NULL
 * out[m,n] = ((raw + (8 - zx[m]) sums[n]) * sx[m]) * sw[n] + bias[n] + residual[m,n]
 * KP must be a positive multiple of 64 (as in the reference).
 */
int dscq_matmul(const uint8_t* a, const uint8_t* b, const float* sx, const int32_t* zx, const float* sw,
                const int32_t* sums, const void* bias, const void* residual, int64_t M, int64_t N, int64_t KP,
                int out_dtype, void* out, int32_t* raw, int variant, void* stream);

/*
 * dscq_matmul with int8 activation codes (no counterpart in the reference, whose
 * activations are packed nibbles): a [M, ld_a >= KP] int8 codes in [-8, 7] (the
 * codes output of dscq_rowquant in a symmetric mode, ld_a a multiple of 16),
 * b [N, KP/2] packed int4 weights. Symmetric activations only (no zero points):
 *   out[m, n] = (sum_k a[m,k] b[n,k]) * sx[m] * sw[n] + bias[n] + residual[m, n]
 * Same result bits as dscq_matmul on the packed form of a; one byte per
 * activation element instead of half, one third less expansion work per K block.
 */
int dscq_matmul_a8(const int8_t* a, int64_t ld_a, const uint8_t* b, const float* sx, const float* sw, const void* bias,
                   const void* residual, int64_t M, int64_t N, int64_t KP, int out_dtype, void* out, int32_t* raw,
                   void* stream);

/*
 * dscq_matmul_a8 with the kernel chosen by `variant` (no counterpart in the
 * reference): DSCQ_GEMM_AUTO (what dscq_matmul_a8 does: CTA pairs with
 * cta_group::2 MMAs for 256-wide tiles, the 1-CTA kernel otherwise),
 * DSCQ_GEMM_LARGE_M (always the 1-CTA kernel) or DSCQ_GEMM_LARGE_M_PAIR
 * (always CTA pairs). Same result bits for every variant; any other variant
 * is DSCQ_ERR_INVALID.
 */
int dscq_matmul_a8_variant(const int8_t* a, int64_t ld_a, const uint8_t* b, const float* sx, const float* sw,
                           const void* bias, const void* residual, int64_t M, int64_t N, int64_t KP, int out_dtype,
                           void* out, int32_t* raw, int variant, void* stream);

/*
 * Column-block form of dscq_matmul (no counterpart in the reference, which has
 * no multi-GPU code): the [M, N] result is written at rows 0..M-1, columns
 * col_off..col_off+N-1 of buffers with row stride ld_out elements, into each of
 * the n_outs (1..8) buffers in `outs` -- in a column-parallel group, the same
 * output buffer of every GPU (peer pointers), so the all-gather of the shards
 * happens in the GEMM epilogue over NVLink. `residual` uses the same indexing.
 */
int dscq_matmul_cols(const uint8_t* a, const uint8_t* b, const float* sx, const int32_t* zx, const float* sw,
                     const int32_t* sums, const void* bias, const void* residual, int64_t M, int64_t N, int64_t KP,
                     int out_dtype, void* const* outs, int n_outs, int64_t ld_out, int64_t col_off, int variant,
                     void* stream);

/*
 * 1 if dscq_rowquant with DSCQ_QUANT_AUTO would take the tcgen05 rotate+quantize
 * for `rows` rotated rows of length K (bf16, symmetric mode, 16-byte aligned),
 * else 0. No counterpart in the reference. A caller that quantises a slice of
 * a larger batch (the column-parallel layer quantises 1/p of the rows on each
 * GPU) passes the whole batch's row count and forces the answer with
 * dscq_rowquant_variant, so every slice gets the codes one call on the whole
 * batch would give.
 */
int dscq_rowquant_auto_tc(int64_t K, int64_t rows);

/*
 * Row-block copy into several buffers (no counterpart in the reference, which
 * has no multi-GPU code): rows x width bytes from `src` (row stride ld_src
 * bytes) to each of the n_dst (1..8) buffers in `dsts` (row stride ld_dst
 * bytes), same offsets. In a column-parallel group this pushes the columns a
 * GPU computed into every peer's output buffer after the GEMM stored them
 * locally; launched on a side stream it overlaps the next GEMM launch.
 * Addresses and strides 16-byte aligned, width a multiple of 16.
 */
int dscq_scatter_block(const void* src, int64_t ld_src, int64_t rows, int64_t width, void* const* dsts, int n_dst,
                       int64_t ld_dst, void* stream);

/*
 * dscq_rowquant's tcgen05 rotate+quantize without any device allocation. No counterpart in the
 * reference: it exists for callers that cannot call cudaMalloc, such as serving engines that
 * reserve all device memory up front for weights and KV cache and allocate only from their own
 * pool, or latency-critical paths that cannot take cudaMalloc's implicit device synchronisation.
 * dscq_rowquant allocates a small buffer once per device and K for the quantizer's Hadamard
 * operand; this entry point instead rebuilds that operand on every call (one extra small launch on
 * `stream`) into a fixed 128 KiB array that the library holds on every device it is loaded on until
 * the process exits. Same arguments, requirements and result bits as dscq_rowquant_variant with
 * DSCQ_QUANT_TC (rotate != 0, K = a' * 64 with 16 <= a' <= 224, DSCQ_ACT_SYM or DSCQ_WEIGHT_SYM,
 * bf16 x, KP == K, 16-byte aligned rows; `zeros` is ignored); anything else, including an operand
 * larger than the array, returns DSCQ_ERR_UNSUPPORTED.
 * The first call on a device looks up the array's device address; make that first call before any
 * stream capture. All calls on a device share the one array: calls that can overlap on the GPU
 * (different streams without ordering between them) race and must not be issued.
 */
int dscq_rowquant_tc_noalloc(const void* x, int x_dtype, int64_t M, int64_t K, int64_t ld_x, int rotate, int rot_a,
                             const int8_t* h_a, int mode, float clip, int64_t rows_out, int64_t KP, uint8_t* packed,
                             int64_t ld_packed, float* scales, int32_t* zeros, int32_t* row_sums, int8_t* codes,
                             int64_t ld_codes, void* stream);

/*
 * Element-wise operators of the Llama prefill workload around the W4A4 linears (no counterpart in the
 * reference, which runs a Hugging Face model around its QuantLinear). bf16 tensors, fp32 arithmetic,
 * rounded to bf16 at the same steps as the torch expressions in the comments.
 *   dscq_rmsnorm:  y[r] = bf16(bf16(x[r] * rsqrt(mean(x[r]^2) + eps)) * w), x, y [rows, H], w [H]
 *   dscq_rope:     in place, q [S, Hq, D] and k [S, Hk, D]: x = bf16(bf16(x * cos) + bf16(rot(x) * sin)),
 *                  rot(x) = [-x[D/2:], x[:D/2]], cos / sin [S, D]
 *   dscq_silu_mul: y = bf16(bf16(silu(g)) * u), n elements
 */
int dscq_rmsnorm(const void* x, const void* w, int64_t rows, int64_t H, float eps, void* y, void* stream);
int dscq_rope(void* q, void* k, const void* cos_t, const void* sin_t, int64_t S, int Hq, int Hk, int D, void* stream);
int dscq_silu_mul(const void* g, const void* u, int64_t n, void* y, void* stream);

/* pack_int4, core/quantization.py:31-40. codes [rows, K] int8 (row stride
 * ld_codes) -> packed [rows, ceil(K/2)] (row stride ld_packed). Codes outside
 * [-8, 7] are counted into *bad_count (device int, caller-zeroed). */
int dscq_pack_int4(const int8_t* codes, int64_t rows, int64_t K, int64_t ld_codes, uint8_t* packed,
                   int64_t ld_packed, int32_t* bad_count, void* stream);

/* unpack_int4, core/quantization.py:42-45. */
int dscq_unpack_int4(const uint8_t* packed, int64_t rows, int64_t ld_packed, int64_t width, int8_t* codes,
                     int64_t ld_codes, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* DSCQ_B200_H_ */
