// W4A4 GEMM for sm_100a: packed-int4 operands -> TMA -> shared memory ->
// int8 expansion in the UMMA canonical 128B-swizzled layout ->
// tcgen05.mma.kind::i8 with int32 accumulators in TMEM -> fused dequant
// epilogue (token scale x channel scale, optional zero-point term, bias,
// residual) -> bf16/f16/f32.
//
// Replaces tensor_gemm / decode_gemm / epilogue of the reference
// (kernel/w4a4.cu:80-161): raw[m,n] = sum_k a_s4[m,k] * b_s4[n,k] in int32,
// then out = ((raw + (8 - zx[m]) * sums[n]) * sx[m]) * sw[n] (+ bias[n]),
// kernel/w4a4.cu:70-78. Rounding is explicit (no FMA contraction) so the
// epilogue is reproducible bit-for-bit from the same int32 accumulators.
//
// int4 -> int8 expansion: each nibble goes to the HIGH half of its byte
// (byte = nibble << 4), i.e. the int8 value 16*code. Both operands are
// expanded this way, so the tensor cores accumulate 256 * sum(a*b) exactly
// (|256 * 64 * KP| < 2^31 for KP <= 65536) and the epilogue shifts right by 8.
// One 32-bit word of 8 nibbles becomes two words with 3 integer ops:
// (w << 4) & 0xF0F0F0F0 (nibbles 0,2,4,6) and w & 0xF0F0F0F0 (1,3,5,7); the
// same permutation inside every 8-element group is applied to both operands,
// so it cancels in the dot product.
//
// Kernels
//   w4a4_gemm_tc<BN, SWAP, SPLIT>  one output tile per CTA; SWAP puts the
//       weights on the 128-row MMA side (small M: tokens become the MMA N
//       dimension, 16..64); SPLIT splits K across the CTAs of a cluster and
//       sums the partial int32 tiles through distributed shared memory.
//   w4a4_gemm_persistent<BN>  large M: persistent CTAs walk the tile list;
//       two TMEM accumulators so the epilogue of one tile overlaps the
//       main loop of the next; raw (TMA) and expanded stages are counted
//       separately (more raw stages in flight to cover load latency).
//
// Warp roles, one-tile kernel (448 threads, one CTA per SM):
//   warps 0-3   epilogue   (warp w owns TMEM lanes 32w..32w+31 = tile rows)
//   warp  4     TMA producer (one lane)
//   warp  5     TMEM allocator + MMA issuer (one lane)
//   warps 6-13  int4 -> int8 expansion (256 threads)
// Persistent kernels (576 threads): warps 0-7 epilogue (two per TMEM lane
// quadrant, each half of the columns), warps 8-9 TMA producer and MMA issuer,
// warps 10-17 expansion.
#pragma once
#include "ptx.cuh"

namespace dscq {

enum OutDtype : int { kOutBF16 = 0, kOutF16 = 1, kOutF32 = 2 };

struct GemmParams {
  int M, N;              // problem size: out is [M, N]
  int kblocks;           // number of 128-element K blocks (64 packed bytes each)
  int tiles_i, tiles_j;  // tile grid over (P rows / 128, Q rows / BN)
  int splits;            // K splits (= cluster size when SPLIT)
  const float* sx;       // [M] token scales
  const int32_t* zx;     // [M] activation zero points, or null (symmetric)
  const float* sw;       // [N] channel scales
  const int32_t* wsum;   // [N] weight code sums (needed when zx != null)
  const void* bias;      // [N] out dtype, or null
  const void* residual;  // [M, N] out dtype, or null
  void* out;             // [M, N] out dtype, or null
  int32_t* raw;          // [M, N] int32 accumulators, or null
  int out_dtype;
  int vec_out;           // 1: out rows allow 16-byte vector stores of 16-column groups
  // direct-load kernels: operand base pointers, packed row length and row counts
  const uint8_t* P;
  const uint8_t* Q;
  int kbytes;
  int rowsP, rowsQ;
  // output placement: out[m * ld_out + col_off + n] in every buffer outs[0..n_outs)
  // (outs[0] == out; more than one buffer = the same tile stored to the peer
  // GPUs of a column-parallel group). residual uses the same indexing.
  int64_t ld_out;
  int col_off;
  int n_outs;
  void* outs[8];
};

constexpr int kGemmThreads = 448;
constexpr int kExpandWarps = 8;
constexpr int kExpandThreads = kExpandWarps * 32;

__device__ __forceinline__ float epi_scale(int32_t acc, float s_row, float s_col) {
  return __fmul_rn(__fmul_rn(__int2float_rn(acc), s_row), s_col);
}

__device__ __forceinline__ float load_as_float(const void* p, int64_t idx, int dtype) {
  if (dtype == kOutBF16) return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[idx]);
  if (dtype == kOutF16) return __half2float(reinterpret_cast<const __half*>(p)[idx]);
  return reinterpret_cast<const float*>(p)[idx];
}

__device__ __forceinline__ void store_from_float(void* p, int64_t idx, int dtype, float v) {
  if (dtype == kOutBF16)
    reinterpret_cast<__nv_bfloat16*>(p)[idx] = __float2bfloat16_rn(v);
  else if (dtype == kOutF16)
    reinterpret_cast<__half*>(p)[idx] = __float2half_rn(v);
  else
    reinterpret_cast<float*>(p)[idx] = v;
}

// Expands one 16-byte chunk (32 nibbles) of row r into 32 bytes at logical
// K-byte offset 32c of that row in a 128B-swizzled operand tile.
__device__ __forceinline__ void expand_chunk(const uint4 w, uint8_t* tile, int r, int c) {
  constexpr uint32_t M = 0xF0F0F0F0u;
  const uint4 o0 = make_uint4((w.x << 4) & M, w.x & M, (w.y << 4) & M, w.y & M);
  const uint4 o1 = make_uint4((w.z << 4) & M, w.z & M, (w.w << 4) & M, w.w & M);
  uint8_t* rowp = tile + r * 128;
  const int sw = r & 7;
  *reinterpret_cast<uint4*>(rowp + (((2 * c) ^ sw) << 4)) = o0;
  *reinterpret_cast<uint4*>(rowp + (((2 * c + 1) ^ sw) << 4)) = o1;
}

// Epilogue for 16 consecutive accumulator columns j0..j0+15 of tile row
// `row_local`; acc[] are the true sums (already divided by 256).
template <int BN, bool SWAP>
__device__ __forceinline__ void epilogue16(const GemmParams& p, int ti, int tj, int row_local, int j0,
                                           const int32_t (&acc)[16]) {
  const bool has_bias = p.bias != nullptr, has_res = p.residual != nullptr;
  const bool asym = p.zx != nullptr;
  if constexpr (!SWAP) {
    const int m = ti * 128 + row_local;
    const int n0 = tj * BN + j0;
    if (m >= p.M) return;
    const float sxm = p.sx[m];
    const int32_t zc = asym ? 8 - p.zx[m] : 0;
    const int64_t r0 = static_cast<int64_t>(m) * p.N + n0;                 // raw index
    const int64_t o0 = static_cast<int64_t>(m) * p.ld_out + p.col_off + n0;  // out index
    const bool full = n0 + 16 <= p.N;
    if (p.raw) {
#pragma unroll
      for (int t = 0; t < 16; ++t)
        if (n0 + t < p.N) p.raw[r0 + t] = acc[t];
    }
    if (p.out) {
      float f[16];
#pragma unroll
      for (int t = 0; t < 16; ++t) {
        const int n = full ? n0 + t : min(n0 + t, p.N - 1);
        f[t] = epi_scale(asym ? acc[t] + zc * p.wsum[n] : acc[t], sxm, p.sw[n]);
        if (has_bias) f[t] = __fadd_rn(f[t], load_as_float(p.bias, n, p.out_dtype));
        if (has_res) f[t] = __fadd_rn(f[t], load_as_float(p.residual, o0 + (n - n0), p.out_dtype));
      }
      if (full && p.vec_out && p.out_dtype == kOutBF16) {
        uint32_t w[8];
#pragma unroll
        for (int t = 0; t < 8; ++t) {
          __nv_bfloat162 h2 = __floats2bfloat162_rn(f[2 * t], f[2 * t + 1]);
          w[t] = *reinterpret_cast<uint32_t*>(&h2);
        }
        for (int b = 0; b < p.n_outs; ++b) {
          uint4* dst = reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(p.outs[b]) + o0);
          dst[0] = make_uint4(w[0], w[1], w[2], w[3]);
          dst[1] = make_uint4(w[4], w[5], w[6], w[7]);
        }
      } else {
        for (int b = 0; b < p.n_outs; ++b)
#pragma unroll
          for (int t = 0; t < 16; ++t)
            if (n0 + t < p.N) store_from_float(p.outs[b], o0 + t, p.out_dtype, f[t]);
      }
    }
  } else {
    const int n = ti * 128 + row_local;
    if (n >= p.N) return;
    const float swn = p.sw[n];
    const int32_t wsn = asym ? p.wsum[n] : 0;
    const float bn = has_bias ? load_as_float(p.bias, n, p.out_dtype) : 0.f;
#pragma unroll
    for (int t = 0; t < 16; ++t) {
      const int m = tj * BN + j0 + t;
      if (m < p.M) {
        const int64_t o = static_cast<int64_t>(m) * p.ld_out + p.col_off + n;
        if (p.raw) p.raw[static_cast<int64_t>(m) * p.N + n] = acc[t];
        if (p.out) {
          const int32_t corr = asym ? acc[t] + (8 - p.zx[m]) * wsn : acc[t];
          float f = epi_scale(corr, p.sx[m], swn);
          if (has_bias) f = __fadd_rn(f, bn);
          if (has_res) f = __fadd_rn(f, load_as_float(p.residual, o, p.out_dtype));
          for (int b = 0; b < p.n_outs; ++b) store_from_float(p.outs[b], o, p.out_dtype, f);
        }
      }
    }
  }
}

// ============================================================ epilogue of the persistent kernels
// Eight epilogue warps: warp e reads TMEM lanes 32*(e & 3).. (its quadrant of
// tile rows) and columns [(e >> 2) * BN/2, +BN/2). The tile's channel scales,
// bias and weight code sums are staged once per tile in shared memory
// (double-buffered by tile parity); accumulators come out of TMEM 16 columns
// per load.
constexpr int kEpiWarps = 8;
constexpr int kEpiThreads = kEpiWarps * 32;
constexpr int kPersistThreads = 576;  // 8 epilogue + 2 control + 8 expansion warps
constexpr int kPairThreads = 576;     // pair kernel: same roles, warp 8 is the peer's relay

template <int BN>
struct EpiStage {
  float sw[2][BN];
  float bias[2][BN];
  int32_t wsum[2][BN];
};

template <int BN>
__device__ __forceinline__ void epilogue_stage(const GemmParams& p, int tj, int par, EpiStage<BN>* st, int et) {
  for (int i = et; i < BN; i += kEpiThreads) {
    const int n = tj * BN + i;
    const bool in = n < p.N;
    st->sw[par][i] = in ? p.sw[n] : 0.f;
    if (p.bias) st->bias[par][i] = in ? load_as_float(p.bias, n, p.out_dtype) : 0.f;
    if (p.zx) st->wsum[par][i] = in ? p.wsum[n] : 0;
  }
}

// SH: the accumulator holds 2^SH * sum(a * b) (8: both operands expanded as 16 * code; 4: int8
// activation codes times expanded weights).
// Multi-buffer output (the column-parallel all-gather writes every tile into every GPU's buffer):
// the warp stages 32 rows x 32 columns of bf16 (2 KB, `stg`) and then writes whole 64-byte row
// segments, four lanes per row, instead of one 32-byte piece per lane and row; peer writes over
// NVLink move in larger, fully used transfers. bf16 output, N a multiple of 32, no raw / residual.
template <int BN, int SH>
__device__ __forceinline__ void epilogue_tile_staged(const GemmParams& p, int ti, int tj, uint32_t t_row, int q, int h,
                                                     int lane, const EpiStage<BN>* st, int par, float sxm, int32_t zc,
                                                     uint8_t* stg) {
  const bool asym = p.zx != nullptr, has_bias = p.bias != nullptr;
#pragma unroll 1
  for (int c0 = h * (BN / 2); c0 < (h + 1) * (BN / 2); c0 += 32) {
    uint32_t r0[16], r1[16];
    tmem_ld16(t_row + static_cast<uint32_t>(c0), r0);
    tmem_ld16(t_row + static_cast<uint32_t>(c0 + 16), r1);
    tmem_ld_wait();
    const int n0 = tj * BN + c0;
    if (n0 >= p.N) continue;  // N is a multiple of 32: the chunk is wholly inside or outside
    uint32_t w[16];
#pragma unroll
    for (int t = 0; t < 16; ++t) {
      float f2[2];
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int c = 2 * t + e;
        int32_t a = static_cast<int32_t>(c < 16 ? r0[c] : r1[c - 16]) >> SH;
        if (asym) a += zc * st->wsum[par][c0 + c];
        float f = epi_scale(a, sxm, st->sw[par][c0 + c]);
        if (has_bias) f = __fadd_rn(f, st->bias[par][c0 + c]);
        f2[e] = f;
      }
      __nv_bfloat162 h2 = __floats2bfloat162_rn(f2[0], f2[1]);
      w[t] = *reinterpret_cast<uint32_t*>(&h2);
    }
#pragma unroll
    for (int j = 0; j < 4; ++j)  // this lane's row: four 16-byte chunks, XOR-swizzled by row
      *reinterpret_cast<uint4*>(stg + lane * 64 + ((j ^ ((lane >> 1) & 3)) << 4)) =
          make_uint4(w[4 * j], w[4 * j + 1], w[4 * j + 2], w[4 * j + 3]);
    __syncwarp();
#pragma unroll
    for (int k = 0; k < 4; ++k) {  // rows 8k .. 8k+7: four lanes per 64-byte row segment
      const int rr = 8 * k + (lane >> 2), ch = lane & 3;
      const int m = ti * 128 + q * 32 + rr;
      if (m < p.M) {
        const uint4 v = *reinterpret_cast<const uint4*>(stg + rr * 64 + ((ch ^ ((rr >> 1) & 3)) << 4));
        const int64_t o = static_cast<int64_t>(m) * p.ld_out + p.col_off + n0 + ch * 8;
        for (int b = 0; b < p.n_outs; ++b)
          *reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(p.outs[b]) + o) = v;
      }
    }
    __syncwarp();
  }
}

template <int BN, int SH = 8>
__device__ __forceinline__ void epilogue_tile(const GemmParams& p, int ti, int tj, uint32_t tmem_acc, int ew, int lane,
                                              const EpiStage<BN>* st, int par, uint8_t* stg = nullptr) {
  const int q = ew & 3, h = ew >> 2;
  const int row_local = q * 32 + lane;
  const int m = ti * 128 + row_local;
  const bool live = m < p.M;
  const uint32_t t_row = tmem_acc + (static_cast<uint32_t>(q * 32) << 16);
  const bool asym = p.zx != nullptr, has_bias = p.bias != nullptr, has_res = p.residual != nullptr;
  const float sxm = live ? p.sx[m] : 0.f;
  const int32_t zc = (asym && live) ? 8 - p.zx[m] : 0;
  if (stg != nullptr && p.n_outs > 1 && p.vec_out && p.out_dtype == kOutBF16 && p.raw == nullptr && !has_res &&
      p.N % 32 == 0) {
    epilogue_tile_staged<BN, SH>(p, ti, tj, t_row, q, h, lane, st, par, sxm, zc, stg);
    return;
  }
#pragma unroll 1
  for (int c0 = h * (BN / 2); c0 < (h + 1) * (BN / 2); c0 += 16) {
    uint32_t r[16];
    tmem_ld16(t_row + static_cast<uint32_t>(c0), r);
    tmem_ld_wait();
    if (!live) continue;
    const int n0 = tj * BN + c0;
    const int64_t o0 = static_cast<int64_t>(m) * p.ld_out + p.col_off + n0;
    const bool full = n0 + 16 <= p.N;
    if (p.raw) {
      const int64_t r0 = static_cast<int64_t>(m) * p.N + n0;
#pragma unroll
      for (int t = 0; t < 16; ++t)
        if (n0 + t < p.N) p.raw[r0 + t] = static_cast<int32_t>(r[t]) >> SH;
    }
    if (!p.out) continue;
    float f[16];
#pragma unroll
    for (int t = 0; t < 16; ++t) {
      int32_t a = static_cast<int32_t>(r[t]) >> SH;
      if (asym) a += zc * st->wsum[par][c0 + t];
      f[t] = epi_scale(a, sxm, st->sw[par][c0 + t]);
      if (has_bias) f[t] = __fadd_rn(f[t], st->bias[par][c0 + t]);
      if (has_res && (full || n0 + t < p.N)) f[t] = __fadd_rn(f[t], load_as_float(p.residual, o0 + t, p.out_dtype));
    }
    if (full && p.vec_out && p.out_dtype == kOutBF16) {
      uint4 vv[2];
#pragma unroll
      for (int v = 0; v < 2; ++v) {
        uint32_t w[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          __nv_bfloat162 h2 = __floats2bfloat162_rn(f[8 * v + 2 * u], f[8 * v + 2 * u + 1]);
          w[u] = *reinterpret_cast<uint32_t*>(&h2);
        }
        vv[v] = make_uint4(w[0], w[1], w[2], w[3]);
      }
      for (int b = 0; b < p.n_outs; ++b) {
        uint4* dst = reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(p.outs[b]) + o0);
        dst[0] = vv[0];
        dst[1] = vv[1];
      }
    } else {
      for (int b = 0; b < p.n_outs; ++b)
#pragma unroll
        for (int t = 0; t < 16; ++t)
          if (n0 + t < p.N) store_from_float(p.outs[b], o0 + t, p.out_dtype, f[t]);
    }
  }
}

// ============================================================ one tile per CTA (small M, split K)
template <int BN>
struct GemmCfg {
  static constexpr int kThreads = kGemmThreads;
  static constexpr int kRows = 128 + BN;           // P rows + Q rows per stage
  static constexpr int kRawStage = kRows * 64;      // packed int4 bytes per stage
  static constexpr int kExpP = 128 * 128;           // expanded int8 bytes, P
  static constexpr int kExpStage = kRows * 128;     // expanded int8 bytes per stage
  static constexpr int kStages = (216 * 1024) / (kRawStage + kExpStage);
  static constexpr int kRedStride = BN + 4;         // int32 words per row of the split-K exchange tile
  static constexpr int kTmemCols = BN < 32 ? 32 : BN;
  static constexpr int kBarBytes = (4 * kStages + 1) * 8 + 16;
  static constexpr int kSmemBytes = 1024 + kStages * (kRawStage + kExpStage) + kBarBytes;
  static_assert(BN % 16 == 0 && BN >= 16 && BN <= 256, "UMMA N for M=128 must be a multiple of 16 in [16,256]");
  static_assert(kStages >= 2, "pipeline needs two stages");
  static_assert(128 * kRedStride * 4 <= kStages * kExpStage, "split-K exchange tile must fit in the stage buffers");
  static_assert((kExpStage % 1024) == 0, "swizzle atoms must stay 1024-byte aligned");
};

template <int BN, bool SWAP, bool SPLIT>
__global__ void __launch_bounds__(kGemmThreads, 1)
    w4a4_gemm_tc(const __grid_constant__ CUtensorMap tmP, const __grid_constant__ CUtensorMap tmQ,
                 const GemmParams p) {
  using C = GemmCfg<BN>;
  constexpr int S = C::kStages;
  extern __shared__ uint8_t smem_dyn[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_dyn) + 1023) & ~uintptr_t(1023));
  uint8_t* exp_base = smem;
  uint8_t* raw_base = smem + S * C::kExpStage;
  uint64_t* bars = reinterpret_cast<uint64_t*>(raw_base + S * C::kRawStage);
  uint64_t* raw_full = bars;
  uint64_t* raw_empty = bars + S;
  uint64_t* exp_full = bars + 2 * S;
  uint64_t* exp_empty = bars + 3 * S;
  uint64_t* tmem_full = bars + 4 * S;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 4 * S + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tile = SPLIT ? blockIdx.x / p.splits : blockIdx.x;
  const int z = SPLIT ? static_cast<int>(cluster_ctarank()) : 0;
  const int ti = tile % p.tiles_i, tj = tile / p.tiles_i;
  const int kb0 = static_cast<int>(static_cast<int64_t>(p.kblocks) * z / p.splits);
  const int kb1 = static_cast<int>(static_cast<int64_t>(p.kblocks) * (z + 1) / p.splits);
  const int nkb = kb1 - kb0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&raw_full[s], 1);
      mbar_init(&raw_empty[s], kExpandWarps);
      mbar_init(&exp_full[s], kExpandWarps);
      mbar_init(&exp_empty[s], 1);
    }
    mbar_init(tmem_full, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 4 && lane == 0) {
    tma_prefetch_desc(&tmP);
    tma_prefetch_desc(&tmQ);
  }
  if (warp == 5) {
    tmem_alloc(tmem_slot, C::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_d = *tmem_slot;
  bool tile_ok = nkb > 0;

  if (warp == 4) {
    // ------------------------------------------------ TMA producer
    if (lane == 0) {
      int issued = 0;
      for (int i = 0; i < nkb; ++i) {
        const int s = i % S;
        const uint32_t ph = (i / S) & 1u;
        if (i >= S && !mbar_wait(&raw_empty[s], ph ^ 1u, abort_flag)) break;
        mbar_arrive_expect_tx(&raw_full[s], C::kRawStage);
        uint8_t* dst = raw_base + s * C::kRawStage;
        const int kx = (kb0 + i) * 64;
        tma_load_2d(dst, &tmP, &raw_full[s], kx, ti * 128);
        tma_load_2d(dst + 128 * 64, &tmQ, &raw_full[s], kx, tj * BN);
        ++issued;
      }
      if (*abort_flag) {
        // Let copies already in flight land before the CTA can exit.
        for (int j = issued > S ? issued - S : 0; j < issued; ++j) mbar_wait(&raw_full[j % S], (j / S) & 1u, nullptr);
      }
    }
  } else if (warp == 5) {
    // ------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = umma_idesc_i8(128, BN);
      for (int i = 0; i < nkb; ++i) {
        const int s = i % S;
        const uint32_t ph = (i / S) & 1u;
        if (!mbar_wait(&exp_full[s], ph, abort_flag)) break;
        tc_fence_after();
        const uint32_t aP = smem_u32(exp_base + s * C::kExpStage);
        const uint64_t da = umma_desc_sw128(aP);
        const uint64_t db = umma_desc_sw128(aP + C::kExpP);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          umma_i8_ss(tmem_d, da + 2 * kk, db + 2 * kk, idesc, (i > 0 || kk > 0) ? 1u : 0u);
        umma_commit(&exp_empty[s]);
      }
      umma_commit(tmem_full);
    }
  } else if (warp >= 6) {
    // ------------------------------------------------ int4 -> int8 expansion
    const int et = threadIdx.x - 6 * 32;
    for (int i = 0; i < nkb; ++i) {
      const int s = i % S;
      const uint32_t ph = (i / S) & 1u;
      if (!mbar_wait(&raw_full[s], ph, abort_flag)) break;
      if (i >= S && !mbar_wait(&exp_empty[s], ph ^ 1u, abort_flag)) break;
      const uint8_t* src = raw_base + s * C::kRawStage;
      uint8_t* dstP = exp_base + s * C::kExpStage;
      for (int u = et; u < C::kRows * 4; u += kExpandThreads) {
        const int row = u >> 2;
        const uint4 w = *reinterpret_cast<const uint4*>(src + u * 16);
        if (row < 128)
          expand_chunk(w, dstP, row, u & 3);
        else
          expand_chunk(w, dstP + C::kExpP, row - 128, u & 3);
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&raw_empty[s]);
        mbar_arrive(&exp_full[s]);
      }
    }
  }

  // ------------------------------------------------ epilogue
  const int row_local = warp * 32 + lane;  // TMEM lane == tile row (warps 0-3)
  const uint32_t t_row = tmem_d + (static_cast<uint32_t>(warp * 32) << 16);
  if (warp < 4) {
    if (!mbar_wait(tmem_full, 0, abort_flag)) tile_ok = false;
    if (*abort_flag) tile_ok = false;
    tile_ok = __all_sync(0xffffffffu, tile_ok);
    tc_fence_after();
  }
  if constexpr (!SPLIT) {
    if (warp < 4 && tile_ok) {
      for (int j0 = 0; j0 < BN; j0 += 16) {
        uint32_t r[16];
        tmem_ld16(t_row + j0, r);
        tmem_ld_wait();
        int32_t acc[16];
#pragma unroll
        for (int t = 0; t < 16; ++t) acc[t] = static_cast<int32_t>(r[t]) >> 8;
        epilogue16<BN, SWAP>(p, ti, tj, row_local, j0, acc);
      }
    }
  } else {
    // Split K: every CTA of the cluster stages its partial tile (true sums) in its shared memory;
    // then the tile's (row, 16-column) chunks are dealt out round-robin over the CTAs, and each CTA
    // sums its chunks over all partials through DSMEM (the loads of one chunk are independent) and
    // runs the epilogue on them with all of its threads.
    int32_t* red = reinterpret_cast<int32_t*>(exp_base);
    if (warp < 4 && tile_ok) {
      for (int j0 = 0; j0 < BN; j0 += 16) {
        uint32_t r[16];
        tmem_ld16(t_row + j0, r);
        tmem_ld_wait();
        int4* dst = reinterpret_cast<int4*>(red + row_local * C::kRedStride + j0);
#pragma unroll
        for (int q = 0; q < 4; ++q)
          dst[q] = make_int4(static_cast<int>(r[4 * q]) >> 8, static_cast<int>(r[4 * q + 1]) >> 8,
                             static_cast<int>(r[4 * q + 2]) >> 8, static_cast<int>(r[4 * q + 3]) >> 8);
      }
    }
    __syncwarp();
    cluster_sync();
    constexpr int kChunksPerRow = BN / 16;
    const int nsplit = p.splits;
    for (int item = z + nsplit * static_cast<int>(threadIdx.x); item < 128 * kChunksPerRow;
         item += nsplit * static_cast<int>(blockDim.x)) {
      const int row = item / kChunksPerRow, j0 = (item % kChunksPerRow) * 16;
      const uint32_t local = smem_u32(red + row * C::kRedStride + j0);
      int32_t acc[16];
#pragma unroll
      for (int t = 0; t < 16; ++t) acc[t] = 0;
      // up to four partials per batch: all of a batch's remote loads are issued before any sum, so a
      // batch costs one DSMEM round trip
#pragma unroll
      for (int q0 = 0; q0 < 8; q0 += 4) {
        if (q0 < nsplit) {
          int4 x[4][4];
#pragma unroll
          for (int qq = 0; qq < 4; ++qq) {
            if (q0 + qq < nsplit) {
              const uint32_t src = dsmem_map(local, static_cast<uint32_t>(q0 + qq));
#pragma unroll
              for (int v = 0; v < 4; ++v) x[qq][v] = dsmem_ld_v4(src + 16 * v);
            } else {
#pragma unroll
              for (int v = 0; v < 4; ++v) x[qq][v] = make_int4(0, 0, 0, 0);
            }
          }
#pragma unroll
          for (int qq = 0; qq < 4; ++qq)
#pragma unroll
            for (int v = 0; v < 4; ++v) {
              acc[4 * v] += x[qq][v].x;
              acc[4 * v + 1] += x[qq][v].y;
              acc[4 * v + 2] += x[qq][v].z;
              acc[4 * v + 3] += x[qq][v].w;
            }
        }
      }
      epilogue16<BN, SWAP>(p, ti, tj, row, j0, acc);
    }
    __syncwarp();
    cluster_sync();  // no CTA leaves while a peer may still read its partial tile
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 5) {
    // All MMAs of this CTA must have retired before TMEM is released.
    if (lane == 0) mbar_wait(tmem_full, 0, nullptr);
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_d, C::kTmemCols);
  }
}

// ============================================================ persistent (large M)
template <int BN>
struct PCfg {
  static constexpr int kRows = 128 + BN;
  static constexpr int kRawStage = kRows * 64;
  static constexpr int kExpP = 128 * 128;
  static constexpr int kExpStage = kRows * 128;
  static constexpr int ES = BN >= 256 ? 2 : 3;                                   // expanded stages
  static constexpr int RS = (216 * 1024 - ES * kExpStage) / kRawStage;           // raw (TMA) stages
  static constexpr int UPT = kRows * 4 / kExpandThreads;                         // 16-B chunks per thread
  static constexpr int kTmemCols = 2 * BN;                                       // two accumulators
  static constexpr int kBarBytes = (2 * RS + 2 * ES + 5) * 8 + 16;
  static constexpr int kEpiBytes = static_cast<int>(sizeof(EpiStage<BN>));
  static constexpr int kSmemBytes = 1024 + ES * kExpStage + RS * kRawStage + kBarBytes + kEpiBytes;
  static_assert(BN == 128 || BN == 256, "persistent kernel uses N tiles of 128 or 256");
  static_assert(RS >= 2, "need two raw stages");
  static_assert(kRows * 4 % kExpandThreads == 0, "expansion chunks must divide evenly");
  static_assert(kSmemBytes <= 227 * 1024, "shared memory budget");
};

template <int BN>
__global__ void __launch_bounds__(kPersistThreads, 1)
    w4a4_gemm_persistent(const __grid_constant__ CUtensorMap tmP, const __grid_constant__ CUtensorMap tmQ,
                         const GemmParams p) {
  using C = PCfg<BN>;
  constexpr int RS = C::RS, ES = C::ES;
  extern __shared__ uint8_t smem_dyn[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_dyn) + 1023) & ~uintptr_t(1023));
  uint8_t* exp_base = smem;
  uint8_t* raw_base = smem + ES * C::kExpStage;
  uint64_t* bars = reinterpret_cast<uint64_t*>(raw_base + RS * C::kRawStage);
  uint64_t* raw_full = bars;
  uint64_t* raw_empty = bars + RS;
  uint64_t* exp_full = bars + 2 * RS;
  uint64_t* exp_empty = bars + 2 * RS + ES;
  uint64_t* tmem_full = bars + 2 * RS + 2 * ES;   // [2]
  uint64_t* tmem_empty = tmem_full + 2;           // [2]
  uint64_t* mma_done = tmem_full + 4;             // [1]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  EpiStage<BN>* est = reinterpret_cast<EpiStage<BN>*>(reinterpret_cast<uint8_t*>(bars) + C::kBarBytes);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ntiles = p.tiles_i * p.tiles_j;
  const int kb_n = p.kblocks;

  if (threadIdx.x == 0) {
    for (int s = 0; s < RS; ++s) {
      mbar_init(&raw_full[s], 1);
      mbar_init(&raw_empty[s], kExpandWarps);
    }
    for (int s = 0; s < ES; ++s) {
      mbar_init(&exp_full[s], kExpandWarps);
      mbar_init(&exp_empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tmem_full[a], 1);
      mbar_init(&tmem_empty[a], kEpiWarps);
    }
    mbar_init(mma_done, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 8 && lane == 0) {
    tma_prefetch_desc(&tmP);
    tma_prefetch_desc(&tmQ);
  }
  if (warp == 9) {
    tmem_alloc(tmem_slot, C::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 8) {
    // ------------------------------------------------ TMA producer
    if (lane == 0) {
      int g = 0;
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < ntiles; tile += gridDim.x) {
        const int ti = tile % p.tiles_i, tj = tile / p.tiles_i;
        for (int kb = 0; kb < kb_n; ++kb, ++g) {
          const int s = g % RS;
          if (g >= RS && !mbar_wait(&raw_empty[s], ((g / RS) & 1u) ^ 1u, abort_flag)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&raw_full[s], C::kRawStage);
          uint8_t* dst = raw_base + s * C::kRawStage;
          tma_load_2d(dst, &tmP, &raw_full[s], kb * 64, ti * 128);
          tma_load_2d(dst + 128 * 64, &tmQ, &raw_full[s], kb * 64, tj * BN);
        }
      }
      if (!ok) {
        for (int j = g > RS ? g - RS : 0; j < g; ++j) mbar_wait(&raw_full[j % RS], (j / RS) & 1u, nullptr);
      }
    }
  } else if (warp == 9) {
    // ------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = umma_idesc_i8(128, BN);
      int g = 0, t = 0;
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < ntiles; tile += gridDim.x, ++t) {
        const int acc = t & 1, use = t >> 1;
        if (use > 0 && !mbar_wait(&tmem_empty[acc], (use - 1) & 1u, abort_flag)) break;
        tc_fence_after();
        const uint32_t d = tmem_base + static_cast<uint32_t>(acc * BN);
        for (int kb = 0; kb < kb_n; ++kb, ++g) {
          const int s = g % ES;
          if (!mbar_wait(&exp_full[s], (g / ES) & 1u, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t aP = smem_u32(exp_base + s * C::kExpStage);
          const uint64_t da = umma_desc_sw128(aP);
          const uint64_t db = umma_desc_sw128(aP + C::kExpP);
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            umma_i8_ss(d, da + 2 * kk, db + 2 * kk, idesc, (kb > 0 || kk > 0) ? 1u : 0u);
          umma_commit(&exp_empty[s]);
        }
        if (ok) umma_commit(&tmem_full[acc]);
      }
      umma_commit(mma_done);
    }
  } else if (warp >= 10) {
    // ------------------------------------------------ int4 -> int8 expansion
    const int et = threadIdx.x - 10 * 32;
    int g = 0;
    bool ok = true;
    for (int tile = blockIdx.x; ok && tile < ntiles; tile += gridDim.x) {
      for (int kb = 0; kb < kb_n; ++kb, ++g) {
        const int rs = g % RS, es = g % ES;
        if (!mbar_wait(&raw_full[rs], (g / RS) & 1u, abort_flag) ||
            (g >= ES && !mbar_wait(&exp_empty[es], ((g / ES) & 1u) ^ 1u, abort_flag))) {
          ok = false;
          break;
        }
        const uint8_t* src = raw_base + rs * C::kRawStage;
        uint8_t* dstP = exp_base + es * C::kExpStage;
        uint4 w[C::UPT];
#pragma unroll
        for (int i = 0; i < C::UPT; ++i) w[i] = *reinterpret_cast<const uint4*>(src + (et + i * kExpandThreads) * 16);
#pragma unroll
        for (int i = 0; i < C::UPT; ++i) {
          const int u = et + i * kExpandThreads;
          const int row = u >> 2;
          if (i * kExpandThreads < 128 * 4)  // compile-time: chunk block i lies in P or in Q
            expand_chunk(w[i], dstP, row, u & 3);
          else
            expand_chunk(w[i], dstP + C::kExpP, row - 128, u & 3);
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&raw_empty[rs]);
          mbar_arrive(&exp_full[es]);
        }
      }
    }
  } else {
    // ------------------------------------------------ epilogue (warps 0-7)
    int t = 0;
    for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x, ++t) {
      const int acc_i = t & 1, use = t >> 1;
      const int ti = tile % p.tiles_i, tj = tile / p.tiles_i;
      epilogue_stage<BN>(p, tj, t & 1, est, threadIdx.x);
      bool ok = mbar_wait(&tmem_full[acc_i], use & 1u, abort_flag);
      // staged scales become visible and all eight warps agree on continuing
      ok = named_bar_and(1, kEpiThreads, ok && !*abort_flag);
      if (!ok) break;
      tc_fence_after();
      epilogue_tile<BN>(p, ti, tj, tmem_base + static_cast<uint32_t>(acc_i * BN), warp, lane, est, t & 1);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tmem_empty[acc_i]);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 9) {
    if (lane == 0) mbar_wait(mma_done, 0, nullptr);  // every issued MMA has retired
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, C::kTmemCols);
  }
}

// ============================================================ persistent, CTA pairs
// Tile 256 x 256 computed by the two CTAs of a cluster pair with
// tcgen05.mma.cta_group::2 (M = 256, N = 256, K = 32 per instruction). CTA r
// of the pair stages, expands and holds rows [128r, 128r+128) of the A tile
// and rows [128r, 128r+128) of the B tile; its TMEM receives rows
// [128r, 128r+128) x all 256 columns of the accumulator. Per SM this halves
// the B-operand bytes that TMA writes, the expansion reads and writes, and
// the tensor cores read from shared memory, for the same MMA throughput.
// Only the leader (rank 0) issues MMAs. Each CTA's expansion warps arrive on
// their own `exp_full`; the peer's relay thread then issues a 16-byte bulk
// copy into the leader whose bytes complete on the leader's `exp_full` of the
// same stage (armed by the leader's first expansion warp), so the leader
// learns of both halves without a blocking remote arrival. The leader's
// commits arrive on `exp_empty`, `tmem_full` and `mma_done` of both CTAs; both
// CTAs' epilogue warps arrive on the leader's `tmem_empty`.
//   warps 0-7 epilogue, warp 8 TMEM allocator + MMA issuer (leader) or relay
//   (peer), warp 9 TMA producer, warps 10-17 expansion (576 threads).
#ifndef DSCQ_PAIR_EXP_GROUPS
#define DSCQ_PAIR_EXP_GROUPS 2
#endif
struct PairCfg {
  static constexpr int BN = 256;                    // pair tile N (128 B rows per CTA)
  // The 8 expansion warps form GROUPS groups that expand alternate K blocks, so the load ->
  // expand -> proxy fence -> arrive latency of one K block overlaps the next one's.
  static constexpr int GROUPS = DSCQ_PAIR_EXP_GROUPS;
  static constexpr int kGroupWarps = kExpandWarps / GROUPS;
  static constexpr int kGroupThreads = kGroupWarps * 32;
  static constexpr int kRows = 256;                 // 128 A rows + 128 B rows per CTA
  static constexpr int kRawStage = kRows * 64;      // 16 KB
  static constexpr int kExpHalf = 128 * 128;        // 16 KB
  static constexpr int kExpStage = kRows * 128;     // 32 KB
  // A pair MMA (256 x 256 x 32) takes ~128 cycles; 4 expanded stages cover the leader -> peer ->
  // leader signalling of a stage, the rest of the budget is raw (TMA) stages.
  static constexpr int ES = 4;
  static constexpr int RS = (212 * 1024 - ES * kExpStage - static_cast<int>(sizeof(EpiStage<256>))) / kRawStage;
  static constexpr int UPT = kRows * 4 / kGroupThreads;  // 16-byte chunks per thread and K block
  static constexpr int kTmemCols = 2 * BN;          // two accumulators x 256 columns
  // barriers, TMEM slot and abort flag, then 16-byte signal slots: [ES] copy targets + 1 source
  static constexpr int kSigOff = ((2 * RS + 2 * ES + 5) * 8 + 8 + 15) / 16 * 16;
  static constexpr int kBarBytes = kSigOff + (ES + 1) * 16;
  static constexpr int kEpiBytes = static_cast<int>(sizeof(EpiStage<BN>));
  static constexpr int kStgBytes = kEpiWarps * 2048;  // staged multi-buffer epilogue, 2 KB per warp
  static constexpr int kSmemBytes = 1024 + ES * kExpStage + RS * kRawStage + kBarBytes + kEpiBytes + kStgBytes;
  static_assert(kSmemBytes <= 227 * 1024, "shared memory budget");
};

__global__ void __launch_bounds__(kPairThreads, 1)
    w4a4_gemm_pair(const __grid_constant__ CUtensorMap tmP, const __grid_constant__ CUtensorMap tmQ,
                   const GemmParams p) {
  using C = PairCfg;
  constexpr int RS = C::RS, ES = C::ES, BN = C::BN;
  extern __shared__ uint8_t smem_dyn[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_dyn) + 1023) & ~uintptr_t(1023));
  uint8_t* exp_base = smem;
  uint8_t* raw_base = smem + ES * C::kExpStage;
  uint64_t* bars = reinterpret_cast<uint64_t*>(raw_base + RS * C::kRawStage);
  uint64_t* raw_full = bars;
  uint64_t* raw_empty = bars + RS;
  uint64_t* exp_full = bars + 2 * RS;            // both: 8 expansion warps; leader: + 16 bytes from the peer
  uint64_t* exp_empty = bars + 2 * RS + ES;      // both: leader's MMA commit
  uint64_t* tmem_full = bars + 2 * RS + 2 * ES;  // [2] both: leader's MMA commit
  uint64_t* tmem_empty = tmem_full + 2;          // [2] leader: 2 x 4 epilogue warps
  uint64_t* mma_done = tmem_full + 4;            // [1] both
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  uint8_t* sig = reinterpret_cast<uint8_t*>(bars) + C::kSigOff;  // [ES] copy targets, then the source
  EpiStage<BN>* est = reinterpret_cast<EpiStage<BN>*>(reinterpret_cast<uint8_t*>(bars) + C::kBarBytes);
  uint8_t* stg_base = reinterpret_cast<uint8_t*>(bars) + C::kBarBytes + C::kEpiBytes;  // 16-byte aligned

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int pair = static_cast<int>(blockIdx.x) >> 1, npairs = static_cast<int>(gridDim.x) >> 1;
  const int tiles_i2 = (p.M + 255) / 256;
  const int ntiles = tiles_i2 * p.tiles_j;
  const int kb_n = p.kblocks;

  if (threadIdx.x == 0) {
    for (int s = 0; s < RS; ++s) {
      mbar_init(&raw_full[s], 1);
      mbar_init(&raw_empty[s], C::kGroupWarps);
    }
    for (int s = 0; s < ES; ++s) {
      // the expansion warps of one group; on the leader its first warp also arms 16 bytes for the
      // peer's signal
      mbar_init(&exp_full[s], C::kGroupWarps);
      mbar_init(&exp_empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tmem_full[a], 1);
      mbar_init(&tmem_empty[a], 2 * kEpiWarps);
    }
    mbar_init(mma_done, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 9 && lane == 0) {
    tma_prefetch_desc(&tmP);
    tma_prefetch_desc(&tmQ);
  }
  if (warp == 8) {
    tmem_alloc_pair(tmem_slot, C::kTmemCols);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncwarp();
  cluster_sync();  // barriers of both CTAs initialised, TMEM of the pair allocated
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  // leader's barriers as seen from this CTA (cluster addresses)
  const uint32_t exp_full_ldr = dsmem_map(smem_u32(exp_full), 0);
  const uint32_t tmem_empty_ldr = dsmem_map(smem_u32(tmem_empty), 0);
  const uint32_t sig_ldr = dsmem_map(smem_u32(sig), 0);

  if (warp == 9) {
    // ------------------------------------------------ TMA producer (both CTAs, own halves)
    if (lane == 0) {
      int g = 0;
      bool ok = true;
      for (int tile = pair; ok && tile < ntiles; tile += npairs) {
        const int ti2 = tile % tiles_i2, tj = tile / tiles_i2;
        for (int kb = 0; kb < kb_n; ++kb, ++g) {
          const int s = g % RS;
          if (g >= RS && !mbar_wait(&raw_empty[s], ((g / RS) & 1u) ^ 1u, abort_flag)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&raw_full[s], C::kRawStage);
          uint8_t* dst = raw_base + s * C::kRawStage;
          tma_load_2d(dst, &tmP, &raw_full[s], kb * 64, ti2 * 256 + static_cast<int>(rank) * 128);
          tma_load_2d(dst + 128 * 64, &tmQ, &raw_full[s], kb * 64, tj * BN + static_cast<int>(rank) * 128);
        }
      }
      if (!ok) {
        for (int j = g > RS ? g - RS : 0; j < g; ++j) mbar_wait(&raw_full[j % RS], (j / RS) & 1u, nullptr);
      }
    }
  } else if (warp == 8) {
    // ------------------------------------------------ relay (peer): once the peer's 8 expansion warps
    // have arrived locally for a K block, a 16-byte bulk copy into the leader completes on the
    // leader's exp_full of that stage. The copy is issued without waiting (a cluster-scope release
    // arrival would hold this thread ~0.7-1 us per K block).
    if (!leader && lane == 0) {
      const int total = (ntiles > pair ? (ntiles - pair + npairs - 1) / npairs : 0) * kb_n;
      int g = 0;
      for (; g < total; ++g) {
        const int s = g % ES;
        if (!mbar_wait(&exp_full[s], (g / ES) & 1u, abort_flag)) break;
        bulk_copy_to_peer(sig_ldr + static_cast<uint32_t>(s * 16), sig + ES * 16, 16,
                          exp_full_ldr + static_cast<uint32_t>(s * 8));
      }
      if (g < total) {  // aborted: copies already issued land within microseconds
        const uint64_t t0 = globaltimer_ns();
        while (globaltimer_ns() - t0 < 100000ull) {
        }
      }
    }
    // ------------------------------------------------ MMA issuer (leader only)
    if (leader && lane == 0) {
      constexpr uint32_t idesc = umma_idesc_i8(256, BN);
      const uint32_t exp_empty_peer = dsmem_map(smem_u32(exp_empty), 1);
      const uint32_t tmem_full_peer = dsmem_map(smem_u32(tmem_full), 1);
      int g = 0, t = 0;
      bool ok = true;
      for (int tile = pair; ok && tile < ntiles; tile += npairs, ++t) {
        const int acc = t & 1, use = t >> 1;
        if (use > 0 && !mbar_wait_cluster(&tmem_empty[acc], (use - 1) & 1u, abort_flag)) break;
        tc_fence_after();
        const uint32_t d = tmem_base + static_cast<uint32_t>(acc * BN);
        for (int kb = 0; kb < kb_n; ++kb, ++g) {
          const int s = g % ES;
          if (!mbar_wait_cluster(&exp_full[s], (g / ES) & 1u, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t aP = smem_u32(exp_base + s * C::kExpStage);
          const uint64_t da = umma_desc_sw128(aP);
          const uint64_t db = umma_desc_sw128(aP + C::kExpHalf);
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            umma_i8_ss_pair(d, da + 2 * kk, db + 2 * kk, idesc, (kb > 0 || kk > 0) ? 1u : 0u);
          umma_commit_pair(smem_u32(&exp_empty[s]));
          umma_commit_pair(exp_empty_peer + static_cast<uint32_t>(s * 8));
        }
        if (ok) {
          umma_commit_pair(smem_u32(&tmem_full[acc]));
          umma_commit_pair(tmem_full_peer + static_cast<uint32_t>(acc * 8));
        }
      }
      umma_commit_pair(smem_u32(mma_done));
      umma_commit_pair(dsmem_map(smem_u32(mma_done), 1));
    }
  } else if (warp >= 10) {
    // ------------------------------------------------ int4 -> int8 expansion (both CTAs)
    const int grp = (warp - 10) / C::kGroupWarps;                    // group: K blocks g = grp (mod GROUPS)
    const int et = threadIdx.x - 10 * 32 - grp * C::kGroupThreads;  // thread within the group
    const bool armer = leader && (warp - 10) % C::kGroupWarps == 0;
    int g = 0;
    bool ok = true;
    for (int tile = pair; ok && tile < ntiles; tile += npairs) {
      for (int kb = 0; kb < kb_n; ++kb, ++g) {
        if (g % C::GROUPS != grp) continue;
        const int rs = g % RS, es = g % ES;
        if (!mbar_wait(&raw_full[rs], (g / RS) & 1u, abort_flag) ||
            (g >= ES && !mbar_wait_cluster(&exp_empty[es], ((g / ES) & 1u) ^ 1u, abort_flag))) {
          ok = false;
          break;
        }
        const uint8_t* src = raw_base + rs * C::kRawStage;
        uint8_t* dstA = exp_base + es * C::kExpStage;
        uint4 w[C::UPT];
#pragma unroll
        for (int i = 0; i < C::UPT; ++i)
          w[i] = *reinterpret_cast<const uint4*>(src + (et + i * C::kGroupThreads) * 16);
#pragma unroll
        for (int i = 0; i < C::UPT; ++i) {
          const int u = et + i * C::kGroupThreads;
          const int row = u >> 2;
          if (i * C::kGroupThreads < 128 * 4)
            expand_chunk(w[i], dstA, row, u & 3);
          else
            expand_chunk(w[i], dstA + C::kExpHalf, row - 128, u & 3);
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&raw_empty[rs]);
          if (armer)
            mbar_arrive_expect_tx(&exp_full[es], 16);  // + the 16 bytes the peer's relay copies in
          else
            mbar_arrive(&exp_full[es]);
        }
      }
    }
  } else {
    // ------------------------------------------------ epilogue (warps 0-7, both CTAs)
    int t = 0;
    for (int tile = pair; tile < ntiles; tile += npairs, ++t) {
      const int acc_i = t & 1, use = t >> 1;
      const int ti2 = tile % tiles_i2, tj = tile / tiles_i2;
      const int ti = ti2 * 2 + static_cast<int>(rank);  // 128-row block of this CTA
      epilogue_stage<BN>(p, tj, t & 1, est, threadIdx.x);
      bool ok = mbar_wait_cluster(&tmem_full[acc_i], use & 1u, abort_flag);
      ok = named_bar_and(1, kEpiThreads, ok && !*abort_flag);
      if (!ok) break;
      tc_fence_after();
      epilogue_tile<BN>(p, ti, tj, tmem_base + static_cast<uint32_t>(acc_i * BN), warp, lane, est, t & 1,
                        stg_base + warp * 2048);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(tmem_empty_ldr + static_cast<uint32_t>(acc_i * 8));
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 8 && lane == 0) mbar_wait_cluster(mma_done, 0, nullptr);  // the pair's MMAs into this CTA retired
  __syncwarp();
  cluster_sync();  // no CTA leaves while its peer may still address its shared memory
  if (warp == 8) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, C::kTmemCols);
  }
}

// ============================================================ persistent, direct loads
// Same tile loop, TMEM double buffering and epilogue as w4a4_gemm_persistent,
// but the expansion warps read the packed int4 bytes straight from L2 with
// 16-byte non-allocating loads, two K blocks ahead in registers, instead of
// staging them through shared memory with TMA. Shared memory then only holds
// the expanded int8 stages (written once by the expansion warps, read once by
// the tensor cores): half the shared-memory traffic per K block.
//   warps 0-3 epilogue, warp 4 TMEM allocator + MMA issuer, warps 5-12 expansion.
template <int BN>
struct LCfg {
  static constexpr int kThreads = 544;  // 8 epilogue + 1 MMA + 8 expansion warps
  static constexpr int kRows = 128 + BN;
  static constexpr int kExpP = 128 * 128;
  static constexpr int kExpStage = kRows * 128;
  static constexpr int ES = (200 * 1024) / kExpStage;
  static constexpr int UPT = kRows * 4 / kExpandThreads;
  static constexpr int D = 2;                      // K blocks in flight per expansion thread
  static constexpr int kTmemCols = 2 * BN;
  static constexpr int kBarBytes = (2 * ES + 5) * 8 + 16;
  static constexpr int kEpiBytes = static_cast<int>(sizeof(EpiStage<BN>));
  static constexpr int kSmemBytes = 1024 + ES * kExpStage + kBarBytes + kEpiBytes;
  static_assert(BN == 128 || BN == 256, "direct-load kernel uses N tiles of 128 or 256");
  static_assert(ES >= 2, "need two expanded stages");
  static_assert(kRows * 4 % kExpandThreads == 0, "expansion chunks must divide evenly");
};

__device__ __forceinline__ uint4 ldg_nc_v4(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

template <int BN>
__global__ void __launch_bounds__(544, 1) w4a4_gemm_persistent_ldg(const GemmParams p) {
  using C = LCfg<BN>;
  constexpr int ES = C::ES, UPT = C::UPT, D = C::D;
  extern __shared__ uint8_t smem_dyn[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_dyn) + 1023) & ~uintptr_t(1023));
  uint8_t* exp_base = smem;
  uint64_t* bars = reinterpret_cast<uint64_t*>(exp_base + ES * C::kExpStage);
  uint64_t* exp_full = bars;
  uint64_t* exp_empty = bars + ES;
  uint64_t* tmem_full = bars + 2 * ES;  // [2]
  uint64_t* tmem_empty = tmem_full + 2;  // [2]
  uint64_t* mma_done = tmem_full + 4;    // [1]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  EpiStage<BN>* est = reinterpret_cast<EpiStage<BN>*>(reinterpret_cast<uint8_t*>(bars) + C::kBarBytes);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ntiles = p.tiles_i * p.tiles_j;
  const int kb_n = p.kblocks;

  if (threadIdx.x == 0) {
    for (int s = 0; s < ES; ++s) {
      mbar_init(&exp_full[s], kExpandWarps);
      mbar_init(&exp_empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tmem_full[a], 1);
      mbar_init(&tmem_empty[a], kEpiWarps);
    }
    mbar_init(mma_done, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 8) {
    tmem_alloc(tmem_slot, C::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 8) {
    // ------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = umma_idesc_i8(128, BN);
      int g = 0, t = 0;
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < ntiles; tile += gridDim.x, ++t) {
        const int acc = t & 1, use = t >> 1;
        if (use > 0 && !mbar_wait(&tmem_empty[acc], (use - 1) & 1u, abort_flag)) break;
        tc_fence_after();
        const uint32_t d = tmem_base + static_cast<uint32_t>(acc * BN);
        for (int kb = 0; kb < kb_n; ++kb, ++g) {
          const int s = g % ES;
          if (!mbar_wait(&exp_full[s], (g / ES) & 1u, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t aP = smem_u32(exp_base + s * C::kExpStage);
          const uint64_t da = umma_desc_sw128(aP);
          const uint64_t db = umma_desc_sw128(aP + C::kExpP);
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            umma_i8_ss(d, da + 2 * kk, db + 2 * kk, idesc, (kb > 0 || kk > 0) ? 1u : 0u);
          umma_commit(&exp_empty[s]);
        }
        if (ok) umma_commit(&tmem_full[acc]);
      }
      umma_commit(mma_done);
    }
  } else if (warp >= 9) {
    // ------------------------------------------------ load + expand (8 warps)
    const int et = threadIdx.x - 9 * 32;
    const int my_tiles = (ntiles - static_cast<int>(blockIdx.x) + static_cast<int>(gridDim.x) - 1) /
                         static_cast<int>(gridDim.x);
    const int total = my_tiles > 0 ? my_tiles * kb_n : 0;
    // per-thread chunk coordinates (fixed across K blocks): row within P/Q and 16-byte column
    auto load = [&](int g, uint4 (&w)[UPT]) {
      if (g >= total) return;
      const int tl = g / kb_n, kb = g - tl * kb_n;
      const int tile = static_cast<int>(blockIdx.x) + tl * static_cast<int>(gridDim.x);
      const int ti = tile % p.tiles_i, tj = tile / p.tiles_i;
#pragma unroll
      for (int i = 0; i < UPT; ++i) {
        const int u = et + i * kExpandThreads;
        const int row = u >> 2, c = u & 3;
        const int kbyte = kb * 64 + c * 16;
        const bool inP = i * kExpandThreads < 128 * 4;  // compile-time per i
        const int grow = inP ? ti * 128 + row : tj * BN + (row - 128);
        const bool valid = (inP ? grow < p.rowsP : grow < p.rowsQ) && kbyte < p.kbytes;
        const uint8_t* base = inP ? p.P : p.Q;
        w[i] = valid ? ldg_nc_v4(base + static_cast<int64_t>(grow) * p.kbytes + kbyte) : make_uint4(0, 0, 0, 0);
      }
    };
    auto expand = [&](int g, const uint4 (&w)[UPT]) -> bool {
      const int es = g % ES;
      if (g >= ES && !mbar_wait(&exp_empty[es], ((g / ES) & 1u) ^ 1u, abort_flag)) return false;
      uint8_t* dstP = exp_base + es * C::kExpStage;
#pragma unroll
      for (int i = 0; i < UPT; ++i) {
        const int u = et + i * kExpandThreads;
        const int row = u >> 2;
        if (i * kExpandThreads < 128 * 4)
          expand_chunk(w[i], dstP, row, u & 3);
        else
          expand_chunk(w[i], dstP + C::kExpP, row - 128, u & 3);
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&exp_full[es]);
      return true;
    };
    uint4 w0[UPT], w1[UPT];
    static_assert(D == 2, "register ring is unrolled for two K blocks");
    load(0, w0);
    load(1, w1);
    for (int g = 0; g < total; g += 2) {
      if (!expand(g, w0)) break;
      load(g + 2, w0);
      if (g + 1 >= total) break;
      if (!expand(g + 1, w1)) break;
      load(g + 3, w1);
    }
  } else {
    // ------------------------------------------------ epilogue (warps 0-7)
    int t = 0;
    for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x, ++t) {
      const int acc_i = t & 1, use = t >> 1;
      const int ti = tile % p.tiles_i, tj = tile / p.tiles_i;
      epilogue_stage<BN>(p, tj, t & 1, est, threadIdx.x);
      bool ok = mbar_wait(&tmem_full[acc_i], use & 1u, abort_flag);
      ok = named_bar_and(1, kEpiThreads, ok && !*abort_flag);
      if (!ok) break;
      tc_fence_after();
      epilogue_tile<BN>(p, ti, tj, tmem_base + static_cast<uint32_t>(acc_i * BN), warp, lane, est, t & 1);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tmem_empty[acc_i]);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 8) {
    if (lane == 0) mbar_wait(mma_done, 0, nullptr);
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, C::kTmemCols);
  }
}

}  // namespace dscq
