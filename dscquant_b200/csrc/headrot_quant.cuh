// Per-head block rotation + symmetric per-row int4 quantisation: the online form of the
// reference's Rotation transform (core/transforms.py:51-52, which core/linear.py:28-37 absorbs
// into the v / o projection weights):
//
//   y[t, 128 h + e] = sum_d x[t, 128 h + d] R_h[d][e]      (R_h orthogonal, 128 x 128, fp32)
//   scale[t] = max(absmax_k(y[t, :]) * clip / 7, 1e-8),  code = rn(y * (1 / scale)) clamped
//
// R_h reaches the kernel split into two bf16 parts, R_h = hi + lo + O(2^-17 |R_h|), stored per
// head transposed (Rt[h][e][d] = R_h[d][e]: the K-major B operand), and D_h = X_h hi + X_h lo runs on
// tcgen05 (kind::f16, bf16 inputs, f32 accumulators in TMEM).
//
// A cluster of C = heads / 4 CTAs takes one 128-token tile; CTA r rotates heads 4r .. 4r+3 into
// its 512 TMEM columns (one lane per token). The row absmax spans all heads: every CTA reduces its
// 512 values per token to one partial maximum and bulk-copies its 128 partials (512 bytes) into
// every CTA of the cluster (shared::cta -> shared::cluster, complete_tx on the receiver's barrier),
// so no thread waits on a remote arrival; each CTA then takes the maximum of the C partials and
// writes the codes of its four heads. Rank 0 writes the scales.
//
// Roles (320 threads): warps 0-7 epilogue (warp w: TMEM lane quadrant w % 4, head pair w / 4),
// warp 8 TMA (two stages of X_h + hi + lo, 96 KB each), warp 9 TMEM + MMA. All waits bounded.
#pragma once
#include "ptx.cuh"
#include "rowquant.cuh"
#include "rotq_tc.cuh"

namespace dscq {

struct HeadRotParams {
  RowQuantParams p;  // x, M, ld_x, rows_out, packed / codes / scales, mode, clip
  int heads;         // K = 128 * heads
  int cluster;       // CTAs per token tile = heads / 4
};

constexpr int kHrThreads = 320;
constexpr int kHrMaxCluster = 16;
constexpr int kHrOperand = 128 * 128 * 2;   // one 128 x 128 bf16 tile (two 64-column SW128 atoms)
constexpr int kHrStage = 3 * kHrOperand;    // X_h, hi, lo
constexpr int kHrSmem = 1024 + 2 * kHrStage + (kHrMaxCluster + 2) * 128 * 4 + 256;

// bf16, both operands K-major, f32 accumulate
__host__ __device__ constexpr uint32_t umma_idesc_bf16_kk(int m, int n) {
  return (1u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(n >> 3) << 17) |
         (static_cast<uint32_t>(m >> 4) << 24);
}

__global__ void __launch_bounds__(kHrThreads, 1)
    headrot_quant(const __grid_constant__ CUtensorMap tmX, const __grid_constant__ CUtensorMap tmHi,
                  const __grid_constant__ CUtensorMap tmLo, const HeadRotParams hp) {
  const RowQuantParams& p = hp.p;
  extern __shared__ uint8_t hr_smem_dyn[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(hr_smem_dyn) + 1023) & ~uintptr_t(1023));
  uint8_t* stage = smem;                                               // [2][X | hi | lo]
  float* pm_all = reinterpret_cast<float*>(smem + 2 * kHrStage);       // [C][128]: partials of every CTA
  float* pm_loc = pm_all + kHrMaxCluster * 128;                        // [2][128]: this CTA's head pairs
  uint64_t* bars = reinterpret_cast<uint64_t*>(pm_loc + 2 * 128);
  uint64_t* full = bars;       // [2]
  uint64_t* empty = bars + 2;  // [2]
  uint64_t* tfull = bars + 4;
  uint64_t* pm_bar = bars + 5;  // C x 512 bytes from the cluster
  uint64_t* mma_done = bars + 6;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 7);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int C = hp.cluster;
  const uint32_t rank = cluster_ctarank();
  const int tile = static_cast<int>(blockIdx.x) / C;
  const int h0 = static_cast<int>(rank) * 4;

  if (threadIdx.x == 0) {
    for (int s = 0; s < 2; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(tfull, 1);
    mbar_init(pm_bar, 1);
    mbar_init(mma_done, 1);
    *abort_flag = 0;
    fence_mbar_init();
    mbar_arrive_expect_tx(pm_bar, static_cast<uint32_t>(C * 512));  // armed before any peer can copy in
  }
  if (warp == 8 && lane == 0) {
    tma_prefetch_desc(&tmX);
    tma_prefetch_desc(&tmHi);
    tma_prefetch_desc(&tmLo);
  }
  if (warp == 9) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncwarp();    // barrier.cluster is .aligned: every warp must arrive converged
  cluster_sync();  // barriers of every CTA of the cluster initialised and armed
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 8) {
    // ------------------------------------------------ TMA: X_h, hi_h, lo_h of the four heads, two stages
    if (lane == 0) {
      int j = 0;
      for (; j < 4; ++j) {
        const int s = j & 1, h = h0 + j;
        if (j >= 2 && !mbar_wait(&empty[s], 0, abort_flag)) break;
        uint8_t* st = stage + s * kHrStage;
        mbar_arrive_expect_tx(&full[s], kHrStage);
        for (int a = 0; a < 2; ++a) {
          tma_load_2d(st + a * (kHrOperand / 2), &tmX, &full[s], h * 128 + a * 64, tile * 128);
          tma_load_2d(st + kHrOperand + a * (kHrOperand / 2), &tmHi, &full[s], a * 64, h * 128);
          tma_load_2d(st + 2 * kHrOperand + a * (kHrOperand / 2), &tmLo, &full[s], a * 64, h * 128);
        }
      }
      for (int i = j > 2 ? j - 2 : 0; i < j; ++i) mbar_wait(&full[i & 1], (i >> 1) & 1u, nullptr);  // landed
    }
  } else if (warp == 9) {
    // ------------------------------------------------ MMA: D_j = X_h hi_h + X_h lo_h, TMEM columns 128 j ..
    if (lane == 0) {
      constexpr uint32_t idesc = umma_idesc_bf16_kk(128, 128);
      bool ok = true;
      for (int j = 0; ok && j < 4; ++j) {
        const int s = j & 1;
        if (!mbar_wait(&full[s], (j >> 1) & 1u, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t x0 = smem_u32(stage + s * kHrStage);
        const uint32_t d = tmem_base + static_cast<uint32_t>(j * 128);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint32_t off = static_cast<uint32_t>((kk >> 2) * (kHrOperand / 2) + (kk & 3) * 32);
          const uint64_t da = umma_desc_sw128(x0 + off);
          umma_f16_ss(d, da, umma_desc_sw128(x0 + kHrOperand + off), idesc, kk > 0 ? 1u : 0u);
          umma_f16_ss(d, da, umma_desc_sw128(x0 + 2 * kHrOperand + off), idesc, 1u);
        }
        umma_commit(&empty[s]);
      }
      if (ok) umma_commit(tfull);
      umma_commit(mma_done);
    }
  } else {
    // ------------------------------------------------ epilogue: token = TMEM lane, two heads per warp
    const int q = warp & 3, hh = warp >> 2;
    const int token = q * 32 + lane;
    const int row = tile * 128 + token;
    const uint32_t taddr = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(hh * 256);
    bool ok = mbar_wait(tfull, 0, abort_flag);
    ok = named_bar_and(1, 256, ok && !*abort_flag);
    float amax = 0.f;
    if (ok) {
      tc_fence_after();
#pragma unroll 1
      for (int c = 0; c < 256; c += 64) {
        float2 v[32];
        tmem_ld64(taddr + static_cast<uint32_t>(c), v);
        amax = fmaxf(amax, absmax64(v));
      }
    }
    pm_loc[hh * 128 + token] = amax;
    named_bar_sync(1, 256);
    if (hh == 0) pm_loc[token] = fmaxf(pm_loc[token], pm_loc[128 + token]);  // this CTA's partial
    fence_proxy_async_smem();  // the partials are read by the bulk copies (async proxy)
    named_bar_sync(1, 256);
    if (warp == 0 && lane == 0) {
      const uint32_t src_slot = smem_u32(pm_all + rank * 128);
      for (int r2 = 0; r2 < C; ++r2)
        bulk_copy_to_peer(dsmem_map(src_slot, static_cast<uint32_t>(r2)), pm_loc, 512,
                          dsmem_map(smem_u32(pm_bar), static_cast<uint32_t>(r2)));
    }
    ok = mbar_wait_cluster(pm_bar, 0, abort_flag) && ok;
    ok = __all_sync(0xffffffffu, ok);  // warp-uniform: the loads below are .sync.aligned
    if (ok) {
      float m = 0.f;
      for (int r2 = 0; r2 < C; ++r2) m = fmaxf(m, pm_all[r2 * 128 + token]);
      const float scale = fmaxf(__fdiv_rn(__fmul_rn(m, p.clip), 7.f), 1e-8f);
      const float cm = __fdiv_rn(1.f, scale);
      const float lo = p.mode == kWeightSym ? -7.f : -8.f;
      const bool clamp = p.clip < 1.f;
      // tcgen05.ld is .sync.aligned: every lane loads, only rows < rows_out store
      const bool store = row < p.rows_out;
      const int k0 = (h0 + 2 * hh) * 128;
#pragma unroll 1
      for (int c = 0; c < 256; c += 64) {
        float2 v[32];
        tmem_ld64(taddr + static_cast<uint32_t>(c), v);
        if (store) {
          uint8_t* prow = p.packed ? p.packed + static_cast<int64_t>(row) * p.ld_packed + (k0 + c) / 2 : nullptr;
          int8_t* crow = p.codes ? p.codes + static_cast<int64_t>(row) * p.ld_codes + k0 + c : nullptr;
          if (clamp)
            quant_row64<true>(v, cm, lo, false, prow, crow);
          else
            quant_row64<false>(v, cm, lo, false, prow, crow);
        }
      }
      if (store && rank == 0 && hh == 0) p.scales[row] = scale;
    }
  }

  tc_fence_before();
  __syncwarp();
  __syncthreads();
  if (warp == 9 && lane == 0) mbar_wait(mma_done, 0, nullptr);  // every issued MMA has retired
  __syncwarp();    // barrier.cluster is .aligned: every warp must arrive converged
  cluster_sync();  // no CTA leaves while a peer may still copy into its shared memory
  if (warp == 9) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 512);
  }
}

}  // namespace dscq
