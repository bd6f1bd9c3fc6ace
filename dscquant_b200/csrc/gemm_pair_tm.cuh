// W4A4 GEMM on CTA pairs with the activations in tensor memory.
//
// The pair kernels are bound by the shared-memory pipe: per K block each CTA
// moves ~96 KB through it (TMA writes, expansion reads and writes, MMA operand
// reads), and the kernel time follows that byte count across variants. Here the
// expanded activations never enter shared memory: the expansion warps write
// them straight into TMEM with tcgen05.st (one lane per activation row, 4 int8
// per 32-bit column), and tcgen05.mma.cta_group::2 reads its A operand from
// TMEM. Per K block and CTA the shared memory then moves the packed activations
// once in and once out (8 + 8 KB), the packed weights in and out (6 + 6 KB), the
// expanded weights in and out of the MMA (12 + 12 KB): 52 KB for a 256 x 192 x
// 128 step instead of 96 KB for 256 x 256 x 128.
//
// TMEM (512 columns per CTA): two accumulators of 192 columns (the epilogue of
// one tile overlaps the main loop of the next) and four 32-column activation
// stages. Hence 256 x 192 output tiles (N = 192: 96 weight rows per CTA).
//
// The packed activation tile arrives by TMA with the 64-byte swizzle, so that
// thread-per-row reads (row r = TMEM lane r) hit distinct banks: logical
// 16-byte chunk c of row r sits at chunk c ^ ((r >> 1) & 3).
//
// Roles (576 threads): warps 0-7 epilogue; warp 8 TMEM allocation + MMA issuer
// (leader) or relay (peer); warp 9 TMA; warps 10-17 expansion: each takes half
// of the K block of the 32 activation rows of its TMEM lane quadrant, plus a
// share of the weight rows into shared memory. The peer signals its expansion
// to the leader with a 16-byte bulk copy completing on the leader's exp_full
// (as in w4a4_gemm_pair). All waits bounded.
#pragma once
#include "gemm_w4a4.cuh"

namespace dscq {

struct PairTmCfg {
  static constexpr int BN = 192;                       // pair tile N
  static constexpr int kBRows = BN / 2;                // weight rows per CTA
  static constexpr int kRawA = 128 * 64;               // packed activations per K block (64-byte swizzle)
  static constexpr int kRawB = kBRows * 64;            // packed weights per K block
  static constexpr int kRawStage = kRawA + kRawB;      // 14 KB (a multiple of 1024)
  static constexpr int kExpStage = kBRows * 128;       // expanded weights, 128-byte swizzle (12 KB)
  static constexpr int ES = 4;                         // operand stages: TMEM activations + smem weights
  static constexpr int kAccCols = BN;                  // one accumulator
  static constexpr int kACol0 = 2 * BN;                // first TMEM column of the activation stages
  static constexpr int kAStageCols = 32;               // 128 int8 per row = 32 columns
  static constexpr int kTmemCols = 512;
  static constexpr int kEpiBytes = static_cast<int>(sizeof(EpiStage<BN>));
  static constexpr int RS_FIT = (212 * 1024 - ES * kExpStage - kEpiBytes) / kRawStage;
  static constexpr int RS = RS_FIT < 8 ? RS_FIT : 8;   // packed (TMA) stages
  static constexpr int kSigOff = ((2 * RS + 2 * ES + 5) * 8 + 8 + 15) / 16 * 16;
  static constexpr int kBarBytes = kSigOff + (ES + 1) * 16;
  static constexpr int kSmemBytes = 1024 + ES * kExpStage + RS * kRawStage + kBarBytes + kEpiBytes;
  static_assert(kACol0 + ES * kAStageCols <= kTmemCols, "TMEM budget");
  static_assert(kRawStage % 1024 == 0 && kExpStage % 1024 == 0, "stages keep swizzle alignment");
  static_assert(RS >= 3, "raw stages");
  static_assert(kSmemBytes <= 227 * 1024, "shared memory budget");
};

__global__ void __launch_bounds__(kPairThreads, 1)
    w4a4_gemm_pair_tm(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                      const GemmParams p) {
  using C = PairTmCfg;
  constexpr int RS = C::RS, ES = C::ES, BN = C::BN;
  extern __shared__ uint8_t smem_dyn[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_dyn) + 1023) & ~uintptr_t(1023));
  uint8_t* exp_base = smem;                       // [ES] expanded weights
  uint8_t* raw_base = smem + ES * C::kExpStage;   // [RS] packed activations + packed weights
  uint64_t* bars = reinterpret_cast<uint64_t*>(raw_base + RS * C::kRawStage);
  uint64_t* raw_full = bars;
  uint64_t* raw_empty = bars + RS;
  uint64_t* exp_full = bars + 2 * RS;            // both: 8 expansion warps; leader: + 16 bytes from the peer
  uint64_t* exp_empty = bars + 2 * RS + ES;      // both: the leader's MMA commit
  uint64_t* tmem_full = bars + 2 * RS + 2 * ES;  // [2] both: the leader's MMA commit
  uint64_t* tmem_empty = tmem_full + 2;          // [2] leader: 2 x 8 epilogue warps
  uint64_t* mma_done = tmem_full + 4;            // [1] both
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  uint8_t* sig = reinterpret_cast<uint8_t*>(bars) + C::kSigOff;  // [ES] copy targets, then the source
  EpiStage<BN>* est = reinterpret_cast<EpiStage<BN>*>(reinterpret_cast<uint8_t*>(bars) + C::kBarBytes);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int pair = static_cast<int>(blockIdx.x) >> 1, npairs = static_cast<int>(gridDim.x) >> 1;
  const int tiles_i2 = (p.M + 255) / 256;
  const int ntiles = tiles_i2 * p.tiles_j;
  const int kb_n = p.kblocks;
  const int total = (ntiles > pair ? (ntiles - pair + npairs - 1) / npairs : 0) * kb_n;

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
      mbar_init(&tmem_empty[a], 2 * kEpiWarps);
    }
    mbar_init(mma_done, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 9 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
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
  const uint32_t exp_full_ldr = dsmem_map(smem_u32(exp_full), 0);
  const uint32_t tmem_empty_ldr = dsmem_map(smem_u32(tmem_empty), 0);
  const uint32_t sig_ldr = dsmem_map(smem_u32(sig), 0);

  if (warp == 9) {
    // ------------------------------------------------ TMA producer (both CTAs, own halves)
    if (lane == 0) {
      int g = 0;
      bool ok = true;
      for (; g < total; ++g) {
        const int s = g % RS;
        if (g >= RS && !mbar_wait(&raw_empty[s], ((g / RS) & 1u) ^ 1u, abort_flag)) {
          ok = false;
          break;
        }
        const int tile = pair + (g / kb_n) * npairs, kb = g % kb_n;
        const int ti2 = tile % tiles_i2, tj = tile / tiles_i2;
        uint8_t* dst = raw_base + s * C::kRawStage;
        mbar_arrive_expect_tx(&raw_full[s], C::kRawStage);
        tma_load_2d(dst, &tmA, &raw_full[s], kb * 64, ti2 * 256 + static_cast<int>(rank) * 128);
        tma_load_2d(dst + C::kRawA, &tmB, &raw_full[s], kb * 64, tj * BN + static_cast<int>(rank) * C::kBRows);
      }
      if (!ok) {
        for (int j = g > RS ? g - RS : 0; j < g; ++j) mbar_wait(&raw_full[j % RS], (j / RS) & 1u, nullptr);
      }
    }
  } else if (warp == 8) {
    // ------------------------------------------------ relay (peer): a 16-byte bulk copy into the leader
    // completes on the leader's exp_full once the peer's 8 expansion warps have arrived locally
    if (!leader && lane == 0) {
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
        const uint32_t d = tmem_base + static_cast<uint32_t>(acc * C::kAccCols);
        for (int kb = 0; kb < kb_n; ++kb, ++g) {
          const int s = g % ES;
          if (!mbar_wait_cluster(&exp_full[s], (g / ES) & 1u, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_t = tmem_base + static_cast<uint32_t>(C::kACol0 + s * C::kAStageCols);
          const uint64_t db = umma_desc_sw128(smem_u32(exp_base + s * C::kExpStage));
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            umma_i8_ts_pair(d, a_t + static_cast<uint32_t>(8 * kk), db + 2 * kk, idesc, (kb > 0 || kk > 0) ? 1u : 0u);
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
    // ------------------------------------------------ expansion (both CTAs)
    // Activations: warp w covers TMEM lane quadrant q = w % 4 (rows 32q .. 32q+31, one row per thread)
    // and half h of the K block (k 64h .. 64h+63 = columns 16h .. 16h+15 of the stage), in the byte
    // order of expand_chunk (each 16 packed bytes -> o0, o1). Weights: 96 rows x 4 chunks of 16 bytes
    // over the 256 threads into the 128-byte-swizzled shared-memory stage.
    const int q = warp & 3, h = (warp - 10) >> 2;
    const int arow = q * 32 + lane;
    const uint32_t a_lane = static_cast<uint32_t>(q * 32) << 16;
    const int et = threadIdx.x - 10 * 32;
    const bool two = et + kExpandThreads < C::kBRows * 4;  // warp-uniform: warps 10-13
    constexpr uint32_t MK = 0xF0F0F0F0u;
    for (int g = 0; g < total; ++g) {
      const int rs = g % RS, es = g % ES;
      if (!mbar_wait(&raw_full[rs], (g / RS) & 1u, abort_flag) ||
          (g >= ES && !mbar_wait_cluster(&exp_empty[es], ((g / ES) & 1u) ^ 1u, abort_flag)))
        break;
      const uint8_t* src = raw_base + rs * C::kRawStage;
      const uint8_t* ap = src + arow * 64;
      const int swz = (arow >> 1) & 3;  // 64-byte swizzle of the packed activation tile
      const uint4 a0 = *reinterpret_cast<const uint4*>(ap + (((2 * h) ^ swz) << 4));
      const uint4 a1 = *reinterpret_cast<const uint4*>(ap + (((2 * h + 1) ^ swz) << 4));
      const uint8_t* bsrc = src + C::kRawA;
      const uint4 wb0 = *reinterpret_cast<const uint4*>(bsrc + et * 16);
      const uint4 wb1 = two ? *reinterpret_cast<const uint4*>(bsrc + (et + kExpandThreads) * 16) : make_uint4(0, 0, 0, 0);
      uint32_t r[16];
      r[0] = (a0.x << 4) & MK;
      r[1] = a0.x & MK;
      r[2] = (a0.y << 4) & MK;
      r[3] = a0.y & MK;
      r[4] = (a0.z << 4) & MK;
      r[5] = a0.z & MK;
      r[6] = (a0.w << 4) & MK;
      r[7] = a0.w & MK;
      r[8] = (a1.x << 4) & MK;
      r[9] = a1.x & MK;
      r[10] = (a1.y << 4) & MK;
      r[11] = a1.y & MK;
      r[12] = (a1.z << 4) & MK;
      r[13] = a1.z & MK;
      r[14] = (a1.w << 4) & MK;
      r[15] = a1.w & MK;
      tmem_st16(tmem_base + a_lane + static_cast<uint32_t>(C::kACol0 + es * C::kAStageCols + 16 * h), r);
      uint8_t* dstB = exp_base + es * C::kExpStage;
      expand_chunk(wb0, dstB, et >> 2, et & 3);
      if (two) expand_chunk(wb1, dstB, (et + kExpandThreads) >> 2, et & 3);
      tmem_st_wait();
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&raw_empty[rs]);
        if (leader && warp == 10)
          mbar_arrive_expect_tx(&exp_full[es], 16);  // + the 16 bytes the peer's relay copies in
        else
          mbar_arrive(&exp_full[es]);
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
      epilogue_tile<BN>(p, ti, tj, tmem_base + static_cast<uint32_t>(acc_i * C::kAccCols), warp, lane, est, t & 1);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(tmem_empty_ldr + static_cast<uint32_t>(acc_i * 8));
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 8 && lane == 0) mbar_wait_cluster(mma_done, 0, nullptr);  // the pair's MMAs into this CTA retired
  __syncwarp();
  cluster_sync();  // no CTA leaves while its peer may still address its shared memory or TMEM
  if (warp == 8) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, C::kTmemCols);
  }
}

}  // namespace dscq
