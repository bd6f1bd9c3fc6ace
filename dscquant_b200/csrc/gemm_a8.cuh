// Persistent W4A4 GEMM with int8 activation codes ("A8"): the activations come
// from the rotate+quantize kernel as one int8 code per element, [M, KP] with a
// 16-byte aligned row stride, instead of packed nibbles. TMA loads each
// 128-row x 128-byte K block of them with the 128-byte swizzle, which is the
// canonical K-major UMMA operand layout, straight into shared memory; only the
// packed int4 weights go through the expansion warps (byte = nibble << 4, int8
// value 16 * code, natural k order). The MMA accumulates 16 * sum(a * b) and the
// epilogue shifts by 4. Compared with the packed-activation kernel this drops
// a third of the expansion work and of the shared-memory traffic per K block
// (activations: one 16 KB TMA write instead of 8 KB TMA + 8 KB read + 16 KB
// write), for one extra byte per activation element written by the quantizer.
//
// Roles as in w4a4_gemm_persistent (576 threads): warps 0-7 epilogue, warp 8
// TMA (activation ring + weight ring), warp 9 TMEM + MMA, warps 10-17 weight
// expansion. Two TMEM accumulators of BN columns; all waits bounded.
#pragma once
#include "gemm_w4a4.cuh"

namespace dscq {

// Expands one 16-byte chunk (32 nibbles, k = 32c .. 32c+31) of weight row r
// into 32 int8 bytes (16 * code) in natural k order at K-byte offset 32c of
// that row of a 128-byte-swizzled tile. (The packed-activation kernels use a
// cheaper expansion whose byte order interleaves even and odd k; that is only
// valid when both operands share it, and here the activations arrive from TMA
// in natural order.)
__device__ __forceinline__ uint32_t nib_pair_spread(uint32_t x, uint32_t sel) {
  const uint32_t t = __byte_perm(x, 0u, sel);  // [b, b, b', b']
  return ((t << 4) & 0x00F000F0u) | (t & 0xF000F000u);
}
__device__ __forceinline__ void expand_chunk_natural(const uint4 w, uint8_t* tile, int r, int c) {
  const uint4 o0 = make_uint4(nib_pair_spread(w.x, 0x1100u), nib_pair_spread(w.x, 0x3322u),
                              nib_pair_spread(w.y, 0x1100u), nib_pair_spread(w.y, 0x3322u));
  const uint4 o1 = make_uint4(nib_pair_spread(w.z, 0x1100u), nib_pair_spread(w.z, 0x3322u),
                              nib_pair_spread(w.w, 0x1100u), nib_pair_spread(w.w, 0x3322u));
  uint8_t* rowp = tile + r * 128;
  const int sw = r & 7;
  *reinterpret_cast<uint4*>(rowp + (((2 * c) ^ sw) << 4)) = o0;
  *reinterpret_cast<uint4*>(rowp + (((2 * c + 1) ^ sw) << 4)) = o1;
}

template <int BN>
struct A8Cfg {
  static constexpr int kAStage = 128 * 128;   // int8 activations, one K block
  static constexpr int kRawStage = BN * 64;   // packed weights, one K block
  static constexpr int kExpStage = BN * 128;  // expanded weights, one K block
  static constexpr int kEpiBytes = static_cast<int>(sizeof(EpiStage<BN>));
  static constexpr int ES = 2;
  static constexpr int RA = 4;
  static constexpr int RS_FIT = (212 * 1024 - ES * kExpStage - RA * kAStage - kEpiBytes) / kRawStage;
  static constexpr int RS = RS_FIT < 8 ? RS_FIT : 8;
  static constexpr int UPT = BN * 4 / kExpandThreads;  // 16-byte raw chunks per expansion thread
  static constexpr int kTmemCols = 2 * BN;
  static constexpr int kBarBytes = (2 * RA + 2 * RS + 2 * ES + 5) * 8 + 16;
  static constexpr int kSmemBytes = 1024 + RA * kAStage + ES * kExpStage + RS * kRawStage + kBarBytes + kEpiBytes;
  static_assert(BN == 128 || BN == 256, "A8 kernel uses N tiles of 128 or 256");
  static_assert(RS >= 2, "need two raw stages");
  static_assert(BN * 4 % kExpandThreads == 0, "expansion chunks must divide evenly");
  static_assert(kSmemBytes <= 227 * 1024, "shared memory budget");
};

template <int BN>
__global__ void __launch_bounds__(kPersistThreads, 1)
    w4a4_gemm_a8(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmQ,
                 const GemmParams p) {
  using C = A8Cfg<BN>;
  constexpr int RS = C::RS, ES = C::ES, RA = C::RA;
  extern __shared__ uint8_t smem_dyn[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_dyn) + 1023) & ~uintptr_t(1023));
  uint8_t* a_base = smem;
  uint8_t* exp_base = a_base + RA * C::kAStage;
  uint8_t* raw_base = exp_base + ES * C::kExpStage;
  uint64_t* bars = reinterpret_cast<uint64_t*>(raw_base + RS * C::kRawStage);
  uint64_t* a_full = bars;
  uint64_t* a_empty = a_full + RA;
  uint64_t* raw_full = a_empty + RA;
  uint64_t* raw_empty = raw_full + RS;
  uint64_t* exp_full = raw_empty + RS;
  uint64_t* exp_empty = exp_full + ES;
  uint64_t* tmem_full = exp_empty + ES;  // [2]
  uint64_t* tmem_empty = tmem_full + 2;  // [2]
  uint64_t* mma_done = tmem_full + 4;    // [1]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  EpiStage<BN>* est = reinterpret_cast<EpiStage<BN>*>(reinterpret_cast<uint8_t*>(bars) + C::kBarBytes);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ntiles = p.tiles_i * p.tiles_j;
  const int kb_n = p.kblocks;

  if (threadIdx.x == 0) {
    for (int s = 0; s < RA; ++s) {
      mbar_init(&a_full[s], 1);
      mbar_init(&a_empty[s], 1);
    }
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
    tma_prefetch_desc(&tmA);
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
    // ------------------------------------------------ TMA producer: activation and weight rings
    if (lane == 0) {
      int g = 0;
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < ntiles; tile += gridDim.x) {
        const int ti = tile % p.tiles_i, tj = tile / p.tiles_i;
        for (int kb = 0; kb < kb_n; ++kb, ++g) {
          const int sa = g % RA, sr = g % RS;
          if ((g >= RA && !mbar_wait(&a_empty[sa], ((g / RA) & 1u) ^ 1u, abort_flag)) ||
              (g >= RS && !mbar_wait(&raw_empty[sr], ((g / RS) & 1u) ^ 1u, abort_flag))) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&a_full[sa], C::kAStage);
          tma_load_2d(a_base + sa * C::kAStage, &tmA, &a_full[sa], kb * 128, ti * 128);
          mbar_arrive_expect_tx(&raw_full[sr], C::kRawStage);
          tma_load_2d(raw_base + sr * C::kRawStage, &tmQ, &raw_full[sr], kb * 64, tj * BN);
        }
      }
      if (!ok) {  // let the loads already issued land before the CTA can exit
        for (int j = g > RA ? g - RA : 0; j < g; ++j) mbar_wait(&a_full[j % RA], (j / RA) & 1u, nullptr);
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
          const int sa = g % RA, se = g % ES;
          if (!mbar_wait(&a_full[sa], (g / RA) & 1u, abort_flag) || !mbar_wait(&exp_full[se], (g / ES) & 1u, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t da = umma_desc_sw128(smem_u32(a_base + sa * C::kAStage));
          const uint64_t db = umma_desc_sw128(smem_u32(exp_base + se * C::kExpStage));
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            umma_i8_ss(d, da + 2 * kk, db + 2 * kk, idesc, (kb > 0 || kk > 0) ? 1u : 0u);
          umma_commit(&a_empty[sa]);
          umma_commit(&exp_empty[se]);
        }
        if (ok) umma_commit(&tmem_full[acc]);
      }
      umma_commit(mma_done);
    }
  } else if (warp >= 10) {
    // ------------------------------------------------ weight int4 -> int8 expansion
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
        uint8_t* dst = exp_base + es * C::kExpStage;
        uint4 w[C::UPT];
#pragma unroll
        for (int i = 0; i < C::UPT; ++i) w[i] = *reinterpret_cast<const uint4*>(src + (et + i * kExpandThreads) * 16);
#pragma unroll
        for (int i = 0; i < C::UPT; ++i) {
          const int u = et + i * kExpandThreads;
          expand_chunk_natural(w[i], dst, u >> 2, u & 3);
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
      ok = named_bar_and(1, kEpiThreads, ok && !*abort_flag);
      if (!ok) break;
      tc_fence_after();
      epilogue_tile<BN, 4>(p, ti, tj, tmem_base + static_cast<uint32_t>(acc_i * BN), warp, lane, est, t & 1);
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

// ============================================================ CTA pairs with int8 activation codes
// 256 x 256 output tiles on a cluster of two CTAs issuing tcgen05.mma.cta_group::2 (M = 256), as in
// w4a4_gemm_pair, but with int8 activation codes: each CTA's 128 activation rows of a K block
// arrive by a cta_group::2 TMA load whose bytes complete on the LEADER's a_full barrier, so the
// activation half needs neither expansion nor a relayed arrival. Only the 128 weight rows of
// each CTA are expanded (natural k order, 16 * code). The peer's relay thread forwards the
// completion of its expansion with a 16-byte shared-to-shared bulk copy into the leader whose
// bytes complete on the leader's exp_full: unlike a cluster-scope release arrival, which holds
// the issuing thread ~0.7-1 us, the copy is issued without waiting, so one relay keeps up with
// every K block. Per K block and CTA the shared memory moves 16 KB (activation TMA)
// + 8 KB (weight TMA) + 8 KB read / 16 KB written by the expansion + 32 KB of MMA operand reads,
// against 96 KB in the packed-activation pair kernel.
//
// Roles (608 threads): warps 0-7 epilogue; warp 8 MMA issuer (leader) or relay (peer); warp 9
// activation TMA; warps 10-17 weight expansion; warp 18 weight TMA.
constexpr int kPairA8Threads = 608;

#ifndef DSCQ_PAIR_A8_ES
#define DSCQ_PAIR_A8_ES 5
#endif
#ifndef DSCQ_PAIR_A8_RS
#define DSCQ_PAIR_A8_RS 7
#endif

template <int ES_, int RS_>
struct PairA8Cfg {
  static constexpr int BN = 256;
  static constexpr int ES = ES_;                       // operand stages (activations + expanded weights)
  static constexpr int RS = RS_;                       // packed weight stages
  static constexpr int kAStage = 128 * 128;            // this CTA's 128 activation rows x 128 K (int8)
  static constexpr int kBStage = 128 * 128;            // this CTA's 128 weight rows x 128 K (expanded)
  static constexpr int kStage = kAStage + kBStage;
  static constexpr int kRawStage = 128 * 64;           // this CTA's 128 weight rows x 128 K (packed)
  static constexpr int UPT = 128 * 4 / kExpandThreads;  // 16-byte raw chunks per expansion thread
  static constexpr int kTmemCols = 2 * BN;
  // barriers, TMEM slot and abort flag, then 16-byte signal slots: [ES] copy targets + 1 source
  static constexpr int kSigOff = ((2 * RS + 3 * ES + 5) * 8 + 8 + 15) / 16 * 16;
  static constexpr int kBarBytes = kSigOff + (ES + 1) * 16;
  static constexpr int kEpiBytes = static_cast<int>(sizeof(EpiStage<BN>));
  static constexpr int kSmemBytes = 1024 + ES * kStage + RS * kRawStage + kBarBytes + kEpiBytes;
  static_assert(ES >= 2 && RS >= 2, "need two stages of each ring");
  static_assert(128 * 4 % kExpandThreads == 0, "expansion chunks must divide evenly");
  static_assert(kSmemBytes <= 227 * 1024, "shared memory budget");
};

template <int ES, int RS>
__global__ void __launch_bounds__(kPairA8Threads, 1)
    w4a4_gemm_pair_a8(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmQ,
                      const GemmParams p) {
  using C = PairA8Cfg<ES, RS>;
  constexpr int BN = C::BN;
  extern __shared__ uint8_t smem_dyn[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_dyn) + 1023) & ~uintptr_t(1023));
  uint8_t* stage_base = smem;  // stage s: activations at +0, expanded weights at +kAStage
  uint8_t* raw_base = smem + ES * C::kStage;
  uint64_t* bars = reinterpret_cast<uint64_t*>(raw_base + RS * C::kRawStage);
  uint64_t* raw_full = bars;
  uint64_t* raw_empty = bars + RS;
  uint64_t* a_full = bars + 2 * RS;      // leader: one armed arrival + both CTAs' activation bytes
  uint64_t* exp_full = a_full + ES;      // both: 8 expansion warps; leader: + 16 bytes copied by the peer
  uint64_t* st_empty = exp_full + ES;    // both: the leader's MMA commit
  uint64_t* tmem_full = st_empty + ES;   // [2] both: the leader's MMA commit
  uint64_t* tmem_empty = tmem_full + 2;  // [2] leader: 2 x 8 epilogue warps
  uint64_t* mma_done = tmem_full + 4;    // [1] both
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
  const int my_tiles = ntiles > pair ? (ntiles - pair + npairs - 1) / npairs : 0;
  const int total = my_tiles * kb_n;  // K blocks this pair processes

  if (threadIdx.x == 0) {
    for (int s = 0; s < RS; ++s) {
      mbar_init(&raw_full[s], 1);
      mbar_init(&raw_empty[s], kExpandWarps);
    }
    for (int s = 0; s < ES; ++s) {
      mbar_init(&a_full[s], 1);
      mbar_init(&exp_full[s], kExpandWarps);
      mbar_init(&st_empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tmem_full[a], 1);
      mbar_init(&tmem_empty[a], 2 * kEpiWarps);
    }
    mbar_init(mma_done, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 9 && lane == 0) tma_prefetch_desc(&tmA);
  if (warp == 18 && lane == 0) tma_prefetch_desc(&tmQ);
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
  const uint32_t a_full_ldr = dsmem_map(smem_u32(a_full), 0);
  const uint32_t sig_ldr = dsmem_map(smem_u32(sig), 0);

  if (warp == 9) {
    // ------------------------------------------------ activation TMA (both CTAs, bytes to the leader)
    if (lane == 0) {
      int g = 0;
      bool ok = true;
      for (; g < total; ++g) {
        const int s = g % ES;
        if (g >= ES && !mbar_wait_cluster(&st_empty[s], ((g / ES) & 1u) ^ 1u, abort_flag)) {
          ok = false;
          break;
        }
        const int tile = pair + (g / kb_n) * npairs, kb = g % kb_n;
        const int ti2 = tile % tiles_i2;
        if (leader) mbar_arrive_expect_tx(&a_full[s], 2 * C::kAStage);
        tma_load_2d_pair(stage_base + s * C::kStage, &tmA, a_full_ldr + static_cast<uint32_t>(s * 8), kb * 128,
                         ti2 * 256 + static_cast<int>(rank) * 128);
      }
      if (!ok) {
        // Loads already issued must land before the CTA can exit. The leader waits for the phases it
        // armed; the peer, whose loads complete on the leader's barriers, waits out a fixed 100 us.
        if (leader) {
          for (int j = g > ES ? g - ES : 0; j < g; ++j) mbar_wait_cluster(&a_full[j % ES], (j / ES) & 1u, nullptr);
        } else {
          const uint64_t t0 = globaltimer_ns();
          while (globaltimer_ns() - t0 < 100000ull) {
          }
        }
      }
    }
  } else if (warp == 18) {
    // ------------------------------------------------ packed weight TMA (both CTAs, own halves)
    if (lane == 0) {
      int g = 0;
      bool ok = true;
      for (; g < total; ++g) {
        const int rs = g % RS;
        if (g >= RS && !mbar_wait(&raw_empty[rs], ((g / RS) & 1u) ^ 1u, abort_flag)) {
          ok = false;
          break;
        }
        const int tile = pair + (g / kb_n) * npairs, kb = g % kb_n;
        const int tj = tile / tiles_i2;
        mbar_arrive_expect_tx(&raw_full[rs], C::kRawStage);
        tma_load_2d(raw_base + rs * C::kRawStage, &tmQ, &raw_full[rs], kb * 64,
                    tj * BN + static_cast<int>(rank) * 128);
      }
      if (!ok) {
        for (int j = g > RS ? g - RS : 0; j < g; ++j) mbar_wait(&raw_full[j % RS], (j / RS) & 1u, nullptr);
      }
    }
  } else if (warp == 8) {
    // ------------------------------------------------ relay (peer): once the peer's 8 expansion warps
    // have arrived locally for a K block, a 16-byte bulk copy into the leader completes on the
    // leader's exp_full of that stage (armed with expect_tx by the leader's first expansion warp).
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
      const uint32_t st_empty_peer = dsmem_map(smem_u32(st_empty), 1);
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
          const uint32_t par = (g / ES) & 1u;
          if (!mbar_wait_cluster(&a_full[s], par, abort_flag) || !mbar_wait_cluster(&exp_full[s], par, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t aS = smem_u32(stage_base + s * C::kStage);
          const uint64_t da = umma_desc_sw128(aS);
          const uint64_t db = umma_desc_sw128(aS + C::kAStage);
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            umma_i8_ss_pair(d, da + 2 * kk, db + 2 * kk, idesc, (kb > 0 || kk > 0) ? 1u : 0u);
          umma_commit_pair(smem_u32(&st_empty[s]));
          umma_commit_pair(st_empty_peer + static_cast<uint32_t>(s * 8));
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
    // ------------------------------------------------ weight int4 -> int8 expansion (both CTAs)
    const int et = threadIdx.x - 10 * 32;
    for (int g = 0; g < total; ++g) {
      const int rs = g % RS, s = g % ES;
      if (!mbar_wait(&raw_full[rs], (g / RS) & 1u, abort_flag) ||
          (g >= ES && !mbar_wait_cluster(&st_empty[s], ((g / ES) & 1u) ^ 1u, abort_flag)))
        break;
      const uint8_t* src = raw_base + rs * C::kRawStage;
      uint8_t* dst = stage_base + s * C::kStage + C::kAStage;
      uint4 w[C::UPT];
#pragma unroll
      for (int i = 0; i < C::UPT; ++i) w[i] = *reinterpret_cast<const uint4*>(src + (et + i * kExpandThreads) * 16);
#pragma unroll
      for (int i = 0; i < C::UPT; ++i) {
        const int u = et + i * kExpandThreads;
        expand_chunk_natural(w[i], dst, u >> 2, u & 3);
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&raw_empty[rs]);
        if (leader && warp == 10)
          mbar_arrive_expect_tx(&exp_full[s], 16);  // + the 16 bytes the peer's relay copies in
        else
          mbar_arrive(&exp_full[s]);
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
      epilogue_tile<BN, 4>(p, ti, tj, tmem_base + static_cast<uint32_t>(acc_i * BN), warp, lane, est, t & 1);
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

}  // namespace dscq
