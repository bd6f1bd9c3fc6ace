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

}  // namespace dscq
