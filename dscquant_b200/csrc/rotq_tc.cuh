// Fused Hadamard rotation + symmetric per-row int4 quantisation on the
// tcgen05 tensor cores, for K = a' * 64 (a' <= 256) and bf16 input:
//
//   y = x (H' (x) H_64) / sqrt(K),  H' = H_a (x) H_(2^s) of order a',  k = i*64 + c
//
// (K = 4096: H' = H_64; K = 8192: H_128; K = 11008: the order-172 matrix;
// K = 14336: H_28 (x) H_8). Per token the row is the matrix X [a'][64]; the
// dense factor is one small GEMM D = H'^T X on the tensor cores, the 64-point
// Walsh-Hadamard transform along c then runs in registers.
//
//   * TMA (3-D map {c, i, token}, 128-byte swizzle) lands one token group's
//     X in shared memory as [token][i][64 c]: a k-by-MN operand whose 128-byte
//     rows hold 64 consecutive c of one i, i.e. the canonical MN-major layout,
//     consumed by tcgen05.mma kind::f16 without any rearrangement;
//   * H'^T (A operand, K-major, 128 rows per M tile, 128-byte swizzle) is a
//     constant of K: rotq_build_operand writes its shared-memory image to global
//     memory once per device and K, and every CTA copies it in (one bulk copy
//     per 16 KB atom, hot in L2) ahead of its first token boxes. For
//     a' <= 64 (a' = 32, 64) P = 128 / a' tokens share one MMA through a
//     block-diagonal A (k = token*a' + i), so all 128 TMEM lanes carry data;
//     a' in (128, 256] uses two M tiles;
//   * D (f32, 128 lanes x 64 columns per M tile) accumulates in TMEM, up to
//     8 token groups in flight (512 columns);
//   * epilogue: each thread owns one TMEM lane (one i' of one token) and its
//     64 columns: tcgen05.ld, 64-point WHT in registers (packed f32x2 adds),
//     row absmax over the token's lanes (shuffles + shared memory), codes by
//     the 1.5*2^23 round-half-even add, 32 contiguous packed bytes per thread.
//
// Warp roles (one CTA per SM, persistent over token groups): epilogue teams
// take token groups round-robin. A team has one warp per 32-lane block of D:
// four for M tile 0 (TMEM lane quadrants 0-3) plus, for two M tiles, one per
// quadrant holding rows of M tile 1, so every thread handles exactly one row
// of 64 values. One warp issues TMA, one owns TMEM and issues the MMAs. All
// waits are bounded.
#pragma once
#include "ptx.cuh"
#include "rowquant.cuh"

namespace dscq {

constexpr int kRqTmemCols = 512;
constexpr int kRqMaxStages = 12;
constexpr int kRqMaxTeams = 4;

struct RotqParams {
  RowQuantParams p;
  int a_base, s_log;     // H' = H_a (x) H_(2^s)
  int ap;                // a' = a_base << s_log
  int ap16;              // a' rounded up to 16: k rows of one token in the B tile
  int P;                 // tokens per MMA group (block-diagonal A when > 1)
  int mt;                // M tiles (1 or 2)
  int groups;            // ceil(rows_out / P)
  int ns;                // B stages in shared memory
  int ksteps;            // k steps of 16 per M tile
  int nkb;               // 64-wide k atoms of A per M tile
  uint32_t a_bytes;      // bytes of the A region (mt * nkb * 16 KB)
  uint32_t stage_bytes;  // P * ap16 * 128
  int log2_ap16;         // log2(ap16) when P > 1
  int nteam;             // epilogue teams
  int tw;                // warps per team
  int team_stride;       // team t owns warps [t * team_stride, t * team_stride + tw)
  int tma_warp, mma_warp;
  int mma_warp2;         // two M tiles: a second MMA issuer taking M tile 1 (-1: mma_warp issues both)
  int split;             // 1: every team takes one block of each MMA group; 0: teams take whole groups
  const uint8_t* a_op;   // global image of the A operand (a_bytes, 16-byte aligned), rotq_build_operand
};

// A operand image (exactly the shared-memory layout rotq_tc feeds to the MMA): 16-byte chunk
// u = (row * nkb + kb) * 8 + ch holds A[row][k0 .. k0+7], k0 = kb * 64 + ch * 8, row = m * 128 + r,
// at byte (m * nkb + kb) * 16384 + r * 128 + ((ch ^ (r & 7)) << 4). A[i'][i] = H'[i][i'] as bf16
// +-1 (0 outside the live i, i' < a' and, for P > 1, outside the token's diagonal block), with
// H'[i][i'] = H_a[i >> s][i' >> s] * (-1)^popc(i & i' & (2^s - 1)). One thread per chunk; runs once
// per device and K, so it reads h_a (a x a, row-major, device memory) straight from global memory.
template <int MT>
__global__ void rotq_build_operand(const RotqParams rp, const int8_t* h_a, uint8_t* out) {
  const int nkb = rp.nkb, ap = rp.ap, ap16 = rp.ap16, P = rp.P;
  const int chunks = MT * 128 * nkb * 8;
  const int s = rp.s_log, a = rp.a_base, msk = (1 << s) - 1;
  for (int u = blockIdx.x * blockDim.x + threadIdx.x; u < chunks; u += gridDim.x * blockDim.x) {
    const int ch = u & 7, rk = u >> 3;
    const int row = rk / nkb, kb = rk - row * nkb;
    const int k0 = kb * 64 + ch * 8;
    int ip, ikb;
    bool row_live;
    if (MT == 1 && P > 1) {
      const int sh = rp.log2_ap16;
      ip = row & (ap16 - 1);
      ikb = k0 & (ap16 - 1);
      row_live = ip < ap && (row >> sh) == (k0 >> sh);
    } else {
      ip = row;
      ikb = k0;
      row_live = ip < ap;
    }
    uint32_t wv[4];
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      uint32_t half[2];
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int i = ikb + 2 * t + e;
        uint32_t v = 0;
        if (row_live && i < ap) {
          bool neg = (__popc(i & ip & msk) & 1) != 0;
          if (a > 1 && h_a[(i >> s) * a + (ip >> s)] < 0) neg = !neg;
          v = neg ? 0xBF80u : 0x3F80u;  // bf16 -1 / +1
        }
        half[e] = v;
      }
      wv[t] = half[0] | (half[1] << 16);
    }
    const int m = row >> 7, r = row & 127;
    uint8_t* dst = out + (m * nkb + kb) * 16384 + r * 128 + ((ch ^ (r & 7)) << 4);
    *reinterpret_cast<uint4*>(dst) = make_uint4(wv[0], wv[1], wv[2], wv[3]);
  }
}

// 64 consecutive TMEM columns of this thread's lane as 32 float2 (natural column order).
__device__ __forceinline__ void tmem_ld64(uint32_t taddr, float2 (&u)[32]) {
  uint32_t r0[32], r1[32];
  tmem_ld32(taddr, r0);
  tmem_ld32(taddr + 32u, r1);
  tmem_ld_wait();
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    u[i] = make_float2(__uint_as_float(r0[2 * i]), __uint_as_float(r0[2 * i + 1]));
    u[16 + i] = make_float2(__uint_as_float(r1[2 * i]), __uint_as_float(r1[2 * i + 1]));
  }
}

// In-place 64-point Walsh-Hadamard transform (Sylvester order, natural index) on u[i] = (v[2i], v[2i+1]):
// one scalar stage inside each pair, five packed f32x2 stages between pairs.
__device__ __forceinline__ void wht64_regs(float2 (&u)[32]) {
#pragma unroll
  for (int i = 0; i < 32; ++i) u[i] = make_float2(u[i].x + u[i].y, u[i].x - u[i].y);
#pragma unroll
  for (int h = 1; h < 32; h <<= 1)
#pragma unroll
    for (int i = 0; i < 32; ++i)
      if (!(i & h)) {
        const float2 a = u[i], b = u[i + h];
        u[i] = __fadd2_rn(a, b);
        u[i + h] = __ffma2_rn(b, make_float2(-1.f, -1.f), a);
      }
}

// Three-operand f32 max (sm_100): half the max instructions of a two-operand chain.
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

// max |u| over the 64 values, four independent chains of three-operand maxima.
__device__ __forceinline__ float absmax64(const float2 (&u)[32]) {
  float m[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int i = 0; i < 32; ++i) m[i & 3] = fmax3(m[i & 3], fabsf(u[i].x), fabsf(u[i].y));
  return fmax3(fmaxf(m[0], m[1]), m[2], m[3]);
}

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t d;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
  return d;
}

// Codes of 64 values -> 32 packed bytes (even k in the low nibble) at prow (if
// not null); optional int8 codes at crow; returns the code sum when SUMS.
// q = v * cm is rounded half to even by adding 1.5 * 2^23 (one FFMA2 per pair without clipping:
// the fused multiply-add rounds once, so codes can differ from a separately rounded product only
// where v * cm lies within an ulp of a .5 tie); the low byte of each result's bit pattern is then
// the two's-complement code. Eight codes go to one word: byte-gather the even and the odd codes
// (PRMT) and interleave their nibbles with one shift and one select (LOP3).
template <bool SUMS, bool CLAMP>
__device__ __forceinline__ int quant_store64(const float2 (&u)[32], float cm, float lo, uint8_t* prow, int8_t* crow) {
  uint32_t w[8], ev[8], od[8];
  int csum = 0;
  const float2 cm2 = make_float2(cm, cm), magic = make_float2(12582912.f, 12582912.f);
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    uint32_t bx[4], by[4];
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      float2 r;
      if (CLAMP) {  // clip < 1: the scaled value may leave [lo, 7]; clamp before rounding
        float2 q = __fmul2_rn(u[4 * j + t], cm2);
        q.x = fminf(fmaxf(q.x, lo), 7.f);
        q.y = fminf(fmaxf(q.y, lo), 7.f);
        r = __fadd2_rn(q, magic);
      } else {
        r = __ffma2_rn(u[4 * j + t], cm2, magic);
      }
      bx[t] = __float_as_uint(r.x);
      by[t] = __float_as_uint(r.y);
      if (SUMS) csum += (static_cast<int>(bx[t] << 28) >> 28) + (static_cast<int>(by[t] << 28) >> 28);
    }
    ev[j] = prmt(prmt(bx[0], bx[1], 0x0040u), prmt(bx[2], bx[3], 0x0040u), 0x5410u);  // codes 8j, 8j+2, +4, +6
    od[j] = prmt(prmt(by[0], by[1], 0x0040u), prmt(by[2], by[3], 0x0040u), 0x5410u);  // codes 8j+1, +3, +5, +7
    uint32_t word;
    asm("lop3.b32 %0, %1, %2, %3, 0xE4;" : "=r"(word) : "r"(ev[j]), "r"(od[j] << 4), "r"(0x0F0F0F0Fu));
    w[j] = word;  // (even & 0x0F..) | ((odd << 4) & 0xF0..)
  }
  if (prow) {
    uint4* dst = reinterpret_cast<uint4*>(prow);
    dst[0] = make_uint4(w[0], w[1], w[2], w[3]);
    dst[1] = make_uint4(w[4], w[5], w[6], w[7]);
  }
  if (crow) {  // the gathered bytes already are the int8 codes: interleave even and odd
    uint4* cd = reinterpret_cast<uint4*>(crow);
#pragma unroll
    for (int j = 0; j < 4; ++j)
      cd[j] = make_uint4(prmt(ev[2 * j], od[2 * j], 0x5140u), prmt(ev[2 * j], od[2 * j], 0x7362u),
                         prmt(ev[2 * j + 1], od[2 * j + 1], 0x5140u), prmt(ev[2 * j + 1], od[2 * j + 1], 0x7362u));
  }
  return csum;
}

template <bool CLAMP>
__device__ __forceinline__ int quant_row64(const float2 (&u)[32], float cm, float lo, bool sums, uint8_t* prow,
                                           int8_t* crow) {
  return sums ? quant_store64<true, CLAMP>(u, cm, lo, prow, crow) : quant_store64<false, CLAMP>(u, cm, lo, prow, crow);
}

// Threads per CTA: one M tile: 18 warps (four teams of 4 that split each group of G = 4 blocks,
// TMA, MMA); two M tiles: up to 16 (two teams of up to 7 for a' <= 224 taking whole groups of
// G = 2 blocks, TMA, MMA).
template <int MT, int G>
struct RqThreads {
  static constexpr int value = MT == 1 ? 576 : 512;
};

template <int MT, int G>
__global__ void __launch_bounds__(RqThreads<MT, G>::value, 1)
    rotq_tc(const __grid_constant__ CUtensorMap tmX, const RotqParams rp) {
  const RowQuantParams& p = rp.p;
  extern __shared__ uint8_t rq_smem_dyn[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(rq_smem_dyn) + 1023) & ~uintptr_t(1023));
  uint8_t* a_base = smem;
  uint8_t* b_base = smem + rp.a_bytes;
  // One MMA covers G consecutive B stages (token blocks) as its N = 64 G columns (MN atoms at the
  // stage stride): an M = 128 tcgen05.mma costs about the same for N = 64 and N = 256.
  constexpr int SLOT = MT * 64 * G;              // TMEM columns per MMA group
  constexpr int S = kRqTmemCols / SLOT;          // TMEM slots (MMA groups in flight)
  uint64_t* bars = reinterpret_cast<uint64_t*>(b_base + rp.ns * rp.stage_bytes);
  uint64_t* full = bars;
  uint64_t* empty = bars + kRqMaxStages;
  uint64_t* tfull = bars + 2 * kRqMaxStages;
  uint64_t* tempty = tfull + S;
  uint64_t* done = tempty + S;
  uint64_t* aready = done + 1;  // A operand copied in
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(aready + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  float* red_max = reinterpret_cast<float*>(tmem_slot + 4);        // [team][parity][8]
  int* red_sum = reinterpret_cast<int*>(red_max + kRqMaxTeams * 16);  // [team][parity][8]

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ap = rp.ap, ap16 = rp.ap16, P = rp.P, ns = rp.ns, tw = rp.tw;

  const int groups = rp.groups;
  const int my_blocks = groups > static_cast<int>(blockIdx.x)
                            ? (groups - static_cast<int>(blockIdx.x) + static_cast<int>(gridDim.x) - 1) /
                                  static_cast<int>(gridDim.x)
                            : 0;
  // The TMA thread initialises every barrier and starts its copies before the CTA barrier, so the
  // DRAM reads overlap the TMEM allocation and the other warps' start-up: first the A operand (a
  // constant of K, prebuilt in global memory and hot in L2, needed before the first MMA), then one
  // ring's worth of token boxes (no stage can be busy yet).
  int n_pre = 0;
  if (warp == rp.tma_warp && lane == 0) {
    tma_prefetch_desc(&tmX);
    for (int s = 0; s < ns; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], rp.mma_warp2 >= 0 ? 2 : 1);  // one commit per MMA issuer
    }
    for (int s = 0; s < S; ++s) {
      mbar_init(&tfull[s], rp.mma_warp2 >= 0 ? 2 : 1);
      mbar_init(&tempty[s], rp.split ? tw * rp.nteam : tw);
    }
    mbar_init(done, rp.mma_warp2 >= 0 ? 2 : 1);
    mbar_init(aready, 1);
    *abort_flag = 0;
    fence_mbar_init();
    mbar_arrive_expect_tx(aready, rp.a_bytes);
    for (uint32_t off = 0; off < rp.a_bytes; off += 16384u) bulk_load_g2s(a_base + off, rp.a_op + off, 16384u, aready);
    n_pre = min(ns, my_blocks);
    for (int n = 0; n < n_pre; ++n) {
      const int g = static_cast<int>(blockIdx.x) + n * static_cast<int>(gridDim.x);
      mbar_arrive_expect_tx(&full[n], rp.stage_bytes);
      tma_load_3d(b_base + n * rp.stage_bytes, &tmX, &full[n], 0, 0, g * P);
    }
  }
  if (warp == rp.mma_warp) {
    tmem_alloc(tmem_slot, kRqTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const int team = warp / rp.team_stride, idx = warp % rp.team_stride;

  if (warp == rp.tma_warp) {
    // ------------------------------------------------ TMA producer: the rest of this CTA's token blocks
    if (lane == 0) {
      int n = n_pre;
      bool ok = true;
      for (int g = static_cast<int>(blockIdx.x) + n * static_cast<int>(gridDim.x); g < groups; g += gridDim.x, ++n) {
        const int s = n % ns;
        if (!mbar_wait(&empty[s], ((n / ns) & 1u) ^ 1u, abort_flag)) {  // n >= ns: the stage was used
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(&full[s], rp.stage_bytes);
        tma_load_3d(b_base + s * rp.stage_bytes, &tmX, &full[s], 0, 0, g * P);
      }
      if (!ok) {  // let the copies already issued land before the CTA can exit
        mbar_wait(aready, 0, nullptr);
        for (int j = n > ns ? n - ns : 0; j < n; ++j) mbar_wait(&full[j % ns], (j / ns) & 1u, nullptr);
      }
    }
  } else if (warp == rp.mma_warp || warp == rp.mma_warp2) {
    // ------------------------------------------------ MMA issuer(s): groups of G token blocks. Each
    // tcgen05.mma costs the issuing thread ~110 cycles whatever N, so with two M tiles (22 MMAs per
    // group at a' = 172) a second issuer takes M tile 1: K = 11008 at 2048 rows 25.6 -> 24.0 us.
    if (lane == 0) {
      constexpr uint32_t idesc = umma_idesc_bf16_bmn(128, 64 * G);
      const uint32_t a0 = smem_u32(a_base);
      bool ok = mbar_wait(aready, 0, abort_flag);
      for (int q = 0; ok && q * G < my_blocks; ++q) {
        const int slot = q % S, use = q / S, n0 = q * G;
        const int nb = min(G, my_blocks - n0);  // blocks of this group that were loaded
        if (use > 0 && !mbar_wait(&tempty[slot], (use - 1) & 1u, abort_flag)) break;
        for (int b = 0; ok && b < nb; ++b) ok = mbar_wait(&full[(n0 + b) % ns], ((n0 + b) / ns) & 1u, abort_flag);
        if (!ok) break;
        tc_fence_after();
        const uint32_t b0 = smem_u32(b_base + (n0 % ns) * rp.stage_bytes);  // ns % G == 0: contiguous stages
        const int m_lo = warp == rp.mma_warp2 ? 1 : 0;
        const int m_hi = rp.mma_warp2 >= 0 ? m_lo + 1 : MT;
        for (int m = m_lo; m < m_hi; ++m) {
          const uint32_t d = tmem_base + static_cast<uint32_t>(slot * SLOT + m * 64 * G);
          for (int ks = 0; ks < rp.ksteps; ++ks) {
            const uint64_t ad = umma_desc_sw128(a0 + (m * rp.nkb + (ks >> 2)) * 16384 + (ks & 3) * 32);
            const uint64_t bd = umma_desc_sw128_mn_atoms(b0 + ks * 2048, rp.stage_bytes);
            umma_f16_ss(d, ad, bd, idesc, ks > 0 ? 1u : 0u);
          }
        }
        for (int b = 0; b < nb; ++b) umma_commit(&empty[(n0 + b) % ns]);
        umma_commit(&tfull[slot]);
      }
      umma_commit(done);
    }
  } else if (team < rp.nteam && idx < tw) {
    // ------------------------------------------------ epilogue team member: one 32-lane block of D
    const int mtile = idx >> 2, qd = idx & 3;  // idx 0-3: M tile 0, idx 4..: M tile 1
    const int r = qd * 32 + lane;              // TMEM lane = row of the M tile
    const float lo = p.mode == kWeightSym ? -7.f : -8.f;
    const bool clamp = p.clip < 1.f;
    int ip, pr;  // i' of this thread's row, token inside the group
    bool live;
    if (MT == 1) {
      pr = r / ap16;
      ip = r % ap16;
      live = pr < P && ip < ap;
    } else {
      pr = 0;
      ip = mtile * 128 + r;
      live = ip < ap;
    }
    const int wtok = P > 1 ? (qd * 32) / ap16 : 0;  // lanes of a warp never straddle two tokens
    const int wpt = P > 1 ? ap16 / 32 : tw;        // team warps per token
    const int first_w = wtok * wpt;
    // the warps of one token meet at their own named barrier (ids 1..8): with two tokens per block,
    // each warp pair exchanges its row maximum without waiting for the team's other pair
    const int bar_id = 1 + team * 2 + wtok;
    const int bar_cnt = wpt * 32;
    float* rmax = red_max + team * 16;
    int* rsum = red_sum + team * 16;
    int it = 0;
    // split: all teams walk every group and team t takes block t of it (the group's TMEM slot is
    // freed once every team has loaded its block); otherwise team t takes groups t, t + nteam, ...
    const int q0 = rp.split ? 0 : team, qstep = rp.split ? 1 : rp.nteam;
    for (int q = q0; q * G < my_blocks; q += qstep) {
      const int slot = q % S, use = q / S, n0 = q * G;
      const int nblk = min(G, my_blocks - n0);
      bool ok = mbar_wait(&tfull[slot], use & 1u, abort_flag);
      ok = named_bar_and(bar_id, bar_cnt, ok && !*abort_flag);
      if (!ok) break;
      tc_fence_after();
      const int b_lo = rp.split ? team : 0;
      const int b_hi = rp.split ? min(team + 1, nblk) : nblk;
      if (b_lo >= b_hi) {  // no block of this group for this team: release the slot right away
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&tempty[slot]);
        continue;
      }
      for (int b = b_lo; b < b_hi; ++b, ++it) {
        const int g = blockIdx.x + (n0 + b) * gridDim.x;  // token block
        const int par = it & 1;
        float2 v[32];
        tmem_ld64(tmem_base + (static_cast<uint32_t>(qd * 32) << 16) +
                      static_cast<uint32_t>(slot * SLOT + mtile * 64 * G + b * 64),
                  v);
        if (b == b_hi - 1) {
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&tempty[slot]);  // the group's columns may be overwritten
        }
        wht64_regs(v);
        float amax = live ? absmax64(v) : 0.f;
  #pragma unroll
        for (int o = 16; o; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
        if (lane == 0) rmax[par * 8 + idx] = amax;
        named_bar_sync(bar_id, bar_cnt);
        amax = 0.f;
        for (int w = 0; w < wpt; ++w) amax = fmaxf(amax, rmax[par * 8 + first_w + w]);

        const int token = g * P + (MT == 1 ? pr : 0);
        const int wtoken = g * P + wtok;
        const float amax_y = __fmul_rn(amax, p.norm);
        const float scale = fmaxf(__fdiv_rn(__fmul_rn(amax_y, p.clip), 7.f), 1e-8f);
        const float cm = __fdiv_rn(p.norm, scale);
        int csum = 0;
        if (live && token < p.rows_out) {
          uint8_t* prow = p.packed ? p.packed + static_cast<int64_t>(token) * p.ld_packed + ip * 32 : nullptr;
          int8_t* crow = p.codes ? p.codes + static_cast<int64_t>(token) * p.ld_codes + ip * 64 : nullptr;
          csum = clamp ? quant_row64<true>(v, cm, lo, p.row_sums != nullptr, prow, crow)
                       : quant_row64<false>(v, cm, lo, p.row_sums != nullptr, prow, crow);
        }
        if (p.row_sums) {
  #pragma unroll
          for (int o = 16; o; o >>= 1) csum += __shfl_xor_sync(0xffffffffu, csum, o);
          if (lane == 0) rsum[par * 8 + idx] = csum;
          named_bar_sync(bar_id, bar_cnt);
        }
        if (idx == first_w && lane == 0 && wtoken < p.rows_out) {
          p.scales[wtoken] = scale;
          if (p.row_sums) {
            int tot = 0;
            for (int w = 0; w < wpt; ++w) tot += rsum[par * 8 + first_w + w];
            p.row_sums[wtoken] = tot;
          }
        }
      }  // blocks of the group
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == rp.mma_warp) {
    if (lane == 0) mbar_wait(done, 0, nullptr);  // every issued MMA has retired
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, kRqTmemCols);
  }
}

}  // namespace dscq
