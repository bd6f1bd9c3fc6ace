// Fused Kronecker-Hadamard rotation + symmetric per-row int4 quantisation for long rows
// K = a * 1024 with a dense +-1 factor of order a <= 32 (K = 28672: a = 28, the Llama-2-70B
// down projection), bf16 input:
//
//   y = x (H_a (x) H_1024) / sqrt(K)       index k = i*1024 + c
//
// One CTA per row at a time (persistent over rows), 16 warps:
//   * the row X [a][1024] bf16 sits in shared memory (cp.async, 16-byte chunks XOR-swizzled by
//     row so ldmatrix.trans is conflict-free; rows a..31 are zero);
//   * the dense factor goes first, on the exact bf16 inputs, as tensor-core tiles (mma.sync
//     m16n8k16 bf16 -> fp32): D = H_a^T X. Warp w owns M tile w & 1 (16 output rows i') and the
//     128-column block w >> 1, i.e. a 16 x 128 tile of D in 16 accumulator fragments;
//   * the 1024-point WHT along c: bits 0..6 (inside a column block) on the fragments -- bit 0 in
//     the thread, bits 1..2 across the lanes of a quad (shuffles), bits 3..6 across the fragments;
//     bits 7..9 (across the eight column blocks) after one exchange through shared memory, where
//     each thread takes the eight blocks' values of a (row, column pair) and finishes the
//     transform in registers;
//   * row absmax over the CTA, then codes and packed bytes straight from those registers (a
//     column pair is one byte, consecutive threads write consecutive bytes);
//   * the next row's cp.async into the input buffer starts as soon as the MMAs have read it.
#pragma once
#include "kron_quant.cuh"
#include "ptx.cuh"
#include "rowquant.cuh"

namespace dscq {

struct KronLongCfg {
  static constexpr int THREADS = 512;
  static constexpr int ROWS = 32;                    // a padded to two 16-row tiles
  static constexpr int XS_BYTES = ROWS * 2048;       // [32][1024] bf16
  static constexpr int YS_BYTES = 32 * 1024 * 4;     // [<= 32][1024] fp32 exchange
  static constexpr int SMEM = XS_BYTES + YS_BYTES + 128;
  static constexpr int ITEMS_MAX = 4;                // (row, column pair) items per thread: 32 * 64 / 512
};

// x rows of K = a * 1024 bf16; p.h_a = H_a ([a, a] +-1, row-major, device memory), 2 <= a <= 32.
__global__ void __launch_bounds__(KronLongCfg::THREADS, 1) kron_long_quant(const RowQuantParams p, int a) {
  using C = KronLongCfg;
  extern __shared__ uint8_t kl_smem[];
  uint8_t* xs = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(kl_smem) + 127) & ~uintptr_t(127));
  float* ys = reinterpret_cast<float*>(xs + C::XS_BYTES);
  __shared__ float s_max[16];
  __shared__ int s_sum[16];

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, q = lane & 3;
  const int mt = warp & 1, cb = warp >> 1;
  const int m0 = mt * 16;

  // A fragments of H_a^T for this warp's 16 output rows: A[r][cc] = H_a[k0 + cc][m0 + r]
  uint32_t afr[2][4];
#pragma unroll
  for (int kt = 0; kt < 2; ++kt) {
    const int k0 = kt * 16;
    auto pair = [&](int r, int cc) {
      return hsign_bf16(p.h_a, a, 0, k0 + cc, m0 + r) | (hsign_bf16(p.h_a, a, 0, k0 + cc + 1, m0 + r) << 16);
    };
    afr[kt][0] = pair(g, 2 * q);
    afr[kt][1] = pair(g + 8, 2 * q);
    afr[kt][2] = pair(g, 2 * q + 8);
    afr[kt][3] = pair(g + 8, 2 * q + 8);
  }
  // rows a..31 of the input buffer stay zero
  for (int i = threadIdx.x; i < (C::ROWS - a) * 128; i += C::THREADS)
    *reinterpret_cast<uint4*>(xs + (a + i / 128) * 2048 + (i % 128) * 16) = make_uint4(0, 0, 0, 0);

  const int chunks = a * 128;  // 16-byte chunks of one row of x
  auto issue = [&](int row) {
    if (row < p.M) {
      const uint8_t* src = reinterpret_cast<const uint8_t*>(p.x) + static_cast<int64_t>(row) * p.ld_x * 2;
      const uint32_t base = smem_u32(xs);
      for (int i = threadIdx.x; i < chunks; i += C::THREADS) {
        const int r = i >> 7, ch = i & 127;
        cp_async16(base + r * 2048 + ((ch ^ (r & 7)) << 4), src + i * 16);
      }
    }
    cp_async_commit();
  };

  const float lo = p.mode == kWeightSym ? -7.f : -8.f;
  const bool clamp = p.clip < 1.f;
  const int stride = gridDim.x;
  int row = blockIdx.x;
  issue(row);
  for (; row < p.rows_out; row += stride) {
    cp_async_wait<0>();
    __syncthreads();
    const bool live = row < p.M;

    // ---- dense factor H_a on the tensor cores: acc[n] = 16 x 8 tile (rows m0.., cols 128 cb + 8n..)
    float acc[16][4];
#pragma unroll
    for (int n = 0; n < 16; ++n) acc[n][0] = acc[n][1] = acc[n][2] = acc[n][3] = 0.f;
    if (live) {
      const uint32_t xb = smem_u32(xs);
      const int mi = lane >> 3, rr = lane & 7;
#pragma unroll
      for (int kt = 0; kt < 2; ++kt) {
#pragma unroll
        for (int np = 0; np < 8; ++np) {
          const int r = kt * 16 + (mi & 1) * 8 + rr;
          const int ch = cb * 16 + 2 * np + (mi >> 1);
          uint32_t b0, b1, b2, b3;
          ldsm_x4_trans(xb + r * 2048 + ((ch ^ (r & 7)) << 4), b0, b1, b2, b3);
          mma_bf16_16816(acc[2 * np], afr[kt], b0, b1);
          mma_bf16_16816(acc[2 * np + 1], afr[kt], b2, b3);
        }
      }
    }
    __syncthreads();     // every warp has read x: the buffer takes the next row
    issue(row + stride);

    // ---- WHT along the block-local column 8n + 2q + e, bits 0..6
#pragma unroll
    for (int n = 0; n < 16; ++n) {  // bit 0 (e)
      float t0 = acc[n][0], t1 = acc[n][1];
      acc[n][0] = t0 + t1;
      acc[n][1] = t0 - t1;
      t0 = acc[n][2];
      t1 = acc[n][3];
      acc[n][2] = t0 + t1;
      acc[n][3] = t0 - t1;
    }
#pragma unroll
    for (int bit = 1; bit <= 2; bit <<= 1) {  // bits 1, 2 (quad lanes)
      const float sgn = (q & bit) ? -1.f : 1.f;
#pragma unroll
      for (int n = 0; n < 16; ++n)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float o = __shfl_xor_sync(0xffffffffu, acc[n][e], bit);
          acc[n][e] = fmaf(acc[n][e], sgn, o);
        }
    }
#pragma unroll
    for (int h = 1; h < 16; h <<= 1)  // bits 3..6 (n)
#pragma unroll
      for (int n = 0; n < 16; ++n)
        if (!(n & h)) {
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float u = acc[n][e], v = acc[n + h][e];
            acc[n][e] = u + v;
            acc[n + h][e] = u - v;
          }
        }

    // ---- exchange: ys[i][c] as float2 units (c / 2) swizzled by ((i & 7) << 2) within 64-unit blocks
    float2* y2 = reinterpret_cast<float2*>(ys);
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      const int i = m0 + g + 8 * half;
      if (i < a) {
#pragma unroll
        for (int n = 0; n < 16; ++n) {
          const int unit = cb * 64 + ((4 * n + q) ^ ((i & 7) << 2));
          y2[i * 512 + unit] = make_float2(acc[n][2 * half], acc[n][2 * half + 1]);
        }
      }
    }
    __syncthreads();

    // ---- bits 7..9: item (i, pair pp) holds columns 128 j + 2 pp + {0, 1}, j = 0..7
    float2 v[C::ITEMS_MAX][8];
    float amax = 0.f;
    const int items = a * 64;
#pragma unroll
    for (int t = 0; t < C::ITEMS_MAX; ++t) {
      const int item = threadIdx.x + t * C::THREADS;
      if (item < items) {
        const int i = item >> 6, pp = item & 63;
        const int su = pp ^ ((i & 7) << 2);
#pragma unroll
        for (int j = 0; j < 8; ++j) v[t][j] = y2[i * 512 + j * 64 + su];
#pragma unroll
        for (int h = 1; h < 8; h <<= 1)
#pragma unroll
          for (int j = 0; j < 8; ++j)
            if (!(j & h)) {
              const float2 x0 = v[t][j], x1 = v[t][j + h];
              v[t][j] = __fadd2_rn(x0, x1);
              v[t][j + h] = __ffma2_rn(x1, make_float2(-1.f, -1.f), x0);
            }
#pragma unroll
        for (int j = 0; j < 8; ++j) amax = fmaxf(amax, fmaxf(fabsf(v[t][j].x), fabsf(v[t][j].y)));
      }
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    if (lane == 0) s_max[warp] = amax;
    __syncthreads();
    amax = 0.f;
#pragma unroll
    for (int w = 0; w < 16; ++w) amax = fmaxf(amax, s_max[w]);

    const float amax_y = __fmul_rn(amax, p.norm);
    const float scale = fmaxf(__fdiv_rn(__fmul_rn(amax_y, p.clip), 7.f), 1e-8f);
    const float cm = __fdiv_rn(p.norm, scale);

    // ---- codes: column pair (128 j + 2 pp, +1) of row i is byte i * 512 + 64 j + pp
    uint8_t* prow = p.packed ? p.packed + static_cast<int64_t>(row) * p.ld_packed : nullptr;
    int8_t* crow = p.codes ? p.codes + static_cast<int64_t>(row) * p.ld_codes : nullptr;
    int csum = 0;
#pragma unroll
    for (int t = 0; t < C::ITEMS_MAX; ++t) {
      const int item = threadIdx.x + t * C::THREADS;
      if (item < items) {
        const int i = item >> 6, pp = item & 63;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          float q0 = v[t][j].x * cm, q1 = v[t][j].y * cm;
          if (clamp) {
            q0 = fminf(fmaxf(q0, lo), 7.f);
            q1 = fminf(fmaxf(q1, lo), 7.f);
          }
          const uint32_t c0 = __float_as_uint(q0 + 12582912.f) & 15u;
          const uint32_t c1 = __float_as_uint(q1 + 12582912.f) & 15u;
          if (prow) prow[i * 512 + j * 64 + pp] = static_cast<uint8_t>(c0 | (c1 << 4));
          if (crow || p.row_sums) {
            const int s0 = static_cast<int>(c0 << 28) >> 28, s1 = static_cast<int>(c1 << 28) >> 28;
            csum += s0 + s1;
            if (crow) {
              crow[i * 1024 + j * 128 + 2 * pp] = static_cast<int8_t>(s0);
              crow[i * 1024 + j * 128 + 2 * pp + 1] = static_cast<int8_t>(s1);
            }
          }
        }
      }
    }
    if (p.row_sums) {
#pragma unroll
      for (int o = 16; o; o >>= 1) csum += __shfl_xor_sync(0xffffffffu, csum, o);
      if (lane == 0) s_sum[warp] = csum;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      p.scales[row] = scale;
      if (p.row_sums) {
        int tot = 0;
        for (int w = 0; w < 16; ++w) tot += s_sum[w];
        p.row_sums[row] = tot;
      }
    }
  }
  cp_async_wait<0>();
}

}  // namespace dscq
