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
//   * the 1024-point WHT along c (column c = 128 cb + 8 n + 2 q + e): bit 0 (e) inside the thread and
//     bits 3..6 (n) across its fragments, then one exchange through shared memory after which each
//     thread holds one (row, n) item -- the 32 column pairs that differ in q and cb -- and finishes
//     bits 1..2 and 7..9 in registers (no shuffles);
//   * row absmax over the CTA, then codes from those registers: the four q of one cb are consecutive
//     bytes, one 32-bit store (and one 8-byte store of int8 codes);
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

    // ---- WHT bits 0 (e, inside the thread) and 3..6 (n, across this thread's fragments); bits 1..2 (q, the
    // quad's lanes) and 7..9 (cb, the column blocks) are done after the exchange, in registers
#pragma unroll
    for (int n = 0; n < 16; ++n) {  // bit 0
      float t0 = acc[n][0], t1 = acc[n][1];
      acc[n][0] = t0 + t1;
      acc[n][1] = t0 - t1;
      t0 = acc[n][2];
      t1 = acc[n][3];
      acc[n][2] = t0 + t1;
      acc[n][3] = t0 - t1;
    }
#pragma unroll
    for (int h = 1; h < 16; h <<= 1)  // bits 3..6, packed over (e = 0, 1)
#pragma unroll
      for (int n = 0; n < 16; ++n)
        if (!(n & h)) {
#pragma unroll
          for (int hf = 0; hf < 2; ++hf) {
            const float2 u = make_float2(acc[n][2 * hf], acc[n][2 * hf + 1]);
            const float2 w = make_float2(acc[n + h][2 * hf], acc[n + h][2 * hf + 1]);
            const float2 s0 = __fadd2_rn(u, w), s1 = __ffma2_rn(w, make_float2(-1.f, -1.f), u);
            acc[n][2 * hf] = s0.x;
            acc[n][2 * hf + 1] = s0.y;
            acc[n + h][2 * hf] = s1.x;
            acc[n + h][2 * hf + 1] = s1.y;
          }
        }

    // ---- exchange: ys[i][c] as float2 units (c / 2 = 64 cb + 4 n + q), groups of four units permuted by
    // (i & 7) within each 64-unit block (unit 4 n + q -> 4 (n ^ (i & 7)) + q)
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

    // ---- item (i, n) = this thread: the 32 column pairs 128 cb + 8 n + 2 q + {0, 1}, cb = 0..7, q = 0..3,
    // read as 32-byte groups; WHT bits 1..2 and 7..9 in registers
    const int it_i = threadIdx.x >> 4, it_n = threadIdx.x & 15;
    const bool item_live = it_i < a;
    float2 v[8][4];
    float amax = 0.f;
    if (item_live) {
      const float2* src = y2 + it_i * 512 + 4 * (it_n ^ (it_i & 7));
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        const float4 g0 = *reinterpret_cast<const float4*>(src + c * 64);
        const float4 g1 = *reinterpret_cast<const float4*>(src + c * 64 + 2);
        v[c][0] = make_float2(g0.x, g0.y);
        v[c][1] = make_float2(g0.z, g0.w);
        v[c][2] = make_float2(g1.x, g1.y);
        v[c][3] = make_float2(g1.z, g1.w);
      }
#pragma unroll
      for (int hq = 1; hq < 4; hq <<= 1)  // bits 1..2
#pragma unroll
        for (int c = 0; c < 8; ++c)
#pragma unroll
          for (int qq = 0; qq < 4; ++qq)
            if (!(qq & hq)) {
              const float2 u = v[c][qq], w = v[c][qq + hq];
              v[c][qq] = __fadd2_rn(u, w);
              v[c][qq + hq] = __ffma2_rn(w, make_float2(-1.f, -1.f), u);
            }
#pragma unroll
      for (int hc = 1; hc < 8; hc <<= 1)  // bits 7..9
#pragma unroll
        for (int c = 0; c < 8; ++c)
          if (!(c & hc)) {
#pragma unroll
            for (int qq = 0; qq < 4; ++qq) {
              const float2 u = v[c][qq], w = v[c + hc][qq];
              v[c][qq] = __fadd2_rn(u, w);
              v[c + hc][qq] = __ffma2_rn(w, make_float2(-1.f, -1.f), u);
            }
          }
#pragma unroll
      for (int c = 0; c < 8; ++c)
#pragma unroll
        for (int qq = 0; qq < 4; ++qq) amax = fmaxf(amax, fmaxf(fabsf(v[c][qq].x), fabsf(v[c][qq].y)));
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

    // ---- codes: column pair (128 cb + 8 n + 2 q, +1) of row i is byte i * 512 + 64 cb + 4 n + q, so the
    // four q of one cb are one 32-bit word (and eight consecutive int8 codes)
    uint8_t* prow = p.packed ? p.packed + static_cast<int64_t>(row) * p.ld_packed : nullptr;
    int8_t* crow = p.codes ? p.codes + static_cast<int64_t>(row) * p.ld_codes : nullptr;
    int csum = 0;
    if (item_live) {
      const float2 cm2 = make_float2(cm, cm), magic = make_float2(12582912.f, 12582912.f);
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        uint32_t word = 0, lo8 = 0, hi8 = 0;
#pragma unroll
        for (int qq = 0; qq < 4; ++qq) {
          float2 qv = __fmul2_rn(v[c][qq], cm2);
          if (clamp) {
            qv.x = fminf(fmaxf(qv.x, lo), 7.f);
            qv.y = fminf(fmaxf(qv.y, lo), 7.f);
          }
          const float2 r = __fadd2_rn(qv, magic);
          const uint32_t c0 = __float_as_uint(r.x) & 15u, c1 = __float_as_uint(r.y) & 15u;
          word |= (c0 | (c1 << 4)) << (8 * qq);
          if (crow || p.row_sums) {
            const int s0 = static_cast<int>(c0 << 28) >> 28, s1 = static_cast<int>(c1 << 28) >> 28;
            csum += s0 + s1;
            const uint32_t pr = (static_cast<uint32_t>(s0) & 0xFFu) | ((static_cast<uint32_t>(s1) & 0xFFu) << 8);
            if (qq < 2) lo8 |= pr << (16 * qq);
            else hi8 |= pr << (16 * (qq - 2));
          }
        }
        if (prow) *reinterpret_cast<uint32_t*>(prow + it_i * 512 + c * 64 + 4 * it_n) = word;
        if (crow) *reinterpret_cast<uint2*>(crow + it_i * 1024 + c * 128 + 8 * it_n) = make_uint2(lo8, hi8);
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
