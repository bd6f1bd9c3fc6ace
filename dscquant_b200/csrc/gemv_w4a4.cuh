// Small-M W4A4 GEMM ("decode", M <= 32 tokens), the role of decode_gemm in
// the reference (kernel/w4a4.cu:135-154), HBM-bound on the weight bytes.
//
// Each CTA owns 16 weight rows (output channels) and splits K across its 8
// warps. A warp streams its weight rows straight from HBM into registers with
// 16-byte loads (a pass's weight and activation loads all issued before its
// first MMA), expands the nibbles in registers (byte = nibble << 4, int8
// value 16*code, as in the tcgen05 kernels) and issues legacy
// mma.sync.m16n8k32 int8 MMAs: A = 16
// weight rows x 32 k, B = 32 k x 8 tokens, int32 accumulators. Any k order
// shared by both operands gives the same dot product, so thread q of a quad
// takes bytes [16q, 16q+16) of every 64-byte (128-element) row chunk and uses
// one 32-bit word of it per k step: every fragment comes from one contiguous
// 16-byte load. Partial sums of the 8 warps meet in shared memory; warp 0
// applies the epilogue (same arithmetic as epilogue16).
#pragma once
#include "gemm_w4a4.cuh"

namespace dscq {

__device__ __forceinline__ void mma_s8_16832(int (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint4 ldg_stream_v4(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

constexpr int kGemvWarps = 8;
constexpr int kGemvChunksPerWarp = 4;  // 128-element K chunks per warp and pass, loaded up front

// NT = number of 8-token MMA column tiles (M <= 8 * NT). Pass p of warp w covers the K chunks
// c = (p * 8 + w) * 4 + i, i < 4: all eight warps share every pass, and each pass issues the
// weight AND activation loads of its four chunks before the first MMA.
template <int NT>
__global__ void __launch_bounds__(kGemvWarps * 32) w4a4_gemv(const GemmParams p) {
  __shared__ int red[kGemvWarps][16][8 * NT];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, q = lane & 3;
  const int n0 = blockIdx.x * 16;  // weight rows of this CTA
  const int kchunks = (p.kbytes + 63) / 64;
  const uint8_t* W = p.Q;  // weights [N, kbytes]
  const uint8_t* X = p.P;  // activations [M, kbytes]

  int acc[NT][4];
#pragma unroll
  for (int t = 0; t < NT; ++t) acc[t][0] = acc[t][1] = acc[t][2] = acc[t][3] = 0;

  const int rA = n0 + g, rB = n0 + g + 8;
  const bool okA = rA < p.N, okB = rB < p.N;
  constexpr int CPW = kGemvChunksPerWarp;
  for (int c_base = warp * CPW; c_base < kchunks; c_base += kGemvWarps * CPW) {
    uint4 wa[CPW], wb[CPW], xv[CPW][NT];
#pragma unroll
    for (int i = 0; i < CPW; ++i) {
      const int c = c_base + i;
      const int off = c * 64 + q * 16;
      const bool inK = c < kchunks && off < p.kbytes;
      wa[i] = (inK && okA) ? ldg_stream_v4(W + static_cast<int64_t>(rA) * p.kbytes + off) : make_uint4(0, 0, 0, 0);
      wb[i] = (inK && okB) ? ldg_stream_v4(W + static_cast<int64_t>(rB) * p.kbytes + off) : make_uint4(0, 0, 0, 0);
#pragma unroll
      for (int t = 0; t < NT; ++t) {
        const int m = t * 8 + g;
        xv[i][t] = (inK && m < p.M)
                       ? __ldg(reinterpret_cast<const uint4*>(X + static_cast<int64_t>(m) * p.kbytes + off))
                       : make_uint4(0, 0, 0, 0);
      }
    }
#pragma unroll
    for (int i = 0; i < CPW; ++i) {
      // Lanes without bytes in a ragged last chunk hold zeros; every lane runs every mma.sync.
      if (c_base + i >= kchunks) continue;  // warp-uniform
      const uint32_t wA[4] = {wa[i].x, wa[i].y, wa[i].z, wa[i].w};
      const uint32_t wB[4] = {wb[i].x, wb[i].y, wb[i].z, wb[i].w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        constexpr uint32_t MSK = 0xF0F0F0F0u;
        const uint32_t a[4] = {(wA[j] << 4) & MSK, (wB[j] << 4) & MSK, wA[j] & MSK, wB[j] & MSK};
#pragma unroll
        for (int t = 0; t < NT; ++t) {
          const uint32_t xw = j == 0 ? xv[i][t].x : (j == 1 ? xv[i][t].y : (j == 2 ? xv[i][t].z : xv[i][t].w));
          mma_s8_16832(acc[t], a, (xw << 4) & MSK, xw & MSK);
        }
      }
    }
  }
  // partial sums: acc[t] = D[row g / g+8][token 8t + 2q, 2q+1]
#pragma unroll
  for (int t = 0; t < NT; ++t) {
    red[warp][g][8 * t + 2 * q] = acc[t][0];
    red[warp][g][8 * t + 2 * q + 1] = acc[t][1];
    red[warp][g + 8][8 * t + 2 * q] = acc[t][2];
    red[warp][g + 8][8 * t + 2 * q + 1] = acc[t][3];
  }
  __syncthreads();
  const bool asym = p.zx != nullptr, has_bias = p.bias != nullptr, has_res = p.residual != nullptr;
  for (int e = threadIdx.x; e < 16 * 8 * NT; e += kGemvWarps * 32) {
    const int r = e / (8 * NT), m = e % (8 * NT);
    const int n = n0 + r;
    if (n >= p.N || m >= p.M) continue;
    int s = 0;
#pragma unroll
    for (int w = 0; w < kGemvWarps; ++w) s += red[w][r][m];
    s >>= 8;
    if (p.raw) p.raw[static_cast<int64_t>(m) * p.N + n] = s;
    if (!p.out) continue;
    const int64_t o = static_cast<int64_t>(m) * p.ld_out + p.col_off + n;
    float f = epi_scale(asym ? s + (8 - p.zx[m]) * p.wsum[n] : s, p.sx[m], p.sw[n]);
    if (has_bias) f = __fadd_rn(f, load_as_float(p.bias, n, p.out_dtype));
    if (has_res) f = __fadd_rn(f, load_as_float(p.residual, o, p.out_dtype));
    for (int b = 0; b < p.n_outs; ++b) store_from_float(p.outs[b], o, p.out_dtype, f);
  }
}

}  // namespace dscq
