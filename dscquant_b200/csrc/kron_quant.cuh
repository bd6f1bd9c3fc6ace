// Fused Kronecker-Hadamard rotation + symmetric per-row int4 quantisation for
// K = a' * 64 with a dense +-1 factor of order a' (K = 11008: a' = 172, the
// order-172 Hadamard matrix; K = 14336: a' = 224 = H_28 (x) H_8), bf16 input.
//
//   y = x (H' (x) H_64) / sqrt(K)       index k = i*64 + c
//
// The dense factor goes first, on the exact bf16 inputs, as tensor-core
// tiles (mma.sync m16n8k16, bf16 x bf16 -> fp32): D = H'^T X with X the row
// viewed as [a', 64]. Each warp owns one 16-row tile of D and keeps its slice
// of H'^T in registers for the CTA's lifetime. The 64-point Walsh-Hadamard
// transform along c then runs on the fp32 accumulator fragments: column bits
// 0 and 3..5 live inside a thread, bits 1..2 across the four lanes of a quad
// (two shuffle stages). Quantisation reads the fragments directly.
//
// Persistent CTAs loop over rows; rows are staged into shared memory with
// cp.async, NBUF deep, in 16-byte chunks XOR-swizzled by row so the
// ldmatrix.trans loads of the B fragments are conflict-free.
#pragma once
#include "ptx.cuh"
#include "rowquant.cuh"

namespace dscq {

template <int AP>
struct KronCfg {
  static constexpr int WARPS = AP / 16;
  static constexpr int THREADS = WARPS * 32;
  static constexpr int KT = AP / 16;              // k tiles of 16
  static constexpr int ROW_BYTES = AP * 128;      // [AP][64] bf16
  static constexpr int NBUF = 3;
  static constexpr int SMEM = NBUF * ROW_BYTES + 1024;
};

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void ldsm_x4_trans(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__device__ __forceinline__ void mma_bf16_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Entry (r, c) of H' = H_a (x) H_(2^s) as bf16 bits (+1 / -1), 0 outside [0, a 2^s)^2.
__device__ __forceinline__ uint32_t hsign_bf16(const int8_t* h_a, int a, int s, int r, int c) {
  const int ap = a << s;
  if (r >= ap || c >= ap) return 0u;
  const int m = (1 << s) - 1;
  const bool neg = (h_a[(r >> s) * a + (c >> s)] < 0) ^ (__popc(r & c & m) & 1);
  return neg ? 0xBF80u : 0x3F80u;
}

// x rows of K = a' * 64 bf16 with a' = a * 2^s; p.h_a = H_a ([a, a] +-1, row-major, device memory).
template <int AP>
__global__ void __launch_bounds__(AP * 2) kron_quant(const RowQuantParams p, int a_base, int s_log) {
  using C = KronCfg<AP>;
  extern __shared__ uint8_t kq_smem[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(kq_smem) + 127) & ~uintptr_t(127));
  __shared__ float s_max[C::WARPS];
  __shared__ int s_sum[C::WARPS];

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, q = lane & 3;
  const int m0 = warp * 16;
  const int a = a_base << s_log;  // order of the dense factor H'

  // A fragments of H'^T for this warp's 16 output rows, all k tiles: A[r][c] = H'[k0 + c][m0 + r]
  uint32_t afr[C::KT][4];
#pragma unroll
  for (int kt = 0; kt < C::KT; ++kt) {
    const int k0 = kt * 16;
    auto pair = [&](int r, int c) {
      return hsign_bf16(p.h_a, a_base, s_log, k0 + c, m0 + r) |
             (hsign_bf16(p.h_a, a_base, s_log, k0 + c + 1, m0 + r) << 16);
    };
    afr[kt][0] = pair(g, 2 * q);
    afr[kt][1] = pair(g + 8, 2 * q);
    afr[kt][2] = pair(g, 2 * q + 8);
    afr[kt][3] = pair(g + 8, 2 * q + 8);
  }
  // zero the padding rows [a, AP) of every buffer once (never written again)
  for (int i = threadIdx.x; i < C::NBUF * (AP - a) * 8; i += C::THREADS) {
    const int b = i / ((AP - a) * 8), r = a + (i % ((AP - a) * 8)) / 8, ch = i % 8;
    *reinterpret_cast<uint4*>(sm + b * C::ROW_BYTES + r * 128 + ch * 16) = make_uint4(0, 0, 0, 0);
  }

  const int chunks = a * 8;  // 16-byte chunks per row
  auto issue = [&](int row, int buf) {
    if (row < p.M) {
      const uint8_t* src = reinterpret_cast<const uint8_t*>(p.x) + static_cast<int64_t>(row) * p.ld_x * 2;
      const uint32_t base = smem_u32(sm + buf * C::ROW_BYTES);
      for (int i = threadIdx.x; i < chunks; i += C::THREADS) {
        const int r = i >> 3, ch = i & 7;
        cp_async16(base + r * 128 + ((ch ^ (r & 7)) << 4), src + i * 16);
      }
    }
    cp_async_commit();
  };

  const int stride = gridDim.x;
  int row = blockIdx.x;
#pragma unroll
  for (int s = 0; s < C::NBUF - 1; ++s) issue(row + s * stride, s);

  const float lo = p.mode == kWeightSym ? -7.f : -8.f;
  const bool clamp = p.clip < 1.f;
  for (int it = 0; row < p.rows_out; ++it, row += stride) {
    const int buf = it % C::NBUF;
    issue(row + (C::NBUF - 1) * stride, (it + C::NBUF - 1) % C::NBUF);
    cp_async_wait<C::NBUF - 1>();
    __syncthreads();

    // ---- dense factor on the tensor cores: acc[n] = 16 x 8 tile (rows m0.., cols 8n..)
    float acc[8][4];
#pragma unroll
    for (int n = 0; n < 8; ++n) acc[n][0] = acc[n][1] = acc[n][2] = acc[n][3] = 0.f;
    const uint32_t xb = smem_u32(sm + buf * C::ROW_BYTES);
    const bool live = row < p.M;
    if (live) {
#pragma unroll
      for (int kt = 0; kt < C::KT; ++kt) {
#pragma unroll
        for (int np = 0; np < 4; ++np) {
          // matrices: (k0..7, n=2np), (k8..15, n=2np), (k0..7, n=2np+1), (k8..15, n=2np+1)
          const int mi = lane >> 3, rr = lane & 7;
          const int r = kt * 16 + (mi & 1) * 8 + rr;
          const int ch = 2 * np + (mi >> 1);
          uint32_t b0, b1, b2, b3;
          ldsm_x4_trans(xb + r * 128 + ((ch ^ (r & 7)) << 4), b0, b1, b2, b3);
          mma_bf16_16816(acc[2 * np], afr[kt], b0, b1);
          mma_bf16_16816(acc[2 * np + 1], afr[kt], b2, b3);
        }
      }
    }
    __syncthreads();  // buffer `buf` is refilled by the next iteration's issue()

    // ---- 64-point WHT along c = 8n + 2q + e
#pragma unroll
    for (int n = 0; n < 8; ++n) {  // bit 0 (e)
      float t0 = acc[n][0], t1 = acc[n][1];
      acc[n][0] = t0 + t1;
      acc[n][1] = t0 - t1;
      t0 = acc[n][2];
      t1 = acc[n][3];
      acc[n][2] = t0 + t1;
      acc[n][3] = t0 - t1;
    }
#pragma unroll
    for (int bit = 1; bit <= 2; bit <<= 1) {  // bits 1, 2 (lane bits 0, 1)
      const float sgn = (q & bit) ? -1.f : 1.f;
#pragma unroll
      for (int n = 0; n < 8; ++n)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float o = __shfl_xor_sync(0xffffffffu, acc[n][e], bit);
          acc[n][e] = fmaf(acc[n][e], sgn, o);
        }
    }
#pragma unroll
    for (int h = 1; h < 8; h <<= 1)  // bits 3..5 (n)
#pragma unroll
      for (int n = 0; n < 8; ++n)
        if (!(n & h)) {
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float u = acc[n][e], v = acc[n + h][e];
            acc[n][e] = u + v;
            acc[n + h][e] = u - v;
          }
        }

    // ---- row absmax over the whole CTA
    float amax = 0.f;
#pragma unroll
    for (int n = 0; n < 8; ++n)
#pragma unroll
      for (int e = 0; e < 4; ++e) amax = fmaxf(amax, fabsf(acc[n][e]));
#pragma unroll
    for (int o = 16; o; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    if (lane == 0) s_max[warp] = amax;
    __syncthreads();
    amax = 0.f;
#pragma unroll
    for (int w = 0; w < C::WARPS; ++w) amax = fmaxf(amax, s_max[w]);

    const float amax_y = __fmul_rn(amax, p.norm);
    const float scale = fmaxf(__fdiv_rn(__fmul_rn(amax_y, p.clip), 7.f), 1e-8f);
    const float cm = __fdiv_rn(p.norm, scale);

    // ---- codes, packed bytes (k = i*64 + 8n + 2q + e -> byte i*32 + 4n + q)
    uint8_t* prow = p.packed ? p.packed + static_cast<int64_t>(row) * p.ld_packed : nullptr;
    int8_t* crow = p.codes ? p.codes + static_cast<int64_t>(row) * p.ld_codes : nullptr;
    int csum = 0;
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      const int i = m0 + g + 8 * half;
      if (i < a) {
#pragma unroll
        for (int n = 0; n < 8; ++n) {
          float q0 = acc[n][2 * half] * cm, q1 = acc[n][2 * half + 1] * cm;
          if (clamp) {
            q0 = fminf(fmaxf(q0, lo), 7.f);
            q1 = fminf(fmaxf(q1, lo), 7.f);
          }
          const uint32_t c0 = __float_as_uint(q0 + 12582912.f) & 15u;
          const uint32_t c1 = __float_as_uint(q1 + 12582912.f) & 15u;
          if (prow) prow[i * 32 + 4 * n + q] = static_cast<uint8_t>(c0 | (c1 << 4));
          if (crow || p.row_sums) {
            const int s0 = static_cast<int>(c0 << 28) >> 28, s1 = static_cast<int>(c1 << 28) >> 28;
            csum += s0 + s1;
            if (crow) {
              crow[i * 64 + 8 * n + 2 * q] = static_cast<int8_t>(s0);
              crow[i * 64 + 8 * n + 2 * q + 1] = static_cast<int8_t>(s1);
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
        for (int w = 0; w < C::WARPS; ++w) tot += s_sum[w];
        p.row_sums[row] = tot;
      }
    }
  }
  cp_async_wait<0>();
}

}  // namespace dscq
