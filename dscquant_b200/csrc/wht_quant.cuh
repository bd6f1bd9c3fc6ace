// Fused online Walsh-Hadamard rotation + symmetric per-row int4 quantisation
// for K = 2^LOGK (LOGK = 10..13), bf16 input. One HBM read of x, one write of
// the packed codes (+ 4 B of scale per row): 2.5 B per element.
//
//   phase 1  each thread loads E contiguous elements (16-byte loads), runs the
//            butterflies over index bits [0, log2 E) in registers (packed
//            f32x2 adds), and stores them to shared memory (XOR-swizzled
//            16-byte chunks: conflict-free stores and column loads)
//   phase 2  each thread reads GPT adjacent columns g.. of the row's
//            [G x E] shared-memory matrix and runs the remaining butterflies
//            over the G = K/E elements of each column in registers
//   quant    row absmax (shuffles; shared memory across warps), one scale per
//            row, q = v * (norm / scale), round-half-even through the 1.5*2^23
//            magic add, nibbles of adjacent columns packed into bytes and
//            stored as 16-bit words (coalesced across the row's threads)
//
// Same definitions as the general kernel (rowquant.cuh): y = x H_K / sqrt(K),
// scale = max(absmax(y)*clip/7, 1e-8), code = clamp(rn(y/scale)) to [-8, 7]
// (activations) or [-7, 7] (weights). The float order differs from a float64
// rotation, so codes can differ by one step only at near ties.
#pragma once
#include "ptx.cuh"
#include "rowquant.cuh"

namespace dscq {

template <int LOGK>
struct WhtCfg {
  static constexpr int K = 1 << LOGK;
  static constexpr int LE = LOGK >= 12 ? 7 : 6;
  static constexpr int E = 1 << LE;   // elements per thread in phase 1
  static constexpr int TR = K / E;    // threads per row
  static constexpr int G = TR;        // phase-2 column height
  static constexpr int GPT = E / G;   // adjacent columns per thread in phase 2
  static constexpr int THREADS = 128;
  static constexpr int ROWS = THREADS / TR;
  static constexpr int SMEM = ROWS * K * 4;
  static_assert(LOGK >= 10 && LOGK <= 13, "K = 1024 .. 8192");
  static_assert(GPT == 2 || GPT == 4, "phase 2 needs 2 or 4 adjacent columns per thread");
  static_assert(TR <= THREADS && THREADS % TR == 0, "rows must tile the CTA");
};

__device__ __forceinline__ float2 f2add(float2 a, float2 b) { return __fadd2_rn(a, b); }
__device__ __forceinline__ float2 f2sub(float2 a, float2 b) { return __ffma2_rn(b, make_float2(-1.f, -1.f), a); }

__device__ __forceinline__ float2 bf16x2_to_f2(uint32_t w) {
  return make_float2(__uint_as_float(w << 16), __uint_as_float(w & 0xFFFF0000u));
}

template <int LOGK>
__global__ void __launch_bounds__(128) wht_quant_pow2(const RowQuantParams p) {
  using C = WhtCfg<LOGK>;
  constexpr int E = C::E, TR = C::TR, G = C::G, GPT = C::GPT, K = C::K;
  constexpr int CM = E / 4 - 1;  // chunk swizzle mask
  extern __shared__ float4 smem_f4[];
  float* sbase = reinterpret_cast<float*>(smem_f4);
  __shared__ float s_red[C::ROWS][2];
  __shared__ int s_sum[C::ROWS][2];

  const int r_local = threadIdx.x / TR;
  const int t = threadIdx.x % TR;
  const int row = blockIdx.x * C::ROWS + r_local;
  const bool live = row < p.M;
  const bool active = row < p.rows_out;
  float* sb = sbase + r_local * K;

  // ---------------- phase 1: contiguous E elements, butterflies over bits [0, LE)
  float2 V[E / 2];
  {
    const uint4* src = reinterpret_cast<const uint4*>(reinterpret_cast<const __nv_bfloat16*>(p.x) +
                                                      static_cast<int64_t>(live ? row : 0) * p.ld_x) +
                       t * (E / 8);
#pragma unroll
    for (int q = 0; q < E / 8; ++q) {
      const uint4 w = live ? __ldcs(src + q) : make_uint4(0, 0, 0, 0);
      V[4 * q + 0] = bf16x2_to_f2(w.x);
      V[4 * q + 1] = bf16x2_to_f2(w.y);
      V[4 * q + 2] = bf16x2_to_f2(w.z);
      V[4 * q + 3] = bf16x2_to_f2(w.w);
    }
  }
#pragma unroll
  for (int m = 0; m < E / 2; ++m) V[m] = make_float2(V[m].x + V[m].y, V[m].x - V[m].y);
#pragma unroll
  for (int hv = 1; hv < E / 2; hv <<= 1) {
#pragma unroll
    for (int m = 0; m < E / 2; ++m) {
      if (!(m & hv)) {
        const float2 a = V[m], b = V[m + hv];
        V[m] = f2add(a, b);
        V[m + hv] = f2sub(a, b);
      }
    }
  }
  {
    float* srow = sb + t * E;
#pragma unroll
    for (int q = 0; q < E / 4; ++q)
      *reinterpret_cast<float4*>(srow + ((q ^ (t & CM)) << 2)) =
          make_float4(V[2 * q].x, V[2 * q].y, V[2 * q + 1].x, V[2 * q + 1].y);
  }
  __syncthreads();

  // ---------------- phase 2: GPT adjacent columns, butterflies over the G rows
  const int g0 = t * GPT;
  float2 Y[GPT / 2][G];
#pragma unroll
  for (int j = 0; j < G; ++j) {
    const float* ps = sb + j * E + (((g0 >> 2) ^ (j & CM)) << 2) + (g0 & 3);
    if constexpr (GPT == 4) {
      const float4 f = *reinterpret_cast<const float4*>(ps);
      Y[0][j] = make_float2(f.x, f.y);
      Y[1][j] = make_float2(f.z, f.w);
    } else {
      Y[0][j] = *reinterpret_cast<const float2*>(ps);
    }
  }
#pragma unroll
  for (int h = 1; h < G; h <<= 1) {
#pragma unroll
    for (int j = 0; j < G; ++j) {
      if (!(j & h)) {
#pragma unroll
        for (int u = 0; u < GPT / 2; ++u) {
          const float2 a = Y[u][j], b = Y[u][j + h];
          Y[u][j] = f2add(a, b);
          Y[u][j + h] = f2sub(a, b);
        }
      }
    }
  }

  // ---------------- row absmax
  float amax = 0.f;
#pragma unroll
  for (int u = 0; u < GPT / 2; ++u)
#pragma unroll
    for (int j = 0; j < G; ++j) amax = fmaxf(amax, fmaxf(fabsf(Y[u][j].x), fabsf(Y[u][j].y)));
#pragma unroll
  for (int o = (TR < 32 ? TR : 32) / 2; o; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  if constexpr (TR > 32) {
    if ((t & 31) == 0) s_red[r_local][t >> 5] = amax;
    __syncthreads();
    amax = fmaxf(s_red[r_local][0], s_red[r_local][1]);
  }

  const float amax_y = __fmul_rn(amax, p.norm);
  const float scale = fmaxf(__fdiv_rn(__fmul_rn(amax_y, p.clip), 7.f), 1e-8f);
  const float cm = __fdiv_rn(p.norm, scale);
  const float lo = p.mode == kWeightSym ? -7.f : -8.f;
  const bool clamp = p.clip < 1.f;
  const float2 cm2 = make_float2(cm, cm);
  const float2 magic2 = make_float2(12582912.f, 12582912.f);  // 1.5 * 2^23: low mantissa bits = rn(q)

  int csum = 0;
  if (active) {
    uint8_t* prow = p.packed ? p.packed + static_cast<int64_t>(row) * p.ld_packed : nullptr;
    int8_t* crow = p.codes ? p.codes + static_cast<int64_t>(row) * p.ld_codes : nullptr;
#pragma unroll
    for (int j = 0; j < G; ++j) {
      uint32_t bytes = 0;
#pragma unroll
      for (int u = 0; u < GPT / 2; ++u) {
        float2 q = __fmul2_rn(Y[u][j], cm2);
        if (clamp) q = make_float2(fminf(fmaxf(q.x, lo), 7.f), fminf(fmaxf(q.y, lo), 7.f));
        const float2 r = f2add(q, magic2);
        const uint32_t c0 = __float_as_uint(r.x) & 15u, c1 = __float_as_uint(r.y) & 15u;
        bytes |= (c0 | (c1 << 4)) << (8 * u);
        if (crow || p.row_sums) {
          const int s0 = static_cast<int>(c0 << 28) >> 28, s1 = static_cast<int>(c1 << 28) >> 28;
          csum += s0 + s1;
          if (crow) {
            crow[g0 + 2 * u + E * j] = static_cast<int8_t>(s0);
            crow[g0 + 2 * u + 1 + E * j] = static_cast<int8_t>(s1);
          }
        }
      }
      if (prow) {
        uint8_t* dst = prow + (E / 2) * j + (g0 >> 1);
        if constexpr (GPT == 4)
          *reinterpret_cast<uint16_t*>(dst) = static_cast<uint16_t>(bytes);
        else
          *dst = static_cast<uint8_t>(bytes);
      }
    }
    if (t == 0) p.scales[row] = scale;
  }
  if (p.row_sums) {  // uniform: every thread of the CTA takes this branch
#pragma unroll
    for (int o = (TR < 32 ? TR : 32) / 2; o; o >>= 1) csum += __shfl_xor_sync(0xffffffffu, csum, o);
    if constexpr (TR > 32) {
      if ((t & 31) == 0) s_sum[r_local][t >> 5] = csum;
      __syncthreads();
      csum = s_sum[r_local][0] + s_sum[r_local][1];
    }
    if (t == 0 && active) p.row_sums[row] = csum;
  }
}

}  // namespace dscq
