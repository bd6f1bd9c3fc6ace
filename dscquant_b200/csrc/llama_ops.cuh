// Element-wise operators around the W4A4 linears of the Llama prefill workload (no counterpart in the
// reference, which runs a Hugging Face model around its QuantLinear): RMSNorm, rotary embeddings on q
// and k, and the SiLU gate. Each is one HBM pass in bf16 with fp32 arithmetic, rounding to bf16 at the
// same steps as the torch expressions they replace:
//   rmsnorm   y = bf16(bf16(x * rsqrt(mean(x^2) + eps)) * w)
//   rope      y = bf16(bf16(x * cos) + bf16(rotate_half(x) * sin)), rotate_half(x) = [-x2, x1]
//   silu_mul  y = bf16(bf16(silu(g)) * u)
#pragma once
#include "ptx.cuh"

namespace dscq {

__device__ __forceinline__ float bf16r(float v) { return __bfloat162float(__float2bfloat16_rn(v)); }

// One CTA of 256 threads per row; H a multiple of 8, x and y rows 16-byte aligned.
__global__ void __launch_bounds__(256) rmsnorm_kernel(const __nv_bfloat16* __restrict__ x,
                                                      const __nv_bfloat16* __restrict__ w, __nv_bfloat16* y, int H,
                                                      float eps) {
  __shared__ float red[8];
  const int64_t row = blockIdx.x;
  const uint4* xr = reinterpret_cast<const uint4*>(x + row * H);
  const int nv = H / 8;
  float ss = 0.f;
  for (int i = threadIdx.x; i < nv; i += 256) {
    const uint4 v = xr[i];
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&v);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 f = __bfloat1622float2(h[j]);
      ss = fmaf(f.x, f.x, fmaf(f.y, f.y, ss));
    }
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int k = 0; k < 8; ++k) tot += red[k];
  const float r = rsqrtf(tot / static_cast<float>(H) + eps);
  uint4* yr = reinterpret_cast<uint4*>(y + row * H);
  const uint4* wr = reinterpret_cast<const uint4*>(w);
  for (int i = threadIdx.x; i < nv; i += 256) {
    const uint4 v = xr[i], wv = wr[i];
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&v);
    const __nv_bfloat162* hw = reinterpret_cast<const __nv_bfloat162*>(&wv);
    uint4 o;
    __nv_bfloat162* ho = reinterpret_cast<__nv_bfloat162*>(&o);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 f = __bfloat1622float2(h[j]), g = __bfloat1622float2(hw[j]);
      ho[j] = __floats2bfloat162_rn(bf16r(f.x * r) * g.x, bf16r(f.y * r) * g.y);
    }
    yr[i] = o;
  }
}

// In place on q [S, Hq, D] and k [S, Hk, D] (rows of D contiguous, D even and <= 256); cos / sin [S, D].
// One thread per (row, pair j < D/2): it owns elements j and j + D/2 of its head row.
__global__ void __launch_bounds__(256) rope_kernel(__nv_bfloat16* q, __nv_bfloat16* k, const __nv_bfloat16* cs,
                                                   const __nv_bfloat16* sn, int S, int Hq, int Hk, int D) {
  const int half = D / 2;
  const int64_t total = static_cast<int64_t>(S) * (Hq + Hk) * half;
  for (int64_t t = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; t < total;
       t += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int j = static_cast<int>(t % half);
    const int64_t hr = t / half;  // head row over q then k
    const int s = static_cast<int>(hr / (Hq + Hk)), hh = static_cast<int>(hr % (Hq + Hk));
    __nv_bfloat16* base = hh < Hq ? q + (static_cast<int64_t>(s) * Hq + hh) * D
                                  : k + (static_cast<int64_t>(s) * Hk + (hh - Hq)) * D;
    const float x1 = __bfloat162float(base[j]), x2 = __bfloat162float(base[j + half]);
    const float c1 = __bfloat162float(cs[static_cast<int64_t>(s) * D + j]);
    const float c2 = __bfloat162float(cs[static_cast<int64_t>(s) * D + j + half]);
    const float s1 = __bfloat162float(sn[static_cast<int64_t>(s) * D + j]);
    const float s2 = __bfloat162float(sn[static_cast<int64_t>(s) * D + j + half]);
    base[j] = __float2bfloat16_rn(bf16r(x1 * c1) + bf16r(-x2 * s1));
    base[j + half] = __float2bfloat16_rn(bf16r(x2 * c2) + bf16r(x1 * s2));
  }
}

// The same rotation, eight consecutive pairs per thread with 16-byte loads and stores (D/2 a multiple of 8,
// every row 16-byte aligned): one thread per (row, group of 8 j).
__global__ void __launch_bounds__(256) rope_vec_kernel(__nv_bfloat16* q, __nv_bfloat16* k, const __nv_bfloat16* cs,
                                                       const __nv_bfloat16* sn, int S, int Hq, int Hk, int D) {
  const int half = D / 2, ng = half / 8;
  const int64_t total = static_cast<int64_t>(S) * (Hq + Hk) * ng;
  for (int64_t t = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; t < total;
       t += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int j = static_cast<int>(t % ng) * 8;
    const int64_t hr = t / ng;
    const int s = static_cast<int>(hr / (Hq + Hk)), hh = static_cast<int>(hr % (Hq + Hk));
    __nv_bfloat16* base = hh < Hq ? q + (static_cast<int64_t>(s) * Hq + hh) * D
                                  : k + (static_cast<int64_t>(s) * Hk + (hh - Hq)) * D;
    const __nv_bfloat16* c = cs + static_cast<int64_t>(s) * D;
    const __nv_bfloat16* n = sn + static_cast<int64_t>(s) * D;
    const uint4 vx1 = *reinterpret_cast<const uint4*>(base + j), vx2 = *reinterpret_cast<const uint4*>(base + j + half);
    const uint4 vc1 = *reinterpret_cast<const uint4*>(c + j), vc2 = *reinterpret_cast<const uint4*>(c + j + half);
    const uint4 vs1 = *reinterpret_cast<const uint4*>(n + j), vs2 = *reinterpret_cast<const uint4*>(n + j + half);
    const __nv_bfloat16* x1 = reinterpret_cast<const __nv_bfloat16*>(&vx1);
    const __nv_bfloat16* x2 = reinterpret_cast<const __nv_bfloat16*>(&vx2);
    const __nv_bfloat16* c1 = reinterpret_cast<const __nv_bfloat16*>(&vc1);
    const __nv_bfloat16* c2 = reinterpret_cast<const __nv_bfloat16*>(&vc2);
    const __nv_bfloat16* s1 = reinterpret_cast<const __nv_bfloat16*>(&vs1);
    const __nv_bfloat16* s2 = reinterpret_cast<const __nv_bfloat16*>(&vs2);
    uint4 o1, o2;
    __nv_bfloat16* y1 = reinterpret_cast<__nv_bfloat16*>(&o1);
    __nv_bfloat16* y2 = reinterpret_cast<__nv_bfloat16*>(&o2);
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const float a = __bfloat162float(x1[e]), b = __bfloat162float(x2[e]);
      y1[e] = __float2bfloat16_rn(bf16r(a * __bfloat162float(c1[e])) + bf16r(-b * __bfloat162float(s1[e])));
      y2[e] = __float2bfloat16_rn(bf16r(b * __bfloat162float(c2[e])) + bf16r(a * __bfloat162float(s2[e])));
    }
    *reinterpret_cast<uint4*>(base + j) = o1;
    *reinterpret_cast<uint4*>(base + j + half) = o2;
  }
}

// y = bf16(bf16(silu(g)) * u) over n elements (n a multiple of 8, 16-byte aligned buffers).
__global__ void __launch_bounds__(256) silu_mul_kernel(const __nv_bfloat16* __restrict__ g,
                                                       const __nv_bfloat16* __restrict__ u, __nv_bfloat16* y,
                                                       int64_t n) {
  const int64_t nv = n / 8;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < nv;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const uint4 gv = reinterpret_cast<const uint4*>(g)[i], uv = reinterpret_cast<const uint4*>(u)[i];
    const __nv_bfloat162* hg = reinterpret_cast<const __nv_bfloat162*>(&gv);
    const __nv_bfloat162* hu = reinterpret_cast<const __nv_bfloat162*>(&uv);
    uint4 o;
    __nv_bfloat162* ho = reinterpret_cast<__nv_bfloat162*>(&o);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 a = __bfloat1622float2(hg[j]), b = __bfloat1622float2(hu[j]);
      const float s0 = bf16r(a.x / (1.f + expf(-a.x))), s1 = bf16r(a.y / (1.f + expf(-a.y)));
      ho[j] = __floats2bfloat162_rn(s0 * b.x, s1 * b.y);
    }
    reinterpret_cast<uint4*>(y)[i] = o;
  }
}

}  // namespace dscq
