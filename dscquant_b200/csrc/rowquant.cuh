// Per-row int4 quantizers with an optional online rotation, all in one pass
// over each row held in shared memory (fp32):
//
//   y = x * (H_a (x) H_b) / sqrt(K)     (optional; H_b Sylvester of order b = 2^j,
//                                        H_a a +-1 matrix of order a, K = a*b)
//   per-row scale / zero point           (mode below)
//   codes -> packed nibbles, even k in the low nibble
//
// Modes (all follow the reference's arithmetic, IEEE division, round half even):
//   kActSym       scale = max(absmax*clip/7, 1e-8), code = clamp(rn(y/scale), -8, 7)
//                 (the symmetric per-token scheme of the W4A4 path)
//   kWeightSym    weight_codes, core/quantization.py:7-11: bound 7,
//                 code = clamp(rn(w/scale), -7, 7); also emits per-row code sums
//   kActAsym      quantize_rows, kernel/w4a4.cu:20-63, bit for bit as nvcc builds it for
//                 sm_100a: lo/hi include 0 and are multiplied by clip, the range hi - lo is one
//                 fused multiply-add fma(max, clip, -lo) (nvcc's default contraction of
//                 maximum - minimum at :43), scale = max(range/15, 1e-8),
//                 zero = clamp(rn(-lo/scale), 0, 15), q = clamp(rn(y/scale + zero), 0, 15)
//                 (the zero point is added before rounding, :50), packed as (q - 8) & 15
//   kActAsymTorch activation_codes, core/quantization.py:13-21: as kActAsym with the range
//                 rounded as hi - lo (two products, one subtraction)
// Rows in [M, rows_out) and columns in [K, KP) are padding and get the codes
// the reference writes there (zero point for the asymmetric modes, 0 otherwise).
#pragma once
#include "ptx.cuh"

namespace dscq {

enum QuantMode : int { kActSym = 0, kWeightSym = 1, kActAsym = 2, kActAsymTorch = 3 };
enum InDtype : int { kInBF16 = 0, kInF16 = 1, kInF32 = 2 };

struct RowQuantParams {
  const void* x;
  int x_dtype;
  int64_t ld_x;      // elements between rows of x
  int M, K, KP;      // real rows, real columns, padded columns (even)
  int rows_out;      // rows written (>= M)
  int rotate;        // 0: identity
  int rot_a;         // order of the dense factor (1: none)
  int log2b;         // b = 1 << log2b, K = rot_a * b
  const int8_t* h_a; // [rot_a, rot_a] +-1, row-major, device memory
  float norm;        // 1/sqrt(K) when rotating
  int mode;
  float clip;
  uint8_t* packed;   // [rows_out, ld_packed], KP/2 bytes used per row
  int64_t ld_packed;
  float* scales;     // [rows_out]
  int32_t* zeros;    // [rows_out] or null
  int32_t* row_sums; // [rows_out] or null (sum of codes over k < K)
  int8_t* codes;     // [rows_out, ld_codes] or null (codes for k < KP)
  int64_t ld_codes;
};

__device__ __forceinline__ float load_in(const void* p, int64_t i, int dtype) {
  if (dtype == kInBF16) return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i]);
  if (dtype == kInF16) return __half2float(reinterpret_cast<const __half*>(p)[i]);
  return reinterpret_cast<const float*>(p)[i];
}

template <int T>
__device__ __forceinline__ float block_reduce_max(float v, float* scratch) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) scratch[w] = v;
  __syncthreads();
  v = (l < T / 32) ? scratch[l] : -INFINITY;
#pragma unroll
  for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

template <int T>
__device__ __forceinline__ int block_reduce_sum(int v, int* scratch) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) scratch[w] = v;
  __syncthreads();
  v = (l < T / 32) ? scratch[l] : 0;
#pragma unroll
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// code for one value; `zero` is the asymmetric zero point (ignored otherwise)
__device__ __forceinline__ int quant_code(float y, float scale, int zero, int mode) {
  const float q = __fdiv_rn(y, scale);
  if (mode == kActSym) return max(-8, min(7, __float2int_rn(q)));
  if (mode == kWeightSym) return max(-7, min(7, __float2int_rn(q)));
  return max(0, min(15, __float2int_rn(__fadd_rn(q, static_cast<float>(zero)))));  // both asymmetric modes
}

__device__ __forceinline__ uint32_t nibble_of(int code, int mode) {
  return static_cast<uint32_t>((mode == kActAsym || mode == kActAsymTorch) ? (code - 8) : code) & 15u;
}

// One CTA per output row. Dynamic shared memory: K floats, plus K more when a
// dense factor of order > 32 is applied (out-of-place stage).
template <int T>
__global__ void __launch_bounds__(T) rowquant_smem(const RowQuantParams p) {
  extern __shared__ float sbuf[];
  __shared__ float fscratch[32];
  __shared__ int iscratch[32];
  const int row = blockIdx.x;
  const int K = p.K;
  const bool live = row < p.M;
  float* buf = sbuf;
  const int64_t xrow = static_cast<int64_t>(row) * p.ld_x;
  for (int k = threadIdx.x; k < K; k += T) buf[k] = live ? load_in(p.x, xrow + k, p.x_dtype) : 0.f;
  __syncthreads();

  float* src = buf;
  float mul = 1.f;
  if (p.rotate) {
    const int b = 1 << p.log2b;
    // Walsh-Hadamard butterflies along the contiguous factor (index k = i*b + c).
    for (int h = 1; h < b; h <<= 1) {
      for (int q = threadIdx.x; q < K / 2; q += T) {
        const int i = q >> (p.log2b - 1);
        const int r = q & ((b >> 1) - 1);
        const int lo = i * b + ((r & ~(h - 1)) << 1) + (r & (h - 1));
        const float u = buf[lo], v = buf[lo + h];
        buf[lo] = u + v;
        buf[lo + h] = u - v;
      }
      __syncthreads();
    }
    if (p.rot_a > 1 && p.rot_a <= 32) {
      // Dense factor, in place, one column c per thread: Y[i2, c] = sum_i H_a[i, i2] * Z[i, c].
      // The signs of column i2 of H_a sit in shared memory as one 32-bit mask per i2 (bit i set
      // where H_a[i, i2] < 0); every thread reads the same word (broadcast).
      __shared__ uint32_t hneg[32];
      const int a = p.rot_a;
      if (threadIdx.x < a) {
        uint32_t m = 0;
        for (int i = 0; i < a; ++i) m |= static_cast<uint32_t>(p.h_a[i * a + threadIdx.x] < 0) << i;
        hneg[threadIdx.x] = m;
      }
      __syncthreads();
      for (int c = threadIdx.x; c < b; c += T) {
        float v[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] = i < a ? buf[(i << p.log2b) + c] : 0.f;
        for (int i2 = 0; i2 < a; ++i2) {
          const uint32_t m = hneg[i2];
          float acc = 0.f;
#pragma unroll
          for (int i = 0; i < 32; ++i) acc += ((m >> i) & 1u) ? -v[i] : v[i];
          buf[(i2 << p.log2b) + c] = acc;
        }
      }
      __syncthreads();
    } else if (p.rot_a > 32) {
      // Dense factor, out of place: Y[i2, c] = sum_i H_a[i, i2] * Z[i, c].
      float* out = sbuf + K;
      const int a = p.rot_a;
      for (int k = threadIdx.x; k < K; k += T) {
        const int i2 = k >> p.log2b, c = k & (b - 1);
        float acc = 0.f;
        for (int i = 0; i < a; ++i) {
          const float v = buf[(i << p.log2b) + c];
          acc = p.h_a[i * a + i2] > 0 ? acc + v : acc - v;
        }
        out[k] = acc;
      }
      __syncthreads();
      src = out;
    }
    mul = p.norm;
  }

  // Row statistics over the real columns.
  const bool asym = p.mode == kActAsym || p.mode == kActAsymTorch;
  float a_max = 0.f, a_min = 0.f;
  for (int k = threadIdx.x; k < K; k += T) {
    const float y = p.rotate ? __fmul_rn(src[k], mul) : src[k];
    if (p.rotate) src[k] = y;
    if (asym) {
      a_max = fmaxf(a_max, y);
      a_min = fminf(a_min, y);
    } else {
      a_max = fmaxf(a_max, fabsf(y));
    }
  }
  a_max = block_reduce_max<T>(a_max, fscratch);
  if (asym) a_min = -block_reduce_max<T>(-a_min, fscratch);

  float scale;
  int zero = 0;
  if (asym) {
    const float lo = __fmul_rn(a_min, p.clip), hi = __fmul_rn(a_max, p.clip);
    const float range = p.mode == kActAsym ? __fmaf_rn(a_max, p.clip, -lo) : __fsub_rn(hi, lo);
    scale = fmaxf(__fdiv_rn(range, 15.f), 1e-8f);
    zero = max(0, min(15, __float2int_rn(__fdiv_rn(-lo, scale))));
  } else {
    scale = fmaxf(__fdiv_rn(__fmul_rn(a_max, p.clip), 7.f), 1e-8f);
  }

  int csum = 0;
  const int pad_code = asym ? zero : 0;
  uint8_t* prow = p.packed ? p.packed + static_cast<int64_t>(row) * p.ld_packed : nullptr;
  int8_t* crow = p.codes ? p.codes + static_cast<int64_t>(row) * p.ld_codes : nullptr;
  for (int pr = threadIdx.x; pr < p.KP / 2; pr += T) {
    const int k = 2 * pr;
    const int c0 = k < K ? quant_code(src[k], scale, zero, p.mode) : pad_code;
    const int c1 = k + 1 < K ? quant_code(src[k + 1], scale, zero, p.mode) : pad_code;
    if (k < K) csum += c0;
    if (k + 1 < K) csum += c1;
    if (prow) prow[pr] = static_cast<uint8_t>(nibble_of(c0, p.mode) | (nibble_of(c1, p.mode) << 4));
    if (crow) {
      crow[k] = static_cast<int8_t>(c0);
      crow[k + 1] = static_cast<int8_t>(c1);
    }
  }
  if (p.row_sums) csum = block_reduce_sum<T>(csum, iscratch);
  if (threadIdx.x == 0) {
    p.scales[row] = scale;
    if (p.zeros) p.zeros[row] = zero;
    if (p.row_sums) p.row_sums[row] = csum;
  }
}

// Rows too long for shared memory (no rotation): one CTA per output row reads the row twice from
// global memory, once for the statistics and once for the codes, as the reference's quantize_rows
// does (kernel/w4a4.cu:20-63, K up to 2^20). Same modes, padding and outputs as rowquant_smem.
template <int T>
__global__ void __launch_bounds__(T) rowquant_stream(const RowQuantParams p) {
  __shared__ float fscratch[32];
  __shared__ int iscratch[32];
  const int row = blockIdx.x;
  const int K = p.K;
  const bool live = row < p.M;
  const int64_t xrow = static_cast<int64_t>(row) * p.ld_x;
  const bool asym = p.mode == kActAsym || p.mode == kActAsymTorch;
  float a_max = 0.f, a_min = 0.f;
  if (live) {
    for (int k = threadIdx.x; k < K; k += T) {
      const float y = load_in(p.x, xrow + k, p.x_dtype);
      if (asym) {
        a_max = fmaxf(a_max, y);
        a_min = fminf(a_min, y);
      } else {
        a_max = fmaxf(a_max, fabsf(y));
      }
    }
  }
  a_max = block_reduce_max<T>(a_max, fscratch);
  if (asym) a_min = -block_reduce_max<T>(-a_min, fscratch);
  float scale;
  int zero = 0;
  if (asym) {
    const float lo = __fmul_rn(a_min, p.clip), hi = __fmul_rn(a_max, p.clip);
    const float range = p.mode == kActAsym ? __fmaf_rn(a_max, p.clip, -lo) : __fsub_rn(hi, lo);
    scale = fmaxf(__fdiv_rn(range, 15.f), 1e-8f);
    zero = max(0, min(15, __float2int_rn(__fdiv_rn(-lo, scale))));
  } else {
    scale = fmaxf(__fdiv_rn(__fmul_rn(a_max, p.clip), 7.f), 1e-8f);
  }
  int csum = 0;
  const int pad_code = asym ? zero : 0;
  uint8_t* prow = p.packed ? p.packed + static_cast<int64_t>(row) * p.ld_packed : nullptr;
  int8_t* crow = p.codes ? p.codes + static_cast<int64_t>(row) * p.ld_codes : nullptr;
  for (int pr = threadIdx.x; pr < p.KP / 2; pr += T) {
    const int k = 2 * pr;
    const int c0 = (live && k < K) ? quant_code(load_in(p.x, xrow + k, p.x_dtype), scale, zero, p.mode) : pad_code;
    const int c1 = (live && k + 1 < K) ? quant_code(load_in(p.x, xrow + k + 1, p.x_dtype), scale, zero, p.mode)
                                       : pad_code;
    if (k < K) csum += c0;
    if (k + 1 < K) csum += c1;
    if (prow) prow[pr] = static_cast<uint8_t>(nibble_of(c0, p.mode) | (nibble_of(c1, p.mode) << 4));
    if (crow) {
      crow[k] = static_cast<int8_t>(c0);
      crow[k + 1] = static_cast<int8_t>(c1);
    }
  }
  if (p.row_sums) csum = block_reduce_sum<T>(csum, iscratch);
  if (threadIdx.x == 0) {
    p.scales[row] = scale;
    if (p.zeros) p.zeros[row] = zero;
    if (p.row_sums) p.row_sums[row] = csum;
  }
}

// ------------------------------------------------------------ pack / unpack
// pack_int4, core/quantization.py:31-40: int8 codes in [-8, 7] -> bytes,
// byte j = (c[2j] & 15) | (c[2j+1] & 15) << 4, odd K padded with code 0.
// Out-of-range codes are counted into *bad (the caller raises).
__global__ void pack_int4_kernel(const int8_t* codes, int64_t rows, int64_t K, int64_t ld_codes, uint8_t* packed,
                                 int64_t ld_packed, int* bad) {
  const int64_t half = (K + 1) / 2;
  const int64_t total = rows * half;
  int nbad = 0;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = i / half, j = i % half;
    const int8_t* c = codes + r * ld_codes;
    const int c0 = c[2 * j];
    const int c1 = (2 * j + 1 < K) ? c[2 * j + 1] : 0;
    nbad += (c0 < -8 || c0 > 7) + (c1 < -8 || c1 > 7);
    packed[r * ld_packed + j] = static_cast<uint8_t>((c0 & 15) | ((c1 & 15) << 4));
  }
  if (nbad) atomicAdd(bad, nbad);
}

// unpack_int4, core/quantization.py:42-45: nibble >= 8 -> nibble - 16.
__global__ void unpack_int4_kernel(const uint8_t* packed, int64_t rows, int64_t ld_packed, int64_t width,
                                   int8_t* codes, int64_t ld_codes) {
  const int64_t total = rows * width;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = i / width, k = i % width;
    const int b = packed[r * ld_packed + k / 2];
    const int v = (k & 1) ? (b >> 4) : (b & 15);
    codes[r * ld_codes + k] = static_cast<int8_t>(v >= 8 ? v - 16 : v);
  }
}

}  // namespace dscq
