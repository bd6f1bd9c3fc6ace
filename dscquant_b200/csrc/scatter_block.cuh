// Copy of one row block [rows, width bytes] (row stride ld_src) into up to 8 destination buffers at the
// same offsets (row stride ld_dst): in a column-parallel group, this GPU's output columns pushed into
// every peer's output buffer over NVLink after the GEMM wrote them locally. No counterpart in the
// reference, which has no multi-GPU code.
//
// The GEMM epilogue can store into the peers itself (dscq_matmul_cols with peer pointers), but then
// remote-store backpressure holds the epilogue warps, which hold the TMEM accumulators, which stall the
// MMAs. As a separate launch the copy runs on a side stream beside the next GEMM launch: a few small
// CTAs per SM co-reside with the one large GEMM CTA. Each warp moves 8 rows x 64 bytes per step with
// 16-byte loads (no L1 allocation) and one 16-byte store per destination (peer stores reached 440-700 GB/s per GPU on
// B200 at this granularity).
#pragma once
#include "ptx.cuh"

namespace dscq {

struct ScatterParams {
  const uint8_t* src;
  int64_t ld_src, ld_dst;  // bytes
  int64_t rows, width;     // width: bytes per row, a multiple of 16
  int n_dst;
  uint8_t* dst[8];
};

__global__ void __launch_bounds__(128) scatter_block_kernel(const ScatterParams p) {
  const int lane = threadIdx.x & 31;
  const int64_t warp = (blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x) >> 5;
  const int64_t nwarps = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
  const int64_t segs = (p.width + 63) / 64;  // 64-byte row segments
  const int64_t units = ((p.rows + 7) / 8) * segs;
  for (int64_t u = warp; u < units; u += nwarps) {
    const int64_t row = (u / segs) * 8 + (lane >> 2);
    const int64_t col = (u % segs) * 64 + (lane & 3) * 16;
    if (row >= p.rows || col >= p.width) continue;
    uint4 v;  // not allocated in L1: L1 is the shared memory of the GEMM running beside this copy
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p.src + row * p.ld_src + col));
    const int64_t o = row * p.ld_dst + col;
    for (int d = 0; d < p.n_dst; ++d) *reinterpret_cast<uint4*>(p.dst[d] + o) = v;
  }
}

}  // namespace dscq
