// C ABI of the W4A4 path (include/dscq_b200.h). One translation unit so the
// device status word is shared by every kernel of the library.
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <map>
#include <mutex>
#include <string>
#include <utility>
#include <vector>

#include "../../include/dscq_b200.h"
#include "gemm_w4a4.cuh"
#include "hadamard.h"
#include "rowquant.cuh"
#include "wht_quant.cuh"
#include "kron_quant.cuh"
#include "kron_long_quant.cuh"
#include "gemv_w4a4.cuh"
#include "gemm_a8.cuh"
#include "gemm_pair_tm.cuh"
#include "headrot_quant.cuh"
#include "rotq_tc.cuh"
#include "llama_ops.cuh"
#include "scatter_block.cuh"

namespace {

thread_local std::string g_err;

int fail(int code, const std::string& msg) {
  g_err = msg;
  return code;
}

#define DSCQ_REQUIRE(cond, msg) \
  do {                          \
    if (!(cond)) return fail(DSCQ_ERR_INVALID, msg); \
  } while (0)

int cuda_fail(cudaError_t e, const char* where) {
  return fail(DSCQ_ERR_CUDA, std::string(where) + ": " + cudaGetErrorString(e));
}

bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

// Row-length limits: the reference's quantize accepts K <= 2^20 (kernel/w4a4.cu:166), which the
// unrotated quantizers match; the online rotation keeps the row in shared memory (K <= 32768). The
// GEMMs accumulate 256 * sum(a b) in int32 (codes shifted into the high nibble), so KP <= 65536.
constexpr int64_t kMaxRowK = 1048576;
constexpr int64_t kMaxRotK = 32768;
constexpr int64_t kMaxGemmKP = 65536;

// sm_100 check, cached per device.
int check_device(int* dev_out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  static int cc_cache[64] = {0};
  int cc = dev < 64 ? cc_cache[dev] : 0;
  if (cc == 0) {
    int major = 0, minor = 0;
    e = cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
    if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceGetAttribute");
    e = cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
    if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceGetAttribute");
    cc = major * 10 + minor;
    if (dev < 64) cc_cache[dev] = cc;
  }
  if (cc != 100)
    return fail(DSCQ_ERR_UNSUPPORTED, "dscq_b200 kernels are built for sm_100a (B200); device " +
                                          std::to_string(dev) + " has compute capability " + std::to_string(cc));
  if (dev_out) *dev_out = dev;
  return DSCQ_OK;
}

// cuTensorMapEncodeTiled through the runtime's driver entry point, so the
// library has no link-time dependency on libcuda.
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

// u8 matrix [rows, cols] with row stride ld bytes, box [box_rows, 64 bytes].
int make_u8_map(CUtensorMap* map, const void* base, int64_t rows, int64_t cols, int64_t ld, int box_rows) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return fail(DSCQ_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld)};
  cuuint32_t box[2] = {64u, static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1u, 1u};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(DSCQ_ERR_CUDA, "cuTensorMapEncodeTiled failed (" + std::to_string(r) + ")");
  return DSCQ_OK;
}

// As make_u8_map with the 64-byte swizzle (16-byte chunk c of box row r lands at chunk
// c ^ ((r >> 1) & 3)), so that one thread per row reads shared memory without bank conflicts.
int make_u8_map_sw64(CUtensorMap* map, const void* base, int64_t rows, int64_t cols, int64_t ld, int box_rows) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return fail(DSCQ_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld)};
  cuuint32_t box[2] = {64u, static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1u, 1u};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(DSCQ_ERR_CUDA, "cuTensorMapEncodeTiled (64B swizzle) failed (" + std::to_string(r) + ")");
  return DSCQ_OK;
}

// bf16 matrix [rows, cols] (row stride ld elements) in boxes of 128 rows x 64 columns landing with
// the 128-byte swizzle: the K-major UMMA operand layout.
int make_bf16_sw128_map(CUtensorMap* map, const void* base, int64_t rows, int64_t cols, int64_t ld) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return fail(DSCQ_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld) * 2u};
  cuuint32_t box[2] = {64u, 128u};
  cuuint32_t estr[2] = {1u, 1u};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(DSCQ_ERR_CUDA, "cuTensorMapEncodeTiled (bf16) failed (" + std::to_string(r) + ")");
  return DSCQ_OK;
}

// x [M, ld_x] bf16 viewed as a 3-D tensor {c: 64, i: ap, token: M} (row k = i*64 + c), boxes of
// {64, ap16, P} landing in shared memory with the 128-byte swizzle (the MN-major UMMA layout).
int make_rows_map(CUtensorMap* map, const void* x, int64_t M, int ap, int64_t ld_x, int ap16, int P) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return fail(DSCQ_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  cuuint64_t dims[3] = {64u, static_cast<cuuint64_t>(ap), static_cast<cuuint64_t>(M)};
  cuuint64_t strides[2] = {128u, static_cast<cuuint64_t>(ld_x) * 2u};
  cuuint32_t box[3] = {64u, static_cast<cuuint32_t>(ap16), static_cast<cuuint32_t>(P)};
  cuuint32_t estr[3] = {1u, 1u, 1u};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(x), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(DSCQ_ERR_CUDA, "cuTensorMapEncodeTiled (rows) failed (" + std::to_string(r) + ")");
  return DSCQ_OK;
}

// int8 activation codes [rows, cols] (row stride ld bytes) in 128 x 128-byte boxes landing with the
// 128-byte swizzle: the K-major UMMA operand layout for the A8 GEMM.
int make_i8_sw128_map(CUtensorMap* map, const void* base, int64_t rows, int64_t cols, int64_t ld) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return fail(DSCQ_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld)};
  cuuint32_t box[2] = {128u, 128u};
  cuuint32_t estr[2] = {1u, 1u};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(DSCQ_ERR_CUDA, "cuTensorMapEncodeTiled (int8 A) failed (" + std::to_string(r) + ")");
  return DSCQ_OK;
}

int g_num_sms = 0;

int num_sms() {
  if (!g_num_sms) {
    int dev = 0, n = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    g_num_sms = n > 0 ? n : 148;
  }
  return g_num_sms;
}

template <int BN, bool SWAP, bool SPLIT>
int launch_gemm_kernel(const CUtensorMap& tmP, const CUtensorMap& tmQ, const dscq::GemmParams& gp,
                       cudaStream_t stream) {
  using C = dscq::GemmCfg<BN>;
  auto kern = dscq::w4a4_gemm_tc<BN, SWAP, SPLIT>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmemBytes);
  if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(w4a4_gemm_tc)");
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(gp.tiles_i * gp.tiles_j * gp.splits));
  cfg.blockDim = dim3(C::kThreads);
  cfg.dynamicSmemBytes = C::kSmemBytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  if (SPLIT) {
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = static_cast<unsigned>(gp.splits);
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
  }
  e = cudaLaunchKernelEx(&cfg, kern, tmP, tmQ, gp);
  if (e != cudaSuccess) return cuda_fail(e, "launch w4a4_gemm_tc");
  return DSCQ_OK;
}

template <int LOGK>
cudaError_t launch_wht(const dscq::RowQuantParams& p, cudaStream_t st) {
  using C = dscq::WhtCfg<LOGK>;
  cudaError_t e = cudaFuncSetAttribute(dscq::wht_quant_pow2<LOGK>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       C::SMEM);
  if (e != cudaSuccess) return e;
  const unsigned grid = static_cast<unsigned>((p.rows_out + C::ROWS - 1) / C::ROWS);
  dscq::wht_quant_pow2<LOGK><<<grid, C::THREADS, C::SMEM, st>>>(p);
  return cudaGetLastError();
}

template <int AP>
cudaError_t launch_kron(const dscq::RowQuantParams& p, int a, int s, cudaStream_t st) {
  using C = dscq::KronCfg<AP>;
  cudaError_t e = cudaFuncSetAttribute(dscq::kron_quant<AP>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
  if (e != cudaSuccess) return e;
  const int grid = std::min(p.rows_out, num_sms());
  dscq::kron_quant<AP><<<grid, C::THREADS, C::SMEM, st>>>(p, a, s);
  return cudaGetLastError();
}

// The tcgen05 quantizer's A operand (H'^T as the MMA reads it from shared memory) is a constant of
// K. It is built once per (device, K) into a library-owned global buffer on the first call and kept
// until the process exits; every launch bulk-copies it into each CTA. The first call synchronises
// its stream and therefore cannot be part of a stream capture.
std::mutex g_operand_mu;
std::map<std::pair<int, int64_t>, uint8_t*> g_operands;

int rotq_operand(int dev, int64_t K, const dscq::RotqParams& rp, const int8_t* h_a, cudaStream_t st,
                 const uint8_t** out) {
  std::lock_guard<std::mutex> lock(g_operand_mu);
  auto it = g_operands.find({dev, K});
  if (it != g_operands.end()) {
    *out = it->second;
    return DSCQ_OK;
  }
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  cudaError_t e = cudaStreamIsCapturing(st, &cs);
  if (e != cudaSuccess) return cuda_fail(e, "cudaStreamIsCapturing");
  if (cs != cudaStreamCaptureStatusNone)
    return fail(DSCQ_ERR_UNSUPPORTED, "the first tcgen05 rotate+quantize call for K=" + std::to_string(K) +
                                          " on a device builds its Hadamard operand and cannot be captured; make "
                                          "one call before capturing");
  const int a = rp.a_base;
  if (a > 1) {  // the operand is cached by K: h_a must be the library's Hadamard factor of order a
    std::vector<int8_t> got(static_cast<size_t>(a) * a), want(static_cast<size_t>(a) * a);
    e = cudaMemcpyAsync(got.data(), h_a, got.size(), cudaMemcpyDeviceToHost, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    if (e != cudaSuccess) return cuda_fail(e, "reading h_a");
    if (!dscq::build_hadamard(a, want.data()) || got != want)
      return fail(DSCQ_ERR_INVALID, "h_a must hold the Hadamard factor dscq_hadamard(" + std::to_string(a) + ")");
  }
  uint8_t* buf = nullptr;
  e = cudaMalloc(&buf, rp.a_bytes);
  if (e != cudaSuccess) return cuda_fail(e, "cudaMalloc(rotate+quantize operand)");
  const int chunks = rp.mt * 128 * rp.nkb * 8;
  if (rp.mt == 1)
    dscq::rotq_build_operand<1><<<(chunks + 255) / 256, 256, 0, st>>>(rp, h_a, buf);
  else
    dscq::rotq_build_operand<2><<<(chunks + 255) / 256, 256, 0, st>>>(rp, h_a, buf);
  e = cudaGetLastError();
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  if (e != cudaSuccess) {
    cudaFree(buf);
    return cuda_fail(e, "building the rotate+quantize operand");
  }
  g_operands[{dev, K}] = buf;
  *out = buf;
  return DSCQ_OK;
}

// AUTO's choice of the tcgen05 rotate+quantize (a' = K / 64 rows of the dense factor). With its
// Hadamard operand prebuilt once per device and K it is as fast as the CUDA-core kernels or faster at
// every row count measured (CUDA-graph replays on B200, 16 to 2048 rows: K = 4096 5.8 vs 6.0 us at
// 16 rows and 11.5 vs 15.1 at 2048; K = 11008 6.2 vs 10.0 and 23.5 vs 59.0; K = 14336 6.6 vs 12.5),
// so AUTO takes it whenever a' >= 32. `rows` is kept for callers that decide for a batch.
bool rowquant_tc_auto(int ap_tc, int64_t rows) {
  return ap_tc >= 32 && rows >= 1;
}

template <int MT, int G>
cudaError_t launch_rotq(const CUtensorMap& tm, const dscq::RotqParams& rp, cudaStream_t st) {
  // at least 120 KB so that one CTA (which allocates all 512 TMEM columns) occupies an SM
  const size_t smem = std::max<size_t>(1024 + rp.a_bytes + static_cast<size_t>(rp.ns) * rp.stage_bytes + 1024,
                                       120 * 1024);
  cudaError_t e = cudaFuncSetAttribute(dscq::rotq_tc<MT, G>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  const int grid = std::min(rp.groups, num_sms());
  const int nwarps = std::max(std::max(rp.tma_warp, rp.mma_warp), rp.mma_warp2) + 1;
  const int threads = std::max(nwarps, (rp.nteam - 1) * rp.team_stride + rp.tw) * 32;
  if (threads > dscq::RqThreads<MT, G>::value) return cudaErrorInvalidConfiguration;
  dscq::rotq_tc<MT, G><<<grid, threads, smem, st>>>(tm, rp);
  return cudaGetLastError();
}

template <int BN>
int launch_gemm_persistent(const CUtensorMap& tmP, const CUtensorMap& tmQ, const dscq::GemmParams& gp,
                           cudaStream_t stream) {
  using C = dscq::PCfg<BN>;
  auto kern = dscq::w4a4_gemm_persistent<BN>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmemBytes);
  if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(w4a4_gemm_persistent)");
  const int tiles = gp.tiles_i * gp.tiles_j;
  const int grid = std::min(tiles, num_sms());
  kern<<<grid, dscq::kPersistThreads, C::kSmemBytes, stream>>>(tmP, tmQ, gp);
  e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "launch w4a4_gemm_persistent");
  return DSCQ_OK;
}

template <int BN>
int launch_gemm_a8(const CUtensorMap& tmA, const CUtensorMap& tmQ, const dscq::GemmParams& gp, cudaStream_t stream) {
  using C = dscq::A8Cfg<BN>;
  auto kern = dscq::w4a4_gemm_a8<BN>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmemBytes);
  if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(w4a4_gemm_a8)");
  const int tiles = gp.tiles_i * gp.tiles_j;
  const int grid = std::min(tiles, num_sms());
  kern<<<grid, dscq::kPersistThreads, C::kSmemBytes, stream>>>(tmA, tmQ, gp);
  e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "launch w4a4_gemm_a8");
  return DSCQ_OK;
}

template <int BN>
int launch_gemm_ldg(const dscq::GemmParams& gp, cudaStream_t stream) {
  using C = dscq::LCfg<BN>;
  auto kern = dscq::w4a4_gemm_persistent_ldg<BN>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmemBytes);
  if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(w4a4_gemm_persistent_ldg)");
  const int tiles = gp.tiles_i * gp.tiles_j;
  const int grid = std::min(tiles, num_sms());
  kern<<<grid, C::kThreads, C::kSmemBytes, stream>>>(gp);
  e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "launch w4a4_gemm_persistent_ldg");
  return DSCQ_OK;
}

int launch_gemm_pair(const CUtensorMap& tmP, const CUtensorMap& tmQ, const dscq::GemmParams& gp,
                     cudaStream_t stream) {
  using C = dscq::PairCfg;
  auto kern = dscq::w4a4_gemm_pair;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmemBytes);
  if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(w4a4_gemm_pair)");
  const int tiles = ((gp.M + 255) / 256) * gp.tiles_j;
  const int pairs = std::min(tiles, num_sms() / 2);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(2 * pairs));
  cfg.blockDim = dim3(dscq::kPairThreads);
  cfg.dynamicSmemBytes = C::kSmemBytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  e = cudaLaunchKernelEx(&cfg, kern, tmP, tmQ, gp);
  if (e != cudaSuccess) return cuda_fail(e, "launch w4a4_gemm_pair");
  return DSCQ_OK;
}

int launch_gemm_pair_a8(const CUtensorMap& tmA, const CUtensorMap& tmQ, const dscq::GemmParams& gp,
                        cudaStream_t stream) {
  using C = dscq::PairA8Cfg<DSCQ_PAIR_A8_ES, DSCQ_PAIR_A8_RS>;
  auto kern = dscq::w4a4_gemm_pair_a8<DSCQ_PAIR_A8_ES, DSCQ_PAIR_A8_RS>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmemBytes);
  if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(w4a4_gemm_pair_a8)");
  const int tiles = ((gp.M + 255) / 256) * gp.tiles_j;
  const int pairs = std::min(tiles, num_sms() / 2);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(2 * pairs));
  cfg.blockDim = dim3(dscq::kPairA8Threads);
  cfg.dynamicSmemBytes = C::kSmemBytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  e = cudaLaunchKernelEx(&cfg, kern, tmA, tmQ, gp);
  if (e != cudaSuccess) return cuda_fail(e, "launch w4a4_gemm_pair_a8");
  return DSCQ_OK;
}

int launch_gemm_pair_tm(const CUtensorMap& tmA, const CUtensorMap& tmB, const dscq::GemmParams& gp,
                        cudaStream_t stream) {
  using C = dscq::PairTmCfg;
  auto kern = dscq::w4a4_gemm_pair_tm;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmemBytes);
  if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(w4a4_gemm_pair_tm)");
  const int tiles = ((gp.M + 255) / 256) * gp.tiles_j;
  const int pairs = std::min(tiles, num_sms() / 2);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(2 * pairs));
  cfg.blockDim = dim3(dscq::kPairThreads);
  cfg.dynamicSmemBytes = C::kSmemBytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  e = cudaLaunchKernelEx(&cfg, kern, tmA, tmB, gp);
  if (e != cudaSuccess) return cuda_fail(e, "launch w4a4_gemm_pair_tm");
  return DSCQ_OK;
}

int launch_gemv(const dscq::GemmParams& gp, cudaStream_t stream) {
  const unsigned grid = static_cast<unsigned>((gp.N + 15) / 16);
  const int nt = (gp.M + 7) / 8;
  const unsigned threads = dscq::kGemvWarps * 32;
  if (nt <= 1)
    dscq::w4a4_gemv<1><<<grid, threads, 0, stream>>>(gp);
  else if (nt <= 2)
    dscq::w4a4_gemv<2><<<grid, threads, 0, stream>>>(gp);
  else
    dscq::w4a4_gemv<4><<<grid, threads, 0, stream>>>(gp);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "launch w4a4_gemv");
  return DSCQ_OK;
}

template <int BN, bool SWAP>
int dispatch_split(const CUtensorMap& tmP, const CUtensorMap& tmQ, const dscq::GemmParams& gp,
                   cudaStream_t stream) {
  return gp.splits > 1 ? launch_gemm_kernel<BN, SWAP, true>(tmP, tmQ, gp, stream)
                       : launch_gemm_kernel<BN, SWAP, false>(tmP, tmQ, gp, stream);
}

}  // namespace

extern "C" {

int dscq_version(void) { return 1; }

const char* dscq_last_error(void) { return g_err.c_str(); }

int dscq_device_status(int device, uint32_t* status, int clear) {
  DSCQ_REQUIRE(status != nullptr, "status must not be null");
  int prev = 0;
  cudaError_t e = cudaGetDevice(&prev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  e = cudaSetDevice(device);
  if (e != cudaSuccess) return cuda_fail(e, "cudaSetDevice");
  e = cudaDeviceSynchronize();
  if (e == cudaSuccess) e = cudaMemcpyFromSymbol(status, dscq::g_status, sizeof(uint32_t));
  if (e == cudaSuccess && clear) {
    const uint32_t zero = 0;
    e = cudaMemcpyToSymbol(dscq::g_status, &zero, sizeof(uint32_t));
  }
  cudaSetDevice(prev);
  if (e != cudaSuccess) return cuda_fail(e, "dscq_device_status");
  return DSCQ_OK;
}

int dscq_hadamard(int n, int8_t* out) {
  DSCQ_REQUIRE(out != nullptr, "out must not be null");
  if (!dscq::build_hadamard(n, out))
    return fail(DSCQ_ERR_UNSUPPORTED, "no Hadamard construction for order " + std::to_string(n));
  return DSCQ_OK;
}

int dscq_rowquant_auto_tc(int64_t K, int64_t rows) {
  int aa = 0, lb = 0;
  if (K < 1 || rows < 1 || !dscq::rotation_split(K, &aa, &lb)) return 0;
  const int ap_tc = lb >= 6 ? static_cast<int>(K / 64) : 0;
  return ap_tc >= 16 && ap_tc <= 224 && rowquant_tc_auto(ap_tc, rows) ? 1 : 0;
}

int dscq_rotation_split(int64_t K, int* a, int* b) {
  DSCQ_REQUIRE(a && b, "a and b must not be null");
  int aa = 0, lb = 0;
  if (!dscq::rotation_split(K, &aa, &lb))
    return fail(DSCQ_ERR_UNSUPPORTED, "K=" + std::to_string(K) + " has no supported Hadamard split");
  *a = aa;
  *b = 1 << lb;
  return DSCQ_OK;
}

int dscq_rowquant_headrot(const void* x, int64_t M, int64_t K, int64_t ld_x, int heads, const void* rot_hi,
                          const void* rot_lo, int mode, float clip, int64_t rows_out, int64_t KP, uint8_t* packed,
                          int64_t ld_packed, float* scales, int8_t* codes, int64_t ld_codes, void* stream) {
  DSCQ_REQUIRE(x && rot_hi && rot_lo && scales, "x, rot_hi, rot_lo and scales must not be null");
  DSCQ_REQUIRE(packed || codes, "need packed or codes output");
  DSCQ_REQUIRE(heads >= 4 && heads % 4 == 0 && heads / 4 <= dscq::kHrMaxCluster && K == 128 * heads,
               "head rotation needs K = 128 * heads with heads a multiple of 4, at most 64");
  DSCQ_REQUIRE(M >= 1 && rows_out >= M && rows_out <= (int64_t(1) << 30) && KP == K, "invalid rows / KP");
  DSCQ_REQUIRE(mode == DSCQ_ACT_SYM || mode == DSCQ_WEIGHT_SYM, "head rotation supports the symmetric modes");
  DSCQ_REQUIRE(clip > 0.f && clip <= 1.f, "clip must be in (0, 1]");
  DSCQ_REQUIRE(ld_x >= K && ld_x % 8 == 0 && aligned(x, 16) && aligned(rot_hi, 16) && aligned(rot_lo, 16),
               "x needs 16-byte aligned rows (ld_x a multiple of 8), rotations 16-byte aligned");
  DSCQ_REQUIRE(!packed || (ld_packed >= K / 2 && ld_packed % 16 == 0 && aligned(packed, 16)),
               "packed rows must be 16-byte aligned");
  DSCQ_REQUIRE(!codes || (ld_codes >= K && ld_codes % 16 == 0 && aligned(codes, 16)), "codes rows must be 16-byte aligned");
  int st = check_device(nullptr);
  if (st) return st;
  dscq::HeadRotParams hp{};
  dscq::RowQuantParams& p = hp.p;
  p.x = x;
  p.x_dtype = DSCQ_BF16;
  p.M = M;
  p.K = K;
  p.ld_x = ld_x;
  p.mode = mode;
  p.clip = clip;
  p.norm = 1.f;
  p.rows_out = rows_out;
  p.KP = KP;
  p.packed = packed;
  p.ld_packed = ld_packed;
  p.scales = scales;
  p.codes = codes;
  p.ld_codes = ld_codes;
  hp.heads = heads;
  hp.cluster = heads / 4;
  CUtensorMap tmX, tmHi, tmLo;
  if ((st = make_bf16_sw128_map(&tmX, x, M, K, ld_x))) return st;
  if ((st = make_bf16_sw128_map(&tmHi, rot_hi, static_cast<int64_t>(heads) * 128, 128, 128))) return st;
  if ((st = make_bf16_sw128_map(&tmLo, rot_lo, static_cast<int64_t>(heads) * 128, 128, 128))) return st;
  auto kern = dscq::headrot_quant;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, dscq::kHrSmem);
  if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(headrot_quant)");
  if (hp.cluster > 8) {
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(non-portable cluster)");
  }
  const int64_t tiles = (rows_out + 127) / 128;
  DSCQ_REQUIRE(tiles * hp.cluster < (int64_t(1) << 31), "problem too large");
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(tiles * hp.cluster));
  cfg.blockDim = dim3(dscq::kHrThreads);
  cfg.dynamicSmemBytes = dscq::kHrSmem;
  cfg.stream = static_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = static_cast<unsigned>(hp.cluster);
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  e = cudaLaunchKernelEx(&cfg, kern, tmX, tmHi, tmLo, hp);
  if (e != cudaSuccess) return cuda_fail(e, "launch headrot_quant");
  return DSCQ_OK;
}

int dscq_rowquant(const void* x, int x_dtype, int64_t M, int64_t K, int64_t ld_x, int rotate, int rot_a,
                  const int8_t* h_a, int mode, float clip, int64_t rows_out, int64_t KP, uint8_t* packed,
                  int64_t ld_packed, float* scales, int32_t* zeros, int32_t* row_sums, int8_t* codes,
                  int64_t ld_codes, void* stream) {
  return dscq_rowquant_variant(x, x_dtype, M, K, ld_x, rotate, rot_a, h_a, mode, clip, rows_out, KP, packed, ld_packed,
                               scales, zeros, row_sums, codes, ld_codes, DSCQ_QUANT_AUTO, stream);
}

int dscq_rowquant_variant(const void* x, int x_dtype, int64_t M, int64_t K, int64_t ld_x, int rotate, int rot_a,
                          const int8_t* h_a, int mode, float clip, int64_t rows_out, int64_t KP, uint8_t* packed,
                          int64_t ld_packed, float* scales, int32_t* zeros, int32_t* row_sums, int8_t* codes,
                          int64_t ld_codes, int variant, void* stream) {
  DSCQ_REQUIRE(variant >= DSCQ_QUANT_AUTO && variant <= DSCQ_QUANT_LEGACY, "unknown quantizer variant");
  DSCQ_REQUIRE(x && (packed || codes) && scales, "x, scales and packed or codes must not be null");
  DSCQ_REQUIRE(x_dtype == DSCQ_BF16 || x_dtype == DSCQ_F16 || x_dtype == DSCQ_F32, "x_dtype must be bf16/f16/f32");
  DSCQ_REQUIRE(M >= 1 && M <= (1 << 24), "require 1 <= M <= 2^24");
  DSCQ_REQUIRE(K >= 1 && K <= kMaxRowK, "require 1 <= K <= 1048576");
  DSCQ_REQUIRE(!rotate || K <= kMaxRotK, "the online rotation supports K <= 32768");
  DSCQ_REQUIRE(ld_x >= K, "ld_x must be >= K");
  DSCQ_REQUIRE(rows_out >= M && rows_out <= (1 << 24), "rows_out must be >= M");
  DSCQ_REQUIRE(KP >= K && KP % 2 == 0 && KP <= kMaxRowK + 64, "KP must be even and >= K");
  DSCQ_REQUIRE(!packed || ld_packed >= KP / 2, "ld_packed must be >= KP/2");
  DSCQ_REQUIRE(mode >= DSCQ_ACT_SYM && mode <= DSCQ_ACT_ASYM_TORCH, "unknown quantizer mode");
  DSCQ_REQUIRE(std::isfinite(clip) && clip > 0.f, "clip must be a positive finite number");
  DSCQ_REQUIRE(!(mode == DSCQ_ACT_ASYM || mode == DSCQ_ACT_ASYM_TORCH) || zeros, "asymmetric modes need zeros");
  DSCQ_REQUIRE(!codes || ld_codes >= KP, "ld_codes must be >= KP");
  int log2b = 0;
  if (rotate) {
    int a = 0;
    if (!dscq::rotation_split(K, &a, &log2b))
      return fail(DSCQ_ERR_UNSUPPORTED, "K=" + std::to_string(K) + " has no supported Hadamard split");
    DSCQ_REQUIRE(a == rot_a, "rot_a does not match the split of K (see dscq_rotation_split)");
    DSCQ_REQUIRE(a == 1 || h_a != nullptr, "h_a must point to the a x a Hadamard factor");
  }
  int st = check_device(nullptr);
  if (st) return st;

  dscq::RowQuantParams p;
  p.x = x;
  p.x_dtype = x_dtype;
  p.ld_x = ld_x;
  p.M = static_cast<int>(M);
  p.K = static_cast<int>(K);
  p.KP = static_cast<int>(KP);
  p.rows_out = static_cast<int>(rows_out);
  p.rotate = rotate ? 1 : 0;
  p.rot_a = rotate ? rot_a : 1;
  p.log2b = log2b;
  p.h_a = h_a;
  p.norm = rotate ? static_cast<float>(1.0 / std::sqrt(static_cast<double>(K))) : 1.f;
  p.mode = mode;
  p.clip = clip;
  p.packed = packed;
  p.ld_packed = ld_packed;
  p.scales = scales;
  p.zeros = zeros;
  p.row_sums = row_sums;
  p.codes = codes;
  p.ld_codes = ld_codes;

  cudaStream_t cst = static_cast<cudaStream_t>(stream);
  // tcgen05 path: K = a' * 64, a' <= 256, symmetric modes, bf16 rows, 16-byte aligned outputs
  const bool sym = mode == DSCQ_ACT_SYM || mode == DSCQ_WEIGHT_SYM;
  const int ap_tc = (rotate && log2b >= 6) ? static_cast<int>(K / 64) : 0;
  const bool tc_ok = rotate && log2b >= 6 && ap_tc >= 16 && ap_tc <= 224 && sym && x_dtype == DSCQ_BF16 &&
                     KP == K && aligned(x, 16) && ld_x % 8 == 0 && (!packed || (aligned(packed, 16) && ld_packed % 16 == 0)) &&
                     (!codes || (aligned(codes, 16) && ld_codes % 16 == 0));
  if (variant == DSCQ_QUANT_TC && !tc_ok)
    return fail(DSCQ_ERR_UNSUPPORTED, "tcgen05 rotate+quantize needs a rotation with K = a' * 64 (a' <= 224), a "
                                      "symmetric mode, bf16 input, KP == K and 16-byte aligned rows");
  const bool tc_auto = rowquant_tc_auto(ap_tc, rows_out);
  if (tc_ok && (variant == DSCQ_QUANT_TC || (variant == DSCQ_QUANT_AUTO && tc_auto))) {
    dscq::RotqParams rp;
    rp.p = p;
    rp.a_base = p.rot_a;
    rp.s_log = log2b - 6;
    rp.ap = ap_tc;
    rp.ap16 = (ap_tc + 15) / 16 * 16;
    rp.P = (rp.ap16 == 32 || rp.ap16 == 64) ? 128 / rp.ap16 : 1;
    rp.log2_ap16 = rp.ap16 == 32 ? 5 : 6;
    rp.mt = rp.ap16 <= 128 ? 1 : 2;
    rp.groups = static_cast<int>((rows_out + rp.P - 1) / rp.P);
    rp.ksteps = (rp.mt == 1 ? rp.P * rp.ap16 : rp.ap16) / 16;
    rp.nkb = (rp.ksteps * 16 + 63) / 64;
    rp.a_bytes = static_cast<uint32_t>(rp.mt * rp.nkb * 16384);
    rp.stage_bytes = static_cast<uint32_t>(rp.P * rp.ap16 * 128);
    rp.ns = std::min<int>(dscq::kRqMaxStages, (210 * 1024 - static_cast<int>(rp.a_bytes)) / static_cast<int>(rp.stage_bytes));
    // one MMA spans G token blocks: G = 4 (N = 256) with one M tile, 2 (N = 128) with two; the
    // stage ring holds whole groups. The epilogue (TMEM load, 64-point WHT, absmax, codes) is the
    // longest role: with one M tile four teams split each group's four blocks
    const int G = rp.mt == 1 ? 4 : 2;
    rp.ns = rp.ns / G * G;
    rp.split = rp.mt == 1 ? 1 : 0;
    if (rp.mt == 1) {  // four teams of four warps (lane quadrants 0-3), then the TMA and MMA warps
      rp.tw = 4;
      rp.team_stride = 4;
      rp.nteam = 4;
      rp.tma_warp = 16;
      rp.mma_warp = 17;
      rp.mma_warp2 = -1;
    } else {  // two teams of 4 + ceil((a' - 128) / 32) warps at warps 0.. and 8..
      rp.tw = 4 + (rp.ap - 128 + 31) / 32;
      rp.team_stride = 8;
      rp.nteam = 2;
      rp.tma_warp = rp.tw <= 6 ? 6 : (rp.tw == 7 ? 7 : 16);
      rp.mma_warp = rp.tw <= 6 ? 7 : (rp.tw == 7 ? 15 : 17);
      rp.mma_warp2 = rp.tw <= 6 ? 15 : -1;  // warp 15 is free when each team has at most 6 warps
    }
    if (rp.ns < 2) return fail(DSCQ_ERR_UNSUPPORTED, "tcgen05 rotate+quantize: shared memory too small");
    int dev = 0;
    cudaError_t ge = cudaGetDevice(&dev);
    if (ge != cudaSuccess) return cuda_fail(ge, "cudaGetDevice");
    st = rotq_operand(dev, K, rp, h_a, cst, &rp.a_op);
    if (st) return st;
    CUtensorMap tm;
    st = make_rows_map(&tm, x, M, rp.ap, ld_x, rp.ap16, rp.P);
    if (st) return st;
    cudaError_t e = rp.mt == 1 ? launch_rotq<1, 4>(tm, rp, cst) : launch_rotq<2, 2>(tm, rp, cst);
    if (e != cudaSuccess) return cuda_fail(e, "launch rotq_tc");
    return DSCQ_OK;
  }
  const bool fast = rotate && p.rot_a == 1 && log2b >= 10 && log2b <= 13 &&
                    (mode == DSCQ_ACT_SYM || mode == DSCQ_WEIGHT_SYM) && x_dtype == DSCQ_BF16 && KP == K &&
                    aligned(x, 16) && ld_x % 8 == 0 && (!packed || (aligned(packed, 2) && ld_packed % 2 == 0));
  if (fast) {
    cudaError_t e = cudaSuccess;
    switch (log2b) {
      case 10: e = launch_wht<10>(p, cst); break;
      case 11: e = launch_wht<11>(p, cst); break;
      case 12: e = launch_wht<12>(p, cst); break;
      default: e = launch_wht<13>(p, cst); break;
    }
    if (e != cudaSuccess) return cuda_fail(e, "launch wht_quant_pow2");
    return DSCQ_OK;
  }

  // Kronecker path: K = a' * 64 with the dense factor H' = H_a (x) H_(2^s), a' <= 224
  const int s_log = log2b - 6;
  const int ap = p.rot_a << (s_log > 0 ? s_log : 0);
  const bool kron = rotate && p.rot_a > 1 && s_log >= 0 && ap <= 224 && (mode == DSCQ_ACT_SYM || mode == DSCQ_WEIGHT_SYM) &&
                    x_dtype == DSCQ_BF16 && KP == K && aligned(x, 16) && ld_x % 8 == 0;
  if (kron) {
    cudaError_t e = ap <= 176 ? launch_kron<176>(p, p.rot_a, s_log, cst) : launch_kron<224>(p, p.rot_a, s_log, cst);
    if (e != cudaSuccess) return cuda_fail(e, "launch kron_quant");
    return DSCQ_OK;
  }

  // long rows K = a * 1024 with a dense factor a <= 32 (K = 28672: H_28 (x) H_1024)
  const bool klong = rotate && p.rot_a > 1 && p.rot_a <= 32 && log2b == 10 &&
                     (mode == DSCQ_ACT_SYM || mode == DSCQ_WEIGHT_SYM) && x_dtype == DSCQ_BF16 && KP == K &&
                     aligned(x, 16) && ld_x % 8 == 0 && (!packed || (aligned(packed, 4) && ld_packed % 4 == 0)) &&
                     (!codes || (aligned(codes, 8) && ld_codes % 8 == 0));
  if (klong) {
    using KC = dscq::KronLongCfg;
    cudaError_t e = cudaFuncSetAttribute(dscq::kron_long_quant, cudaFuncAttributeMaxDynamicSharedMemorySize, KC::SMEM);
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(kron_long_quant)");
    const int grid = static_cast<int>(std::min<int64_t>(rows_out, num_sms()));
    dscq::kron_long_quant<<<grid, KC::THREADS, KC::SMEM, cst>>>(p, p.rot_a);
    e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e, "launch kron_long_quant");
    return DSCQ_OK;
  }

  constexpr int T = 512;
  if (!rotate && K > kMaxRotK) {  // long rows: two passes over global memory, as kernel/w4a4.cu:20-63
    dscq::rowquant_stream<T><<<static_cast<unsigned>(rows_out), T, 0, cst>>>(p);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e, "launch rowquant_stream");
    return DSCQ_OK;
  }
  size_t smem = static_cast<size_t>(K) * sizeof(float) * ((rotate && p.rot_a > 32) ? 2 : 1);
  if (smem > 220 * 1024)
    return fail(DSCQ_ERR_UNSUPPORTED, "row of K=" + std::to_string(K) + " does not fit in shared memory");
  cudaError_t e = cudaFuncSetAttribute(dscq::rowquant_smem<T>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(smem));
  if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(rowquant)");
  dscq::rowquant_smem<T><<<static_cast<unsigned>(rows_out), T, smem, cst>>>(p);
  e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "launch rowquant");
  return DSCQ_OK;
}

int dscq_quantize(const void* x, int x_dtype, int64_t M, int64_t K, float clip, int fused, uint8_t* packed,
                  float* scales, int32_t* zeros, void* stream) {
  (void)fused;
  DSCQ_REQUIRE(M >= 1 && M <= 65535 && K >= 1 && K <= 1048576, "Require 1<=M<=65535 and 1<=K<=1048576");
  DSCQ_REQUIRE(clip >= 0.5f && clip <= 1.f, "Activation clip must be in [0.5,1]");
  DSCQ_REQUIRE(zeros != nullptr, "zeros must not be null");
  const int64_t MP = (M + 7) / 8 * 8, KP = (K + 63) / 64 * 64;
  return dscq_rowquant(x, x_dtype, M, K, K, 0, 1, nullptr, DSCQ_ACT_ASYM, clip, MP, KP, packed, KP / 2, scales,
                       zeros, nullptr, nullptr, 0, stream);
}

static int matmul_impl(const uint8_t* a, const uint8_t* b, const float* sx, const int32_t* zx, const float* sw,
                       const int32_t* sums, const void* bias, const void* residual, int64_t M, int64_t N, int64_t KP,
                       int out_dtype, void* const* outs, int n_outs, int64_t ld_out, int64_t col_off, int32_t* raw,
                       int variant, void* stream) {
  void* out = n_outs > 0 ? outs[0] : nullptr;
  DSCQ_REQUIRE(a && b && sx && sw, "a, b, sx and sw must not be null");
  DSCQ_REQUIRE(out || raw, "at least one of out / raw must be given");
  DSCQ_REQUIRE(n_outs >= 0 && n_outs <= 8, "at most 8 output buffers");
  for (int i = 0; i < n_outs; ++i) DSCQ_REQUIRE(outs[i] != nullptr, "output buffers must not be null");
  DSCQ_REQUIRE(col_off >= 0 && ld_out >= col_off + N, "ld_out must cover col_off + N");
  DSCQ_REQUIRE(M > 0 && M <= (1 << 24) && N > 0 && N <= (1 << 24) && KP > 0 && KP <= 1048576 && KP % 64 == 0,
               "Invalid dimensions (need M, N > 0 and KP a positive multiple of 64)");
  DSCQ_REQUIRE(!zx || sums, "asymmetric activations (zx) need weight code sums");
  DSCQ_REQUIRE(out_dtype == DSCQ_BF16 || out_dtype == DSCQ_F16 || out_dtype == DSCQ_F32, "out_dtype must be bf16/f16/f32");
  DSCQ_REQUIRE(aligned(a, 16) && aligned(b, 16), "packed operands must be 16-byte aligned");
  DSCQ_REQUIRE(variant >= DSCQ_GEMM_AUTO && variant <= DSCQ_GEMM_LARGE_M_PAIR_TMEM, "unknown GEMM variant");
  if (KP > kMaxGemmKP)
    return fail(DSCQ_ERR_UNSUPPORTED, "KP > 65536 is not supported: the int8 tensor-core accumulation (256 * sum) "
                                      "would overflow int32 (the reference's s4 WMMA path accepts KP <= 2^20)");
  int st = check_device(nullptr);
  if (st) return st;
  const int64_t kbytes = KP / 2;
  const int kblocks = static_cast<int>((KP + 127) / 128);
  const bool decode = M <= 32 && (variant == DSCQ_GEMM_AUTO || variant == DSCQ_GEMM_SMALL_M);
  const bool swap = variant == DSCQ_GEMM_SMALL_M || variant == DSCQ_GEMM_SMALL_M_TC ||
                    (variant == DSCQ_GEMM_AUTO && M <= 64);
  const int nsm = num_sms();
  int BN;
  int64_t ti, tj;
  int splits = 1;
  bool persistent = false;
  if (swap) {
    BN = M <= 16 ? 16 : (M <= 32 ? 32 : 64);
    ti = (N + 127) / 128;
    tj = (M + BN - 1) / BN;
    while (splits < 8 && ti * tj * splits * 2 <= nsm && kblocks >= splits * 2 * 2) splits *= 2;
  } else {
    ti = (M + 127) / 128;
    const int64_t t256 = ti * ((N + 255) / 256), t128 = ti * ((N + 127) / 128);
    if (t128 * 2 <= nsm) {
      BN = 128;  // too few tiles: split K across a cluster
      while (splits < 8 && t128 * splits * 2 <= nsm && kblocks >= splits * 2 * 2) splits *= 2;
    } else {
      // 256-wide tiles (the CTA-pair kernel) whenever every pair gets at least one: a pair tile runs
      // about 1.9x the int ops per SM-second of a 128-wide 1-CTA tile, which outweighs the better
      // wave quantisation of the smaller tiles (M = N = 4096, K = 8192 on 128-wide tiles: 0.20 ms,
      // as long as N = 8192 on pair tiles)
      BN = t256 >= nsm / 2 ? 256 : 128;
    }
    if (variant == DSCQ_GEMM_LARGE_M_PAIR_TMEM) {  // 256 x 192 pair tiles, activations in TMEM
      BN = 192;
      splits = 1;
    }
    tj = (N + BN - 1) / BN;
    persistent = splits == 1;
  }
  const int64_t tiles = ti * tj;
  DSCQ_REQUIRE(tiles * 8 < (int64_t(1) << 31), "problem too large");

  CUtensorMap tmP, tmQ;
  const uint8_t* P = swap ? b : a;
  const uint8_t* Q = swap ? a : b;
  const int64_t rowsP = swap ? N : M, rowsQ = swap ? M : N;
  const bool pair_tm = variant == DSCQ_GEMM_LARGE_M_PAIR_TMEM;
  st = pair_tm ? make_u8_map_sw64(&tmP, P, rowsP, kbytes, kbytes, 128) : make_u8_map(&tmP, P, rowsP, kbytes, kbytes, 128);
  if (st) return st;
  // AUTO takes the CTA-pair kernel whenever the 256-wide tile is chosen (2-SM MMAs); LARGE_M keeps
  // the 1-CTA persistent kernel for A/B timing
  const bool pair = persistent && BN == 256 && (variant == DSCQ_GEMM_LARGE_M_PAIR || variant == DSCQ_GEMM_AUTO);
  st = make_u8_map(&tmQ, Q, rowsQ, kbytes, kbytes, pair_tm ? dscq::PairTmCfg::kBRows : (pair ? 128 : BN));
  if (st) return st;

  dscq::GemmParams gp;
  gp.M = static_cast<int>(M);
  gp.N = static_cast<int>(N);
  gp.kblocks = kblocks;
  gp.tiles_i = static_cast<int>(ti);
  gp.tiles_j = static_cast<int>(tj);
  gp.splits = splits;
  gp.sx = sx;
  gp.zx = zx;
  gp.sw = sw;
  gp.wsum = sums;
  gp.bias = bias;
  gp.residual = residual;
  gp.out = out;
  gp.raw = raw;
  gp.out_dtype = out_dtype;
  bool vec = out != nullptr && ld_out % 8 == 0 && col_off % 8 == 0;
  for (int i = 0; i < n_outs; ++i) vec = vec && aligned(outs[i], 16);
  gp.vec_out = vec ? 1 : 0;
  gp.ld_out = ld_out;
  gp.col_off = static_cast<int>(col_off);
  gp.n_outs = n_outs;
  for (int i = 0; i < 8; ++i) gp.outs[i] = i < n_outs ? outs[i] : nullptr;
  gp.P = P;
  gp.Q = Q;
  gp.kbytes = static_cast<int>(kbytes);
  gp.rowsP = static_cast<int>(rowsP);
  gp.rowsQ = static_cast<int>(rowsQ);

  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (decode) {
    gp.P = a;  // activations
    gp.Q = b;  // weights
    return launch_gemv(gp, s);
  }
  if (pair_tm) return launch_gemm_pair_tm(tmP, tmQ, gp, s);
  if (pair) return launch_gemm_pair(tmP, tmQ, gp, s);
  if (persistent && variant == DSCQ_GEMM_LARGE_M_DIRECT)
    return BN == 256 ? launch_gemm_ldg<256>(gp, s) : launch_gemm_ldg<128>(gp, s);
  if (persistent)
    return BN == 256 ? launch_gemm_persistent<256>(tmP, tmQ, gp, s) : launch_gemm_persistent<128>(tmP, tmQ, gp, s);
  if (swap) {
    if (BN == 16) return dispatch_split<16, true>(tmP, tmQ, gp, s);
    if (BN == 32) return dispatch_split<32, true>(tmP, tmQ, gp, s);
    return dispatch_split<64, true>(tmP, tmQ, gp, s);
  }
  if (BN == 256) return dispatch_split<256, false>(tmP, tmQ, gp, s);
  return dispatch_split<128, false>(tmP, tmQ, gp, s);
}

int dscq_matmul(const uint8_t* a, const uint8_t* b, const float* sx, const int32_t* zx, const float* sw,
                const int32_t* sums, const void* bias, const void* residual, int64_t M, int64_t N, int64_t KP,
                int out_dtype, void* out, int32_t* raw, int variant, void* stream) {
  void* outs[1] = {out};
  return matmul_impl(a, b, sx, zx, sw, sums, bias, residual, M, N, KP, out_dtype, outs, out ? 1 : 0, N, 0, raw, variant,
                     stream);
}

int dscq_matmul_cols(const uint8_t* a, const uint8_t* b, const float* sx, const int32_t* zx, const float* sw,
                     const int32_t* sums, const void* bias, const void* residual, int64_t M, int64_t N, int64_t KP,
                     int out_dtype, void* const* outs, int n_outs, int64_t ld_out, int64_t col_off, int variant,
                     void* stream) {
  DSCQ_REQUIRE(outs != nullptr && n_outs >= 1, "need at least one output buffer");
  return matmul_impl(a, b, sx, zx, sw, sums, bias, residual, M, N, KP, out_dtype, outs, n_outs, ld_out, col_off,
                     nullptr, variant, stream);
}

int dscq_scatter_block(const void* src, int64_t ld_src, int64_t rows, int64_t width, void* const* dsts, int n_dst,
                       int64_t ld_dst, void* stream) {
  DSCQ_REQUIRE(src != nullptr && dsts != nullptr && n_dst >= 1 && n_dst <= 8, "need a source and 1..8 destinations");
  DSCQ_REQUIRE(rows >= 0 && width >= 0 && width % 16 == 0, "width must be a non-negative multiple of 16 bytes");
  DSCQ_REQUIRE(ld_src % 16 == 0 && ld_dst % 16 == 0 && ld_src >= width && ld_dst >= width,
               "row strides must be multiples of 16 bytes and cover the width");
  DSCQ_REQUIRE(aligned(src, 16), "source must be 16-byte aligned");
  dscq::ScatterParams p{};
  p.src = static_cast<const uint8_t*>(src);
  p.ld_src = ld_src;
  p.ld_dst = ld_dst;
  p.rows = rows;
  p.width = width;
  p.n_dst = n_dst;
  for (int i = 0; i < n_dst; ++i) {
    DSCQ_REQUIRE(dsts[i] != nullptr && aligned(dsts[i], 16), "destinations must be non-null and 16-byte aligned");
    p.dst[i] = static_cast<uint8_t*>(dsts[i]);
  }
  if (rows == 0 || width == 0) return DSCQ_OK;
  int st = check_device(nullptr);
  if (st) return st;
  const int64_t units = ((rows + 7) / 8) * ((width + 63) / 64);
  const int64_t want = (units + 3) / 4;  // 4 warps per CTA
  const unsigned grid = static_cast<unsigned>(std::max<int64_t>(1, std::min<int64_t>(want, 4 * num_sms())));
  dscq::scatter_block_kernel<<<grid, 128, 0, static_cast<cudaStream_t>(stream)>>>(p);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "launch scatter_block");
  return DSCQ_OK;
}

int dscq_matmul_a8(const int8_t* a, int64_t ld_a, const uint8_t* b, const float* sx, const float* sw, const void* bias,
                   const void* residual, int64_t M, int64_t N, int64_t KP, int out_dtype, void* out, int32_t* raw,
                   void* stream) {
  return dscq_matmul_a8_variant(a, ld_a, b, sx, sw, bias, residual, M, N, KP, out_dtype, out, raw, DSCQ_GEMM_AUTO,
                                stream);
}

int dscq_matmul_a8_variant(const int8_t* a, int64_t ld_a, const uint8_t* b, const float* sx, const float* sw,
                           const void* bias, const void* residual, int64_t M, int64_t N, int64_t KP, int out_dtype,
                           void* out, int32_t* raw, int variant, void* stream) {
  DSCQ_REQUIRE(variant == DSCQ_GEMM_AUTO || variant == DSCQ_GEMM_LARGE_M || variant == DSCQ_GEMM_LARGE_M_PAIR,
               "dscq_matmul_a8 variant must be AUTO, LARGE_M or LARGE_M_PAIR");
  DSCQ_REQUIRE(a && b && sx && sw, "a, b, sx and sw must not be null");
  DSCQ_REQUIRE(out || raw, "at least one of out / raw must be given");
  DSCQ_REQUIRE(M > 0 && M <= (1 << 24) && N > 0 && N <= (1 << 24) && KP > 0 && KP <= 1048576 && KP % 64 == 0,
               "Invalid dimensions (need M, N > 0 and KP a positive multiple of 64)");
  DSCQ_REQUIRE(ld_a >= KP && ld_a % 16 == 0, "ld_a must be >= KP and a multiple of 16");
  if (KP > kMaxGemmKP) return fail(DSCQ_ERR_UNSUPPORTED, "KP > 65536 is not supported by the int8 GEMMs");
  DSCQ_REQUIRE(aligned(a, 16) && aligned(b, 16), "operands must be 16-byte aligned");
  DSCQ_REQUIRE(out_dtype == DSCQ_BF16 || out_dtype == DSCQ_F16 || out_dtype == DSCQ_F32, "out_dtype must be bf16/f16/f32");
  int st = check_device(nullptr);
  if (st) return st;
  const int64_t kbytes = KP / 2;
  const int nsm = num_sms();
  const int64_t ti = (M + 127) / 128;
  const int64_t t256 = ti * ((N + 255) / 256), t128 = ti * ((N + 127) / 128);
  auto eff = [&](int64_t t) { return static_cast<double>(t) / (((t + nsm - 1) / nsm) * nsm); };
  const int BN = variant == DSCQ_GEMM_LARGE_M_PAIR || (t256 >= nsm / 2 && eff(t256) + 0.1 >= eff(t128)) ? 256 : 128;
  // LARGE_M keeps the 1-CTA kernel; AUTO and LARGE_M_PAIR take the CTA-pair kernel for 256-wide tiles
  const bool pair = BN == 256 && variant != DSCQ_GEMM_LARGE_M;
  const int64_t tj = (N + BN - 1) / BN;
  DSCQ_REQUIRE(ti * tj * 8 < (int64_t(1) << 31), "problem too large");
  CUtensorMap tmA, tmQ;
  st = make_i8_sw128_map(&tmA, a, M, KP, ld_a);
  if (st) return st;
  st = make_u8_map(&tmQ, b, N, kbytes, kbytes, pair ? 128 : BN);
  if (st) return st;
  dscq::GemmParams gp;
  gp.M = static_cast<int>(M);
  gp.N = static_cast<int>(N);
  gp.kblocks = static_cast<int>((KP + 127) / 128);
  gp.tiles_i = static_cast<int>(ti);
  gp.tiles_j = static_cast<int>(tj);
  gp.splits = 1;
  gp.sx = sx;
  gp.zx = nullptr;
  gp.sw = sw;
  gp.wsum = nullptr;
  gp.bias = bias;
  gp.residual = residual;
  gp.out = out;
  gp.raw = raw;
  gp.out_dtype = out_dtype;
  gp.vec_out = (out != nullptr && N % 8 == 0 && aligned(out, 16)) ? 1 : 0;
  gp.P = nullptr;
  gp.Q = b;
  gp.kbytes = static_cast<int>(kbytes);
  gp.rowsP = static_cast<int>(M);
  gp.rowsQ = static_cast<int>(N);
  gp.ld_out = N;
  gp.col_off = 0;
  gp.n_outs = out ? 1 : 0;
  for (int i = 0; i < 8; ++i) gp.outs[i] = nullptr;
  gp.outs[0] = out;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (pair) return launch_gemm_pair_a8(tmA, tmQ, gp, s);
  return BN == 256 ? launch_gemm_a8<256>(tmA, tmQ, gp, s) : launch_gemm_a8<128>(tmA, tmQ, gp, s);
}

int dscq_rmsnorm(const void* x, const void* w, int64_t rows, int64_t H, float eps, void* y, void* stream) {
  DSCQ_REQUIRE(x && w && y, "x, w and y must not be null");
  DSCQ_REQUIRE(rows >= 1 && rows < (int64_t(1) << 31) && H >= 8 && H % 8 == 0 && H <= (1 << 20),
               "rmsnorm needs rows >= 1 and H a positive multiple of 8");
  DSCQ_REQUIRE(aligned(x, 16) && aligned(w, 16) && aligned(y, 16), "rmsnorm buffers must be 16-byte aligned");
  int st = check_device(nullptr);
  if (st) return st;
  dscq::rmsnorm_kernel<<<static_cast<unsigned>(rows), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(x), static_cast<const __nv_bfloat16*>(w), static_cast<__nv_bfloat16*>(y),
      static_cast<int>(H), eps);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "launch rmsnorm");
  return DSCQ_OK;
}

int dscq_rope(void* q, void* k, const void* cos_t, const void* sin_t, int64_t S, int Hq, int Hk, int D, void* stream) {
  DSCQ_REQUIRE(q && k && cos_t && sin_t, "q, k, cos and sin must not be null");
  DSCQ_REQUIRE(S >= 1 && Hq >= 1 && Hk >= 1 && D >= 2 && D % 2 == 0 && D <= 1024, "invalid rope shape");
  int st = check_device(nullptr);
  if (st) return st;
  const bool vec = (D / 2) % 8 == 0 && aligned(q, 16) && aligned(k, 16) && aligned(cos_t, 16) && aligned(sin_t, 16);
  const int64_t total = S * (Hq + Hk) * (D / 2) / (vec ? 8 : 1);
  const unsigned grid = static_cast<unsigned>(std::min<int64_t>((total + 255) / 256, int64_t(num_sms()) * 16));
  auto* qq = static_cast<__nv_bfloat16*>(q);
  auto* kk = static_cast<__nv_bfloat16*>(k);
  const auto* cc = static_cast<const __nv_bfloat16*>(cos_t);
  const auto* ss = static_cast<const __nv_bfloat16*>(sin_t);
  if (vec)
    dscq::rope_vec_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(qq, kk, cc, ss, static_cast<int>(S), Hq,
                                                                               Hk, D);
  else
    dscq::rope_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(qq, kk, cc, ss, static_cast<int>(S), Hq, Hk,
                                                                           D);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "launch rope");
  return DSCQ_OK;
}

int dscq_silu_mul(const void* g, const void* u, int64_t n, void* y, void* stream) {
  DSCQ_REQUIRE(g && u && y, "g, u and y must not be null");
  DSCQ_REQUIRE(n >= 8 && n % 8 == 0, "silu_mul needs n a positive multiple of 8");
  DSCQ_REQUIRE(aligned(g, 16) && aligned(u, 16) && aligned(y, 16), "silu_mul buffers must be 16-byte aligned");
  int st = check_device(nullptr);
  if (st) return st;
  const unsigned grid = static_cast<unsigned>(std::min<int64_t>((n / 8 + 255) / 256, int64_t(num_sms()) * 16));
  dscq::silu_mul_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(g), static_cast<const __nv_bfloat16*>(u), static_cast<__nv_bfloat16*>(y), n);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "launch silu_mul");
  return DSCQ_OK;
}

int dscq_pack_int4(const int8_t* codes, int64_t rows, int64_t K, int64_t ld_codes, uint8_t* packed,
                   int64_t ld_packed, int32_t* bad_count, void* stream) {
  DSCQ_REQUIRE(codes && packed && bad_count, "codes, packed and bad_count must not be null");
  DSCQ_REQUIRE(rows >= 0 && K >= 1 && ld_codes >= K && ld_packed >= (K + 1) / 2, "invalid pack_int4 shape");
  int st = check_device(nullptr);
  if (st) return st;
  if (rows == 0) return DSCQ_OK;
  const int64_t total = rows * ((K + 1) / 2);
  const unsigned grid = static_cast<unsigned>(std::min<int64_t>((total + 255) / 256, 148 * 32));
  dscq::pack_int4_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(codes, rows, K, ld_codes, packed,
                                                                             ld_packed, bad_count);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "launch pack_int4");
  return DSCQ_OK;
}

int dscq_unpack_int4(const uint8_t* packed, int64_t rows, int64_t ld_packed, int64_t width, int8_t* codes,
                     int64_t ld_codes, void* stream) {
  DSCQ_REQUIRE(codes && packed, "codes and packed must not be null");
  DSCQ_REQUIRE(rows >= 0 && width >= 0 && ld_codes >= width && ld_packed >= (width + 1) / 2,
               "invalid unpack_int4 shape");
  int st = check_device(nullptr);
  if (st) return st;
  if (rows == 0 || width == 0) return DSCQ_OK;
  const int64_t total = rows * width;
  const unsigned grid = static_cast<unsigned>(std::min<int64_t>((total + 255) / 256, 148 * 32));
  dscq::unpack_int4_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(packed, rows, ld_packed, width,
                                                                               codes, ld_codes);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "launch unpack_int4");
  return DSCQ_OK;
}

}  // extern "C"

// ------------------------------------------------------------ rotate+quantize without allocation
// For callers that must not allocate device memory: serving engines that reserve all of HBM up
// front for weights and KV cache and hand out memory only from their own pool, or latency-critical
// paths that cannot take cudaMalloc's implicit device synchronisation. dscq_rowquant builds the
// tcgen05 quantizer's Hadamard operand once per device and K into a buffer it allocates with
// cudaMalloc; this variant keeps that operand in a fixed array instead, rebuilt by every call.

// Largest operand of the tcgen05 quantizer: two 128-row M tiles x four 64-wide k atoms (a' <= 256).
constexpr uint32_t kRotqScratchBytes = 128u * 1024u;

// The operand scratch: one array per device, loaded with the library and held until the process
// exits. Host code must not use this name as a device address; see rotq_scratch_address.
static __device__ __align__(256) uint8_t g_rotq_scratch[kRotqScratchBytes];

namespace {

std::mutex g_scratch_mu;
void* g_scratch_addr[64] = {};

// Device address of g_rotq_scratch for device `dev` (which must be current): looked up once per
// device with cudaGetSymbolAddress, then cached.
int rotq_scratch_address(int dev, void** out) {
  if (dev < 0 || dev >= 64) return fail(DSCQ_ERR_UNSUPPORTED, "device index out of range for the scratch cache");
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (g_scratch_addr[dev] == nullptr) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_rotq_scratch);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(rotate+quantize scratch)");
    g_scratch_addr[dev] = p;
  }
  *out = g_scratch_addr[dev];
  return DSCQ_OK;
}

}  // namespace

extern "C" int dscq_rowquant_tc_noalloc(const void* x, int x_dtype, int64_t M, int64_t K, int64_t ld_x, int rotate,
                                        int rot_a, const int8_t* h_a, int mode, float clip, int64_t rows_out,
                                        int64_t KP, uint8_t* packed, int64_t ld_packed, float* scales,
                                        int32_t* zeros, int32_t* row_sums, int8_t* codes, int64_t ld_codes,
                                        void* stream) {
  (void)zeros;  // symmetric modes only: no zero points
  DSCQ_REQUIRE(x && (packed || codes) && scales, "x, scales and packed or codes must not be null");
  DSCQ_REQUIRE(M >= 1 && M <= (1 << 24) && rows_out >= M && rows_out <= (1 << 24), "require 1 <= M <= rows_out <= 2^24");
  DSCQ_REQUIRE(K >= 1 && K <= kMaxRotK && ld_x >= K, "require 1 <= K <= 32768 and ld_x >= K");
  DSCQ_REQUIRE(!packed || ld_packed >= KP / 2, "ld_packed must be >= KP/2");
  DSCQ_REQUIRE(!codes || ld_codes >= KP, "ld_codes must be >= KP");
  DSCQ_REQUIRE(std::isfinite(clip) && clip > 0.f, "clip must be a positive finite number");
  int log2b = 0, a = 0;
  if (!rotate || !dscq::rotation_split(K, &a, &log2b))
    return fail(DSCQ_ERR_UNSUPPORTED, "dscq_rowquant_tc_noalloc needs the online rotation with a supported split of K");
  DSCQ_REQUIRE(a == rot_a && (a == 1 || h_a != nullptr), "rot_a / h_a must be the Hadamard factor of K's split");
  const int ap = log2b >= 6 ? static_cast<int>(K / 64) : 0;
  const bool sym = mode == DSCQ_ACT_SYM || mode == DSCQ_WEIGHT_SYM;
  if (!(ap >= 16 && ap <= 224 && sym && x_dtype == DSCQ_BF16 && KP == K && aligned(x, 16) && ld_x % 8 == 0 &&
        (!packed || (aligned(packed, 16) && ld_packed % 16 == 0)) && (!codes || (aligned(codes, 16) && ld_codes % 16 == 0))))
    return fail(DSCQ_ERR_UNSUPPORTED, "dscq_rowquant_tc_noalloc: needs K = a' * 64 (16 <= a' <= 224), a symmetric "
                                      "mode, bf16 input, KP == K and 16-byte aligned rows");
  int dev = 0;
  int st = check_device(&dev);
  if (st) return st;

  dscq::RotqParams rp;
  dscq::RowQuantParams& p = rp.p;
  p.x = x;
  p.x_dtype = x_dtype;
  p.ld_x = ld_x;
  p.M = static_cast<int>(M);
  p.K = static_cast<int>(K);
  p.KP = static_cast<int>(KP);
  p.rows_out = static_cast<int>(rows_out);
  p.rotate = 1;
  p.rot_a = a;
  p.log2b = log2b;
  p.h_a = h_a;
  p.norm = static_cast<float>(1.0 / std::sqrt(static_cast<double>(K)));
  p.mode = mode;
  p.clip = clip;
  p.packed = packed;
  p.ld_packed = ld_packed;
  p.scales = scales;
  p.zeros = nullptr;
  p.row_sums = row_sums;
  p.codes = codes;
  p.ld_codes = ld_codes;
  rp.a_base = a;
  rp.s_log = log2b - 6;
  rp.ap = ap;
  rp.ap16 = (ap + 15) / 16 * 16;
  rp.P = (rp.ap16 == 32 || rp.ap16 == 64) ? 128 / rp.ap16 : 1;
  rp.log2_ap16 = rp.ap16 == 32 ? 5 : 6;
  rp.mt = rp.ap16 <= 128 ? 1 : 2;
  rp.groups = static_cast<int>((rows_out + rp.P - 1) / rp.P);
  rp.ksteps = (rp.mt == 1 ? rp.P * rp.ap16 : rp.ap16) / 16;
  rp.nkb = (rp.ksteps * 16 + 63) / 64;
  rp.a_bytes = static_cast<uint32_t>(rp.mt * rp.nkb * 16384);
  rp.stage_bytes = static_cast<uint32_t>(rp.P * rp.ap16 * 128);
  rp.ns = std::min<int>(dscq::kRqMaxStages, (210 * 1024 - static_cast<int>(rp.a_bytes)) / static_cast<int>(rp.stage_bytes));
  const int G = rp.mt == 1 ? 4 : 2;
  rp.ns = rp.ns / G * G;
  rp.split = rp.mt == 1 ? 1 : 0;
  if (rp.mt == 1) {
    rp.tw = 4;
    rp.team_stride = 4;
    rp.nteam = 4;
    rp.tma_warp = 16;
    rp.mma_warp = 17;
    rp.mma_warp2 = -1;
  } else {
    rp.tw = 4 + (rp.ap - 128 + 31) / 32;
    rp.team_stride = 8;
    rp.nteam = 2;
    rp.tma_warp = rp.tw <= 6 ? 6 : (rp.tw == 7 ? 7 : 16);
    rp.mma_warp = rp.tw <= 6 ? 7 : (rp.tw == 7 ? 15 : 17);
    rp.mma_warp2 = rp.tw <= 6 ? 15 : -1;
  }
  if (rp.ns < 2) return fail(DSCQ_ERR_UNSUPPORTED, "tcgen05 rotate+quantize: shared memory too small");
  if (rp.a_bytes > kRotqScratchBytes)
    return fail(DSCQ_ERR_UNSUPPORTED, "K=" + std::to_string(K) + " needs " + std::to_string(rp.a_bytes) +
                                          " bytes of operand scratch; the static scratch holds " +
                                          std::to_string(kRotqScratchBytes));
  void* scratch = nullptr;
  st = rotq_scratch_address(dev, &scratch);
  if (st) return st;
  cudaStream_t cst = static_cast<cudaStream_t>(stream);
  // The builder writes every byte of the operand region, so nothing left by an earlier call (of
  // another K) survives into this one.
  const int chunks = rp.mt * 128 * rp.nkb * 8;
  if (rp.mt == 1)
    dscq::rotq_build_operand<1><<<(chunks + 255) / 256, 256, 0, cst>>>(rp, h_a, static_cast<uint8_t*>(scratch));
  else
    dscq::rotq_build_operand<2><<<(chunks + 255) / 256, 256, 0, cst>>>(rp, h_a, static_cast<uint8_t*>(scratch));
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "launch rotq_build_operand (static scratch)");
  rp.a_op = static_cast<const uint8_t*>(scratch);
  CUtensorMap tm;
  st = make_rows_map(&tm, x, M, rp.ap, ld_x, rp.ap16, rp.P);
  if (st) return st;
  e = rp.mt == 1 ? launch_rotq<1, 4>(tm, rp, cst) : launch_rotq<2, 2>(tm, rp, cst);
  if (e != cudaSuccess) return cuda_fail(e, "launch rotq_tc (static scratch)");
  return DSCQ_OK;
}
