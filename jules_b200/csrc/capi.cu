// C ABI of the jules_b200 library (include/jules_kernels.h): argument
// validation, path selection (tensor-core vs CUDA-core kernel) and launches.
//
// Single translation unit for all device code, so the device error word
// (jb::g_dev_error) is one symbol without relocatable device code.
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <map>
#include <set>
#include <mutex>
#include <string>
#include <utility>
#include <type_traits>

#include "../../include/jules_kernels.h"
#include "attn_tc.cuh"
#include "attn_bwd.cuh"
#include "gemm_tc.cuh"
#include "gemm_i8.cuh"
#include "sm100.cuh"
#include "simt.cuh"
#include "rowwise.cuh"
#include "train.cuh"

namespace {

thread_local char g_errbuf[512];

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_errbuf, sizeof(g_errbuf), fmt, ap);
  va_end(ap);
  return code;
}

int cuda_fail(cudaError_t e, const char* what) {
  return fail(JULES_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

int ok() {
  g_errbuf[0] = 0;
  return JULES_OK;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// ---------------------------------------------------------------------------
// Per-device facts, looked up once.
// ---------------------------------------------------------------------------
constexpr int kMaxDevices = 64;
struct DeviceInfo {
  int sms = 0;
};
DeviceInfo g_dev[kMaxDevices];
std::mutex g_dev_mu;

int current_device(int* dev) {
  cudaError_t e = cudaGetDevice(dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (*dev < 0 || *dev >= kMaxDevices) return fail(JULES_ERR_CUDA, "device index %d", *dev);
  return JULES_OK;
}

int device_sms(int dev) {
  if (g_dev[dev].sms == 0) {
    int v = 0;
    cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
    g_dev[dev].sms = v > 0 ? v : 148;
  }
  return g_dev[dev].sms;
}

// ---------------------------------------------------------------------------
// Tensor maps (driver entry point, so the library needs no -lcuda).
// ---------------------------------------------------------------------------
PFN_cuTensorMapEncodeTiled_v12000 tmap_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// rank-2 or rank-3 map of 16-bit elements (bf16 or f16) with 128-byte swizzle.
int make_tmap_bf16(CUtensorMap* map, const void* base, int rank, const uint64_t* dims,
                   const uint64_t* strides_bytes, const uint32_t* box,
                   CUtensorMapDataType dt = CU_TENSOR_MAP_DATA_TYPE_BFLOAT16) {
  auto enc = tmap_encoder();
  if (!enc) return fail(JULES_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  cuuint64_t d[3];
  cuuint64_t st[2];
  cuuint32_t bx[3];
  cuuint32_t es[3] = {1, 1, 1};
  for (int i = 0; i < rank; ++i) {
    d[i] = dims[i];
    bx[i] = box[i];
  }
  for (int i = 0; i < rank - 1; ++i) st[i] = strides_bytes[i];
  CUresult r = enc(map, dt, rank, const_cast<void*>(base), d, st,
                   bx, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(JULES_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return JULES_OK;
}

// 2-D int8 tensor map (row-major [rows, cols], cols contiguous), 128-byte
// swizzle.
int make_tmap_i8(CUtensorMap* map, const void* base, uint64_t cols, uint64_t rows,
                 uint32_t box_cols, uint32_t box_rows) {
  auto enc = tmap_encoder();
  if (!enc) return fail(JULES_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  cuuint64_t d[2] = {cols, rows};
  cuuint64_t st[1] = {cols};
  cuuint32_t bx[2] = {box_cols, box_rows};
  cuuint32_t es[2] = {1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), d, st, bx, es,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(JULES_ERR_CUDA, "cuTensorMapEncodeTiled (int8) failed (%d)", (int)r);
  return JULES_OK;
}

// Dynamic shared memory limit of a kernel, raised once per (device, kernel).
int ensure_smem_attr(const void* kern, size_t smem, int dev) {
  static std::set<std::pair<int, const void*>> done;
  std::lock_guard<std::mutex> lk(g_dev_mu);
  if (done.count({dev, kern})) return JULES_OK;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute");
  done.insert({dev, kern});
  return JULES_OK;
}

int check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, what);
  return ok();
}

// ---------------------------------------------------------------------------
// GEMM paths
// ---------------------------------------------------------------------------
constexpr int kGemmBN = 256;
constexpr int kGemmStages = 4;

template <typename TIn>
constexpr CUtensorMapDataType tmap_dtype() {
  return std::is_same<TIn, __half>::value   ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
         : std::is_same<TIn, float>::value ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                           : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
}

// TIn: __nv_bfloat16 or __half operands (and residual); TOut: TIn or float.
template <typename TIn, typename TOut>
int gemm_tc(const TIn* A, const TIn* W, const float* bias, const TIn* res, TOut* C, int64_t M,
            int64_t N, int64_t K, int act, cudaStream_t st, const float2* ln_stats = nullptr,
            const float* ln_colsum = nullptr) {
  int dev;
  if (int rc = current_device(&dev)) return rc;
  CUtensorMap ta, tw;
  {
    const uint64_t dims[2] = {(uint64_t)K, (uint64_t)M};
    const uint64_t strides[1] = {(uint64_t)K * 2};
    const uint32_t box[2] = {64, 128};
    if (int rc = make_tmap_bf16(&ta, A, 2, dims, strides, box, tmap_dtype<TIn>())) return rc;
  }
  {
    const uint64_t dims[2] = {(uint64_t)N, (uint64_t)K};
    const uint64_t strides[1] = {(uint64_t)N * 2};
    const uint32_t box[2] = {64, 64};
    if (int rc = make_tmap_bf16(&tw, W, 2, dims, strides, box, tmap_dtype<TIn>())) return rc;
  }
  auto kern = jb::gemm::gemm_bf16_tc_kernel<kGemmBN, kGemmStages, TIn, TOut>;
  const size_t smem = sizeof(jb::gemm::Smem<kGemmBN, kGemmStages>) + 1024;
  if (int rc = ensure_smem_attr((const void*)kern, smem, dev)) return rc;
  const int64_t tiles = ((M + 127) / 128) * ((N + kGemmBN - 1) / kGemmBN);
  const int grid = (int)(tiles < device_sms(dev) ? tiles : device_sms(dev));
  kern<<<grid, jb::gemm::kThreads, smem, st>>>(ta, tw, bias, res, C, (int)M, (int)N, (int)K, act,
                                               ln_stats, ln_colsum);
  return check_launch("gemm_bf16_tc_kernel launch");
}

// CTA-pair tcgen05 GEMM (256 x 256 tiles, cluster of 2).
// out: the local C, or every rank's C for the sharded GEMM with the gather
// fused into the epilogue (M = this rank's rows).
template <int TN, typename TIn, typename TOut>
int gemm_tc2(const TIn* A, const TIn* W, const float* bias,
             const TIn* res, const jb::gemm::OutDest<TOut>& out, int64_t M, int64_t N,
             int64_t K, int act, cudaStream_t st, const float2* ln_stats = nullptr,
             const float* ln_colsum = nullptr, int64_t ld_a = 0, int64_t ld_w = 0) {
  // ld_a: A's row stride in elements (0: K).  ld_w: the transposed fp32 W's
  // row stride (0: K); 16-bit W is [K,N] with row stride N.
  if (ld_a == 0) ld_a = K;
  if (ld_w == 0) ld_w = K;
  int dev;
  if (int rc = current_device(&dev)) return rc;
  CUtensorMap ta, tw;
  constexpr uint32_t kE = sizeof(TIn), kRow = 128 / kE;  // elements per 128-byte row
  {
    const uint64_t dims[2] = {(uint64_t)K, (uint64_t)M};
    const uint64_t strides[1] = {(uint64_t)ld_a * kE};
    const uint32_t box[2] = {kRow, 128};
    if (int rc = make_tmap_bf16(&ta, A, 2, dims, strides, box, tmap_dtype<TIn>())) return rc;
  }
  if constexpr (kE == 4) {  // fp32 (tf32) W comes transposed: [N,K], boxes of 64 N rows
    const uint64_t dims[2] = {(uint64_t)K, (uint64_t)N};
    const uint64_t strides[1] = {(uint64_t)ld_w * kE};
    const uint32_t box[2] = {kRow, 64};
    if (int rc = make_tmap_bf16(&tw, W, 2, dims, strides, box, tmap_dtype<TIn>())) return rc;
  } else {
    const uint64_t dims[2] = {(uint64_t)N, (uint64_t)K};
    const uint64_t strides[1] = {(uint64_t)N * kE};
    const uint32_t box[2] = {kRow, kRow};
    if (int rc = make_tmap_bf16(&tw, W, 2, dims, strides, box, tmap_dtype<TIn>())) return rc;
  }
  constexpr int kStages = TN == 256 ? 6 : 8;
  auto kern = jb::gemm::gemm_bf16_tc2_kernel<kStages, TN, TIn, TOut>;
  const size_t smem = sizeof(jb::gemm::Smem2<kStages, TN>) + 1024;
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.blockDim = dim3(jb::gemm::kThreads2);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  // resident CTA pairs of this kernel, queried once per device
  static std::map<std::pair<int, const void*>, int> pairs_of;
  int max_pairs = 0;
  {
    std::lock_guard<std::mutex> lk(g_dev_mu);
    auto it = pairs_of.find({dev, (const void*)kern});
    if (it != pairs_of.end()) max_pairs = it->second;
  }
  if (max_pairs == 0) {
    if (int rc = ensure_smem_attr((const void*)kern, smem, dev)) return rc;
    cfg.gridDim = dim3(2 * (device_sms(dev) / 2));
    int clusters = 0;
    cudaError_t e = cudaOccupancyMaxActiveClusters(&clusters, kern, &cfg);
    if (e != cudaSuccess || clusters <= 0) {
      (void)cudaGetLastError();
      clusters = device_sms(dev) / 2;
    }
    max_pairs = clusters;
    std::lock_guard<std::mutex> lk(g_dev_mu);
    pairs_of[{dev, (const void*)kern}] = clusters;
  }
  const int64_t tiles = ((M + 255) / 256) * ((N + TN - 1) / TN);
  // Tail split (see gemm_bf16_tc2_kernel): the r tiles of the last, partial
  // round run as 2r half-width units when they fit in one round.  At C2
  // (4096^3: 256 tiles on 74 pairs) the last round's 34 tiles become 68
  // halves; with 512 rows per GPU (32 tiles) every tile is split.
  const int64_t tail = tiles % max_pairs;
  const int whole = (int)(tiles - (2 * tail <= max_pairs ? tail : 0));
  const int units = (int)(whole + 2 * (tiles - whole));
  const int pairs = units < max_pairs ? units : max_pairs;
  cfg.gridDim = dim3(2 * pairs);
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, ta, tw, bias, res, out, (int)M, (int)N, (int)K,
                                     act, whole, units, ln_stats, ln_colsum);
  if (e != cudaSuccess) return cuda_fail(e, "gemm_bf16_tc2_kernel launch");
  return check_launch("gemm_bf16_tc2_kernel launch");
}

// Tile choice for the tensor-core GEMM: 256 x 256 CTA-pair tiles once M and
// N fill them, 128 x 256 single-CTA tiles below that.  (256 x 128 pair tiles
// measured slower: their N=128 MMAs leave the tensor pipe idle between
// instructions.)
template <typename TIn, typename TOut>
int gemm_tc_dispatch(const TIn* A, const TIn* W, const float* bias,
                     const TIn* res, TOut* C, int64_t M, int64_t N, int64_t K, int act,
                     cudaStream_t st, const float2* ln_stats = nullptr,
                     const float* ln_colsum = nullptr) {
  if (M < 256 || N < 256) return gemm_tc(A, W, bias, res, C, M, N, K, act, st, ln_stats, ln_colsum);
  jb::gemm::OutDest<TOut> out{};
  out.c[0] = C;
  out.n = 1;
  out.row_off = 0;
  return gemm_tc2<256>(A, W, bias, res, out, M, N, K, act, st, ln_stats, ln_colsum);
}

template <typename TIn, typename TOut>
int gemm_simt(const void* A, const void* W, const float* bias, const void* res, void* C, int64_t M,
              int64_t N, int64_t K, int act, int exact, cudaStream_t st) {
  dim3 grid((unsigned)((N + jb::simt::GBN - 1) / jb::simt::GBN),
            (unsigned)((M + jb::simt::GBM - 1) / jb::simt::GBM));
  if (grid.y > 65535u) return fail(JULES_ERR_SHAPE, "M=%lld too large for the CUDA-core GEMM", (long long)M);
  jb::simt::gemm_kernel<TIn, TOut><<<grid, 256, 0, st>>>(
      static_cast<const TIn*>(A), static_cast<const TIn*>(W), bias,
      static_cast<const TIn*>(res), static_cast<TOut*>(C), (int)M, (int)N, (int)K, act, exact);
  return check_launch("gemm_kernel launch");
}

// ---------------------------------------------------------------------------
// Attention paths
// ---------------------------------------------------------------------------
template <typename TIn, typename TOut, int DPL>
int attn_simt_launch(const void* Q, const void* K, const void* V, void* O, float* lse, int B, int Hq,
                     int Hkv, int S, int D, float scale, int causal, cudaStream_t st) {
  constexpr int DMAX = DPL * 32;
  const size_t smem = sizeof(float) * (jb::simt::ABQ * DMAX + jb::simt::ABK * (DMAX + 1) +
                                       jb::simt::ABK * DMAX);
  auto kern = jb::simt::attn_kernel<TIn, TOut, DPL>;
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(attn)");
  }
  dim3 grid((unsigned)((S + jb::simt::ABQ - 1) / jb::simt::ABQ), (unsigned)(B * Hq));
  kern<<<grid, 128, smem, st>>>(static_cast<const TIn*>(Q), static_cast<const TIn*>(K),
                                static_cast<const TIn*>(V), static_cast<TOut*>(O), lse, Hq, Hkv, S,
                                D, scale, causal);
  return check_launch("attn_kernel launch");
}

template <typename TIn, typename TOut, int D>
int attn_tile_launch(const void* Q, const void* K, const void* V, void* O, float* lse, int B, int Hq,
                     int Hkv, int S, float scale, int causal, cudaStream_t st) {
  namespace sm = jb::simt;
  const size_t smem = sizeof(float) * sm::attn_tile_smem_floats<D>();
  auto kern = sm::attn_tile_kernel<TIn, TOut, D>;
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(attn_tile)");
  }
  dim3 grid((unsigned)((S + sm::TBQ - 1) / sm::TBQ), (unsigned)(B * Hq));
  kern<<<grid, sm::kTileThreads, smem, st>>>(static_cast<const TIn*>(Q), static_cast<const TIn*>(K),
                                             static_cast<const TIn*>(V), static_cast<TOut*>(O), lse,
                                             Hq, Hkv, S, scale, causal);
  return check_launch("attn_tile_kernel launch");
}

template <typename T>
int attn_simt(const void* Q, const void* K, const void* V, void* O, float* lse, int B, int Hq,
              int Hkv, int S, int D, float scale, int causal, cudaStream_t st) {
  // register-tiled kernel: vector loads of K / V need 16-byte aligned bases
  if (aligned16(Q) && aligned16(K) && aligned16(V)) {
    if (D == 32) return attn_tile_launch<T, T, 32>(Q, K, V, O, lse, B, Hq, Hkv, S, scale, causal, st);
    if (D == 64) return attn_tile_launch<T, T, 64>(Q, K, V, O, lse, B, Hq, Hkv, S, scale, causal, st);
    if (D == 128) return attn_tile_launch<T, T, 128>(Q, K, V, O, lse, B, Hq, Hkv, S, scale, causal, st);
  }
  if (D <= 32) return attn_simt_launch<T, T, 1>(Q, K, V, O, lse, B, Hq, Hkv, S, D, scale, causal, st);
  if (D <= 64) return attn_simt_launch<T, T, 2>(Q, K, V, O, lse, B, Hq, Hkv, S, D, scale, causal, st);
  if (D <= 128) return attn_simt_launch<T, T, 4>(Q, K, V, O, lse, B, Hq, Hkv, S, D, scale, causal, st);
  return attn_simt_launch<T, T, 8>(Q, K, V, O, lse, B, Hq, Hkv, S, D, scale, causal, st);
}

// out: the local O / lse, or every rank's for the sharded call with the
// gather fused in (B, Hq, Hkv: this rank's units).  D is 64 or 128; f16
// selects fp16 operands and output (else bf16).
template <int HDIM, typename TEl, bool G>
int attn_tc_launch(const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv,
                   const jb::attn::AttnOut& out, int B, int Hq, int Hkv, int S, float scale_log2,
                   int causal, int dev, int grid, cudaStream_t st) {
  auto kern = jb::attn::attn_fwd_tc_kernel<HDIM, TEl, G>;
  // with the gather fused in: the staged epilogue's shared memory after Smem
  const size_t smem = ((sizeof(jb::attn::Smem) + 127) & ~size_t(127)) + 1024 +
                      (G ? jb::attn::kEpiBytes : 0);
  if (int rc = ensure_smem_attr((const void*)kern, smem, dev)) return rc;
  kern<<<grid, jb::attn::kThreads, smem, st>>>(tq, tk, tv, out, B, Hq, Hkv, S, scale_log2, causal);
  return check_launch("attn_fwd_tc_kernel launch");
}

int attn_tc(const void* Q, const void* K, const void* V, const jb::attn::AttnOut& out, int B, int Hq,
            int Hkv, int S, int D, float scale, int causal, bool f16, cudaStream_t st) {
  int dev;
  if (int rc = current_device(&dev)) return rc;
  CUtensorMap tq, tk, tv;
  const uint32_t box[3] = {64, (uint32_t)jb::attn::BQ, 1};
  const uint32_t boxkv[3] = {64, (uint32_t)jb::attn::BKV, 1};
  const CUtensorMapDataType dt = f16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  {
    const uint64_t dims[3] = {(uint64_t)D, (uint64_t)S, (uint64_t)B * Hq};
    const uint64_t strides[2] = {(uint64_t)D * 2, (uint64_t)S * D * 2};
    if (int rc = make_tmap_bf16(&tq, Q, 3, dims, strides, box, dt)) return rc;
  }
  {
    const uint64_t dims[3] = {(uint64_t)D, (uint64_t)S, (uint64_t)B * Hkv};
    const uint64_t strides[2] = {(uint64_t)D * 2, (uint64_t)S * D * 2};
    if (int rc = make_tmap_bf16(&tk, K, 3, dims, strides, boxkv, dt)) return rc;
    if (int rc = make_tmap_bf16(&tv, V, 3, dims, strides, boxkv, dt)) return rc;
  }
  constexpr int kRowsPerItem = jb::attn::NQT * jb::attn::BQ;
  const int n_pairs = (S + kRowsPerItem - 1) / kRowsPerItem;
  const int64_t work = (int64_t)n_pairs * B * Hq;
  const int grid = (int)(work < device_sms(dev) ? work : device_sms(dev));
  const float scale_log2 = scale * 1.4426950408889634f;
  const bool g = out.n > 1;
#define JB_ATTN(HDIM, T, G) \
  attn_tc_launch<HDIM, T, G>(tq, tk, tv, out, B, Hq, Hkv, S, scale_log2, causal, dev, grid, st)
  if (D == 128) {
    if (f16) return g ? JB_ATTN(128, __half, true) : JB_ATTN(128, __half, false);
    return g ? JB_ATTN(128, __nv_bfloat16, true) : JB_ATTN(128, __nv_bfloat16, false);
  }
  if (f16) return g ? JB_ATTN(64, __half, true) : JB_ATTN(64, __half, false);
  return g ? JB_ATTN(64, __nv_bfloat16, true) : JB_ATTN(64, __nv_bfloat16, false);
#undef JB_ATTN
}

size_t align256(size_t n) { return (n + 255) & ~size_t(255); }

size_t attn_bwd_ws_bytes(int64_t BH, int S, int tensor_path) {
  const int64_t rows = BH * (tensor_path ? jb::attn_bwd::padded_len(S) : S);
  return 2 * align256((size_t)rows * 4);
}

// Attention backward, tcgen05 path (bf16, D = 128, 16-byte aligned).
int attn_bwd_tc(const void* Q, const void* K, const void* V, const void* O, const void* dO,
                const float* lse, void* dQ, void* dK, void* dV, int B, int Hq, int Hkv, int S,
                float scale, int causal, void* ws, cudaStream_t st) {
  namespace ab = jb::attn_bwd;
  int dev;
  if (int rc = current_device(&dev)) return rc;
  const int Sp = ab::padded_len(S);
  const int64_t BHq = (int64_t)B * Hq, BHkv = (int64_t)B * Hkv;
  const int n_t = Sp / ab::BT;
  if (BHq * n_t > INT32_MAX || BHkv * n_t > INT32_MAX)
    return fail(JULES_ERR_SHAPE, "attention bwd: too many tiles");
  float* lse2 = static_cast<float*>(ws);
  float* delta = reinterpret_cast<float*>(static_cast<char*>(ws) + align256((size_t)BHq * Sp * 4));
  {
    const int64_t warps = BHq * Sp;
    const int grid = (int)std::min<int64_t>((warps * 32 + 255) / 256, (int64_t)device_sms(dev) * 16);
    ab::bwd_prep_kernel<<<grid, 256, 0, st>>>(static_cast<const __nv_bfloat16*>(O),
                                              static_cast<const __nv_bfloat16*>(dO), lse, lse2,
                                              delta, (int)BHq, S, Sp);
    if (int rc = check_launch("bwd_prep_kernel launch")) return rc;
  }
  CUtensorMap tq, tk, tv, tdo;
  const uint32_t box[3] = {64, (uint32_t)ab::BT, 1};
  {
    const uint64_t dims[3] = {(uint64_t)ab::HD, (uint64_t)S, (uint64_t)BHq};
    const uint64_t strides[2] = {(uint64_t)ab::HD * 2, (uint64_t)S * ab::HD * 2};
    if (int rc = make_tmap_bf16(&tq, Q, 3, dims, strides, box)) return rc;
    if (int rc = make_tmap_bf16(&tdo, dO, 3, dims, strides, box)) return rc;
  }
  {
    const uint64_t dims[3] = {(uint64_t)ab::HD, (uint64_t)S, (uint64_t)BHkv};
    const uint64_t strides[2] = {(uint64_t)ab::HD * 2, (uint64_t)S * ab::HD * 2};
    if (int rc = make_tmap_bf16(&tk, K, 3, dims, strides, box)) return rc;
    if (int rc = make_tmap_bf16(&tv, V, 3, dims, strides, box)) return rc;
  }
  const size_t smem_kv = sizeof(ab::SmemKV) + 1024, smem_q = sizeof(ab::SmemQ) + 1024;
  static bool attr_set[kMaxDevices] = {};
  if (!attr_set[dev]) {
    std::lock_guard<std::mutex> lk(g_dev_mu);
    cudaError_t e = cudaFuncSetAttribute(ab::bwd_dkdv_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem_kv);
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(ab::bwd_dq_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem_q);
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(attention bwd)");
    attr_set[dev] = true;
  }
  ab::bwd_dkdv_kernel<<<(unsigned)(BHkv * n_t), ab::kThreads, smem_kv, st>>>(
      tq, tk, tv, tdo, lse2, delta, static_cast<__nv_bfloat16*>(dK),
      static_cast<__nv_bfloat16*>(dV), B, Hq, Hkv, S, scale, causal);
  if (int rc = check_launch("bwd_dkdv_kernel launch")) return rc;
  ab::bwd_dq_kernel<<<(unsigned)(BHq * n_t), ab::kThreads, smem_q, st>>>(
      tq, tk, tv, tdo, lse2, delta, static_cast<const __nv_bfloat16*>(Q),
      static_cast<const __nv_bfloat16*>(dO), static_cast<__nv_bfloat16*>(dQ), B, Hq, Hkv, S, scale,
      causal);
  return check_launch("bwd_dq_kernel launch");
}

// Attention backward, CUDA cores (any dtype of T, head dim <= 256).
template <typename T>
int attn_bwd_simt(const void* Q, const void* K, const void* V, const void* O, const void* dO,
                  const float* lse, void* dQ, void* dK, void* dV, int B, int Hq, int Hkv, int S,
                  int D, float scale, int causal, void* ws, cudaStream_t st) {
  namespace ab = jb::attn_bwd;
  int dev;
  if (int rc = current_device(&dev)) return rc;
  float* delta = static_cast<float*>(ws);
  const int64_t rq = (int64_t)B * Hq * S, rk = (int64_t)B * Hkv * S;
  const int cap = device_sms(dev) * 16;
  auto grid_for = [&](int64_t rows) { return (int)std::min<int64_t>((rows * 32 + 255) / 256, cap); };
  ab::bwd_simt_delta_kernel<T><<<grid_for(rq), 256, 0, st>>>(
      static_cast<const T*>(O), static_cast<const T*>(dO), delta, rq, D);
  if (int rc = check_launch("bwd_simt_delta_kernel launch")) return rc;
  ab::bwd_simt_dq_kernel<T><<<grid_for(rq), 256, 0, st>>>(
      static_cast<const T*>(Q), static_cast<const T*>(K), static_cast<const T*>(V),
      static_cast<const T*>(dO), lse, delta, static_cast<T*>(dQ), B, Hq, Hkv, S, D, scale, causal);
  if (int rc = check_launch("bwd_simt_dq_kernel launch")) return rc;
  ab::bwd_simt_dkdv_kernel<T><<<grid_for(rk), 256, 0, st>>>(
      static_cast<const T*>(Q), static_cast<const T*>(K), static_cast<const T*>(V),
      static_cast<const T*>(dO), lse, delta, static_cast<T*>(dK), static_cast<T*>(dV), B, Hq, Hkv,
      S, D, scale, causal);
  return check_launch("bwd_simt_dkdv_kernel launch");
}

// Self-test of the bounded wait: one thread waits on an mbarrier that nothing
// arrives on, with the given limit.  The wait gives up, records
// kDevErrTimeout with site kSelftestWaitSite in the device error word and the
// kernel returns; the context stays usable.
constexpr uint32_t kSelftestWaitSite = 250;
__global__ void wait_selftest_kernel(uint64_t limit_ns) {
  __shared__ uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    jb::mbar_init(&bar, 1);
    abort_flag = 0;
    jb::fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) (void)jb::mbar_wait_for(&bar, 0, kSelftestWaitSite, &abort_flag, limit_ns);
}

}  // namespace

namespace {
// bf16 LayerNorm / row statistics, one warp per row (N % 8 == 0, N <= 8192).
int layernorm_warp_launch(const __nv_bfloat16* in, const float* gamma, const float* beta,
                          __nv_bfloat16* out, float* mean_out, float* rstd_out, float2* stats,
                          int64_t M, int N, float eps, cudaStream_t st) {
  const unsigned grid = (unsigned)((M + 7) / 8);
  const int nv = N / 8;
#define JB_LN_WARP(NV)                                                                         \
  jb::simt::layernorm_bf16_warp_kernel<NV><<<grid, 256, 0, st>>>(in, gamma, beta, out, mean_out, \
                                                                 rstd_out, stats, M, N, eps)
  if (nv <= 32) JB_LN_WARP(1);
  else if (nv <= 64) JB_LN_WARP(2);
  else if (nv <= 128) JB_LN_WARP(4);
  else if (nv <= 256) JB_LN_WARP(8);
  else if (nv <= 512) JB_LN_WARP(16);
  else if (nv <= 1024) JB_LN_WARP(32);
  else return fail(JULES_ERR_SHAPE, "layernorm: row of %d too long for the warp kernel", N);
#undef JB_LN_WARP
  return check_launch("layernorm_bf16_warp_kernel launch");
}
}  // namespace

#include "dist.cuh"

// ===========================================================================
// Exported C ABI
// ===========================================================================
namespace {

// Launch an 8-bit CTA-pair kernel (cluster of 2) over the 256 x 256 tiles of
// an M x N output: one pair per tile up to the number of co-resident pairs
// (queried once per device and kernel, cached in max_pairs).
template <typename... KArgs, typename... Args>
int launch_pair8(void (*kern)(KArgs...), size_t smem, int dev, int64_t M, int64_t N,
                 int (&max_pairs)[64], cudaStream_t st, const char* what, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.blockDim = dim3(jb::gemm8::kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int mp;
  {
    std::lock_guard<std::mutex> lk(g_dev_mu);
    mp = max_pairs[dev & 63];
    if (mp == 0) {
      cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      if (e != cudaSuccess) return cuda_fail(e, what);
      cfg.gridDim = dim3(2 * (device_sms(dev) / 2));
      int clusters = 0;
      e = cudaOccupancyMaxActiveClusters(&clusters, kern, &cfg);
      if (e != cudaSuccess || clusters <= 0) {
        (void)cudaGetLastError();
        clusters = device_sms(dev) / 2;
      }
      mp = max_pairs[dev & 63] = clusters;
    }
  }
  const int64_t tiles = ((M + 255) / 256) * ((N + 255) / 256);
  cfg.gridDim = dim3((unsigned)(2 * (tiles < mp ? tiles : mp)));
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
  if (e != cudaSuccess) return cuda_fail(e, what);
  return check_launch(what);
}

// fp8 GEMM (E4M3 / E5M2 operands, fp32 accumulation): tcgen05 kind::f8f6f4
// on CTA pairs when K and N are multiples of 16 and the pointers 16-byte
// aligned, CUDA cores otherwise.
template <typename TOut>
int gemm_f8(const uint8_t* A, const uint8_t* W, const float* bias, const __nv_bfloat16* res,
            TOut* C, int64_t M, int64_t N, int64_t K, float scale, int a_fmt, int w_fmt, int act,
            cudaStream_t st) {
  int dev;
  if (int rc = current_device(&dev)) return rc;
  if (K % 16 == 0 && N % 16 == 0 && aligned16(A) && aligned16(W) && aligned16(C) &&
      (!bias || aligned16(bias)) && (!res || aligned16(res))) {
    constexpr int STAGES = 6;
    CUtensorMap ta, tb;
    if (int rc = make_tmap_i8(&ta, A, (uint64_t)K, (uint64_t)M, jb::gemm8::BK, 128)) return rc;
    if (int rc = make_tmap_i8(&tb, W, (uint64_t)N, (uint64_t)K, 128, jb::gemm8::BK)) return rc;
    static int max_pairs[64] = {};
    const uint32_t idesc = jb::gemm8::idesc_f8_f32(256, 256, a_fmt, w_fmt, true);
    return launch_pair8(jb::gemm8::gemm_f8_tc2_kernel<STAGES, TOut>,
                        sizeof(jb::gemm8::Smem8p<STAGES>) + 1024, dev, M, N, max_pairs, st,
                        "gemm_f8_tc2_kernel", ta, tb, bias, res, C, (int)M, (int)N, (int)K, scale,
                        idesc, act);
  }
  dim3 grid((unsigned)((N + 15) / 16), (unsigned)((M + 15) / 16));
  if (grid.y > 65535u) return fail(JULES_ERR_SHAPE, "gemm_fp8: M too large for the CUDA-core path");
  jb::gemm8::gemm_f8_simt_kernel<TOut><<<grid, 256, 0, st>>>(A, W, bias, res, C, (int)M, (int)N,
                                                             (int)K, scale, a_fmt, w_fmt, act);
  return check_launch("gemm_f8_simt_kernel launch");
}

// int8 GEMM: tcgen05 kind::i8 when K and N are multiples of 16 and the
// pointers 16-byte aligned, CUDA cores otherwise.
int gemm_s8(const int8_t* A, const int8_t* B, const float* bias, float* C, int64_t M, int64_t N,
            int64_t K, float scale, cudaStream_t st) {
  int dev;
  if (int rc = current_device(&dev)) return rc;
  const bool tc_ok = K % 16 == 0 && N % 16 == 0 && aligned16(A) && aligned16(B) && aligned16(C) &&
                     (!bias || aligned16(bias));
  if (tc_ok && M >= 256 && N >= 256) {
    // CTA pairs, 256 x 256 tiles
    constexpr int STAGES = 6;
    CUtensorMap ta, tb;
    if (int rc = make_tmap_i8(&ta, A, (uint64_t)K, (uint64_t)M, jb::gemm8::BK, 128)) return rc;
    if (int rc = make_tmap_i8(&tb, B, (uint64_t)N, (uint64_t)K, 128, jb::gemm8::BK)) return rc;
    static int max_pairs[64] = {};
    return launch_pair8(jb::gemm8::gemm_s8_tc2_kernel<STAGES>,
                        sizeof(jb::gemm8::Smem8p<STAGES>) + 1024, dev, M, N, max_pairs, st,
                        "gemm_s8_tc2_kernel", ta, tb, bias, C, (int)M, (int)N, (int)K, scale);
  }
  if (tc_ok) {
    constexpr int BN = 256, STAGES = 4;
    CUtensorMap ta, tb;
    if (int rc = make_tmap_i8(&ta, A, (uint64_t)K, (uint64_t)M, jb::gemm8::BK, jb::gemm8::BM)) return rc;
    if (int rc = make_tmap_i8(&tb, B, (uint64_t)N, (uint64_t)K, 128, jb::gemm8::BK)) return rc;
    auto kern = jb::gemm8::gemm_s8_tc_kernel<BN, STAGES>;
    const size_t smem = sizeof(jb::gemm8::Smem8<BN, STAGES>) + 1024;
    static bool attr_set[64] = {};
    if (!attr_set[dev & 63]) {
      std::lock_guard<std::mutex> lk(g_dev_mu);
      cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(gemm_s8)");
      attr_set[dev & 63] = true;
    }
    const int64_t tiles = ((M + jb::gemm8::BM - 1) / jb::gemm8::BM) * ((N + BN - 1) / BN);
    const int grid = (int)(tiles < device_sms(dev) ? tiles : device_sms(dev));
    kern<<<grid, jb::gemm8::kThreads, smem, st>>>(ta, tb, bias, C, (int)M, (int)N, (int)K, scale);
    return check_launch("gemm_s8_tc_kernel launch");
  }
  dim3 grid((unsigned)((N + 15) / 16), (unsigned)((M + 15) / 16));
  jb::gemm8::gemm_s8_simt_kernel<<<grid, 256, 0, st>>>(A, B, bias, C, (int)M, (int)N, (int)K, scale);
  return check_launch("gemm_s8_simt_kernel launch");
}

// Register-resident CTA-per-row softmax when the types match, rows are
// 16-byte aligned and a row fits THREADS x NV vectors; returns false when it
// does not apply.
template <int THREADS, int NV, typename T, bool XENT>
void rows_reg_go(const T* x, T* y, const int32_t* targets, float* loss, int64_t M, int64_t N,
                 float inv_M, int sms, cudaStream_t st) {
  int64_t blocks = M;
  const int64_t cap = (int64_t)sms * (2048 / THREADS);
  if (blocks > cap) blocks = cap;
  jb::rows::softmax_reg_kernel<THREADS, NV, T, XENT>
      <<<(unsigned)blocks, THREADS, 0, st>>>(x, y, targets, loss, M, (int)N, inv_M);
}

// Rows of 32 KB and more: one persistent 1024-thread CTA per SM with the
// next row staged in shared memory (softmax_stage_kernel).
template <int THREADS, int NV, typename T, bool XENT>
bool rows_stage_go(const T* x, T* y, const int32_t* targets, float* loss, int64_t M, int64_t N,
                   float inv_M, int sms, cudaStream_t st) {
  const size_t smem = (size_t)N * sizeof(T);
  auto kern = jb::rows::softmax_stage_kernel<THREADS, NV, T, XENT>;
  static bool attr_set[kMaxDevices] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return false;
  if (!attr_set[dev]) {
    std::lock_guard<std::mutex> lk(g_dev_mu);
    constexpr size_t kMax = (size_t)THREADS * NV * 16;  // the largest row this instance takes
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kMax) != cudaSuccess) {
      (void)cudaGetLastError();
      return false;
    }
    attr_set[dev] = true;
  }
  int64_t blocks = M < sms ? M : sms;
  kern<<<(unsigned)blocks, THREADS, smem, st>>>(x, y, targets, loss, M, (int)N, inv_M);
  return true;
}

template <typename TIn, typename TOut, bool XENT>
bool rows_reg_launch(const TIn* x, TOut* y, const int32_t* targets, float* loss, int64_t M,
                     int64_t N, float inv_M, int sms, cudaStream_t st) {
  if constexpr (!std::is_same<TIn, TOut>::value) {
    return false;
  } else {
    constexpr int E = jb::rows::Vec16<TIn>::kN;
    if (N % E || !aligned16(x) || (y && !aligned16(y)) || (N * sizeof(TIn)) % 16) return false;
    if (N <= 256 * 4 * E) rows_reg_go<256, 4, TIn, XENT>(x, y, targets, loss, M, N, inv_M, sms, st);
    else if (N <= 512 * 4 * E) rows_reg_go<512, 4, TIn, XENT>(x, y, targets, loss, M, N, inv_M, sms, st);
    else if (N <= 1024 * 4 * E) return rows_stage_go<1024, 4, TIn, XENT>(x, y, targets, loss, M, N, inv_M, sms, st);
    else if (E == 4 && N <= 1024 * 8 * E)  // 8 vectors of bf16 would spill at 1024 threads
      return rows_stage_go<1024, (E == 4 ? 8 : 4), TIn, XENT>(x, y, targets, loss, M, N, inv_M, sms, st);
    else return false;
    return true;
  }
}

// Row softmax / fused cross-entropy launcher: one warp per row up to
// kWarpRowMax columns, one CTA per row beyond.  Grids are capped at a few
// waves of resident blocks; the kernels stride over rows.
template <typename TIn, typename TOut, bool XENT>
int rows_launch(const void* in, void* out, const int32_t* targets, float* loss, int64_t M,
                int64_t N, cudaStream_t st) {
  int dev;
  if (int rc = current_device(&dev)) return rc;
  const float inv_M = 1.0f / (float)M;
  const auto* x = static_cast<const TIn*>(in);
  auto* y = static_cast<TOut*>(out);
  if (N <= jb::rows::kWarpRowMax) {
    int64_t blocks = (M + 7) / 8;
    const int64_t cap = (int64_t)device_sms(dev) * 8;
    if (blocks > cap) blocks = cap;
    jb::rows::softmax_warp_kernel<TIn, TOut, XENT>
        <<<(unsigned)blocks, 256, 0, st>>>(x, y, targets, loss, M, (int)N, inv_M);
  } else if (!rows_reg_launch<TIn, TOut, XENT>(x, y, targets, loss, M, N, inv_M, device_sms(dev), st)) {
    int64_t blocks = M;
    const int64_t cap = (int64_t)device_sms(dev) * 8;
    if (blocks > cap) blocks = cap;
    jb::rows::softmax_cta_kernel<TIn, TOut, XENT>
        <<<(unsigned)blocks, jb::rows::kCtaThreads, 0, st>>>(x, y, targets, loss, M, (int)N, inv_M);
  }
  return check_launch(XENT ? "cross_entropy launch" : "softmax launch");
}

}  // namespace

extern "C" {

int jules_version(void) { return (0 << 16) | 1; }

const char* jules_last_error_string(void) { return g_errbuf; }

const char* jules_status_string(int s) {
  switch (s) {
    case JULES_OK: return "ok";
    case JULES_ERR_SHAPE: return "bad shape";
    case JULES_ERR_ALIGN: return "bad alignment";
    case JULES_ERR_DTYPE: return "unsupported dtype";
    case JULES_ERR_CUDA: return "cuda error";
    case JULES_ERR_TIMEOUT: return "device wait timed out";
    case JULES_ERR_ARG: return "bad argument";
    case JULES_ERR_UNSUPPORTED: return "not implemented";
    case JULES_ERR_WORKSPACE: return "workspace too small";
    case JULES_ERR_COMM: return "collective communication error";
    default: return "unknown status";
  }
}

int jules_device_error(uint32_t* word, int clear) {
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceSynchronize");
  uint32_t w = 0;
  e = cudaMemcpyFromSymbol(&w, jb::g_dev_error, sizeof(w));
  if (e != cudaSuccess) return cuda_fail(e, "read device error word");
  if (clear && w) {
    const uint32_t z = 0;
    e = cudaMemcpyToSymbol(jb::g_dev_error, &z, sizeof(z));
    if (e != cudaSuccess) return cuda_fail(e, "clear device error word");
  }
  if (word) *word = w;
  if (w & jb::kDevErrTimeout)
    return fail(JULES_ERR_TIMEOUT, "device wait timed out (site %u)", (w >> 8) & 0xffu);
  if (w) return fail(JULES_ERR_SHAPE, "device reported error word 0x%x", w);
  return ok();
}

int jules_selftest_bounded_wait(uint64_t limit_ns, void* stream) {
  if (limit_ns == 0 || limit_ns > jb::kWaitLimitNs)
    return fail(JULES_ERR_ARG, "selftest_bounded_wait: limit %llu ns outside (0, %llu]",
                (unsigned long long)limit_ns, (unsigned long long)jb::kWaitLimitNs);
  wait_selftest_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(limit_ns);
  return check_launch("wait_selftest_kernel launch");
}

int jules_gemm_bias_act(const void* A, const void* W, const float* bias, const void* residual,
                        void* C, int64_t M, int64_t N, int64_t K, int act, int in_dtype,
                        int out_dtype, void* stream) {
  if (!A || !W || !C) return fail(JULES_ERR_ARG, "gemm: NULL A, W or C");
  if (M < 0 || N <= 0 || K <= 0) return fail(JULES_ERR_SHAPE, "gemm: M=%lld N=%lld K=%lld", (long long)M, (long long)N, (long long)K);
  if (M > INT32_MAX || N > INT32_MAX || K > INT32_MAX) return fail(JULES_ERR_SHAPE, "gemm: dimension exceeds 2^31-1");
  if (act < JULES_ACT_NONE || act > JULES_ACT_GELU) return fail(JULES_ERR_ARG, "gemm: act=%d", act);
  if (M == 0) return ok();
  if (in_dtype == JULES_DTYPE_FP8E4M3 || in_dtype == JULES_DTYPE_FP8E5M2)
    return jules_gemm_fp8(A, W, bias, residual, C, M, N, K, 1.0f, act, in_dtype, in_dtype,
                          out_dtype, stream);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (in_dtype == JULES_DTYPE_F16 || out_dtype == JULES_DTYPE_F16) {
    if (in_dtype != JULES_DTYPE_F16 || (out_dtype != JULES_DTYPE_F16 && out_dtype != JULES_DTYPE_F32))
      return fail(JULES_ERR_DTYPE, "gemm: dtypes %d/%d (f16 operands give f16 or fp32 C)", in_dtype, out_dtype);
    const bool out_h = out_dtype == JULES_DTYPE_F16;
    if (N % 8 == 0 && K % 8 == 0 && aligned16(A) && aligned16(W) && aligned16(C) &&
        (!bias || aligned16(bias)) && (!residual || aligned16(residual))) {
      const auto* a = static_cast<const __half*>(A);
      const auto* w = static_cast<const __half*>(W);
      const auto* r = static_cast<const __half*>(residual);
      if (out_h) return gemm_tc_dispatch(a, w, bias, r, static_cast<__half*>(C), M, N, K, act, st);
      return gemm_tc_dispatch(a, w, bias, r, static_cast<float*>(C), M, N, K, act, st);
    }
    if (out_h) return gemm_simt<__half, __half>(A, W, bias, residual, C, M, N, K, act, 0, st);
    return gemm_simt<__half, float>(A, W, bias, residual, C, M, N, K, act, 1, st);
  }
  const bool in_bf = in_dtype == JULES_DTYPE_BF16, out_bf = out_dtype == JULES_DTYPE_BF16;
  if ((in_dtype != JULES_DTYPE_F32 && !in_bf) || (out_dtype != JULES_DTYPE_F32 && !out_bf))
    return fail(JULES_ERR_DTYPE, "gemm: dtypes %d/%d", in_dtype, out_dtype);
  if (in_bf && N % 8 == 0 && K % 8 == 0 && aligned16(A) && aligned16(W) && aligned16(C) &&
      (!bias || aligned16(bias)) && (!residual || aligned16(residual))) {
    const auto* a = static_cast<const __nv_bfloat16*>(A);
    const auto* w = static_cast<const __nv_bfloat16*>(W);
    const auto* r = static_cast<const __nv_bfloat16*>(residual);
    if (out_bf)
      return gemm_tc_dispatch(a, w, bias, r, static_cast<__nv_bfloat16*>(C), M, N, K, act, st);
    return gemm_tc_dispatch(a, w, bias, r, static_cast<float*>(C), M, N, K, act, st);
  }
  if (in_bf && out_bf) return gemm_simt<__nv_bfloat16, __nv_bfloat16>(A, W, bias, residual, C, M, N, K, act, 0, st);
  if (in_bf) return gemm_simt<__nv_bfloat16, float>(A, W, bias, residual, C, M, N, K, act, 1, st);
  if (out_bf) return gemm_simt<float, __nv_bfloat16>(A, W, bias, residual, C, M, N, K, act, 0, st);
  return gemm_simt<float, float>(A, W, bias, residual, C, M, N, K, act, 1, st);
}

// 3xTF32 chunking: K is accumulated on the tensor cores in chunks of at most
// kF32Chunk columns (each 3 x kF32Chunk tf32 columns, at most 128 MMA steps
// at full magnitude); each chunk's epilogue adds the fp32 sum of the earlier
// chunks (held in C) with a round-to-nearest add, the last one then bias and
// activation.
constexpr int64_t kF32Chunk = 1024;

int64_t f32_chunks(int64_t K) { return (K + kF32Chunk - 1) / kF32Chunk; }

size_t jules_gemm_f32_tc_workspace_bytes(int64_t M, int64_t N, int64_t K) {
  if (M <= 0 || N <= 0 || K <= 0) return 0;
  return align256((size_t)M * 3 * (size_t)K * 4) + (size_t)3 * K * N * 4;
}

int jules_gemm_f32_tc(const float* A, const float* W, const float* bias, float* C, int64_t M,
                      int64_t N, int64_t K, int act, void* workspace, size_t workspace_bytes,
                      void* stream) {
  if (!A || !W || !C) return fail(JULES_ERR_ARG, "gemm_f32_tc: NULL A, W or C");
  if (M < 0 || N <= 0 || K <= 0 || M > INT32_MAX || N > INT32_MAX || K > INT32_MAX)
    return fail(JULES_ERR_SHAPE, "gemm_f32_tc: M=%lld N=%lld K=%lld", (long long)M, (long long)N, (long long)K);
  if (act < JULES_ACT_NONE || act > JULES_ACT_GELU) return fail(JULES_ERR_ARG, "gemm_f32_tc: act=%d", act);
  if (M == 0) return ok();
  const bool tc = M >= 256 && N >= 256 && N % 8 == 0 && K % 4 == 0 && 3 * K <= INT32_MAX &&
                  (K + 63) / 64 <= 65535 && aligned16(A) && aligned16(W) && aligned16(C) &&
                  (!bias || aligned16(bias));
  if (!tc)  // the fp32 CUDA-core GEMM (exact fp32 products)
    return jules_gemm_bias_act(A, W, bias, nullptr, C, M, N, K, act, JULES_DTYPE_F32, JULES_DTYPE_F32, stream);
  const size_t need = jules_gemm_f32_tc_workspace_bytes(M, N, K);
  if (!workspace || workspace_bytes < need)
    return fail(JULES_ERR_WORKSPACE, "gemm_f32_tc: workspace %zu bytes, need %zu", workspace_bytes, need);
  if (!aligned16(workspace)) return fail(JULES_ERR_ALIGN, "gemm_f32_tc: workspace not 16-byte aligned");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int dev;
  if (int rc = current_device(&dev)) return rc;
  char* ws = static_cast<char*>(workspace);
  float* A3 = reinterpret_cast<float*>(ws);
  float* W3T = reinterpret_cast<float*>(ws + align256((size_t)M * 3 * K * 4));
  const int Kc = (int)std::min<int64_t>(K, kF32Chunk);
  const int64_t chunks = f32_chunks(K);
  const int cap = device_sms(dev) * 8;
  const int64_t na = M * (K / 4);
  jb::simt::split3_a_kernel<<<(int)std::min<int64_t>((na + 255) / 256, cap), 256, 0, st>>>(
      reinterpret_cast<const float4*>(A), A3, M, (int)K, Kc);
  if (int rc = check_launch("split3_a_kernel launch")) return rc;
  constexpr int64_t T = jb::simt::kSplitTile;
  jb::simt::split3_wt_kernel<<<dim3((unsigned)((N + T - 1) / T), (unsigned)((K + T - 1) / T)), dim3(32, 8), 0, st>>>(
      W, W3T, (int)K, (int)N, Kc);
  if (int rc = check_launch("split3_wt_kernel launch")) return rc;
  for (int64_t c = 0; c < chunks; ++c) {
    const int64_t k0 = c * kF32Chunk, L = std::min<int64_t>(kF32Chunk, K - k0);
    const bool last = c == chunks - 1;
    jb::gemm::OutDest<float> out{};
    out.c[0] = C;
    out.n = 1;
    if (int rc = gemm_tc2<256>(static_cast<const float*>(A3 + 3 * k0), static_cast<const float*>(W3T + 3 * k0),
                               last ? bias : nullptr, c == 0 ? nullptr : static_cast<const float*>(C), out,
                               M, N, 3 * L, last ? act : JULES_ACT_NONE, st, nullptr, nullptr, 3 * K, 3 * K))
      return rc;
  }
  return JULES_OK;
}

int jules_sgemm(int transA, int transB, int64_t M, int64_t N, int64_t K, float alpha,
                const float* A, int64_t lda, const float* B, int64_t ldb, float beta, float* C,
                int64_t ldc, void* stream) {
  if (!A || !B || !C) return fail(JULES_ERR_ARG, "sgemm: NULL pointer");
  if (M < 0 || N < 0 || K < 0 || M > INT32_MAX || N > INT32_MAX || K > INT32_MAX)
    return fail(JULES_ERR_SHAPE, "sgemm: M=%lld N=%lld K=%lld", (long long)M, (long long)N, (long long)K);
  if (ldc < N || lda < (transA ? M : K) || ldb < (transB ? K : N))
    return fail(JULES_ERR_SHAPE, "sgemm: leading dimension too small");
  if (M == 0 || N == 0) return ok();
  dim3 grid((unsigned)((N + jb::simt::GBN - 1) / jb::simt::GBN),
            (unsigned)((M + jb::simt::GBM - 1) / jb::simt::GBM));
  if (grid.y > 65535u) return fail(JULES_ERR_SHAPE, "sgemm: M too large");
  jb::simt::sgemm_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      transA ? 1 : 0, transB ? 1 : 0, (int)M, (int)N, (int)K, alpha, A, (int)lda, B, (int)ldb,
      beta, C, (int)ldc);
  return check_launch("sgemm_kernel launch");
}

int jules_flash_attention_fwd(const void* Q, const void* K, const void* V, void* O, float* lse,
                              int B, int Hq, int Hkv, int S, int D, float scale, int causal,
                              int dtype, void* stream) {
  if (!Q || !K || !V || !O) return fail(JULES_ERR_ARG, "attention: NULL Q, K, V or O");
  if (B < 0 || Hq <= 0 || Hkv <= 0 || S < 0 || D <= 0 || Hq % Hkv != 0)
    return fail(JULES_ERR_SHAPE, "attention: B=%d Hq=%d Hkv=%d S=%d D=%d", B, Hq, Hkv, S, D);
  if (D > 256) return fail(JULES_ERR_SHAPE, "attention: head_dim %d > 256", D);
  if ((int64_t)B * Hq > 65535 * 1024LL) return fail(JULES_ERR_SHAPE, "attention: too many heads");
  if (B == 0 || S == 0) return ok();
  if (!(scale > 0.0f)) scale = 1.0f / sqrtf((float)D);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (dtype == JULES_DTYPE_F32)
    return attn_simt<float>(Q, K, V, O, lse, B, Hq, Hkv, S, D, scale, causal ? 1 : 0, st);
  const bool f16 = dtype == JULES_DTYPE_F16;
  if (dtype != JULES_DTYPE_BF16 && !f16) return fail(JULES_ERR_DTYPE, "attention: dtype %d", dtype);
  if ((D == 128 || D == 64) && aligned16(Q) && aligned16(K) && aligned16(V) && aligned16(O)) {
    jb::attn::AttnOut out{};
    out.o[0] = static_cast<__nv_bfloat16*>(O);
    out.lse[0] = lse;
    out.n = 1;
    return attn_tc(Q, K, V, out, B, Hq, Hkv, S, D, scale, causal ? 1 : 0, f16, st);
  }
  if (f16) return attn_simt<__half>(Q, K, V, O, lse, B, Hq, Hkv, S, D, scale, causal ? 1 : 0, st);
  return attn_simt<__nv_bfloat16>(Q, K, V, O, lse, B, Hq, Hkv, S, D, scale, causal ? 1 : 0, st);
}

size_t jules_flash_attention_bwd_workspace_bytes(int B, int Hq, int S, int D, int dtype) {
  if (B <= 0 || Hq <= 0 || S <= 0) return 0;
  const int tensor_path = dtype == JULES_DTYPE_BF16 && D == jb::attn_bwd::HD;
  return attn_bwd_ws_bytes((int64_t)B * Hq, S, tensor_path);
}

int jules_flash_attention_bwd(const void* Q, const void* K, const void* V, const void* O,
                              const void* dO, const float* lse, void* dQ, void* dK, void* dV,
                              int B, int Hq, int Hkv, int S, int D, float scale, int causal,
                              int dtype, void* workspace, size_t workspace_bytes, void* stream) {
  if (!Q || !K || !V || !O || !dO || !lse || !dQ || !dK || !dV)
    return fail(JULES_ERR_ARG, "attention bwd: NULL pointer");
  if (B < 0 || Hq <= 0 || Hkv <= 0 || S < 0 || D <= 0 || Hq % Hkv != 0)
    return fail(JULES_ERR_SHAPE, "attention bwd: B=%d Hq=%d Hkv=%d S=%d D=%d", B, Hq, Hkv, S, D);
  if (D > 32 * jb::attn_bwd::kSimtDPL) return fail(JULES_ERR_SHAPE, "attention bwd: head_dim %d > 256", D);
  if (dtype != JULES_DTYPE_F32 && dtype != JULES_DTYPE_BF16)
    return fail(JULES_ERR_DTYPE, "attention bwd: dtype %d", dtype);
  if (B == 0 || S == 0) return ok();
  const size_t need = jules_flash_attention_bwd_workspace_bytes(B, Hq, S, D, dtype);
  if (!workspace || workspace_bytes < need || !aligned16(workspace))
    return fail(JULES_ERR_WORKSPACE, "attention bwd: workspace %zu < %zu bytes (or unaligned)", workspace_bytes, need);
  if (!(scale > 0.0f)) scale = 1.0f / sqrtf((float)D);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int c = causal ? 1 : 0;
  if (dtype == JULES_DTYPE_F32)
    return attn_bwd_simt<float>(Q, K, V, O, dO, lse, dQ, dK, dV, B, Hq, Hkv, S, D, scale, c, workspace, st);
  if (D == jb::attn_bwd::HD && aligned16(Q) && aligned16(K) && aligned16(V) && aligned16(O) &&
      aligned16(dO) && aligned16(dQ) && aligned16(dK) && aligned16(dV) && aligned16(lse))
    return attn_bwd_tc(Q, K, V, O, dO, lse, dQ, dK, dV, B, Hq, Hkv, S, scale, c, workspace, st);
  // other head dims and unaligned buffers: CUDA cores (as the forward)
  return attn_bwd_simt<__nv_bfloat16>(Q, K, V, O, dO, lse, dQ, dK, dV, B, Hq, Hkv, S, D, scale, c, workspace, st);
}

int jules_layernorm(const void* in, const float* gamma, const float* beta, void* out, int64_t M,
                    int64_t N, float eps, int in_dtype, int out_dtype, float* mean_out,
                    float* rstd_out, void* stream) {
  if (!in || !out || (!gamma != !beta)) return fail(JULES_ERR_ARG, "layernorm: NULL pointer");
  if (M < 0 || N <= 0 || M > INT32_MAX) return fail(JULES_ERR_SHAPE, "layernorm: M=%lld N=%lld", (long long)M, (long long)N);
  if (M == 0) return ok();
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const bool in_bf = in_dtype == JULES_DTYPE_BF16, out_bf = out_dtype == JULES_DTYPE_BF16;
  if ((in_dtype != JULES_DTYPE_F32 && !in_bf) || (out_dtype != JULES_DTYPE_F32 && !out_bf))
    return fail(JULES_ERR_DTYPE, "layernorm: dtypes %d/%d", in_dtype, out_dtype);
  const unsigned grid = (unsigned)M;
  if (in_bf && out_bf && N % 8 == 0 && N <= 256 * 32 && aligned16(in) && aligned16(out) &&
      (!gamma || (aligned16(gamma) && aligned16(beta)))) {
    if (int rc = layernorm_warp_launch(static_cast<const __nv_bfloat16*>(in), gamma, beta,
                                       static_cast<__nv_bfloat16*>(out), mean_out, rstd_out,
                                       nullptr, M, (int)N, eps, st))
      return rc;
  } else if (in_bf && out_bf && gamma && N % 8 == 0 && N <= 8 * 256 * 4 && aligned16(in) &&
             aligned16(out) && aligned16(gamma) && aligned16(beta)) {
    jb::simt::layernorm_bf16_vec_kernel<4><<<grid, 256, 0, st>>>(
        static_cast<const __nv_bfloat16*>(in), gamma, beta, static_cast<__nv_bfloat16*>(out),
        mean_out, rstd_out, M, (int)N, eps);
  } else if (in_bf && out_bf) {
    jb::simt::layernorm_kernel<__nv_bfloat16, __nv_bfloat16><<<grid, 256, 0, st>>>(
        static_cast<const __nv_bfloat16*>(in), gamma, beta, static_cast<__nv_bfloat16*>(out),
        mean_out, rstd_out, M, N, eps);
  } else if (in_bf) {
    jb::simt::layernorm_kernel<__nv_bfloat16, float><<<grid, 256, 0, st>>>(
        static_cast<const __nv_bfloat16*>(in), gamma, beta, static_cast<float*>(out), mean_out,
        rstd_out, M, N, eps);
  } else if (out_bf) {
    jb::simt::layernorm_kernel<float, __nv_bfloat16><<<grid, 256, 0, st>>>(
        static_cast<const float*>(in), gamma, beta, static_cast<__nv_bfloat16*>(out), mean_out,
        rstd_out, M, N, eps);
  } else {
    jb::simt::layernorm_kernel<float, float><<<grid, 256, 0, st>>>(
        static_cast<const float*>(in), gamma, beta, static_cast<float*>(out), mean_out, rstd_out,
        M, N, eps);
  }
  return check_launch("layernorm launch");
}

int jules_gelu(const void* in, void* out, int64_t n, int dtype, void* stream) {
  if (!in || !out) return fail(JULES_ERR_ARG, "gelu: NULL pointer");
  if (n < 0) return fail(JULES_ERR_SHAPE, "gelu: n=%lld", (long long)n);
  if (n == 0) return ok();
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int64_t blocks = (n + 255) / 256;
  if (blocks > 148 * 16) blocks = 148 * 16;
  if (dtype == JULES_DTYPE_F32)
    jb::simt::gelu_kernel<float><<<(unsigned)blocks, 256, 0, st>>>(static_cast<const float*>(in), static_cast<float*>(out), n);
  else if (dtype == JULES_DTYPE_BF16)
    jb::simt::gelu_kernel<__nv_bfloat16><<<(unsigned)blocks, 256, 0, st>>>(
        static_cast<const __nv_bfloat16*>(in), static_cast<__nv_bfloat16*>(out), n);
  else
    return fail(JULES_ERR_DTYPE, "gelu: dtype %d", dtype);
  return check_launch("gelu launch");
}

int jules_matmul_int8(const int8_t* A, const int8_t* B, float* C, int64_t M, int64_t N,
                      int64_t K, float scale_a, float scale_b, const float* bias, void* stream) {
  if (!A || !B || !C) return fail(JULES_ERR_ARG, "matmul_int8: NULL A, B or C");
  if (M < 0 || N <= 0 || K <= 0) return fail(JULES_ERR_SHAPE, "matmul_int8: M=%lld N=%lld K=%lld", (long long)M, (long long)N, (long long)K);
  if (M > INT32_MAX || N > INT32_MAX || K > INT32_MAX) return fail(JULES_ERR_SHAPE, "matmul_int8: dimension exceeds 2^31-1");
  if (M == 0) return ok();
  return gemm_s8(A, B, bias, C, M, N, K, scale_a * scale_b, static_cast<cudaStream_t>(stream));
}

int jules_gemm_fp8(const void* A, const void* W, const float* bias, const void* residual, void* C,
                   int64_t M, int64_t N, int64_t K, float scale, int act, int a_dtype,
                   int w_dtype, int out_dtype, void* stream) {
  if (!A || !W || !C) return fail(JULES_ERR_ARG, "gemm_fp8: NULL A, W or C");
  if (M < 0 || N <= 0 || K <= 0) return fail(JULES_ERR_SHAPE, "gemm_fp8: M=%lld N=%lld K=%lld", (long long)M, (long long)N, (long long)K);
  if (M > INT32_MAX || N > INT32_MAX || K > INT32_MAX) return fail(JULES_ERR_SHAPE, "gemm_fp8: dimension exceeds 2^31-1");
  if (act < JULES_ACT_NONE || act > JULES_ACT_GELU) return fail(JULES_ERR_ARG, "gemm_fp8: act=%d", act);
  auto fmt = [](int dt) {
    return dt == JULES_DTYPE_FP8E4M3 ? jb::gemm8::kFmtE4M3 : (dt == JULES_DTYPE_FP8E5M2 ? jb::gemm8::kFmtE5M2 : -1);
  };
  const int af = fmt(a_dtype), wf = fmt(w_dtype);
  if (af < 0 || wf < 0 || (out_dtype != JULES_DTYPE_F32 && out_dtype != JULES_DTYPE_BF16))
    return fail(JULES_ERR_DTYPE, "gemm_fp8: dtypes %d/%d/%d", a_dtype, w_dtype, out_dtype);
  if (M == 0) return ok();
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const auto* a = static_cast<const uint8_t*>(A);
  const auto* w = static_cast<const uint8_t*>(W);
  const auto* r = static_cast<const __nv_bfloat16*>(residual);
  if (out_dtype == JULES_DTYPE_BF16)
    return gemm_f8(a, w, bias, r, static_cast<__nv_bfloat16*>(C), M, N, K, scale, af, wf, act, st);
  return gemm_f8(a, w, bias, r, static_cast<float*>(C), M, N, K, scale, af, wf, act, st);
}

int jules_cast(const void* src, void* dst, int64_t n, int src_dtype, int dst_dtype, void* stream) {
  if (!src || !dst) return fail(JULES_ERR_ARG, "cast: NULL pointer");
  if (n < 0) return fail(JULES_ERR_SHAPE, "cast: n=%lld", (long long)n);
  auto valid = [](int d) { return d >= JULES_DTYPE_F32 && d <= JULES_DTYPE_FP8E5M2; };
  if (!valid(src_dtype) || !valid(dst_dtype)) return fail(JULES_ERR_DTYPE, "cast: dtypes %d -> %d", src_dtype, dst_dtype);
  if (n == 0) return ok();
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int dev;
  if (int rc = current_device(&dev)) return rc;
  const int grid_cap = device_sms(dev) * 8;
  const bool to_f8 = dst_dtype == JULES_DTYPE_FP8E4M3 || dst_dtype == JULES_DTYPE_FP8E5M2;
  const int f = dst_dtype == JULES_DTYPE_FP8E5M2 ? jb::gemm8::kFmtE5M2 : jb::gemm8::kFmtE4M3;
  if (to_f8 && (src_dtype == JULES_DTYPE_F32 || src_dtype == JULES_DTYPE_BF16) && n % 8 == 0 &&
      aligned16(src) && aligned16(dst)) {
    const int64_t n8 = n / 8;
    const int grid = (int)std::min<int64_t>((n8 + 255) / 256, grid_cap);
    if (src_dtype == JULES_DTYPE_F32)
      jb::gemm8::cast_to_f8_vec_kernel<float><<<grid, 256, 0, st>>>(
          static_cast<const float*>(src), static_cast<uint8_t*>(dst), n8, f);
    else
      jb::gemm8::cast_to_f8_vec_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>(
          static_cast<const __nv_bfloat16*>(src), static_cast<uint8_t*>(dst), n8, f);
    return check_launch("cast_to_f8_vec_kernel launch");
  }
  const int grid = (int)std::min<int64_t>((n + 255) / 256, grid_cap);
  jb::gemm8::cast_kernel<<<grid, 256, 0, st>>>(src, dst, n, src_dtype, dst_dtype);
  return check_launch("cast_kernel launch");
}

int jules_softmax(const void* in, void* out, int64_t M, int64_t N, int in_dtype, int out_dtype,
                  void* stream) {
  if (!in || !out) return fail(JULES_ERR_ARG, "softmax: NULL pointer");
  if (M < 0 || N < 0 || N > INT32_MAX) return fail(JULES_ERR_SHAPE, "softmax: M=%lld N=%lld", (long long)M, (long long)N);
  if (M == 0 || N == 0) return ok();
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const bool fi = in_dtype == JULES_DTYPE_F32, bi = in_dtype == JULES_DTYPE_BF16;
  const bool fo = out_dtype == JULES_DTYPE_F32, bo = out_dtype == JULES_DTYPE_BF16;
  if (fi && fo) return rows_launch<float, float, false>(in, out, nullptr, nullptr, M, N, st);
  if (fi && bo) return rows_launch<float, __nv_bfloat16, false>(in, out, nullptr, nullptr, M, N, st);
  if (bi && fo) return rows_launch<__nv_bfloat16, float, false>(in, out, nullptr, nullptr, M, N, st);
  if (bi && bo) return rows_launch<__nv_bfloat16, __nv_bfloat16, false>(in, out, nullptr, nullptr, M, N, st);
  return fail(JULES_ERR_DTYPE, "softmax: dtypes %d -> %d", in_dtype, out_dtype);
}

int jules_cross_entropy_loss(const void* logits, const int32_t* targets, void* grad, float* loss,
                             int64_t M, int64_t N, int dtype, void* stream) {
  if (!logits || !targets || !loss) return fail(JULES_ERR_ARG, "cross_entropy: NULL pointer");
  if (M <= 0 || N <= 0 || N > INT32_MAX) return fail(JULES_ERR_SHAPE, "cross_entropy: M=%lld N=%lld", (long long)M, (long long)N);
  if (dtype != JULES_DTYPE_F32 && dtype != JULES_DTYPE_BF16) return fail(JULES_ERR_DTYPE, "cross_entropy: dtype %d", dtype);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaMemsetAsync(loss, 0, sizeof(float), st);
  if (e != cudaSuccess) return cuda_fail(e, "cross_entropy: clear loss");
  if (dtype == JULES_DTYPE_F32)
    return rows_launch<float, float, true>(logits, grad, targets, loss, M, N, st);
  return rows_launch<__nv_bfloat16, __nv_bfloat16, true>(logits, grad, targets, loss, M, N, st);
}

int jules_custom_call(const char* name, void* stream, void** buffers, int n_buffers,
                      const void* opaque, size_t opaque_len) {
  const int id = jules_kernel_by_name(name);
  if (id < 0) return fail(JULES_ERR_ARG, "custom_call: unknown kernel name");
  if (!jules_kernel_implemented(id)) return fail(JULES_ERR_UNSUPPORTED, "custom_call: kernel not implemented");
  if (!opaque || opaque_len != sizeof(jules_call_desc))
    return fail(JULES_ERR_ARG, "custom_call: opaque must be one jules_call_desc");
  if (!buffers || n_buffers <= 0) return fail(JULES_ERR_ARG, "custom_call: no buffers");
  jules_call_desc d;
  std::memcpy(&d, opaque, sizeof(d));
  const std::string n(name);
  auto need = [&](int a, int b = -1) { return n_buffers == a || n_buffers == b; };
  void** B = buffers;
  // fusedMatmul<Act> / fusedMatmulBias<Act>
  static const std::pair<const char*, int> kActs[] = {
      {"Relu", JULES_ACT_RELU}, {"Sigmoid", JULES_ACT_SIGMOID}, {"Tanh", JULES_ACT_TANH},
      {"Gelu", JULES_ACT_GELU}};
  for (const auto& a : kActs) {
    const bool plain = n == std::string("fusedMatmul") + a.first;
    const bool bias = n == std::string("fusedMatmulBias") + a.first;
    if (!plain && !bias) continue;
    if (!need(bias ? 4 : 3)) return fail(JULES_ERR_ARG, "custom_call: matmul buffer count");
    const int out_dt = (d.dtype == JULES_DTYPE_BF16 && (d.flags & 1)) ? JULES_DTYPE_F32 : d.dtype;
    return jules_gemm_bias_act(B[0], B[1], bias ? static_cast<const float*>(B[2]) : nullptr,
                               nullptr, B[bias ? 3 : 2], d.dims[0], d.dims[1], d.dims[2], a.second,
                               d.dtype, out_dt, stream);
  }
  if (n == "blasMatmul") {
    if (!need(3)) return fail(JULES_ERR_ARG, "custom_call: blasMatmul buffer count");
    const int64_t M = d.dims[0], N = d.dims[1], K = d.dims[2];
    const int ta = d.flags & 1, tb = (d.flags >> 1) & 1;
    return jules_sgemm(ta, tb, M, N, K, d.fparams[0], static_cast<const float*>(B[0]), ta ? M : K,
                       static_cast<const float*>(B[1]), tb ? K : N, d.fparams[1],
                       static_cast<float*>(B[2]), N, stream);
  }
  if (n == "matmulInt8") {
    if (!need(3, 4)) return fail(JULES_ERR_ARG, "custom_call: matmulInt8 buffer count");
    const bool bias = n_buffers == 4;
    return jules_matmul_int8(static_cast<const int8_t*>(B[0]), static_cast<const int8_t*>(B[1]),
                             static_cast<float*>(B[bias ? 3 : 2]),
                             d.dims[0], d.dims[1], d.dims[2], d.fparams[0], d.fparams[1],
                             bias ? static_cast<const float*>(B[2]) : nullptr, stream);
  }
  if (n == "fusedLayerNorm") {
    if (!need(2, 4)) return fail(JULES_ERR_ARG, "custom_call: fusedLayerNorm buffer count");
    const bool affine = n_buffers == 4;
    const float eps = d.fparams[0] > 0.0f ? d.fparams[0] : 1e-5f;
    return jules_layernorm(B[0], affine ? static_cast<const float*>(B[1]) : nullptr,
                           affine ? static_cast<const float*>(B[2]) : nullptr, B[affine ? 3 : 1],
                           d.dims[0], d.dims[1], eps, d.dtype, d.dtype, nullptr, nullptr, stream);
  }
  if (n == "fusedGelu") {
    if (!need(2)) return fail(JULES_ERR_ARG, "custom_call: fusedGelu buffer count");
    return jules_gelu(B[0], B[1], d.dims[0], d.dtype, stream);
  }
  if (n == "fusedSoftmax") {
    if (!need(2)) return fail(JULES_ERR_ARG, "custom_call: fusedSoftmax buffer count");
    return jules_softmax(B[0], B[1], d.dims[0], d.dims[1], d.dtype, d.dtype, stream);
  }
  if (n == "fusedCrossEntropyLoss") {
    if (!need(3, 4)) return fail(JULES_ERR_ARG, "custom_call: fusedCrossEntropyLoss buffer count");
    const bool grad = n_buffers == 4;
    return jules_cross_entropy_loss(B[0], static_cast<const int32_t*>(B[1]), grad ? B[2] : nullptr,
                                    static_cast<float*>(B[grad ? 3 : 2]), d.dims[0], d.dims[1],
                                    d.dtype, stream);
  }
  if (n == "flashAttention") {
    if (!need(4, 5)) return fail(JULES_ERR_ARG, "custom_call: flashAttention buffer count");
    return jules_flash_attention_fwd(B[0], B[1], B[2], B[3],
                                     n_buffers == 5 ? static_cast<float*>(B[4]) : nullptr,
                                     (int)d.dims[0], (int)d.dims[1], (int)d.dims[2],
                                     (int)d.dims[3], (int)d.dims[4], d.fparams[0], d.flags & 1,
                                     d.dtype, stream);
  }
  if (n == "fusedMLPForward") {
    if (!need(8)) return fail(JULES_ERR_ARG, "custom_call: fusedMLPForward buffer count");
    const float eps = d.fparams[0] > 0.0f ? d.fparams[0] : 1e-5f;
    return jules_mlp_block_noalloc(B[0], static_cast<const float*>(B[1]),
                                   static_cast<const float*>(B[2]), B[3],
                                   static_cast<const float*>(B[4]), B[5],
                                   static_cast<const float*>(B[6]), B[7],
                                   (d.flags & 1) ? JULES_DTYPE_F32 : JULES_DTYPE_BF16, d.dims[0],
                                   d.dims[1], d.dims[2], eps, stream);
  }
  return fail(JULES_ERR_UNSUPPORTED, "custom_call: no dispatch for this name");
}

size_t jules_mlp_fwd_bwd_workspace_bytes(int64_t M, int64_t N1, int64_t N2) {
  if (M <= 0 || N1 <= 0 || N2 <= 0) return 0;
  const size_t a = ((size_t)M * N1 * 4 + 255) & ~size_t(255);
  const size_t dout = ((size_t)M * N2 * 4 + 255) & ~size_t(255);
  return 2 * a + dout;
}

int jules_mlp_fwd_bwd(const float* X, const float* W1, const float* b1, const float* W2,
                      const float* b2, const int32_t* targets, float* output, float* loss,
                      float* dW1, float* db1, float* dW2, float* db2, float* dX, int64_t M,
                      int64_t K1, int64_t N1, int64_t N2, void* workspace, size_t workspace_bytes,
                      void* stream) {
  if (!X || !W1 || !b1 || !W2 || !b2 || !targets || !output || !loss || !dW1 || !db1 || !dW2 ||
      !db2)
    return fail(JULES_ERR_ARG, "mlp_fwd_bwd: NULL pointer");
  if (M <= 0 || K1 <= 0 || N1 <= 0 || N2 <= 0 || M > INT32_MAX || K1 > INT32_MAX || N1 > INT32_MAX ||
      N2 > INT32_MAX)
    return fail(JULES_ERR_SHAPE, "mlp_fwd_bwd: M=%lld K1=%lld N1=%lld N2=%lld", (long long)M,
                (long long)K1, (long long)N1, (long long)N2);
  const size_t need = jules_mlp_fwd_bwd_workspace_bytes(M, N1, N2);
  if (!workspace || workspace_bytes < need)
    return fail(JULES_ERR_WORKSPACE, "mlp_fwd_bwd: workspace %zu < %zu bytes", workspace_bytes, need);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  char* ws = static_cast<char*>(workspace);
  const size_t a_bytes = ((size_t)M * N1 * 4 + 255) & ~size_t(255);
  float* a = reinterpret_cast<float*>(ws);                  // relu(X W1 + b1)   [M, N1]
  float* dh = reinterpret_cast<float*>(ws + a_bytes);       // dL/dh             [M, N1]
  float* dout = reinterpret_cast<float*>(ws + 2 * a_bytes); // dL/dout           [M, N2]
  auto blocks = [](int64_t n) { return (unsigned)std::min<int64_t>((n + 255) / 256, 148 * 16); };
  // forward
  if (int rc = jules_sgemm(0, 0, M, N1, K1, 1.0f, X, K1, W1, N1, 0.0f, a, N1, stream)) return rc;
  jb::train::bias_relu_kernel<<<blocks(M * N1), 256, 0, st>>>(a, b1, M, N1);
  if (int rc = jules_sgemm(0, 0, M, N2, N1, 1.0f, a, N1, W2, N2, 0.0f, output, N2, stream)) return rc;
  jb::train::bias_add_kernel<<<blocks(M * N2), 256, 0, st>>>(output, b2, M, N2);
  if (int rc = check_launch("mlp_fwd_bwd forward")) return rc;
  // loss and dL/dout = (softmax - onehot) / M
  if (int rc = jules_cross_entropy_loss(output, targets, dout, loss, M, N2, JULES_DTYPE_F32, stream))
    return rc;
  // backward
  if (int rc = jules_sgemm(1, 0, N1, N2, M, 1.0f, a, N1, dout, N2, 0.0f, dW2, N2, stream)) return rc;
  jb::train::colsum_kernel<<<(unsigned)((N2 + 31) / 32), 256, 0, st>>>(dout, db2, M, N2);
  if (int rc = jules_sgemm(0, 1, M, N1, N2, 1.0f, dout, N2, W2, N2, 0.0f, dh, N1, stream)) return rc;
  jb::train::relu_grad_kernel<<<blocks(M * N1), 256, 0, st>>>(dh, a, M * N1);
  if (int rc = jules_sgemm(1, 0, K1, N1, M, 1.0f, X, K1, dh, N1, 0.0f, dW1, N1, stream)) return rc;
  jb::train::colsum_kernel<<<(unsigned)((N1 + 31) / 32), 256, 0, st>>>(dh, db1, M, N1);
  if (dX)
    if (int rc = jules_sgemm(0, 1, M, K1, N1, 1.0f, dh, N1, W1, N1, 0.0f, dX, K1, stream)) return rc;
  return check_launch("mlp_fwd_bwd backward");
}

size_t jules_mlp_block_workspace_bytes(int64_t T, int64_t d, int64_t dff) {
  if (T <= 0 || d <= 0 || dff <= 0) return 0;
  const size_t xn = ((size_t)T * d * 2 + 255) & ~size_t(255);
  const size_t h = ((size_t)T * dff * 2 + 255) & ~size_t(255);
  return xn + h;
}

int jules_mlp_block(const void* X, const float* gamma, const float* beta, const void* W1,
                    const float* b1, const void* W2, const float* b2, void* out, int out_dtype,
                    int64_t T, int64_t d, int64_t dff, float eps, void* workspace,
                    size_t workspace_bytes, void* stream) {
  if (!X || !gamma || !beta || !W1 || !W2 || !out) return fail(JULES_ERR_ARG, "mlp_block: NULL pointer");
  if (out_dtype != JULES_DTYPE_BF16 && out_dtype != JULES_DTYPE_F32)
    return fail(JULES_ERR_DTYPE, "mlp_block: out dtype %d", out_dtype);
  if (T < 0 || d <= 0 || dff <= 0) return fail(JULES_ERR_SHAPE, "mlp_block: T=%lld d=%lld dff=%lld", (long long)T, (long long)d, (long long)dff);
  if (T == 0) return ok();
  const size_t need = jules_mlp_block_workspace_bytes(T, d, dff);
  if (!workspace || workspace_bytes < need)
    return fail(JULES_ERR_WORKSPACE, "mlp_block: workspace %zu < %zu bytes", workspace_bytes, need);
  if (!aligned16(workspace)) return fail(JULES_ERR_ALIGN, "mlp_block: workspace not 16-byte aligned");
  const size_t xn_bytes = ((size_t)T * d * 2 + 255) & ~size_t(255);
  void* xn = workspace;
  void* hid = static_cast<char*>(workspace) + xn_bytes;
  if (int rc = jules_layernorm(X, gamma, beta, xn, T, d, eps, JULES_DTYPE_BF16, JULES_DTYPE_BF16,
                               nullptr, nullptr, stream))
    return rc;
  if (int rc = jules_gemm_bias_act(xn, W1, b1, nullptr, hid, T, dff, d, JULES_ACT_GELU,
                                   JULES_DTYPE_BF16, JULES_DTYPE_BF16, stream))
    return rc;
  return jules_gemm_bias_act(hid, W2, b2, X, out, T, d, dff, JULES_ACT_NONE, JULES_DTYPE_BF16,
                             out_dtype, stream);
}

int jules_mlp_block_fold_weights(const float* gamma, const float* beta, const void* W1,
                                 const float* b1, void* W1f, float* colsum, float* c, int64_t d,
                                 int64_t dff, void* stream) {
  if (!gamma || !beta || !W1 || !W1f || !colsum || !c)
    return fail(JULES_ERR_ARG, "mlp_block_fold_weights: NULL pointer");
  if (d <= 0 || dff <= 0 || d > INT32_MAX || dff > INT32_MAX)
    return fail(JULES_ERR_SHAPE, "mlp_block_fold_weights: d=%lld dff=%lld", (long long)d, (long long)dff);
  jb::simt::ln_fold_weights_kernel<<<(unsigned)((dff + 255) / 256), 256, 0,
                                     static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(W1), gamma, beta, b1, static_cast<__nv_bfloat16*>(W1f),
      colsum, c, (int)d, (int)dff);
  return check_launch("ln_fold_weights_kernel launch");
}

size_t jules_mlp_block_folded_workspace_bytes(int64_t T, int64_t d, int64_t dff) {
  if (T <= 0 || d <= 0 || dff <= 0) return 0;
  return (((size_t)T * 8 + 255) & ~size_t(255)) + (((size_t)T * dff * 2 + 255) & ~size_t(255));
}

int jules_mlp_block_folded(const void* X, const void* W1f, const float* colsum, const float* c,
                           const void* W2, const float* b2, void* out, int out_dtype, int64_t T,
                           int64_t d, int64_t dff, float eps, void* workspace,
                           size_t workspace_bytes, void* stream) {
  if (!X || !W1f || !colsum || !c || !W2 || !out)
    return fail(JULES_ERR_ARG, "mlp_block_folded: NULL pointer");
  if (out_dtype != JULES_DTYPE_BF16 && out_dtype != JULES_DTYPE_F32)
    return fail(JULES_ERR_DTYPE, "mlp_block_folded: out dtype %d", out_dtype);
  if (T < 0 || d <= 0 || dff <= 0 || T > INT32_MAX || d > 8192 || dff > INT32_MAX ||
      d % 8 != 0 || dff % 8 != 0)
    return fail(JULES_ERR_SHAPE,
                "mlp_block_folded: T=%lld d=%lld dff=%lld (needs d, dff multiples of 8, d <= 8192; "
                "jules_mlp_block takes any shape)", (long long)T, (long long)d, (long long)dff);
  if (!aligned16(X) || !aligned16(W1f) || !aligned16(colsum) || !aligned16(c) || !aligned16(W2) ||
      !aligned16(out) || (b2 && !aligned16(b2)))
    return fail(JULES_ERR_ALIGN, "mlp_block_folded: buffers must be 16-byte aligned");
  if (T == 0) return ok();
  const size_t need = jules_mlp_block_folded_workspace_bytes(T, d, dff);
  if (!workspace || workspace_bytes < need)
    return fail(JULES_ERR_WORKSPACE, "mlp_block_folded: workspace %zu < %zu bytes", workspace_bytes, need);
  if (!aligned16(workspace)) return fail(JULES_ERR_ALIGN, "mlp_block_folded: workspace not 16-byte aligned");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  float2* stats = static_cast<float2*>(workspace);
  auto* hid = reinterpret_cast<__nv_bfloat16*>(static_cast<char*>(workspace) +
                                               (((size_t)T * 8 + 255) & ~size_t(255)));
  // row statistics of X (one read of X), then GEMM1 on the raw rows with the
  // LayerNorm applied in its epilogue, then GEMM2 + bias + residual
  if (int rc = layernorm_warp_launch(static_cast<const __nv_bfloat16*>(X), nullptr, nullptr, nullptr,
                                     nullptr, nullptr, stats, T, (int)d, eps, st))
    return rc;
  if (int rc = gemm_tc_dispatch<__nv_bfloat16, __nv_bfloat16>(
          static_cast<const __nv_bfloat16*>(X), static_cast<const __nv_bfloat16*>(W1f), c,
          nullptr, hid, T, dff, d, JULES_ACT_GELU, st, stats, colsum))
    return rc;
  return jules_gemm_bias_act(hid, W2, b2, X, out, T, d, dff, JULES_ACT_NONE, JULES_DTYPE_BF16,
                             out_dtype, stream);
}

}  // extern "C"

// ===========================================================================
// MLP block without allocation (jules_mlp_block_noalloc).
//
// Some callers cannot allocate device memory: a runtime's custom-call handler
// (the route jules.extern_kernel -> stablehlo.custom_call takes) receives only
// its operand and result buffers, and the device memory belongs to that
// runtime's allocator, so the handler may neither cudaMalloc nor keep a
// workspace of its own.  This entry point takes its workspace from a
// fixed-size array compiled into the library instead.
// ===========================================================================

// Workspace of jules_mlp_block_noalloc: LN(X) and the hidden activation, bf16.
// Every device that loads the library holds these 32 MiB until the process
// exits.  All calls on a device share it: calls whose kernels overlap on the
// GPU (different streams, no ordering between them) race on it.  Nothing in
// it needs to start at zero (each call writes both parts before reading
// them), so stale contents from the previous call are harmless.
constexpr size_t kNoAllocScratchBytes = 32ull << 20;
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

namespace {

// Device address of g_noalloc_scratch per device.  In host code the array's
// name is only a host-side stand-in, so the address is looked up once per
// device, with that device current.
void* g_noalloc_ptr[kMaxDevices] = {};

int noalloc_scratch(void** out) {
  int dev;
  if (int rc = current_device(&dev)) return rc;
  std::lock_guard<std::mutex> lk(g_dev_mu);
  if (!g_noalloc_ptr[dev]) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(noalloc scratch)");
    g_noalloc_ptr[dev] = p;
  }
  *out = g_noalloc_ptr[dev];
  return JULES_OK;
}

}  // namespace

extern "C" {

size_t jules_mlp_block_noalloc_max_workspace_bytes(void) { return kNoAllocScratchBytes; }

int jules_mlp_block_noalloc(const void* X, const float* gamma, const float* beta, const void* W1,
                            const float* b1, const void* W2, const float* b2, void* out,
                            int out_dtype, int64_t T, int64_t d, int64_t dff, float eps,
                            void* stream) {
  if (!X || !gamma || !beta || !W1 || !W2 || !out)
    return fail(JULES_ERR_ARG, "mlp_block_noalloc: NULL pointer");
  if (T < 0 || d <= 0 || dff <= 0 || T > INT32_MAX || d > INT32_MAX || dff > INT32_MAX)
    return fail(JULES_ERR_SHAPE, "mlp_block_noalloc: T=%lld d=%lld dff=%lld", (long long)T,
                (long long)d, (long long)dff);
  if (out_dtype != JULES_DTYPE_BF16 && out_dtype != JULES_DTYPE_F32)
    return fail(JULES_ERR_DTYPE, "mlp_block_noalloc: out dtype %d", out_dtype);
  const size_t need = jules_mlp_block_workspace_bytes(T, d, dff);
  if (need > kNoAllocScratchBytes)
    return fail(JULES_ERR_WORKSPACE,
                "mlp_block_noalloc: T=%lld d=%lld dff=%lld needs %zu bytes of workspace; the "
                "built-in array holds %zu (use jules_mlp_block with a caller workspace)",
                (long long)T, (long long)d, (long long)dff, need, kNoAllocScratchBytes);
  if (T == 0) return ok();
  void* ws = nullptr;
  if (int rc = noalloc_scratch(&ws)) return rc;
  const size_t xn_bytes = ((size_t)T * d * 2 + 255) & ~size_t(255);
  void* xn = ws;
  void* hid = static_cast<char*>(ws) + xn_bytes;
  if (int rc = jules_layernorm(X, gamma, beta, xn, T, d, eps, JULES_DTYPE_BF16, JULES_DTYPE_BF16,
                               nullptr, nullptr, stream))
    return rc;
  // The GEMMs allocate nothing (their tail split needs no scratch).
  if (int rc = jules_gemm_bias_act(xn, W1, b1, nullptr, hid, T, dff, d, JULES_ACT_GELU,
                                   JULES_DTYPE_BF16, JULES_DTYPE_BF16, stream))
    return rc;
  return jules_gemm_bias_act(hid, W2, b2, X, out, T, d, dff, JULES_ACT_NONE, JULES_DTYPE_BF16,
                             out_dtype, stream);
}

}  // extern "C"

// ===========================================================================
// Multi-GPU entry points (dist.cuh).
// ===========================================================================
extern "C" {

int jules_dist_shard(int64_t units, int world, int rank, int64_t* begin, int64_t* end) {
  if (!begin || !end) return fail(JULES_ERR_ARG, "dist_shard: NULL output");
  if (units < 0 || world <= 0 || rank < 0 || rank >= world)
    return fail(JULES_ERR_ARG, "dist_shard: units=%lld world=%d rank=%d", (long long)units, world, rank);
  const int64_t base = units / world, extra = units % world;
  *begin = rank * base + (rank < extra ? rank : extra);
  *end = *begin + base + (rank < extra ? 1 : 0);
  return ok();
}

int jules_dist_unique_id(void* id) {
  if (!id) return fail(JULES_ERR_ARG, "dist_unique_id: NULL");
  if (int rc = need_nccl()) return rc;
  ncclUniqueId u;
  ncclResult_t r = nccl_lib().get_unique_id(&u);
  if (r != ncclSuccess) return nccl_fail(r, "ncclGetUniqueId");
  static_assert(sizeof(u) == JULES_DIST_ID_BYTES, "NCCL unique id size");
  std::memcpy(id, &u, sizeof(u));
  return ok();
}

int jules_dist_init(void** comm, int world, int rank, const void* id) {
  if (!comm || !id) return fail(JULES_ERR_ARG, "dist_init: NULL");
  *comm = nullptr;
  if (world < 1 || world > jb::dist::kMaxRanks || rank < 0 || rank >= world)
    return fail(JULES_ERR_ARG, "dist_init: world=%d rank=%d (1 <= world <= %d)", world, rank,
                jb::dist::kMaxRanks);
  if (int rc = need_nccl()) return rc;
  auto* c = new DistComm();
  c->world = world;
  c->rank = rank;
  if (int rc = current_device(&c->dev)) {
    delete c;
    return rc;
  }
  ncclUniqueId u;
  std::memcpy(&u, id, sizeof(u));
  ncclResult_t r = nccl_lib().comm_init_rank(&c->comm, world, u, rank);
  if (r != ncclSuccess) {
    delete c;
    return nccl_fail(r, "ncclCommInitRank");
  }
  int rc = shared_alloc(c, 256, &c->flags);
  if (!rc) {
    unsigned long long* h[jb::dist::kMaxRanks];
    for (int q = 0; q < world; ++q) h[q] = static_cast<unsigned long long*>(c->flags.peers[q]);
    cudaError_t e = cudaMalloc(&c->d_counters, sizeof(h));
    if (e == cudaSuccess) e = cudaMemcpy(c->d_counters, h, sizeof(h), cudaMemcpyHostToDevice);
    if (e != cudaSuccess) rc = cuda_fail(e, "dist_init: counter table");
  }
  if (rc) {
    jules_dist_destroy(c);
    return rc;
  }
#if JULES_NCCL_DEVICE_API
  multicast_setup(c);
#endif
  if (const char* g = std::getenv("JULES_DIST_GATHER")) {
    if (!std::strcmp(g, "stores") || !std::strcmp(g, "fused")) c->gather_mode = 1;
    if (!std::strcmp(g, "pull")) c->gather_mode = 2;
  }
  *comm = c;
  return ok();
}

int jules_dist_destroy(void* comm) {
  if (!comm) return ok();
  auto* c = static_cast<DistComm*>(comm);
  cudaDeviceSynchronize();
  side_release(c);
  for (auto& b : c->shared) shared_release(c, b);
  shared_release(c, c->flags);
  if (c->d_counters) cudaFree(c->d_counters);
#if JULES_NCCL_DEVICE_API
  if (c->has_devcomm) nccl_lib().devcomm_destroy(c->comm, &c->devcomm);
#endif
  if (c->comm) nccl_lib().comm_destroy(c->comm);
  delete c;
  return ok();
}

int jules_dist_multicast(void* comm, int* on) {
  if (!on) return fail(JULES_ERR_ARG, "dist_multicast: NULL");
  *on = 0;
  DistComm* c;
  if (int rc = dist_check(comm, &c)) return rc;
  *on = c->multicast ? 1 : 0;
  return ok();
}

int jules_dist_gather_route(void* comm, size_t out_bytes, int* route) {
  if (!route) return fail(JULES_ERR_ARG, "dist_gather_route: NULL");
  *route = JULES_GATHER_STORES;
  DistComm* c;
  if (int rc = dist_check(comm, &c)) return rc;
  *route = c->multicast ? JULES_GATHER_MULTICAST
                        : use_pull_gather(c, out_bytes) ? JULES_GATHER_PULL : JULES_GATHER_STORES;
  return ok();
}

int jules_dist_barrier(void* comm, void* stream) {
  DistComm* c;
  if (int rc = dist_check(comm, &c)) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // one in-place all-reduce of the spare word after the counter
  auto* w = reinterpret_cast<unsigned long long*>(static_cast<char*>(c->flags.local) + 64);
  ncclResult_t r = nccl_lib().all_reduce(w, w, 1, ncclUint64, ncclSum, c->comm, st);
  return r == ncclSuccess ? ok() : nccl_fail(r, "ncclAllReduce(barrier)");
}

int jules_dist_alloc_shared(void* comm, size_t bytes, void** local) {
  if (!local) return fail(JULES_ERR_ARG, "dist_alloc_shared: NULL");
  *local = nullptr;
  DistComm* c;
  if (int rc = dist_check(comm, &c)) return rc;
  if (bytes == 0) return fail(JULES_ERR_ARG, "dist_alloc_shared: 0 bytes");
  SharedBuf b;
#if JULES_NCCL_DEVICE_API
  if (c->multicast) {
    if (int rc = shared_alloc_window(c, bytes, &b)) return rc;
  } else
#endif
  if (int rc = shared_alloc(c, bytes, &b)) return rc;
  std::lock_guard<std::mutex> lk(c->mu);
  c->shared.push_back(b);
  *local = b.local;
  return ok();
}

int jules_dist_free_shared(void* comm, void* local) {
  DistComm* c;
  if (int rc = dist_check(comm, &c)) return rc;
  std::lock_guard<std::mutex> lk(c->mu);
  for (size_t i = 0; i < c->shared.size(); ++i) {
    if (c->shared[i].local == local) {
      cudaDeviceSynchronize();
      shared_release(c, c->shared[i]);
      c->shared.erase(c->shared.begin() + (long)i);
      return ok();
    }
  }
  return fail(JULES_ERR_ARG, "dist_free_shared: not a shared buffer of this communicator");
}

int jules_dist_gemm_bias_act(void* comm, const void* A, const void* W, const float* bias,
                             const void* residual, void* C, int64_t M, int64_t N, int64_t K,
                             int act, int in_dtype, int out_dtype, void* stream) {
  DistComm* c;
  if (int rc = dist_check(comm, &c)) return rc;
  if (!A || !W || !C) return fail(JULES_ERR_ARG, "dist_gemm: NULL A, W or C");
  if (M < 0 || N <= 0 || K <= 0 || M > INT32_MAX || N > INT32_MAX || K > INT32_MAX)
    return fail(JULES_ERR_SHAPE, "dist_gemm: M=%lld N=%lld K=%lld", (long long)M, (long long)N, (long long)K);
  if (out_dtype != JULES_DTYPE_F32 && out_dtype != JULES_DTYPE_BF16)
    return fail(JULES_ERR_DTYPE, "dist_gemm: out dtype %d", out_dtype);
  if (in_dtype != JULES_DTYPE_F32 && in_dtype != JULES_DTYPE_BF16 && in_dtype != JULES_DTYPE_FP8E4M3 &&
      in_dtype != JULES_DTYPE_FP8E5M2)
    return fail(JULES_ERR_DTYPE, "dist_gemm: in dtype %d", in_dtype);
  if (M == 0) return ok();
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int64_t b, e;
  jules_dist_shard(M, c->world, c->rank, &b, &e);
  const size_t ein = dtype_bytes(in_dtype), eout = dtype_bytes(out_dtype);
  const size_t eres = in_dtype == JULES_DTYPE_F32 ? 4 : 2;  // fp8 operands take a bf16 residual
  const char* A_l = static_cast<const char*>(A) + (size_t)b * K * ein;
  const char* R_l = residual ? static_cast<const char*>(residual) + (size_t)b * N * eres : nullptr;
  SharedBuf shared_c;  // C's peer mappings when it is a shared buffer
  const bool is_shared = find_shared(c, C, (size_t)M * N * eout, &shared_c);
  // The fused path depends only on values every rank shares, so all ranks
  // take the same path.
  const bool fused = is_shared && in_dtype == JULES_DTYPE_BF16 && N % 8 == 0 && K % 8 == 0 && N >= 256 &&
                     M / c->world >= 256 && aligned16(A) && aligned16(W) && aligned16(C) &&
                     (!bias || aligned16(bias)) && (!residual || aligned16(residual));
  if (fused) {
    const auto* a = reinterpret_cast<const __nv_bfloat16*>(A_l);
    const auto* w = static_cast<const __nv_bfloat16*>(W);
    const auto* r = reinterpret_cast<const __nv_bfloat16*>(R_l);
    // pull: the kernel stores this rank's rows locally; the copy engines
    // fetch the other ranks' rows after the signal/wait round.
    const bool pull = use_pull_gather(c, (size_t)M * N * eout) && !c->multicast;
    const int n_dest = pull ? 1 : c->world;
    int rc;
    if (out_dtype == JULES_DTYPE_BF16) {
      jb::gemm::OutDest<__nv_bfloat16> od{};
      od.n = n_dest;
      od.row_off = (int)b;
      od.c[0] = static_cast<__nv_bfloat16*>(C);
      od.mc = static_cast<__nv_bfloat16*>(shared_c.mc);
      for (int q = 1; q < c->world; ++q)
        od.c[q] = static_cast<__nv_bfloat16*>(shared_c.peers[(c->rank + q) % c->world]);
      rc = gemm_tc2<256>(a, w, bias, r, od, e - b, N, K, act, st);
    } else {
      jb::gemm::OutDest<float> od{};
      od.n = n_dest;
      od.row_off = (int)b;
      od.c[0] = static_cast<float*>(C);
      od.mc = static_cast<float*>(shared_c.mc);
      for (int q = 1; q < c->world; ++q)
        od.c[q] = static_cast<float*>(shared_c.peers[(c->rank + q) % c->world]);
      rc = gemm_tc2<256>(a, w, bias, r, od, e - b, N, K, act, st);
    }
    if (rc) return rc;
    const unsigned long long target = (++c->calls) * (unsigned long long)c->world;
    jb::dist::dist_signal_wait_kernel<<<1, 32, 0, st>>>(
        c->d_counters, c->world, static_cast<const unsigned long long*>(c->flags.local), target,
        jb::kWaitLimitNs);
    if (int rc2 = check_launch("dist_signal_wait_kernel launch")) return rc2;
    return pull ? pull_gather(c, shared_c, M, (size_t)N * eout, nullptr, 0, st) : ok();
  }
  if (e > b) {
    char* C_l = static_cast<char*>(C) + (size_t)b * N * eout;
    if (int rc = jules_gemm_bias_act(A_l, W, bias, R_l, C_l, e - b, N, K, act, in_dtype, out_dtype, stream))
      return rc;
  }
  ncclDataType_t t;
  if (int rc = nccl_type(out_dtype, &t)) return rc;
  return gather_in_place(c, C, M, N, t, eout, st);
}

int jules_dist_flash_attention_fwd(void* comm, const void* Q, const void* K, const void* V, void* O,
                                   float* lse, int B, int Hq, int Hkv, int S, int D, float scale,
                                   int causal, int dtype, void* stream) {
  DistComm* c;
  if (int rc = dist_check(comm, &c)) return rc;
  if (!Q || !K || !V || !O) return fail(JULES_ERR_ARG, "dist_attention: NULL Q, K, V or O");
  if (B < 0 || Hq <= 0 || Hkv <= 0 || S < 0 || D <= 0 || Hq % Hkv != 0)
    return fail(JULES_ERR_SHAPE, "dist_attention: B=%d Hq=%d Hkv=%d S=%d D=%d", B, Hq, Hkv, S, D);
  if (dtype != JULES_DTYPE_F32 && dtype != JULES_DTYPE_BF16 && dtype != JULES_DTYPE_F16)
    return fail(JULES_ERR_DTYPE, "dist_attention: dtype %d", dtype);
  if (B == 0 || S == 0) return ok();
  // Units: (batch, kv head) pairs, each one kv head and the Hq/Hkv query
  // heads reading it, contiguous in every tensor.  Each rank's units must
  // form whole batches or lie inside one batch, so its share is one call.
  const int64_t units = (int64_t)B * Hkv;
  const int w = c->world;
  if (units % w != 0)
    return fail(JULES_ERR_SHAPE, "dist_attention: %lld units do not split over %d ranks", (long long)units, w);
  const int64_t upr = units / w, u0 = upr * c->rank;
  if (upr % Hkv != 0 && Hkv % upr != 0)
    return fail(JULES_ERR_SHAPE, "dist_attention: %lld units per rank neither whole batches nor a part of one", (long long)upr);
  const int G = Hq / Hkv;
  const int64_t b0 = u0 / Hkv, g0 = u0 % Hkv;
  const int Bl = upr % Hkv == 0 ? (int)(upr / Hkv) : 1;
  const int Hkvl = upr % Hkv == 0 ? Hkv : (int)upr;
  const int Hql = Hkvl * G;
  const size_t elt = dtype_bytes(dtype);
  const size_t q_off = ((size_t)b0 * Hq + (size_t)g0 * G) * S * D;
  const size_t kv_off = ((size_t)b0 * Hkv + (size_t)g0) * S * D;
  const char* q = static_cast<const char*>(Q) + q_off * elt;
  const char* k = static_cast<const char*>(K) + kv_off * elt;
  const char* v = static_cast<const char*>(V) + kv_off * elt;
  char* o = static_cast<char*>(O) + q_off * elt;
  float* l = lse ? lse + ((size_t)b0 * Hq + (size_t)g0 * G) * S : nullptr;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  SharedBuf so, sl;
  const bool o_shared = find_shared(c, O, (size_t)B * Hq * S * D * elt, &so);
  const bool l_shared = !lse || find_shared(c, lse, (size_t)B * Hq * S * 4, &sl);
  if (o_shared && l_shared && (dtype == JULES_DTYPE_BF16 || dtype == JULES_DTYPE_F16) &&
      (D == 128 || D == 64) && aligned16(Q) &&
      aligned16(K) && aligned16(V) && aligned16(O)) {
    // Gather fused into the attention epilogue: each finished O tile (and
    // its lse) is stored into every rank's buffers.
    const bool pull = use_pull_gather(c, (size_t)B * Hq * S * D * elt) && !c->multicast;
    jb::attn::AttnOut out{};
    out.n = pull ? 1 : w;  // pull: local stores, the copy engines fetch the rest
    for (int qq = 0; qq < w; ++qq) {
      const int peer = (c->rank + qq) % w;
      out.o[qq] = reinterpret_cast<__nv_bfloat16*>(static_cast<char*>(so.peers[peer]) + q_off * elt);
      out.lse[qq] = lse ? reinterpret_cast<float*>(static_cast<char*>(sl.peers[peer]) +
                                                   ((size_t)b0 * Hq + (size_t)g0 * G) * S * 4)
                        : nullptr;
    }
    if (c->multicast && so.mc && (!lse || sl.mc)) {  // O and lse alike
      out.o_mc = reinterpret_cast<__nv_bfloat16*>(static_cast<char*>(so.mc) + q_off * elt);
      out.lse_mc = lse ? reinterpret_cast<float*>(static_cast<char*>(sl.mc) +
                                                  ((size_t)b0 * Hq + (size_t)g0 * G) * S * 4)
                       : nullptr;
    }
    if (!(scale > 0.0f)) scale = 1.0f / sqrtf((float)D);
    if (int rc = attn_tc(q, k, v, out, Bl, Hql, Hkvl, S, D, scale, causal ? 1 : 0,
                         dtype == JULES_DTYPE_F16, st))
      return rc;
    const unsigned long long target = (++c->calls) * (unsigned long long)w;
    jb::dist::dist_signal_wait_kernel<<<1, 32, 0, st>>>(
        c->d_counters, w, static_cast<const unsigned long long*>(c->flags.local), target,
        jb::kWaitLimitNs);
    if (int rc = check_launch("dist_signal_wait_kernel launch")) return rc;
    return pull ? pull_gather(c, so, units, (size_t)G * S * D * elt, lse ? &sl : nullptr,
                              (size_t)G * S * 4, st)
                : ok();
  }
  if (int rc = jules_flash_attention_fwd(q, k, v, o, l, Bl, Hql, Hkvl, S, D, scale, causal, dtype, stream))
    return rc;
  ncclDataType_t t;
  if (int rc = nccl_type(dtype, &t)) return rc;
  ncclResult_t r = nccl_lib().group_start();
  if (r != ncclSuccess) return nccl_fail(r, "ncclGroupStart");
  int rc = gather_in_place(c, O, units, (int64_t)G * S * D, t, elt, st);
  if (!rc && lse) rc = gather_in_place(c, lse, units, (int64_t)G * S, ncclFloat32, 4, st);
  r = nccl_lib().group_end();
  if (rc) return rc;
  return r == ncclSuccess ? ok() : nccl_fail(r, "ncclGroupEnd");
}

}  // extern "C"
