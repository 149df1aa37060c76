// Host side of the drop-in boundary:
//  - the reference's C++ kernel API (namespace jules::kernel, host float*
//    arguments, same signatures as AVmakeralt/jules
//    include/jules/Kernel/{FusedKernels,FlashAttention}.h), implemented by
//    staging to the current GPU and calling the C ABI;
//  - the extern_kernel name registry (jules_kernel_by_name & co.).
//
// Staging uses a per-thread, grow-only device buffer and the legacy default
// stream, so each call is synchronous like the reference's.
#include <cuda_runtime.h>

#include <cmath>
#include <cstring>
#include <stdexcept>
#include <string>

#include "jules/Kernel/ExecutionArena.h"
#include "jules/Kernel/FlashAttention.h"
#include "jules/Kernel/FusedKernels.h"
#include "jules/Kernel/InterleavedAutodiff.h"
#include "jules/Kernel/TilePlanner.h"
#include "jules_kernels.h"

namespace {

void check(cudaError_t e, const char* what) {
  if (e != cudaSuccess) throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
}

void check_status(int rc, const char* what) {
  if (rc != JULES_OK)
    throw std::runtime_error(std::string(what) + ": " + jules_status_string(rc) + " (" +
                             jules_last_error_string() + ")");
}

// Grow-only device staging area for one host thread and device.
class Staging {
 public:
  ~Staging() {
    if (ptr_) cudaFree(ptr_);
  }
  // Returns device pointers for `n` buffers of the given byte sizes.
  static constexpr int kMaxBuffers = 16;
  void reserve(const size_t* bytes, int n, char** out) {
    if (n < 0 || n > kMaxBuffers) throw std::runtime_error("jules: too many staging buffers");
    size_t total = 0;
    size_t off[kMaxBuffers];
    for (int i = 0; i < n; ++i) {
      off[i] = total;
      total += (bytes[i] + 255) & ~size_t(255);
    }
    int dev = 0;
    check(cudaGetDevice(&dev), "cudaGetDevice");
    if (total > cap_ || dev != dev_) {
      if (ptr_) cudaFree(ptr_);
      ptr_ = nullptr;
      cap_ = 0;
      check(cudaMalloc(&ptr_, total ? total : 256), "cudaMalloc(staging)");
      cap_ = total;
      dev_ = dev;
    }
    for (int i = 0; i < n; ++i) out[i] = static_cast<char*>(ptr_) + off[i];
  }

 private:
  void* ptr_ = nullptr;
  size_t cap_ = 0;
  int dev_ = -1;
};

Staging& staging() {
  thread_local Staging s;
  return s;
}

void h2d(void* d, const void* h, size_t n) {
  if (n) check(cudaMemcpy(d, h, n, cudaMemcpyHostToDevice), "cudaMemcpy H2D");
}
void d2h(void* h, const void* d, size_t n) {
  if (n) check(cudaMemcpy(h, d, n, cudaMemcpyDeviceToHost), "cudaMemcpy D2H");
}

// act(X.W + bias), host pointers, fp32: the 3xTF32 tensor-core GEMM (its
// operand-split workspace in the staging area) where the shape allows, the
// fp32 CUDA-core GEMM otherwise.
void gemm_host(const float* X, const float* W, const float* bias, float* out, int M, int K, int N,
               int act) {
  if (M <= 0 || N <= 0 || K <= 0) return;
  const size_t bx = (size_t)M * K * 4, bw = (size_t)K * N * 4, bb = bias ? (size_t)N * 4 : 0,
               bo = (size_t)M * N * 4, bws = jules_gemm_f32_tc_workspace_bytes(M, N, K);
  const size_t sizes[5] = {bx, bw, bb ? bb : 4, bo, bws};
  char* d[5];
  staging().reserve(sizes, 5, d);
  h2d(d[0], X, bx);
  h2d(d[1], W, bw);
  if (bias) h2d(d[2], bias, bb);
  check_status(jules_gemm_f32_tc(reinterpret_cast<float*>(d[0]), reinterpret_cast<float*>(d[1]),
                                 bias ? reinterpret_cast<float*>(d[2]) : nullptr,
                                 reinterpret_cast<float*>(d[3]), M, N, K, act, d[4], bws, nullptr),
               "jules_gemm_f32_tc");
  d2h(out, d[3], bo);
}

void attention_host(float* out, const float* Q, const float* K, const float* V, int B, int H,
                    int S, int D) {
  if (B <= 0 || H <= 0 || S <= 0 || D <= 0) return;
  const size_t n = (size_t)B * H * S * D * 4;
  const size_t sizes[4] = {n, n, n, n};
  char* d[4];
  staging().reserve(sizes, 4, d);
  h2d(d[0], Q, n);
  h2d(d[1], K, n);
  h2d(d[2], V, n);
  check_status(jules_flash_attention_fwd(d[0], d[1], d[2], d[3], nullptr, B, H, H, S, D, 0.0f, 0,
                                         JULES_DTYPE_F32, nullptr),
               "jules_flash_attention_fwd");
  d2h(out, d[3], n);
}

}  // namespace

namespace jules {
namespace kernel {

CacheInfo CacheInfo::detect() {
  CacheInfo c{};
  int dev = 0, smem = 0, l2 = 0, sms = 0;
  if (cudaGetDevice(&dev) == cudaSuccess) {
    cudaDeviceGetAttribute(&smem, cudaDevAttrMaxSharedMemoryPerMultiprocessor, dev);
    cudaDeviceGetAttribute(&l2, cudaDevAttrL2CacheSize, dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  }
  c.l1d_bytes = smem > 0 ? (size_t)smem : 228 * 1024;
  c.l2_bytes = l2 > 0 ? (size_t)l2 : 126u * 1024 * 1024;
  c.l3_bytes = c.l2_bytes;
  c.line_bytes = 128;
  c.num_cores = sms > 0 ? sms : 148;
  return c;
}

ExecutionArena::ExecutionArena(size_t maxSize)
    : buffer_(nullptr), maxSize_(maxSize), offset_(0), highWaterMark_(0) {
  void* p = nullptr;
  if (cudaMalloc(&p, maxSize_ ? maxSize_ : 256) != cudaSuccess) throw std::bad_alloc();
  buffer_ = static_cast<char*>(p);
}

ExecutionArena::~ExecutionArena() {
  if (buffer_) cudaFree(buffer_);
}

void* ExecutionArena::allocateBytes(size_t bytes) {
  const size_t aligned = (offset_ + 63) & ~size_t(63);
  if (aligned + bytes > maxSize_) throw std::bad_alloc();
  offset_ = aligned + bytes;
  if (offset_ > highWaterMark_) highWaterMark_ = offset_;
  return buffer_ + aligned;
}

void ExecutionArena::resetAndZero() {
  if (offset_) check(cudaMemset(buffer_, 0, offset_), "cudaMemset(arena)");
  offset_ = 0;
}

void tiledMatmulWithActivation(const float* A, const float* B, float* C, int M, int N, int K,
                               const TileConfig& cfg, ActivationType act) {
  (void)cfg;  // the GPU kernel's tile is fixed
  gemm_host(A, B, nullptr, C, M, K, N, static_cast<int>(act));
}

void fusedMatmulRelu(const float* X, const float* W, float* output, int M, int K, int N) {
  gemm_host(X, W, nullptr, output, M, K, N, JULES_ACT_RELU);
}

void fusedMatmulBiasRelu(const float* X, const float* W, const float* bias, float* output, int M,
                         int K, int N) {
  gemm_host(X, W, bias, output, M, K, N, JULES_ACT_RELU);
}

void fusedMatmulBiasGelu(const float* X, const float* W, const float* bias, float* output, int M,
                         int K, int N) {
  gemm_host(X, W, bias, output, M, K, N, JULES_ACT_GELU);
}

void fusedLayerNorm(float* output, const float* input, const float* gamma, const float* beta, int M,
                    int N, float epsilon) {
  if (M <= 0 || N <= 0) return;
  const size_t bx = (size_t)M * N * 4, bg = (size_t)N * 4;
  const size_t sizes[4] = {bx, bg, bg, bx};
  char* d[4];
  staging().reserve(sizes, 4, d);
  h2d(d[0], input, bx);
  h2d(d[1], gamma, bg);
  h2d(d[2], beta, bg);
  check_status(jules_layernorm(d[0], reinterpret_cast<float*>(d[1]), reinterpret_cast<float*>(d[2]),
                               d[3], M, N, epsilon, JULES_DTYPE_F32, JULES_DTYPE_F32, nullptr,
                               nullptr, nullptr),
               "jules_layernorm");
  d2h(output, d[3], bx);
}

void fusedGelu(float* output, const float* input, int N) {
  if (N <= 0) return;
  const size_t b = (size_t)N * 4;
  const size_t sizes[2] = {b, b};
  char* d[2];
  staging().reserve(sizes, 2, d);
  h2d(d[0], input, b);
  check_status(jules_gelu(d[0], d[1], N, JULES_DTYPE_F32, nullptr), "jules_gelu");
  d2h(output, d[1], b);
}

void fusedSoftmax(float* output, const float* input, int M, int N) {
  if (M <= 0 || N <= 0) return;
  const size_t b = (size_t)M * N * 4;
  const size_t sizes[2] = {b, b};
  char* d[2];
  staging().reserve(sizes, 2, d);
  h2d(d[0], input, b);
  check_status(jules_softmax(d[0], d[1], M, N, JULES_DTYPE_F32, JULES_DTYPE_F32, nullptr),
               "jules_softmax");
  d2h(output, d[1], b);
}

float fusedCrossEntropyLoss(const float* logits, const int32_t* targets, float* grad, int M,
                            int N) {
  if (M <= 0 || N <= 0) return 0.0f;
  const size_t bl = (size_t)M * N * 4, bt = (size_t)M * 4;
  const size_t sizes[4] = {bl, bt, bl, 256};
  char* d[4];
  staging().reserve(sizes, 4, d);
  h2d(d[0], logits, bl);
  h2d(d[1], targets, bt);
  check_status(jules_cross_entropy_loss(d[0], reinterpret_cast<const int32_t*>(d[1]), d[2],
                                        reinterpret_cast<float*>(d[3]), M, N, JULES_DTYPE_F32,
                                        nullptr),
               "jules_cross_entropy_loss");
  d2h(grad, d[2], bl);
  float loss = 0.0f;
  d2h(&loss, d[3], sizeof(float));
  check_status(jules_device_error(nullptr, 1), "fusedCrossEntropyLoss (target outside [0, N))");
  return loss;
}

void matmulInt8(const int8_t* A, const int8_t* B, float* C, int M, int N, int K, float scale_A,
                float scale_B, const float* bias, ExecutionArena* /*arena*/) {
  if (M <= 0 || N <= 0) return;
  const size_t ba = (size_t)M * K, bb = (size_t)K * N, bc = (size_t)M * N * 4;
  const size_t sizes[4] = {ba ? ba : 16, bb ? bb : 16, bc, (size_t)N * 4};
  char* d[4];
  staging().reserve(sizes, 4, d);
  h2d(d[0], A, ba);
  h2d(d[1], B, bb);
  if (bias) h2d(d[3], bias, (size_t)N * 4);
  check_status(jules_matmul_int8(reinterpret_cast<const int8_t*>(d[0]),
                                 reinterpret_cast<const int8_t*>(d[1]),
                                 reinterpret_cast<float*>(d[2]), M, N, K, scale_A, scale_B,
                                 bias ? reinterpret_cast<const float*>(d[3]) : nullptr, nullptr),
               "jules_matmul_int8");
  d2h(C, d[2], bc);
}

InterleavedMLPResult interleavedMLPForwardBackward(const float* X, const float* W1,
                                                   const float* b1, const float* W2,
                                                   const float* b2, const int32_t* targets,
                                                   float* output, float* dW1, float* db1,
                                                   float* dW2, float* db2, float* dX, int M,
                                                   int K1, int N1, int N2, ExecutionArena&,
                                                   TilePlanner&) {
  InterleavedMLPResult res{0.0f, MLPGradients{dW1, db1, dW2, db2, dX}};
  if (M <= 0) return res;
  const size_t bx = (size_t)M * K1 * 4, bw1 = (size_t)K1 * N1 * 4, bw2 = (size_t)N1 * N2 * 4;
  const size_t bo = (size_t)M * N2 * 4, bt = (size_t)M * 4;
  const size_t ws = jules_mlp_fwd_bwd_workspace_bytes(M, N1, N2);
  // X W1 b1 W2 b2 t out loss dW1 db1 dW2 db2 dX ws
  const size_t sizes[14] = {bx, bw1, (size_t)N1 * 4, bw2, (size_t)N2 * 4, bt, bo, 256,
                            bw1, (size_t)N1 * 4, bw2, (size_t)N2 * 4, dX ? bx : 16, ws};
  char* d[14];
  staging().reserve(sizes, 14, d);
  h2d(d[0], X, bx);
  h2d(d[1], W1, bw1);
  h2d(d[2], b1, (size_t)N1 * 4);
  h2d(d[3], W2, bw2);
  h2d(d[4], b2, (size_t)N2 * 4);
  h2d(d[5], targets, bt);
  auto f = [&](int i) { return reinterpret_cast<float*>(d[i]); };
  check_status(jules_mlp_fwd_bwd(f(0), f(1), f(2), f(3), f(4), reinterpret_cast<const int32_t*>(d[5]),
                                 f(6), f(7), f(8), f(9), f(10), f(11), dX ? f(12) : nullptr, M, K1,
                                 N1, N2, d[13], ws, nullptr),
               "jules_mlp_fwd_bwd");
  d2h(output, d[6], bo);
  d2h(&res.loss, d[7], 4);
  d2h(dW1, d[8], bw1);
  d2h(db1, d[9], (size_t)N1 * 4);
  d2h(dW2, d[10], bw2);
  d2h(db2, d[11], (size_t)N2 * 4);
  if (dX) d2h(dX, d[12], bx);
  check_status(jules_device_error(nullptr, 1), "interleavedMLPForwardBackward (target outside [0, N2))");
  return res;
}

void blasMatmul(const float* A, const float* B, float* C, int M, int N, int K, float alpha,
                float beta, bool transA, bool transB) {
  if (M <= 0 || N <= 0) return;
  // The plain product (no transposes, alpha 1, beta 0) runs the 3xTF32
  // tensor-core GEMM; everything else the fp32 SGEMM kernel.
  const bool plain = !transA && !transB && alpha == 1.0f && beta == 0.0f && K > 0;
  const size_t ba = (size_t)M * K * 4, bb = (size_t)K * N * 4, bc = (size_t)M * N * 4,
               bws = plain ? jules_gemm_f32_tc_workspace_bytes(M, N, K) : 0;
  const size_t sizes[4] = {ba ? ba : 4, bb ? bb : 4, bc, bws ? bws : 4};
  char* d[4];
  staging().reserve(sizes, 4, d);
  h2d(d[0], A, ba);
  h2d(d[1], B, bb);
  if (beta != 0.0f) h2d(d[2], C, bc);
  if (plain)
    check_status(jules_gemm_f32_tc(reinterpret_cast<float*>(d[0]), reinterpret_cast<float*>(d[1]),
                                   nullptr, reinterpret_cast<float*>(d[2]), M, N, K, JULES_ACT_NONE,
                                   d[3], bws, nullptr),
                 "jules_gemm_f32_tc");
  else
    check_status(jules_sgemm(transA, transB, M, N, K, alpha, reinterpret_cast<float*>(d[0]),
                             transA ? M : K, reinterpret_cast<float*>(d[1]), transB ? K : N, beta,
                             reinterpret_cast<float*>(d[2]), N, nullptr),
                 "jules_sgemm");
  d2h(C, d[2], bc);
}

void fusedMLPForward(float* output, const float* X, const MLPParams& p, ExecutionArena& arena,
                     TilePlanner& planner) {
  (void)planner;
  const int M = p.batch_size, K1 = p.in_features, N1 = p.hidden_features, N2 = p.out_features;
  if (M <= 0 || K1 <= 0 || N1 <= 0 || N2 <= 0) return;
  // Operands live in the caller's device arena (the reference's arena holds
  // the hidden activation, FusedKernels.h:669-700).
  float* dX = arena.allocate<float>((size_t)M * K1);
  float* dW1 = arena.allocate<float>((size_t)K1 * N1);
  float* db1 = arena.allocate<float>(N1);
  float* dW2 = arena.allocate<float>((size_t)N1 * N2);
  float* db2 = arena.allocate<float>(N2);
  float* dH = arena.allocate<float>((size_t)M * N1);
  float* dO = arena.allocate<float>((size_t)M * N2);
  h2d(dX, X, (size_t)M * K1 * 4);
  h2d(dW1, p.W1, (size_t)K1 * N1 * 4);
  h2d(db1, p.b1, (size_t)N1 * 4);
  h2d(dW2, p.W2, (size_t)N1 * N2 * 4);
  h2d(db2, p.b2, (size_t)N2 * 4);
  // The GEMMs' operand-split workspace lives in the staging area, not the
  // caller's arena (which is sized for the reference's own buffers).
  const size_t ws1 = jules_gemm_f32_tc_workspace_bytes(M, N1, K1),
               ws2 = jules_gemm_f32_tc_workspace_bytes(M, N2, N1);
  const size_t wsb[1] = {ws1 > ws2 ? ws1 : ws2};
  char* ws[1];
  staging().reserve(wsb, 1, ws);
  check_status(jules_gemm_f32_tc(dX, dW1, db1, dH, M, N1, K1, JULES_ACT_RELU, ws[0], wsb[0], nullptr),
               "mlp gemm1");
  check_status(jules_gemm_f32_tc(dH, dW2, db2, dO, M, N2, N1, JULES_ACT_NONE, ws[0], wsb[0], nullptr),
               "mlp gemm2");
  d2h(output, dO, (size_t)M * N2 * 4);
  arena.reset();
}

bool shouldUseFlashAttention(int seq_len, int head_dim, size_t l3_bytes) {
  const size_t attn_matrix_bytes = (size_t)seq_len * seq_len * sizeof(float);
  if (attn_matrix_bytes > l3_bytes) return true;
  return seq_len >= 64 && head_dim <= 256;
}

void flashAttention(float* output, const float* Q, const float* K, const float* V, int batch,
                    int heads, int seq, int head_dim, ExecutionArena& arena, TilePlanner& planner) {
  (void)arena;
  (void)planner;
  attention_host(output, Q, K, V, batch, heads, seq, head_dim);
}

void standardAttention(float* output, const float* Q, const float* K, const float* V, int batch,
                       int heads, int seq, int head_dim, ExecutionArena& arena) {
  // On the GPU the tiled kernel is the standard path too; the result is the
  // same softmax(QK^T/sqrt(D))V.
  attention_host(output, Q, K, V, batch, heads, seq, head_dim);
  arena.reset();
}

void attention(float* output, const float* Q, const float* K, const float* V, int batch, int heads,
               int seq, int head_dim, ExecutionArena& arena, TilePlanner& planner) {
  flashAttention(output, Q, K, V, batch, heads, seq, head_dim, arena, planner);
}

int flashAttentionBf16(uint16_t* output, float* lse, const uint16_t* Q, const uint16_t* K,
                       const uint16_t* V, int batch, int q_heads, int kv_heads, int seq,
                       int head_dim, bool causal, void* stream) {
  return jules_flash_attention_fwd(Q, K, V, output, lse, batch, q_heads, kv_heads, seq, head_dim,
                                   0.0f, causal ? 1 : 0, JULES_DTYPE_BF16, stream);
}

}  // namespace kernel
}  // namespace jules

// ---------------------------------------------------------------------------
// extern_kernel name registry
// ---------------------------------------------------------------------------
namespace {

struct KernelEntry {
  const char* name;
  int implemented;
};

// Names emitted by KernelRoutingPass (lib/Passes/KernelRoutingPass.cpp:
// 134-419) and documented in include/jules/Passes/KernelRoutingPass.h:13-23,
// plus the GELU forms the routing pass has no name for.
const KernelEntry kKernels[] = {
    {"fusedMatmulRelu", 1},        {"fusedMatmulSigmoid", 1},   {"fusedMatmulTanh", 1},
    {"fusedMatmulGelu", 1},        {"fusedMatmulBiasRelu", 1},  {"fusedMatmulBiasSigmoid", 1},
    {"fusedMatmulBiasTanh", 1},    {"fusedMatmulBiasGelu", 1},  {"fusedLayerNorm", 1},
    {"fusedGelu", 1},              {"fusedMLPForward", 1},      {"flashAttention", 1},
    {"blasMatmul", 1},             {"fusedSoftmax", 1},         {"fusedCrossEntropyLoss", 1},
    {"matmulInt8", 1},             {"interleavedMLPForwardBackward", 1},
};
constexpr int kNumKernels = sizeof(kKernels) / sizeof(kKernels[0]);

}  // namespace

extern "C" {

int jules_kernel_by_name(const char* name) {
  if (!name) return -1;
  for (int i = 0; i < kNumKernels; ++i)
    if (std::strcmp(kKernels[i].name, name) == 0) return i;
  return -1;
}

const char* jules_kernel_name(int id) {
  return (id >= 0 && id < kNumKernels) ? kKernels[id].name : nullptr;
}

int jules_kernel_count(void) { return kNumKernels; }

int jules_kernel_implemented(int id) {
  return (id >= 0 && id < kNumKernels) ? kKernels[id].implemented : 0;
}


}  // extern "C"
