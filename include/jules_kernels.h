/*
 * jules_kernels.h - C ABI of the B200 (sm_100a) implementation of the Jules
 * fused-kernel layer.
 *
 * Every entry point takes DEVICE pointers, plain sizes and a CUDA stream
 * (cudaStream_t passed as void*; NULL = legacy default stream), enqueues its
 * kernels and returns a status code without synchronising.  Inputs are
 * dense row-major, like the reference (include/jules/Kernel/*.h of
 * AVmakeralt/jules).  Outputs are fully overwritten.
 *
 * The reference's C++ API (jules::kernel::flashAttention etc., host float*)
 * is kept verbatim in include/jules/Kernel/*.h and is implemented on top of
 * these functions.
 *
 * Errors: 0 = success; otherwise a JULES_ERR_* code, with a message from
 * jules_last_error_string() (thread-local).  Shapes are validated (the
 * reference does no validation and aborts on arena overflow,
 * ExecutionArena.h:140-143).  Kernels never trap: a pipeline wait that
 * exceeds its time limit sets a device error word that
 * jules_device_error() reports.
 */
#ifndef JULES_KERNELS_H
#define JULES_KERNELS_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes. */
#define JULES_OK 0
#define JULES_ERR_SHAPE 1       /* invalid or unsupported dimensions */
#define JULES_ERR_ALIGN 2       /* pointer alignment the kernel needs */
#define JULES_ERR_DTYPE 3       /* unsupported dtype combination */
#define JULES_ERR_CUDA 4        /* CUDA runtime / launch error */
#define JULES_ERR_TIMEOUT 5     /* device pipeline wait timed out */
#define JULES_ERR_ARG 6         /* NULL pointer or bad enum */
#define JULES_ERR_UNSUPPORTED 7 /* name known but not implemented */
#define JULES_ERR_WORKSPACE 8   /* caller workspace too small */
#define JULES_ERR_COMM 9        /* NCCL missing or a collective failed */

/* Element types. */
#define JULES_DTYPE_F32 0
#define JULES_DTYPE_BF16 1
/* 8-bit floats (OCP FP8): E4M3 (finite only, max 448) and E5M2 (max 57344),
 * the two fp8 types of the reference's mixed-precision pass
 * (lib/Passes/MixedPrecisionPass.cpp:55-62, lib/Dialect/JulesDialect.cpp:41). */
#define JULES_DTYPE_FP8E4M3 2
#define JULES_DTYPE_FP8E5M2 3
/* IEEE half: the other 16-bit type of the reference's mixed-precision pass,
 * which treats f16 like bf16 (lib/Passes/MixedPrecisionPass.cpp:76). */
#define JULES_DTYPE_F16 4

/* Activations: same order as jules::kernel::ActivationType
 * (include/jules/Kernel/FusedKernels.h:61-67). */
#define JULES_ACT_NONE 0
#define JULES_ACT_RELU 1
#define JULES_ACT_SIGMOID 2
#define JULES_ACT_TANH 3
#define JULES_ACT_GELU 4

/* Library version, (major << 16) | minor. */
int jules_version(void);

/* Message for the last error on this host thread ("" if none). */
const char* jules_last_error_string(void);

/* Name of a status code. */
const char* jules_status_string(int status);

/*
 * Device error word: synchronises the current device, copies the word into
 * *word (may be NULL) and clears it when clear != 0.  Returns JULES_OK when
 * the word is zero, JULES_ERR_TIMEOUT when a bounded wait expired.
 */
int jules_device_error(uint32_t* word, int clear);

/*
 * Failure-detection self-test: launches one thread that waits, with a limit
 * of limit_ns (0 < limit_ns <= 2 s), on a pipeline barrier that nothing
 * completes.  The wait gives up the way every pipeline wait of the library
 * does (the device error word gets JULES_ERR_TIMEOUT's kind with site 250)
 * and the kernel returns, so jules_device_error() then reports
 * JULES_ERR_TIMEOUT and the context stays usable.  No counterpart in the
 * reference, whose kernels have no bounded waits.
 */
int jules_selftest_bounded_wait(uint64_t limit_ns, void* stream);

/*
 * C = act(A . W + bias) (+ residual)
 *   A [M,K], W [K,N], C and residual [M,N], bias [N] (fp32, nullable),
 *   residual nullable (same dtype as A and W).
 *   in_dtype: dtype of A, W and residual; out_dtype: dtype of C.
 * bf16 in (bf16 or fp32 out) or f16 in (f16 or fp32 out) with N % 8 == 0,
 * K % 8 == 0 and 16-byte aligned pointers runs on tcgen05 tensor cores (fp32
 * accumulate, fp32 epilogue, one cast at the store); everything else on CUDA
 * cores in fp32.
 * in_dtype JULES_DTYPE_FP8E4M3 / FP8E5M2 runs jules_gemm_fp8 with scale 1
 * (residual then bf16).
 * Replaces tiledMatmulWithActivation (FusedKernels.h:378-458),
 * fusedMatmulRelu (:203-259), fusedMatmulBiasRelu (:265-372) and
 * blasMatmul with alpha=1, beta=0, no transposes (:633-644).
 */
int jules_gemm_bias_act(const void* A, const void* W, const float* bias, const void* residual,
                        void* C, int64_t M, int64_t N, int64_t K, int act, int in_dtype,
                        int out_dtype, void* stream);

/*
 * fp32 C = act(A . W + bias) on tensor cores with fp32-level accuracy
 * (3xTF32): each operand is split into tf32 hi + lo parts (one HBM pass into
 * the caller's workspace, W transposed) and the tcgen05 pair GEMM (kind::tf32,
 * fp32 accumulation in TMEM) computes loA.hiW + hiA.loW + hiA.hiW, dropping
 * only loA.loW (relative size <= 2^-22).  K runs in chunks of 1024, each
 * chunk's epilogue adding the sum of the earlier ones in fp32 with a
 * round-to-nearest add (the MMA accumulation truncates, so long
 * accumulations would drift).  Activations in the accurate fp32 forms.
 *   A [M,K], W [K,N], C [M,N], bias [N] (nullable), all fp32, row-major.
 * Tensor cores for M >= 256, N >= 256, N % 8 == 0, K % 4 == 0 and 16-byte
 * aligned buffers; other shapes run the fp32 CUDA-core GEMM (no workspace
 * used).  workspace: jules_gemm_f32_tc_workspace_bytes(M, N, K) bytes of
 * device memory, 16-byte aligned (JULES_ERR_WORKSPACE when smaller).
 * Replaces tiledMatmulWithActivation (FusedKernels.h:378-458) and, through
 * the C++ API, blasMatmul / fusedMLPForward's GEMMs (:633-644, :650-760) on
 * the reference's float* path.
 */
size_t jules_gemm_f32_tc_workspace_bytes(int64_t M, int64_t N, int64_t K);
int jules_gemm_f32_tc(const float* A, const float* W, const float* bias, float* C, int64_t M,
                      int64_t N, int64_t K, int act, void* workspace, size_t workspace_bytes,
                      void* stream);

/*
 * Row-major fp32 SGEMM, C = alpha op(A) op(B) + beta C, with op = transpose
 * when transA / transB != 0; lda/ldb/ldc in elements.  The cblas_sgemm
 * contract the reference relies on (FusedKernels.h:633-644,
 * FlashAttention.h:74,92,184).  CUDA cores, fp32.
 */
int jules_sgemm(int transA, int transB, int64_t M, int64_t N, int64_t K, float alpha,
                const float* A, int64_t lda, const float* B, int64_t ldb, float beta, float* C,
                int64_t ldc, void* stream);

/*
 * Flash-attention forward.
 *   Q, O [B,Hq,S,D]; K, V [B,Hkv,S,D]; lse [B,Hq,S] fp32 (nullable),
 *   lse = log(sum_j exp(scale * q.k_j)) per query row, natural log.
 *   Hq % Hkv == 0 (grouped-query heads: kv head = h / (Hq/Hkv)).
 *   causal != 0 masks key j > query i.  scale <= 0 means 1/sqrt(D).
 *   dtype F32 (fp32 in/out, CUDA cores), BF16 or F16 (16-bit in/out, fp32
 *   softmax statistics; D == 128 or 64 with 16-byte aligned buffers runs on
 *   tcgen05, P in the operand type).
 * Replaces flashAttention (FlashAttention.h:130-309), standardAttention
 * (:52-100) and attention (:114-124), which are the non-causal, Hq == Hkv,
 * fp32 special case.
 */
int jules_flash_attention_fwd(const void* Q, const void* K, const void* V, void* O, float* lse,
                              int B, int Hq, int Hkv, int S, int D, float scale, int causal,
                              int dtype, void* stream);

/*
 * Flash-attention backward: dQ, dK, dV of O = softmax(scale * Q K^T [causal])
 * V for a given dO, from the forward's O and logsumexp (lse [B,Hq,S] fp32,
 * natural log, as jules_flash_attention_fwd writes it).  Q, O, dO, dQ
 * [B,Hq,S,D]; K, V, dK, dV [B,Hkv,S,D]; all of `dtype` (JULES_DTYPE_BF16 or
 * F32).  Grouped-query heads: dK / dV of a kv head sum over its Hq/Hkv
 * query heads.  scale <= 0 means 1/sqrt(D).  bf16 with D == 128 (16-byte
 * aligned buffers) runs on tcgen05 (bf16 P and dS, fp32 accumulation);
 * fp32, other head dims (<= 256) and unaligned buffers on CUDA cores in fp32.  No atomics: the
 * result is deterministic.  workspace: caller-provided device memory of
 * jules_flash_attention_bwd_workspace_bytes() bytes (16-byte aligned).
 * The reference has no attention backward; this is the gradient of the
 * forward that replaces flashAttention (FlashAttention.h:130-309), the
 * training-side neighbour of interleavedMLPForwardBackward
 * (InterleavedAutodiff.h:55-160).
 */
size_t jules_flash_attention_bwd_workspace_bytes(int B, int Hq, int S, int D, int dtype);
int jules_flash_attention_bwd(const void* Q, const void* K, const void* V, const void* O,
                              const void* dO, const float* lse, void* dQ, void* dK, void* dV,
                              int B, int Hq, int Hkv, int S, int D, float scale, int causal,
                              int dtype, void* workspace, size_t workspace_bytes, void* stream);

/*
 * Row LayerNorm: out = (x - mean) * inv_std * gamma + beta, biased variance,
 * inv_std = 1/sqrt(var + eps).  in [M,N], gamma/beta [N] fp32, optional
 * mean_out / rstd_out [M] fp32.  gamma and beta may both be NULL (no affine
 * transform, the form KernelRoutingPass routes).
 * Replaces fusedLayerNorm (FusedKernels.h:532-600).
 */
int jules_layernorm(const void* in, const float* gamma, const float* beta, void* out, int64_t M,
                    int64_t N, float eps, int in_dtype, int out_dtype, float* mean_out,
                    float* rstd_out, void* stream);

/*
 * GELU (tanh form) elementwise, n elements.
 * Replaces fusedGelu (FusedKernels.h:606-627).
 */
int jules_gelu(const void* in, void* out, int64_t n, int dtype, void* stream);

/*
 * int8 GEMM: C = float(A . B) * (scale_a * scale_b) (+ bias), int32
 * accumulation.  A [M,K], B [K,N] int8 row-major; C [M,N] and bias [N]
 * (nullable) fp32.  K and N multiples of 16 with 16-byte aligned pointers run
 * on tcgen05 (kind::i8); other shapes on CUDA cores.
 * Replaces matmulInt8 (FusedKernels.h:867-1073), whose int32 product is the
 * one its scalar branch (:1046-1057) computes.
 */
int jules_matmul_int8(const int8_t* A, const int8_t* B, float* C, int64_t M, int64_t N,
                      int64_t K, float scale_a, float scale_b, const float* bias, void* stream);

/*
 * fp8 GEMM: C = act((A . W) * scale + bias) (+ residual), fp32 accumulation
 * of products of 8-bit floats, fp32 epilogue, one cast at the store.
 *   A [M,K] (a_dtype), W [K,N] (w_dtype), each JULES_DTYPE_FP8E4M3 or
 *   JULES_DTYPE_FP8E5M2; bias [N] fp32 (nullable); residual [M,N] bf16
 *   (nullable); C [M,N] fp32 or bf16 (out_dtype).  scale: the product of the
 *   operands' dequantisation scales (1 for a plain cast).
 * The matmul of the reference's mixed-precision pass at target "fp8"
 * (lib/Passes/MixedPrecisionPass.cpp:1-28,125-140: inputs cast to fp8,
 * accumulation in f32, result cast back), with the epilogue of
 * tiledMatmulWithActivation (FusedKernels.h:378-458).  K and N multiples of
 * 16 with 16-byte aligned pointers run on tcgen05 (kind::f8f6f4); other
 * shapes on CUDA cores.
 */
int jules_gemm_fp8(const void* A, const void* W, const float* bias, const void* residual, void* C,
                   int64_t M, int64_t N, int64_t K, float scale, int act, int a_dtype,
                   int w_dtype, int out_dtype, void* stream);

/*
 * Element type conversion, n elements, any pair of JULES_DTYPE_* codes: the
 * reference's jules.cast (include/jules/Dialect/JulesOps.td:369, inserted by
 * lib/Passes/MixedPrecisionPass.cpp:176-184 createCastOp).  To bf16: round to nearest even.
 * To fp8: round to nearest even, saturating to the largest finite value
 * (E4M3 +-448, E5M2 +-57344); NaN stays NaN.  Widening casts are exact.
 */
int jules_cast(const void* src, void* dst, int64_t n, int src_dtype, int dst_dtype, void* stream);

/*
 * Row softmax: out[i,:] = exp(x[i,:] - max_i) / sum_j exp(x[i,j] - max_i),
 * in/out [M,N] row-major, fp32 arithmetic.  in_dtype and out_dtype each F32
 * or BF16.
 * Replaces fusedSoftmax (FusedKernels.h:464-526).
 */
int jules_softmax(const void* in, void* out, int64_t M, int64_t N, int in_dtype, int out_dtype,
                  void* stream);

/*
 * Fused softmax + cross-entropy over logits [M,N] and int32 targets [M]:
 *   p = softmax(logits[i,:]),  loss = mean_i -log(p[i, targets[i]] + 1e-10),
 *   grad[i,:] = (p - onehot(targets[i])) / M.
 * loss points to ONE device float, overwritten with the mean loss (row losses
 * are added atomically, so the last bits may vary between runs).  grad may be
 * NULL (loss only); otherwise it has the logits' dtype (F32 or BF16).  A
 * target outside [0, N) adds nothing to the loss and sets the device error
 * word (jules_device_error reports JULES_ERR_SHAPE).
 * Replaces fusedCrossEntropyLoss (FusedKernels.h:766-854), which returns the
 * loss on the host and always writes grad.
 */
int jules_cross_entropy_loss(const void* logits, const int32_t* targets, void* grad, float* loss,
                             int64_t M, int64_t N, int dtype, void* stream);

/*
 * 2-layer MLP training step, fp32 (the reference's
 * interleavedMLPForwardBackward, InterleavedAutodiff.h:55-160, computed over
 * the whole batch; its tiling only changes summation order):
 *   a = relu(X . W1 + b1), output = a . W2 + b2,
 *   *loss = mean_i -log(softmax(output_i)[targets_i] + 1e-10),
 *   dout = (softmax(output) - onehot) / M, dW2 = a^T dout, db2 = colsum(dout),
 *   dh = (dout . W2^T) * (a > 0), dW1 = X^T dh, db1 = colsum(dh),
 *   dX = dh . W1^T (skipped when dX is NULL).
 * X [M,K1], W1 [K1,N1], W2 [N1,N2], output [M,N2], targets [M] int32; loss is
 * one device float.  workspace: at least jules_mlp_fwd_bwd_workspace_bytes().
 */
size_t jules_mlp_fwd_bwd_workspace_bytes(int64_t M, int64_t N1, int64_t N2);
int jules_mlp_fwd_bwd(const float* X, const float* W1, const float* b1, const float* W2,
                      const float* b2, const int32_t* targets, float* output, float* loss,
                      float* dW1, float* db1, float* dW2, float* db2, float* dX, int64_t M,
                      int64_t K1, int64_t N1, int64_t N2, void* workspace, size_t workspace_bytes,
                      void* stream);

/*
 * Transformer MLP block, bf16:
 *   out = GELU(LN(X) . W1 + b1) . W2 + b2 + X
 *   X, out [T,d]; W1 [d,dff]; W2 [dff,d]; gamma, beta, b2 [d] and b1 [dff]
 *   fp32.  LN statistics, bias, GELU and residual in fp32; LN(X) and the
 *   hidden activation are stored as bf16 (matmul operands).  out_dtype
 *   BF16 or F32 (the cast back to the caller's type happens once, at the
 *   final store).
 * workspace: device buffer of at least jules_mlp_block_workspace_bytes().
 * Generalises fusedMLPForward (FusedKernels.h:650-760).
 */
size_t jules_mlp_block_workspace_bytes(int64_t T, int64_t d, int64_t dff);
int jules_mlp_block(const void* X, const float* gamma, const float* beta, const void* W1,
                    const float* b1, const void* W2, const float* b2, void* out, int out_dtype,
                    int64_t T, int64_t d, int64_t dff, float eps, void* workspace,
                    size_t workspace_bytes, void* stream);

/*
 * The MLP block with the LayerNorm folded into the first GEMM's epilogue.
 * With W1' = diag(gamma) W1,
 *   LN(x) . W1 + b1 = rstd * (x . W1' - mean * colsum(W1')) + (beta . W1 + b1),
 * so the first GEMM runs on the raw rows of X (no normalised copy of X in
 * HBM) after a pass that reads X once for its row statistics.
 * jules_mlp_block_fold_weights prepares, once per weights: W1f [d,dff] bf16
 * (= bf16(gamma[k] * W1[k][n])), colsum [dff] fp32 (column sums of W1f) and
 * c [dff] fp32 (= beta . W1 + b1).  jules_mlp_block_folded then computes
 * jules_mlp_block's result: out = GELU(LN(X) . W1 + b1) . W2 + b2 + X.
 * d and dff multiples of 8, d <= 8192, 16-byte aligned buffers; workspace of
 * jules_mlp_block_folded_workspace_bytes() (row statistics + the hidden
 * activation).  Rounding differs from jules_mlp_block (W1' is rounded to
 * bf16 instead of LN(X)); in fp32 accumulation the fold loses accuracy
 * when a row's |mean| is large against its standard deviation, where
 * jules_mlp_block is the form to use.
 * Implements fusedMLPForward's LayerNorm + first layer (FusedKernels.h:
 * 532-600, 650-760) with the normalisation inside the GEMM epilogue.
 */
int jules_mlp_block_fold_weights(const float* gamma, const float* beta, const void* W1,
                                 const float* b1, void* W1f, float* colsum, float* c, int64_t d,
                                 int64_t dff, void* stream);
size_t jules_mlp_block_folded_workspace_bytes(int64_t T, int64_t d, int64_t dff);
int jules_mlp_block_folded(const void* X, const void* W1f, const float* colsum, const float* c,
                           const void* W2, const float* b2, void* out, int out_dtype, int64_t T,
                           int64_t d, int64_t dff, float eps, void* workspace,
                           size_t workspace_bytes, void* stream);

/*
 * The MLP block of jules_mlp_block without any allocation: no counterpart in
 * the reference.  For callers that cannot allocate device memory, such as a
 * runtime's custom-call handler (the jules.extern_kernel ->
 * stablehlo.custom_call route), which receives only its operand and result
 * buffers while the device memory belongs to the runtime's allocator.
 * The workspace is an array compiled into the library, of
 * jules_mlp_block_noalloc_max_workspace_bytes() (32 MiB) on every device
 * that loads it; a call whose jules_mlp_block_workspace_bytes(T, d, dff)
 * exceeds that fails with JULES_ERR_WORKSPACE (e.g. d = 4096, dff = 16384
 * allows T <= 819).  All calls on a device share the array: calls that
 * overlap on the GPU race.  The first call on a device looks up the array's
 * device address (set-up); make that first call before any stream capture.
 * It calls no cudaMalloc / cudaFree and no allocating routine.
 */
size_t jules_mlp_block_noalloc_max_workspace_bytes(void);
int jules_mlp_block_noalloc(const void* X, const float* gamma, const float* beta, const void* W1,
                            const float* b1, const void* W2, const float* b2, void* out,
                            int out_dtype, int64_t T, int64_t d, int64_t dff, float eps,
                            void* stream);

/*
 * Custom-call entry: runs the kernel registered under `name` on the buffers a
 * runtime's custom-call handler receives (the jules.extern_kernel ->
 * stablehlo.custom_call call_target_name route, StableHLOLowering.cpp:
 * 1175-1214), inputs first, then outputs.  Shapes and scalars travel in the
 * opaque bytes as one jules_call_desc (opaque_len == sizeof).  Allocates
 * nothing (the MLP block runs as jules_mlp_block_noalloc).  Buffers per name:
 *   fusedMatmul{Relu,Sigmoid,Tanh,Gelu}   A, W, C          dims {M, N, K}
 *   fusedMatmulBias{Relu,Sigmoid,Tanh,Gelu} A, W, bias(f32), C   dims {M, N, K}
 *       dtype F32 or BF16 (operands); flags bit 0: C is fp32 for bf16 operands
 *   blasMatmul      A, B, C (f32)   dims {M, N, K}, fparams {alpha, beta},
 *                   flags bit 0 transA, bit 1 transB (dense row-major)
 *   fusedLayerNorm  x, out  or  x, gamma, beta, out   dims {M, N}, fparams[0]
 *                   eps (0 means 1e-5)
 *   fusedGelu       x, out          dims {n}
 *   fusedSoftmax    x, out          dims {M, N}
 *   fusedCrossEntropyLoss  logits, targets(int32), [grad,] loss(f32 scalar)
 *                   dims {M, N}
 *   flashAttention  Q, K, V, O [, lse]   dims {B, Hq, Hkv, S, D},
 *                   fparams[0] scale (0 means 1/sqrt(D)), flags bit 0 causal
 *   fusedMLPForward X, gamma, beta, W1, b1, W2, b2, out   dims {T, d, dff},
 *                   fparams[0] eps (0 means 1e-5), flags bit 0: out is fp32
 *   matmulInt8      A, B [, bias], C   dims {M, N, K}, fparams {scale_a, scale_b}
 * A registered name without an implementation returns JULES_ERR_UNSUPPORTED;
 * an unknown name, a wrong buffer count or opaque size JULES_ERR_ARG.
 */
typedef struct jules_call_desc {
  int64_t dims[6];
  float fparams[2];
  int32_t dtype; /* JULES_DTYPE_* of the floating-point operands */
  int32_t flags;
} jules_call_desc;

int jules_custom_call(const char* name, void* stream, void** buffers, int n_buffers,
                      const void* opaque, size_t opaque_len);

/*
 * Kernel registry keyed by the jules.extern_kernel names that
 * KernelRoutingPass emits (lib/Passes/KernelRoutingPass.cpp:134-419) plus
 * the documented fusedMLPForward / flashAttention and the GELU variants the
 * routing pass cannot name (activationToString has no GELU case,
 * KernelRoutingPass.cpp:88-94).
 * jules_kernel_by_name returns an id >= 0, or -1 for an unknown name.
 * jules_kernel_implemented returns 1 when the id has a CUDA implementation.
 */
int jules_kernel_by_name(const char* name);
const char* jules_kernel_name(int id);
int jules_kernel_count(void);
int jules_kernel_implemented(int id);

/*
 * ---------------------------------------------------------------------------
 * Multi-GPU: one process per GPU (1 <= world <= 8, one node).  The hot path is
 * split into independent units - token rows of the GEMM, (batch, kv head)
 * units of attention - and the outputs are gathered over NVLink, the one
 * exchange the partition needs.  The reference names that exchange only as an
 * IR collective (include/jules/Dialect/JulesOps.td:660-684, lowering in
 * lib/Passes/StableHLOLowering.cpp:1100-1170 that never runs); these entry
 * points are what a dispatch table binds for it.  NCCL is loaded at run time
 * (libnccl.so.2); without it these calls return JULES_ERR_COMM.
 *
 * All dist calls are collective: every rank makes the same calls in the same
 * order, with the same shapes.  Buffers use the single-GPU layouts; each rank
 * reads only its own units of the inputs and every rank's output holds the
 * whole result when the call's work on `stream` has finished.
 * ---------------------------------------------------------------------------
 */
#define JULES_DIST_ID_BYTES 128

/* Balanced contiguous partition: rank's units are [*begin, *end) of units. */
int jules_dist_shard(int64_t units, int world, int rank, int64_t* begin, int64_t* end);

/* Rank 0 creates the id (JULES_DIST_ID_BYTES bytes) and passes it to every
 * rank out of band; each rank then calls jules_dist_init with its own device
 * current.  jules_dist_destroy releases the communicator and its buffers. */
int jules_dist_unique_id(void* id);
int jules_dist_init(void** comm, int world, int rank, const void* id);
int jules_dist_destroy(void* comm);

/* Stream-ordered barrier over all ranks (an 8-byte all-reduce). */
int jules_dist_barrier(void* comm, void* stream);

/* Output buffer that every rank can write: each rank allocates `bytes`, and
 * the peers' buffers are mapped into every process.  With NVLink multicast
 * (below) it is an NCCL symmetric window bound to the communicator's
 * multicast object; otherwise cudaMalloc + CUDA IPC (handles exchanged over
 * the communicator).  Both calls are collective (same buffers, same order on
 * every rank).  The memory is zeroed. */
int jules_dist_alloc_shared(void* comm, size_t bytes, void** local);
int jules_dist_free_shared(void* comm, void* local);

/* *on = 1 when this communicator's shared buffers have an NVLink multicast
 * address (NVSwitch multicast, NCCL >= 2.28 with its device API): the fused
 * gathers then store each chunk once and the switch replicates it to every
 * rank.  Opt-in: set JULES_DIST_MULTICAST=1 in every rank before
 * jules_dist_init (it measured no reproducible gain over peer stores on 2-8
 * B200s; it needs NVLS, so NCCL_NVLS_ENABLE=0 also keeps it off). */
int jules_dist_multicast(void* comm, int* on);

/* How the sharded calls gather an output of out_bytes (total, all ranks)
 * held in a shared buffer:
 *   JULES_GATHER_STORES     the kernel's epilogue stores every finished tile
 *                           into every rank's buffer over NVLink;
 *   JULES_GATHER_MULTICAST  the same through the buffer's multicast address;
 *   JULES_GATHER_PULL       the kernel stores this rank's share locally and,
 *                           once every rank has signalled, the copy engines
 *                           fetch the other ranks' shares (one transfer per
 *                           peer on its own stream).
 * Chosen from the world size and out_bytes (the same on every rank);
 * JULES_DIST_GATHER=stores or pull in the environment forces one. */
#define JULES_GATHER_STORES 0
#define JULES_GATHER_MULTICAST 1
#define JULES_GATHER_PULL 2
int jules_dist_gather_route(void* comm, size_t out_bytes, int* route);

/*
 * Sharded jules_gemm_bias_act: rank r computes rows jules_dist_shard(M) of
 * C = act(A . W + bias) (+ residual) from its rows of A (and residual); W and
 * bias are replicated.  When C comes from jules_dist_alloc_shared (bf16
 * operands, N % 8 == 0, K % 8 == 0, M / world >= 256, N >= 256), the gather
 * is fused into the GEMM: the epilogue stores every finished tile into all
 * ranks' C over NVLink while later tiles compute, then the ranks signal each
 * other through counters in peer memory (a bounded wait; an expired wait
 * reports JULES_ERR_TIMEOUT through jules_device_error).  Otherwise the rows
 * are computed locally and gathered with an in-place ncclAllGather.
 * Replaces tiledMatmulWithActivation (FusedKernels.h:378-458) run across the
 * GPUs of one node.
 */
int jules_dist_gemm_bias_act(void* comm, const void* A, const void* W, const float* bias,
                             const void* residual, void* C, int64_t M, int64_t N, int64_t K,
                             int act, int in_dtype, int out_dtype, void* stream);

/*
 * Sharded jules_flash_attention_fwd: the B x Hkv (batch, kv head) units are
 * split evenly over the ranks (B * Hkv % world == 0, and each rank's units
 * whole batches or a part of one); each rank computes O (and lse) of its
 * units, then O and lse are gathered in place with ncclAllGather.
 * Replaces flashAttention (FlashAttention.h:130-309) run across the GPUs of
 * one node.
 */
int jules_dist_flash_attention_fwd(void* comm, const void* Q, const void* K, const void* V, void* O,
                                   float* lse, int B, int Hq, int Hkv, int S, int D, float scale,
                                   int causal, int dtype, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* JULES_KERNELS_H */
