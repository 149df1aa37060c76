/*
 * CPU restatement of the Jules fused-kernel hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the parity checker for the CUDA
 * kernels in jules_b200/csrc and the "port" CPU baseline.  Only tests/,
 * __graft_entry__.smoke() and bench.py's CPU legs may load it; the shipped
 * library never links it and has no CPU fallback.
 *
 * Each routine restates a reference routine (paths are within the
 * AVmakeralt/jules project) and is itself pinned against the reference's
 * own code, compiled from source into oracle/_ref by oracle/Makefile, by the
 * golden fixtures under tests/golden (tests/test_oracle.py).  Where the
 * reference lacks a feature the configs need (causal mask, grouped-query
 * heads, logsumexp output, bias+GELU, LayerNorm->MLP->residual), the
 * extension is written into the reference's own loop structure and marked.
 *
 * Numerics: fp32 accumulation in the reference's loop order; expf() stands
 * in for the reference's fast_exp_zmm polynomial (FusedKernels.h:90-133),
 * which differs by ~1 ulp.
 */
#include <float.h>
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

/* ------------------------------------------------------------------ */
/* Casts.  The reference's MixedPrecisionPass lowers casts to           */
/* stablehlo.convert (lib/Passes/StableHLOLowering.cpp:461-470), i.e.   */
/* round-to-nearest-even.                                               */
/* ------------------------------------------------------------------ */
static inline float bf16_rne(float x) {
  uint32_t u;
  memcpy(&u, &x, 4);
  if ((u & 0x7f800000u) == 0x7f800000u) {
    if (u & 0x007fffffu) u |= 0x00400000u; /* keep NaN quiet */
    u &= 0xffff0000u;
  } else {
    u += 0x7fffu + ((u >> 16) & 1u);
    u &= 0xffff0000u;
  }
  memcpy(&x, &u, 4);
  return x;
}

void orc_round_bf16(float* x, int64_t n) {
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < n; i++) x[i] = bf16_rne(x[i]);
}

/* bf16 bit patterns <-> float (the GPU consumes the same bits). */
void orc_f32_to_bf16_bits(const float* x, uint16_t* out, int64_t n) {
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < n; i++) {
    float r = bf16_rne(x[i]);
    uint32_t u;
    memcpy(&u, &r, 4);
    out[i] = (uint16_t)(u >> 16);
  }
}

void orc_bf16_bits_to_f32(const uint16_t* in, float* out, int64_t n) {
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < n; i++) {
    uint32_t u = (uint32_t)in[i] << 16;
    memcpy(&out[i], &u, 4);
  }
}

/* ------------------------------------------------------------------ */
/* Activations: FusedKernels.h:61-67 (ActivationType), 137-164 (tanh,   */
/* sigmoid, GELU), 425-428 (scalar forms).                              */
/* ------------------------------------------------------------------ */
enum { ORC_ACT_NONE = 0, ORC_ACT_RELU = 1, ORC_ACT_SIGMOID = 2, ORC_ACT_TANH = 3,
       ORC_ACT_GELU = 4 };

/* exp with the reference's +-88 clamp (FusedKernels.h:91-96). */
static inline float clamped_exp(float x) {
  if (x > 88.0f) x = 88.0f;
  if (x < -88.0f) x = -88.0f;
  return expf(x);
}

/* tanh(x) = (e^{2x}-1)/(e^{2x}+1)  (FusedKernels.h:137-143) */
static inline float ref_tanh(float x) {
  float e = clamped_exp(2.0f * x);
  return (e - 1.0f) / (e + 1.0f);
}

/* GELU-tanh, formula pinned by GeluOp (include/jules/Dialect/JulesOps.td:256-265)
 * and gelu_zmm (FusedKernels.h:155-164). */
static inline float ref_gelu(float x) {
  float inner = 0.7978845608f * (x + 0.044715f * (x * x * x));
  return 0.5f * (x * (1.0f + ref_tanh(inner)));
}

static inline float apply_act(float v, int act) {
  switch (act) {
    case ORC_ACT_RELU: return v > 0.0f ? v : 0.0f;
    case ORC_ACT_SIGMOID: return 1.0f / (1.0f + clamped_exp(-v));
    case ORC_ACT_TANH: return ref_tanh(v);
    case ORC_ACT_GELU: return ref_gelu(v);
    default: return v;
  }
}

/* FusedKernels.h:606-627 */
void orc_gelu(float* out, const float* in, int64_t n) {
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < n; i++) out[i] = ref_gelu(in[i]);
}

/* ------------------------------------------------------------------ */
/* GEMM + bias + activation (+ residual).                               */
/* Loop structure of tiledMatmulWithActivation (FusedKernels.h:378-458): */
/* each C element accumulates A[i,k]*B[k,j] in k order in fp32; the     */
/* activation is applied after the last K tile (:407-415).  Bias is     */
/* added before the activation as in fusedMatmulBiasRelu (:308-313).    */
/* Residual (extension for the MLP block): added after the activation.  */
/* A [M,K], B [K,N], C [M,N], all row-major; argument order (M,N,K).    */
/* ------------------------------------------------------------------ */
void orc_gemm_bias_act(const float* A, const float* B, const float* bias,
                       const float* residual, float* C, int64_t M, int64_t N,
                       int64_t K, int act) {
#pragma omp parallel for schedule(dynamic, 1)
  for (int64_t i = 0; i < M; i++) {
    float* c = C + i * N;
    for (int64_t j = 0; j < N; j++) c[j] = 0.0f;
    const float* a = A + i * K;
    for (int64_t k = 0; k < K; k++) {
      const float av = a[k];
      const float* b = B + k * N;
      for (int64_t j = 0; j < N; j++) c[j] += av * b[j];
    }
    for (int64_t j = 0; j < N; j++) {
      float v = c[j];
      if (bias) v += bias[j];
      v = apply_act(v, act);
      if (residual) v += residual[i * N + j];
      c[j] = v;
    }
  }
}

/* ------------------------------------------------------------------ */
/* LayerNorm: FusedKernels.h:532-600.  Two passes over the row (mean,   */
/* then biased variance), inv_std = 1/sqrt(var+eps),                    */
/* y = (x-mean)*inv_std*gamma + beta.  16 partial sums mimic the        */
/* 16-lane AVX-512 accumulation (:545-566).                             */
/* Optional outputs: per-row mean and inv_std.                          */
/* ------------------------------------------------------------------ */
/*
 * 2-layer MLP training step.  InterleavedAutodiff.h:55-160 (per tile: :127-
 * 160 forward, :162-185 loss and dL/do, :187-258 backward), over the whole
 * batch at once (the tiling only changes summation order):
 *   h = X W1 + b1, a = relu(h), out = a W2 + b2,
 *   p = softmax(out row), loss = sum_i -log(p[i, t_i] + 1e-10) / M,
 *   do = (p - onehot(t)) / M, dW2 = a^T do, db2 = colsum(do),
 *   dh = (do W2^T) * (h > 0), dW1 = X^T dh, db1 = colsum(dh), dX = dh W1^T.
 * Accumulation in double here (the fixtures pin it to the reference within
 * the fp32 tolerance).  dX may be NULL.
 */
float orc_mlp_fwd_bwd(const float* X, const float* W1, const float* b1, const float* W2,
                      const float* b2, const int32_t* t, float* out, float* dW1, float* db1,
                      float* dW2, float* db2, float* dX, int64_t M, int64_t K1, int64_t N1,
                      int64_t N2) {
  float* a = (float*)malloc(sizeof(float) * (size_t)(M * N1));
  float* dout = (float*)malloc(sizeof(float) * (size_t)(M * N2));
  float* dh = (float*)malloc(sizeof(float) * (size_t)(M * N1));
  double loss = 0.0;
  for (int64_t i = 0; i < M; i++) {
    for (int64_t j = 0; j < N1; j++) {
      double s = b1[j];
      for (int64_t k = 0; k < K1; k++) s += (double)X[i * K1 + k] * W1[k * N1 + j];
      a[i * N1 + j] = s > 0.0 ? (float)s : 0.0f;
    }
    for (int64_t j = 0; j < N2; j++) {
      double s = b2[j];
      for (int64_t k = 0; k < N1; k++) s += (double)a[i * N1 + k] * W2[k * N2 + j];
      out[i * N2 + j] = (float)s;
    }
    double mx = -DBL_MAX, sum = 0.0;
    for (int64_t j = 0; j < N2; j++) mx = fmax(mx, out[i * N2 + j]);
    for (int64_t j = 0; j < N2; j++) sum += exp(out[i * N2 + j] - mx);
    for (int64_t j = 0; j < N2; j++) {
      const double p = exp(out[i * N2 + j] - mx) / sum;
      dout[i * N2 + j] = (float)((p - (j == t[i] ? 1.0 : 0.0)) / (double)M);
      if (j == t[i]) loss += -log(p + 1e-10);
    }
  }
  for (int64_t i = 0; i < M; i++)
    for (int64_t j = 0; j < N1; j++) {
      double s = 0.0;
      for (int64_t k = 0; k < N2; k++) s += (double)dout[i * N2 + k] * W2[j * N2 + k];
      dh[i * N1 + j] = a[i * N1 + j] > 0.0f ? (float)s : 0.0f;
    }
  for (int64_t r = 0; r < N1; r++)
    for (int64_t c = 0; c < N2; c++) {
      double s = 0.0;
      for (int64_t i = 0; i < M; i++) s += (double)a[i * N1 + r] * dout[i * N2 + c];
      dW2[r * N2 + c] = (float)s;
    }
  for (int64_t c = 0; c < N2; c++) {
    double s = 0.0;
    for (int64_t i = 0; i < M; i++) s += dout[i * N2 + c];
    db2[c] = (float)s;
  }
  for (int64_t r = 0; r < K1; r++)
    for (int64_t c = 0; c < N1; c++) {
      double s = 0.0;
      for (int64_t i = 0; i < M; i++) s += (double)X[i * K1 + r] * dh[i * N1 + c];
      dW1[r * N1 + c] = (float)s;
    }
  for (int64_t c = 0; c < N1; c++) {
    double s = 0.0;
    for (int64_t i = 0; i < M; i++) s += dh[i * N1 + c];
    db1[c] = (float)s;
  }
  if (dX)
    for (int64_t i = 0; i < M; i++)
      for (int64_t k = 0; k < K1; k++) {
        double s = 0.0;
        for (int64_t j = 0; j < N1; j++) s += (double)dh[i * N1 + j] * W1[k * N1 + j];
        dX[i * K1 + k] = (float)s;
      }
  free(a);
  free(dout);
  free(dh);
  return (float)(loss / (double)M);
}

/*
 * int8 GEMM.  FusedKernels.h:867-1073: int32 accumulation as its scalar
 * branch (:1046-1057), C = (float)acc * (scale_a * scale_b), plus bias[j]
 * (:1060-1065).  (The reference's AVX-512 branches load 32 columns of B per
 * 16-column step and sum adjacent columns pairwise; the scalar branch is the
 * routine's stated contract.)
 */
void orc_matmul_int8(const int8_t* A, const int8_t* B, float* C, int64_t M, int64_t N, int64_t K,
                     float scale_a, float scale_b, const float* bias) {
  const float s = scale_a * scale_b;
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < M; i++) {
    int32_t* acc = (int32_t*)calloc((size_t)N, sizeof(int32_t));
    for (int64_t k = 0; k < K; k++) {
      const int32_t a = A[i * K + k];
      const int8_t* b = B + k * N;
      for (int64_t j = 0; j < N; j++) acc[j] += a * (int32_t)b[j];
    }
    for (int64_t j = 0; j < N; j++) {
      C[i * N + j] = (float)acc[j] * s;
      if (bias) C[i * N + j] += bias[j];
    }
    free(acc);
  }
}

/*
 * 8-bit floats: the E4M3 and E5M2 types of the reference's mixed-precision
 * pass (lib/Passes/MixedPrecisionPass.cpp:55-62; lib/Dialect/JulesDialect.cpp
 * :41-77), which the reference names but never evaluates.  Restated from
 * the OCP 8-bit floating point specification (v1.0): sign, exponent,
 * mantissa = 1/4/3 bits with bias 7 (E4M3) or 1/5/2 bits with bias 15
 * (E5M2); exponent field 0 holds subnormals m * 2^(1 - bias - mbits).  E4M3
 * has no infinities: S.1111.111 is its only NaN and 448 its largest value.
 * E5M2 follows IEEE 754: exponent 31 with mantissa 0 is infinity, else NaN;
 * 57344 is its largest finite value.
 * fmt: 0 = E4M3, 1 = E5M2.
 */
float orc_fp8_to_f32(uint8_t x, int fmt) {
  const int mbits = fmt == 0 ? 3 : 2, bias = fmt == 0 ? 7 : 15;
  const int e = (x & 0x7F) >> mbits, m = x & ((1 << mbits) - 1);
  const double sign = (x & 0x80) ? -1.0 : 1.0;
  if (fmt == 0 && e == 15 && m == 7) return NAN;
  if (fmt == 1 && e == 31) return m ? NAN : (float)(sign * INFINITY);
  if (e == 0) return (float)(sign * ldexp((double)m, 1 - bias - mbits));
  return (float)(sign * ldexp((double)((1 << mbits) + m), e - bias - mbits));
}

/*
 * fp32 -> 8-bit float: round to nearest, ties to even, saturating to the
 * largest finite value (the conversion jules_cast documents); NaN -> the
 * format's NaN (E4M3 S.1111.111, E5M2 S.11111.11).
 */
uint8_t orc_f32_to_fp8(float x, int fmt) {
  const int mbits = fmt == 0 ? 3 : 2, bias = fmt == 0 ? 7 : 15;
  const uint8_t sign = signbit(x) ? 0x80 : 0x00;
  const uint8_t max_code = fmt == 0 ? 0x7E : 0x7B;
  if (isnan(x)) return sign | 0x7F;
  const double a = fabs((double)x);
  if (a >= (double)orc_fp8_to_f32(max_code, fmt)) return sign | max_code;
  const int emin = 1 - bias;  /* exponent of the smallest normal */
  int e2;
  frexp(a, &e2);              /* a = f * 2^e2, f in [0.5, 1) */
  int e = e2 - 1;             /* a in [2^e, 2^(e+1)) */
  if (a == 0.0 || e < emin) {
    /* subnormal spacing 2^(emin - mbits); k = 2^mbits rolls into the smallest normal */
    const double k = rint(ldexp(a, mbits - emin));
    return sign | (uint8_t)k;
  }
  double k = rint(ldexp(a, mbits - e));   /* in [2^mbits, 2^(mbits+1)] */
  if (k == (double)(1 << (mbits + 1))) {
    k = (double)(1 << mbits);
    e += 1;
  }
  const int code = ((e + bias) << mbits) | ((int)k - (1 << mbits));
  return sign | (uint8_t)(code > max_code ? max_code : code);
}

void orc_fp8_decode(const uint8_t* in, float* out, int64_t n, int fmt) {
  for (int64_t i = 0; i < n; i++) out[i] = orc_fp8_to_f32(in[i], fmt);
}

void orc_fp8_encode(const float* in, uint8_t* out, int64_t n, int fmt) {
  for (int64_t i = 0; i < n; i++) out[i] = orc_f32_to_fp8(in[i], fmt);
}

/*
 * fp8 GEMM, the matmul the mixed-precision pass forms at target "fp8"
 * (MixedPrecisionPass.cpp:1-28: operands cast to fp8, accumulation in f32,
 * result cast back), with the tiledMatmulWithActivation epilogue
 * (FusedKernels.h:378-458): C = act((A . W) * scale + bias) (+ residual).
 * Products of decoded operands summed in double (the exact sum, rounded
 * once), then the fp32 epilogue.
 */
void orc_gemm_fp8(const uint8_t* A, const uint8_t* W, const float* bias, const float* residual,
                  float* C, int64_t M, int64_t N, int64_t K, float scale, int act, int a_fmt,
                  int w_fmt) {
  float* wd = (float*)malloc((size_t)(K * N) * sizeof(float));
  for (int64_t i = 0; i < K * N; i++) wd[i] = orc_fp8_to_f32(W[i], w_fmt);
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < M; i++) {
    double* acc = (double*)calloc((size_t)N, sizeof(double));
    for (int64_t k = 0; k < K; k++) {
      const double a = orc_fp8_to_f32(A[i * K + k], a_fmt);
      const float* w = wd + k * N;
      for (int64_t j = 0; j < N; j++) acc[j] += a * (double)w[j];
    }
    for (int64_t j = 0; j < N; j++) {
      float v = (float)acc[j] * scale;
      if (bias) v += bias[j];
      v = apply_act(v, act);
      if (residual) v += residual[i * N + j];
      C[i * N + j] = v;
    }
    free(acc);
  }
  free(wd);
}

/*
 * Row softmax.  FusedKernels.h:464-526, in the summation order of its
 * AVX-512 branch (:466-505): max over the row (from -FLT_MAX); e = exp(x -
 * max) stored and summed in 16 lanes over 16-wide chunks, the lanes reduced,
 * then the scalar tail added; each e multiplied by 1/sum (the tail divided).
 */
void orc_softmax(float* out, const float* in, int64_t M, int64_t N) {
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < M; i++) {
    const float* x = in + i * N;
    float* y = out + i * N;
    float mx = -FLT_MAX;
    for (int64_t j = 0; j < N; j++) mx = fmaxf(mx, x[j]);
    float lane[16] = {0};
    int64_t j = 0;
    for (; j + 15 < N; j += 16)
      for (int l = 0; l < 16; l++) {
        y[j + l] = expf(x[j + l] - mx);
        lane[l] += y[j + l];
      }
    /* lane reduction as a halving tree */
    for (int w = 8; w > 0; w >>= 1)
      for (int l = 0; l < w; l++) lane[l] += lane[l + w];
    float sum = lane[0];
    const int64_t vec_end = j;
    for (; j < N; j++) {
      y[j] = expf(x[j] - mx);
      sum += y[j];
    }
    const float inv = 1.0f / sum;
    for (j = 0; j < vec_end; j++) y[j] *= inv;
    for (; j < N; j++) y[j] /= sum;
  }
}

/*
 * Softmax + cross-entropy.  FusedKernels.h:766-854 (scalar branch :827-850):
 * grad = softmax(row); row loss = -log(grad[target] + 1e-10); grad[target]
 * -= 1; grad /= M; returns the sum of row losses / M.  The row losses are
 * summed in row order here (the reference sums them in an OpenMP reduction).
 */
float orc_cross_entropy(const float* logits, const int32_t* targets, float* grad, int64_t M,
                        int64_t N) {
  orc_softmax(grad, logits, M, N);
  double total = 0.0;
  for (int64_t i = 0; i < M; i++) {
    float* g = grad + i * N;
    const int32_t t = targets[i];
    total += -logf(g[t] + 1e-10f);
    g[t] -= 1.0f;
    for (int64_t j = 0; j < N; j++) g[j] /= (float)M;
  }
  return (float)(total / (double)M);
}

void orc_layernorm(float* out, const float* in, const float* gamma,
                   const float* beta, int64_t M, int64_t N, float eps,
                   float* mean_out, float* rstd_out) {
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < M; i++) {
    const float* x = in + i * N;
    float lanes[16] = {0};
    int64_t j = 0;
    for (; j + 15 < N; j += 16)
      for (int l = 0; l < 16; l++) lanes[l] += x[j + l];
    float mean = 0.0f;
    for (int l = 0; l < 16; l++) mean += lanes[l];
    for (; j < N; j++) mean += x[j];
    mean /= (float)N;

    float vl[16] = {0};
    j = 0;
    for (; j + 15 < N; j += 16)
      for (int l = 0; l < 16; l++) {
        float d = x[j + l] - mean;
        vl[l] += d * d;
      }
    float var = 0.0f;
    for (int l = 0; l < 16; l++) var += vl[l];
    for (; j < N; j++) {
      float d = x[j] - mean;
      var += d * d;
    }
    var /= (float)N;
    float inv_std = 1.0f / sqrtf(var + eps);
    float* y = out + i * N;
    for (j = 0; j < N; j++) y[j] = (x[j] - mean) * inv_std * gamma[j] + beta[j];
    if (mean_out) mean_out[i] = mean;
    if (rstd_out) rstd_out[i] = inv_std;
  }
}

/*
 * Attention backward (no reference routine: the reference has no gradient
 * for attention).  The exact gradient of the forward restated below,
 * O = softmax(scale * Q K^T [causal]) V, for a given dO, in double:
 *   P = softmax row by row (from the scores, not from a stored lse),
 *   dV_j = sum_i P_ij dO_i, dP_ij = dO_i . v_j, D_i = sum_j P_ij dP_ij,
 *   dS_ij = P_ij (dP_ij - D_i), dQ_i = scale sum_j dS_ij k_j,
 *   dK_j = scale sum_i dS_ij q_i; grouped-query heads sum into their kv head.
 * Layout as orc_flash_attention.  dK, dV are zeroed here.
 */
void orc_attention_bwd(float* dQ, float* dK, float* dV, const float* Q, const float* K,
                       const float* V, const float* dO, int B, int Hq, int Hkv, int S, int D,
                       float scale, int causal) {
  const int group = Hq / Hkv;
  const size_t nkv = (size_t)B * Hkv * S * D;
  double* dk = (double*)calloc(nkv, sizeof(double));
  double* dv = (double*)calloc(nkv, sizeof(double));
  double* P = (double*)malloc(sizeof(double) * (size_t)S * S);   /* P_ij, row i */
  double* dS = (double*)malloc(sizeof(double) * (size_t)S * S);  /* dS_ij */
  for (int b = 0; b < B; b++)
    for (int h = 0; h < Hq; h++) {
      const size_t zq = (size_t)b * Hq + h, zk = (size_t)b * Hkv + h / group;
      const float* q = Q + zq * S * D;
      const float* g = dO + zq * S * D;
      const float* k = K + zk * S * D;
      const float* v = V + zk * S * D;
#pragma omp parallel for schedule(dynamic, 4)
      for (int i = 0; i < S; i++) {
        double* pr = P + (size_t)i * S;
        double* dsr = dS + (size_t)i * S;
        const int n = causal ? i + 1 : S;
        double m = -INFINITY, l = 0.0, dsum = 0.0;
        for (int j = 0; j < S; j++) {
          pr[j] = 0.0;
          dsr[j] = 0.0;
        }
        for (int j = 0; j < n; j++) {
          double t = 0.0;
          for (int d = 0; d < D; d++) t += (double)q[(size_t)i * D + d] * k[(size_t)j * D + d];
          pr[j] = t * scale;
          if (pr[j] > m) m = pr[j];
        }
        for (int j = 0; j < n; j++) {
          pr[j] = exp(pr[j] - m);
          l += pr[j];
        }
        for (int j = 0; j < n; j++) {
          double t = 0.0;
          pr[j] /= l;
          for (int d = 0; d < D; d++) t += (double)g[(size_t)i * D + d] * v[(size_t)j * D + d];
          dsr[j] = t;            /* dP_ij for now */
          dsum += pr[j] * t;
        }
        for (int j = 0; j < n; j++) dsr[j] = pr[j] * (dsr[j] - dsum);
        for (int d = 0; d < D; d++) {
          double t = 0.0;
          for (int j = 0; j < n; j++) t += dsr[j] * k[(size_t)j * D + d];
          dQ[(zq * S + i) * D + d] = (float)(t * scale);
        }
      }
#pragma omp parallel for schedule(static)
      for (int j = 0; j < S; j++) {
        double* acck = dk + (zk * S + j) * D;
        double* accv = dv + (zk * S + j) * D;
        for (int i = causal ? j : 0; i < S; i++) {
          const double pij = P[(size_t)i * S + j], dsij = dS[(size_t)i * S + j];
          for (int d = 0; d < D; d++) {
            accv[d] += pij * g[(size_t)i * D + d];
            acck[d] += dsij * scale * q[(size_t)i * D + d];
          }
        }
      }
    }
  for (size_t x = 0; x < nkv; x++) {
    dK[x] = (float)dk[x];
    dV[x] = (float)dv[x];
  }
  free(P);
  free(dS);
  free(dk);
  free(dv);
}

/* ------------------------------------------------------------------ */
/* Flash attention forward: FlashAttention.h:130-309.                   */
/* Per (b,h) unit and query tile: running max/sum and an accumulator;   */
/* per key tile: scores = scale*q.k (:184-188), new_max = max(old,       */
/* tile max) (:195-204), rescale acc and sum by exp(old-new) when old    */
/* is finite (:206-220), p = exp(s-new) (:222-235), acc += p*V (:237-    */
/* 250), final acc/sum (:287-305).                                      */
/* Extensions (absent from the reference):                              */
/*  - causal: key j > query i is excluded; key tiles entirely above the  */
/*    diagonal are skipped;                                              */
/*  - grouped-query heads: kv head = h / (Hq/Hkv);                       */
/*  - lse (nullable) = running_max + log(running_sum), natural log, in   */
/*    the scaled-score domain;                                           */
/*  - a query-row window [q_begin, q_end) and a unit list so large       */
/*    configs can be checked on samples.                                 */
/* Layout: Q,O [B,Hq,S,D]; K,V [B,Hkv,S,D]; lse [B,Hq,S]; row-major.     */
/* units: n_units entries of (b*Hq + h); NULL means all B*Hq units.      */
/* ------------------------------------------------------------------ */
void orc_flash_attention(float* out, float* lse, const float* Q,
                         const float* K, const float* V, int B, int Hq,
                         int Hkv, int S, int D, float scale, int causal,
                         const int* units, int n_units, int q_begin, int q_end,
                         int tile_q, int tile_k) {
  if (tile_q <= 0) tile_q = 32; /* FlashAttention.h:137 */
  if (tile_k <= 0) tile_k = 64; /* FlashAttention.h:138 */
  if (q_end <= 0 || q_end > S) q_end = S;
  if (q_begin < 0) q_begin = 0;
  const int total_units = units ? n_units : B * Hq;
  const int group = Hq / Hkv;
  const int n_qt = (q_end - q_begin + tile_q - 1) / tile_q;

#pragma omp parallel
  {
    float* acc = (float*)malloc(sizeof(float) * (size_t)tile_q * D);
    float* rmax = (float*)malloc(sizeof(float) * tile_q);
    float* rsum = (float*)malloc(sizeof(float) * tile_q);
    float* sc = (float*)malloc(sizeof(float) * (size_t)tile_q * tile_k);

#pragma omp for collapse(2) schedule(dynamic, 1)
    for (int u = 0; u < total_units; u++) {
      for (int qt = 0; qt < n_qt; qt++) {
        const int unit = units ? units[u] : u;
        const int b = unit / Hq, h = unit % Hq;
        const int hk = h / group;
        const float* q = Q + ((size_t)(b * Hq + h)) * S * D;
        const float* k = K + ((size_t)(b * Hkv + hk)) * S * D;
        const float* v = V + ((size_t)(b * Hkv + hk)) * S * D;
        float* o = out + ((size_t)(b * Hq + h)) * S * D;
        const int tq = q_begin + qt * tile_q;
        const int tq_curr = (tile_q < q_end - tq) ? tile_q : (q_end - tq);

        for (int i = 0; i < tq_curr; i++) {
          rmax[i] = -FLT_MAX;
          rsum[i] = 0.0f;
        }
        memset(acc, 0, sizeof(float) * (size_t)tq_curr * D);

        const int k_stop = causal ? (tq + tq_curr) : S; /* keys < k_stop */
        for (int tk = 0; tk < k_stop; tk += tile_k) {
          int tk_curr = (tile_k < S - tk) ? tile_k : (S - tk);
          /* scores = scale * q k^T (cblas_sgemm alpha=scale, :184-188) */
          for (int i = 0; i < tq_curr; i++) {
            const float* qi = q + (size_t)(tq + i) * D;
            for (int j = 0; j < tk_curr; j++) {
              const float* kj = k + (size_t)(tk + j) * D;
              float s = 0.0f;
              for (int d = 0; d < D; d++) s += qi[d] * kj[d];
              sc[i * tile_k + j] = scale * s;
            }
          }
          for (int i = 0; i < tq_curr; i++) {
            const int qpos = tq + i;
            float* srow = sc + i * tile_k;
            int jn = tk_curr;
            if (causal) {
              int lim = qpos - tk + 1; /* keys tk..qpos allowed */
              if (lim < jn) jn = lim;
              if (jn <= 0) continue; /* whole tile masked for this row */
            }
            float new_max = -FLT_MAX;
            for (int j = 0; j < jn; j++) new_max = srow[j] > new_max ? srow[j] : new_max;
            const float old_max = rmax[i];
            if (old_max > new_max) new_max = old_max;
            if (old_max > -FLT_MAX) {
              const float rescale = expf(old_max - new_max);
              for (int d = 0; d < D; d++) acc[i * D + d] *= rescale;
              rsum[i] *= rescale;
            }
            float row_sum = 0.0f;
            for (int j = 0; j < jn; j++) {
              float e = expf(srow[j] - new_max);
              srow[j] = e;
              row_sum += e;
            }
            for (int j = 0; j < jn; j++) {
              const float w = srow[j];
              const float* vj = v + (size_t)(tk + j) * D;
              for (int d = 0; d < D; d++) acc[i * D + d] += w * vj[d];
            }
            rmax[i] = new_max;
            rsum[i] += row_sum;
          }
        }
        for (int i = 0; i < tq_curr; i++) {
          const float inv = 1.0f / rsum[i];
          for (int d = 0; d < D; d++)
            o[(size_t)(tq + i) * D + d] = acc[i * D + d] * inv;
          if (lse)
            lse[((size_t)(b * Hq + h)) * S + tq + i] = rmax[i] + logf(rsum[i]);
        }
      }
    }
    free(acc);
    free(rmax);
    free(rsum);
    free(sc);
  }
}

/* ------------------------------------------------------------------ */
/* Transformer MLP block (config C4), composed from the reference's     */
/* pieces with the mixed-precision rules of                             */
/* lib/Passes/MixedPrecisionPass.cpp: matmul operands cast to bf16      */
/* (:350-459), fp32 accumulation, reductions (LayerNorm stats) in fp32  */
/* (:288-340), activation and elementwise ops after a matmul stay fp32  */
/* (:490, :632).  The GPU casts the result to bf16 once at the end; the  */
/* oracle returns the fp32 result it is compared against.               */
/*   Xn  = bf16(LayerNorm(X))                  FusedKernels.h:532-600    */
/*   Hd  = bf16(GELU(Xn.W1 + b1))              :378-458, :606-627        */
/*   out = Hd.W2 + b2 + X   (fp32)             residual: extension       */
/* X holds bf16 values (as float).  rows selects which token rows are    */
/* computed (NULL = all T); out is [n_rows, d].                          */
/* ------------------------------------------------------------------ */
void orc_mlp_block(float* out, const float* X, const float* gamma,
                   const float* beta, const float* W1, const float* b1,
                   const float* W2, const float* b2, int64_t T, int64_t d,
                   int64_t dff, float eps, const int64_t* rows,
                   int64_t n_rows) {
  if (!rows) n_rows = T;
  float* xs = (float*)malloc(sizeof(float) * n_rows * d);
  float* xn = (float*)malloc(sizeof(float) * n_rows * d);
  float* hd = (float*)malloc(sizeof(float) * n_rows * dff);
  for (int64_t r = 0; r < n_rows; r++) {
    int64_t src = rows ? rows[r] : r;
    memcpy(xs + r * d, X + src * d, sizeof(float) * d);
  }
  orc_layernorm(xn, xs, gamma, beta, n_rows, d, eps, NULL, NULL);
  orc_round_bf16(xn, n_rows * d);
  orc_gemm_bias_act(xn, W1, b1, NULL, hd, n_rows, dff, d, ORC_ACT_GELU);
  orc_round_bf16(hd, n_rows * dff);
  orc_gemm_bias_act(hd, W2, b2, xs, out, n_rows, d, dff, ORC_ACT_NONE);
  free(xs);
  free(xn);
  free(hd);
}

int orc_num_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}
