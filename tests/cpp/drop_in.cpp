// A caller written against the reference's jules::kernel API
// (benchmarks/bench_kernel.cpp style), compiled against this repository's
// headers and linked to libjules_b200.so.  Reads inputs from <dir>/in_*.bin,
// writes results to <dir>/out_*.bin.
#include <cstdio>
#include <cstdlib>
#include <string>
#include <vector>

#include "jules/Kernel/ExecutionArena.h"
#include "jules/Kernel/FlashAttention.h"
#include "jules/Kernel/FusedKernels.h"
#include "jules/Kernel/InterleavedAutodiff.h"
#include "jules/Kernel/TilePlanner.h"

using namespace jules::kernel;

static std::vector<float> load(const std::string& p, size_t n) {
  std::vector<float> v(n);
  FILE* f = std::fopen(p.c_str(), "rb");
  if (!f || std::fread(v.data(), 4, n, f) != n) { std::fprintf(stderr, "read %s\n", p.c_str()); std::exit(2); }
  std::fclose(f);
  return v;
}
static std::vector<int8_t> load_i8(const std::string& p, size_t n) {
  std::vector<int8_t> v(n);
  FILE* f = std::fopen(p.c_str(), "rb");
  if (!f || std::fread(v.data(), 1, n, f) != n) { std::fprintf(stderr, "read %s\n", p.c_str()); std::exit(2); }
  std::fclose(f);
  return v;
}
static void save(const std::string& p, const std::vector<float>& v) {
  FILE* f = std::fopen(p.c_str(), "wb");
  std::fwrite(v.data(), 4, v.size(), f);
  std::fclose(f);
}

int main(int argc, char** argv) {
  const std::string d = argc > 1 ? argv[1] : ".";
  // attention [1,8,512,64]
  const int B = 1, H = 8, S = 512, D = 64, n = B * H * S * D;
  auto Q = load(d + "/in_q.bin", n), K = load(d + "/in_k.bin", n), V = load(d + "/in_v.bin", n);
  std::vector<float> O(n);
  ExecutionArena arena(64UL << 20);
  TilePlanner planner;
  flashAttention(O.data(), Q.data(), K.data(), V.data(), B, H, S, D, arena, planner);
  save(d + "/out_flash.bin", O);
  attention(O.data(), Q.data(), K.data(), V.data(), B, H, S, D, arena, planner);
  save(d + "/out_attention.bin", O);
  standardAttention(O.data(), Q.data(), K.data(), V.data(), B, H, S, D, arena);
  save(d + "/out_standard.bin", O);
  // tiled matmul + GELU [96,200]x[200,136]
  const int M = 96, Kd = 200, N = 136;
  auto A = load(d + "/in_a.bin", M * Kd), W = load(d + "/in_w.bin", Kd * N);
  auto bias = load(d + "/in_bias.bin", N);
  std::vector<float> C(M * N);
  TileConfig cfg = planner.getTileConfig(M, N, Kd);
  tiledMatmulWithActivation(A.data(), W.data(), C.data(), M, N, Kd, cfg, ActivationType::Gelu);
  save(d + "/out_tiled_gelu.bin", C);
  fusedMatmulBiasRelu(A.data(), W.data(), bias.data(), C.data(), M, Kd, N);
  save(d + "/out_bias_relu.bin", C);
  fusedMatmulRelu(A.data(), W.data(), C.data(), M, Kd, N);  // argument order (M, K, N)
  save(d + "/out_relu.bin", C);
  blasMatmul(A.data(), W.data(), C.data(), M, N, Kd);
  save(d + "/out_blas.bin", C);
  // [320,200]x[200,264]: M, N >= 256, the 3xTF32 tensor-core path
  {
    const int Mt = 320, Nt = 264;
    auto At = load(d + "/in_a_tc.bin", Mt * Kd), Wt = load(d + "/in_w_tc.bin", Kd * Nt);
    std::vector<float> Ct(Mt * Nt);
    TileConfig cfg_t = planner.getTileConfig(Mt, Nt, Kd);
    tiledMatmulWithActivation(At.data(), Wt.data(), Ct.data(), Mt, Nt, Kd, cfg_t, ActivationType::Gelu);
    save(d + "/out_tiled_gelu_tc.bin", Ct);
    blasMatmul(At.data(), Wt.data(), Ct.data(), Mt, Nt, Kd);
    save(d + "/out_blas_tc.bin", Ct);
  }
  // layernorm [96,200] and gelu
  std::vector<float> g(Kd, 1.0f), be(Kd, 0.0f), L(M * Kd);
  fusedLayerNorm(L.data(), A.data(), g.data(), be.data(), M, Kd);
  save(d + "/out_layernorm.bin", L);
  fusedGelu(L.data(), A.data(), M * Kd);
  save(d + "/out_gelu.bin", L);
  // MLP forward [96,200] -> 136 -> 24
  auto W2 = load(d + "/in_w2.bin", N * 24), b2 = load(d + "/in_b2.bin", 24);
  MLPParams p{W.data(), bias.data(), W2.data(), b2.data(), M, Kd, N, 24};
  std::vector<float> out(M * 24);
  fusedMLPForward(out.data(), A.data(), p, arena, planner);
  save(d + "/out_mlp.bin", out);
  // softmax and cross-entropy over the [96,136] GEMM output, targets i % 136
  std::vector<float> sm(M * N), grad(M * N);
  fusedSoftmax(sm.data(), C.data(), M, N);
  save(d + "/out_softmax.bin", sm);
  std::vector<int32_t> tgt(M);
  for (int i = 0; i < M; ++i) tgt[i] = (i * 7) % N;
  std::vector<float> loss(1, fusedCrossEntropyLoss(C.data(), tgt.data(), grad.data(), M, N));
  save(d + "/out_xent_grad.bin", grad);
  save(d + "/out_xent_loss.bin", loss);
  // interleavedMLPForwardBackward [96,200] -> 136 -> 24 (ReLU), targets i % 24
  {
    std::vector<int32_t> t24(M);
    for (int i = 0; i < M; ++i) t24[i] = i % 24;
    std::vector<float> o(M * 24), gW1(Kd * N), gb1(N), gW2(N * 24), gb2(24), gX(M * Kd);
    auto r = interleavedMLPForwardBackward(A.data(), W.data(), bias.data(), W2.data(), b2.data(),
                                           t24.data(), o.data(), gW1.data(), gb1.data(),
                                           gW2.data(), gb2.data(), gX.data(), M, Kd, N, 24, arena,
                                           planner);
    save(d + "/out_train_out.bin", o);
    save(d + "/out_train_dW1.bin", gW1);
    save(d + "/out_train_dX.bin", gX);
    save(d + "/out_train_loss.bin", std::vector<float>(1, r.loss));
  }
  // matmulInt8: [96,200]x[200,136] (CUDA cores: N not a multiple of 16) and
  // [256,256]x[256,512] (tcgen05 kind::i8), scales 0.5 / 0.25, with bias
  {
    auto A8 = load_i8(d + "/in_a8.bin", M * Kd), B8 = load_i8(d + "/in_b8.bin", Kd * N);
    std::vector<float> C8(M * N);
    matmulInt8(A8.data(), B8.data(), C8.data(), M, N, Kd, 0.5f, 0.25f, bias.data());
    save(d + "/out_int8_small.bin", C8);
    const int M2 = 256, K2 = 256, N2 = 512;
    auto A9 = load_i8(d + "/in_a9.bin", M2 * K2), B9 = load_i8(d + "/in_b9.bin", K2 * N2);
    auto b9 = load(d + "/in_b9bias.bin", N2);
    std::vector<float> C9(M2 * N2);
    matmulInt8(A9.data(), B9.data(), C9.data(), M2, N2, K2, 0.5f, 0.25f, b9.data());
    save(d + "/out_int8_tc.bin", C9);
    matmulInt8(A9.data(), B9.data(), C9.data(), M2, N2, K2, 1.0f, 1.0f);  // no bias
    save(d + "/out_int8_tc_nobias.bin", C9);
  }
  std::printf("drop-in ok\n");
  return 0;
}
