// The sharded GEMM driven from C++ through the C ABI only (no Python, no
// PyTorch): one process per GPU, rank 0 creates the NCCL id and passes it
// through a file.  Every rank checks that its gathered C equals the
// single-GPU result bit for bit.
//   dist_gemm <rank> <world> <id file>
#include <cuda_runtime.h>

#include <chrono>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>
#include <thread>
#include <vector>

#include "jules_kernels.h"

#define CHECK(x)                                                                   \
  do {                                                                             \
    int rc_ = (x);                                                                 \
    if (rc_) {                                                                     \
      std::fprintf(stderr, "%s failed: %d %s\n", #x, rc_, jules_last_error_string()); \
      return 1;                                                                    \
    }                                                                              \
  } while (0)

static uint16_t bf16_bits(float f) {  // round to nearest even
  uint32_t u;
  std::memcpy(&u, &f, 4);
  u += 0x7fffu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}

int main(int argc, char** argv) {
  if (argc < 4) return 2;
  const int rank = std::atoi(argv[1]), world = std::atoi(argv[2]);
  const std::string idf = argv[3];
  if (cudaSetDevice(rank) != cudaSuccess) return 3;
  unsigned char id[JULES_DIST_ID_BYTES];
  if (rank == 0) {
    CHECK(jules_dist_unique_id(id));
    const std::string tmp = idf + ".tmp";
    FILE* f = std::fopen(tmp.c_str(), "wb");
    std::fwrite(id, 1, sizeof(id), f);
    std::fclose(f);
    std::rename(tmp.c_str(), idf.c_str());
  } else {
    FILE* f = nullptr;
    for (int i = 0; i < 600 && !f; ++i) {
      f = std::fopen(idf.c_str(), "rb");
      if (!f) std::this_thread::sleep_for(std::chrono::milliseconds(100));
    }
    if (!f || std::fread(id, 1, sizeof(id), f) != sizeof(id)) return 4;
    std::fclose(f);
  }
  void* comm = nullptr;
  CHECK(jules_dist_init(&comm, world, rank, id));

  const int64_t M = 2048, N = 1024, K = 512;
  std::vector<uint16_t> hA(M * K), hW(K * N);
  std::vector<float> hb(N);
  uint32_t s = 12345u;  // the same inputs on every rank
  auto rnd = [&] { s = s * 1664525u + 1013904223u; return (float)(s >> 8) / 16777216.0f - 0.5f; };
  for (auto& x : hA) x = bf16_bits(rnd());
  for (auto& x : hW) x = bf16_bits(rnd() / 8.0f);
  for (auto& x : hb) x = 0.02f * rnd();
  void *A, *W, *b, *Cref, *C;
  if (cudaMalloc(&A, M * K * 2) || cudaMalloc(&W, K * N * 2) || cudaMalloc(&b, N * 4) ||
      cudaMalloc(&Cref, M * N * 2))
    return 5;
  cudaMemcpy(A, hA.data(), M * K * 2, cudaMemcpyHostToDevice);
  cudaMemcpy(W, hW.data(), K * N * 2, cudaMemcpyHostToDevice);
  cudaMemcpy(b, hb.data(), N * 4, cudaMemcpyHostToDevice);
  CHECK(jules_dist_alloc_shared(comm, M * N * 2, &C));
  CHECK(jules_gemm_bias_act(A, W, (const float*)b, nullptr, Cref, M, N, K, JULES_ACT_GELU,
                            JULES_DTYPE_BF16, JULES_DTYPE_BF16, nullptr));
  for (int it = 0; it < 3; ++it)
    CHECK(jules_dist_gemm_bias_act(comm, A, W, (const float*)b, nullptr, C, M, N, K, JULES_ACT_GELU,
                                   JULES_DTYPE_BF16, JULES_DTYPE_BF16, nullptr));
  CHECK(jules_device_error(nullptr, 1));
  std::vector<uint16_t> got(M * N), want(M * N);
  cudaMemcpy(got.data(), C, M * N * 2, cudaMemcpyDeviceToHost);
  cudaMemcpy(want.data(), Cref, M * N * 2, cudaMemcpyDeviceToHost);
  CHECK(jules_dist_barrier(comm, nullptr));  // no rank frees C while another still writes it
  CHECK(jules_device_error(nullptr, 1));
  const bool same = std::memcmp(got.data(), want.data(), M * N * 2) == 0;
  CHECK(jules_dist_free_shared(comm, C));
  CHECK(jules_dist_destroy(comm));
  if (!same) {
    std::fprintf(stderr, "rank %d: gathered C differs from the single-GPU result\n", rank);
    return 6;
  }
  std::printf("rank %d: dist_gemm ok\n", rank);
  return 0;
}
