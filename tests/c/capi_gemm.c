/* A C caller of libgemm3_b200.so, as an integration outside Python would be (test support).
 *
 * Builds seeded A [M,K] and B [N,K] in FP32 on the host, copies them to the GPU, quantises both
 * with nvfp4_quantize (global scale 1), runs nvfp4_gemm_run into an FP16 C and, with the same
 * operands, nvfp4_gemm_run_gather into columns [64, 64 + N) of a wider buffer. The host then
 * decodes the packed codes and linear scales the library wrote, forms the FP64 product and
 * requires a relative Frobenius error below 1e-3 for C, and the gathered block to equal C bit
 * for bit. Exit status 0 on success.
 *
 * Usage: capi_gemm M N K   (N and K multiples of 64). Link: -lgemm3_b200 -lcudart. */
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "nvfp4_gemm.h"

#define CHECK_CUDA(x)                                                     \
  do {                                                                    \
    cudaError_t e_ = (x);                                                 \
    if (e_ != cudaSuccess) {                                              \
      fprintf(stderr, "%s:%d %s\n", __FILE__, __LINE__, cudaGetErrorString(e_)); \
      return 2;                                                           \
    }                                                                     \
  } while (0)
#define CHECK_G3(x)                                                       \
  do {                                                                    \
    int r_ = (x);                                                         \
    if (r_ != NVFP4_OK) {                                                 \
      fprintf(stderr, "%s:%d %s\n", __FILE__, __LINE__, nvfp4_strerror(r_)); \
      return 3;                                                           \
    }                                                                     \
  } while (0)

static uint64_t rng = 0x9E3779B97F4A7C15ull;
static double next_normal(void) { /* Box-Muller on a 64-bit LCG */
  rng = rng * 6364136223846793005ull + 1442695040888963407ull;
  double u1 = ((rng >> 11) + 1.0) / 9007199254740993.0;
  rng = rng * 6364136223846793005ull + 1442695040888963407ull;
  double u2 = (rng >> 11) / 9007199254740992.0;
  return sqrt(-2.0 * log(u1)) * cos(6.283185307179586 * u2);
}

static double e4m3_value(uint8_t b) { /* UE4M3 as written by the quantiser (sign bit clear) */
  int e = (b >> 3) & 15, m = b & 7;
  if (e == 15 && m == 7) return NAN;
  return e == 0 ? ldexp(m / 8.0, -6) : ldexp(1.0 + m / 8.0, e - 7);
}

static const double kE2M1[8] = {0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0};

/* dequantised [rows, k] from packed codes (low nibble first) and linear scales [rows, k/16] */
static void dequant(const uint8_t* q, const uint8_t* sf, int rows, int k, double* out) {
  for (int r = 0; r < rows; ++r)
    for (int c = 0; c < k; ++c) {
      uint8_t byte = q[(size_t)r * (k / 2) + c / 2];
      uint8_t code = (c & 1) ? (byte >> 4) : (byte & 15);
      double v = kE2M1[code & 7] * ((code & 8) ? -1.0 : 1.0);
      out[(size_t)r * k + c] = v * e4m3_value(sf[(size_t)r * (k / 16) + c / 16]);
    }
}

static double half_to_double(uint16_t h) {
  int s = h >> 15, e = (h >> 10) & 31, m = h & 1023;
  double v = e == 0 ? ldexp(m, -24) : ldexp(1024 + m, e - 25);
  return s ? -v : v;
}

int main(int argc, char** argv) {
  if (argc != 4) return 1;
  const int M = atoi(argv[1]), N = atoi(argv[2]), K = atoi(argv[3]);
  const size_t sf_a = (size_t)((M + 127) / 128) * 128 * (K / 64) * 4, sf_b = (size_t)((N + 127) / 128) * 128 * (K / 64) * 4;
  float* ha = malloc(sizeof(float) * M * K);
  float* hb = malloc(sizeof(float) * N * K);
  for (size_t i = 0; i < (size_t)M * K; ++i) ha[i] = (float)next_normal();
  for (size_t i = 0; i < (size_t)N * K; ++i) hb[i] = (float)next_normal();

  float *da, *db, *dalpha;
  uint8_t *qa, *qb, *sa, *sb, *la, *lb;
  uint16_t *dc, *dwide;
  const int col0 = 64, ldc = N + 128;
  CHECK_CUDA(cudaMalloc((void**)&da, sizeof(float) * M * K));
  CHECK_CUDA(cudaMalloc((void**)&db, sizeof(float) * N * K));
  CHECK_CUDA(cudaMalloc((void**)&qa, (size_t)M * K / 2));
  CHECK_CUDA(cudaMalloc((void**)&qb, (size_t)N * K / 2));
  CHECK_CUDA(cudaMalloc((void**)&sa, sf_a));
  CHECK_CUDA(cudaMalloc((void**)&sb, sf_b));
  CHECK_CUDA(cudaMalloc((void**)&la, (size_t)M * K / 16));
  CHECK_CUDA(cudaMalloc((void**)&lb, (size_t)N * K / 16));
  CHECK_CUDA(cudaMalloc((void**)&dc, sizeof(uint16_t) * M * N));
  CHECK_CUDA(cudaMalloc((void**)&dwide, sizeof(uint16_t) * M * ldc));
  CHECK_CUDA(cudaMalloc((void**)&dalpha, sizeof(float)));
  const float one = 1.0f;
  CHECK_CUDA(cudaMemcpy(da, ha, sizeof(float) * M * K, cudaMemcpyHostToDevice));
  CHECK_CUDA(cudaMemcpy(db, hb, sizeof(float) * N * K, cudaMemcpyHostToDevice));
  CHECK_CUDA(cudaMemcpy(dalpha, &one, sizeof(float), cudaMemcpyHostToDevice));
  CHECK_CUDA(cudaMemset(dwide, 0, sizeof(uint16_t) * M * ldc));

  cudaStream_t s;
  CHECK_CUDA(cudaStreamCreate(&s));
  CHECK_G3(nvfp4_quantize(da, NVFP4_DTYPE_F32, M, K, 1.0f, NULL, 0, 0, qa, sa, la, NULL, s));
  CHECK_G3(nvfp4_quantize(db, NVFP4_DTYPE_F32, N, K, 1.0f, NULL, 0, 0, qb, sb, lb, NULL, s));
  nvfp4_gemm_config cfg;
  memset(&cfg, 0, sizeof cfg);
  cfg.struct_size = sizeof cfg;
  CHECK_G3(nvfp4_gemm_run(qa, qb, sa, sb, dc, dalpha, M, N, K, NVFP4_DTYPE_F16, &cfg, NULL, s));
  void* dst[1] = {dwide};
  CHECK_G3(nvfp4_gemm_run_gather(qa, qb, sa, sb, dst, 1, ldc, col0, dalpha, M, N, K, NVFP4_DTYPE_F16, &cfg, NULL, s));
  CHECK_CUDA(cudaStreamSynchronize(s));

  uint8_t* hqa = malloc((size_t)M * K / 2);
  uint8_t* hqb = malloc((size_t)N * K / 2);
  uint8_t* hla = malloc((size_t)M * K / 16);
  uint8_t* hlb = malloc((size_t)N * K / 16);
  uint16_t* hc = malloc(sizeof(uint16_t) * M * N);
  uint16_t* hw = malloc(sizeof(uint16_t) * M * ldc);
  CHECK_CUDA(cudaMemcpy(hqa, qa, (size_t)M * K / 2, cudaMemcpyDeviceToHost));
  CHECK_CUDA(cudaMemcpy(hqb, qb, (size_t)N * K / 2, cudaMemcpyDeviceToHost));
  CHECK_CUDA(cudaMemcpy(hla, la, (size_t)M * K / 16, cudaMemcpyDeviceToHost));
  CHECK_CUDA(cudaMemcpy(hlb, lb, (size_t)N * K / 16, cudaMemcpyDeviceToHost));
  CHECK_CUDA(cudaMemcpy(hc, dc, sizeof(uint16_t) * M * N, cudaMemcpyDeviceToHost));
  CHECK_CUDA(cudaMemcpy(hw, dwide, sizeof(uint16_t) * M * ldc, cudaMemcpyDeviceToHost));

  double* A = malloc(sizeof(double) * M * K);
  double* B = malloc(sizeof(double) * N * K);
  dequant(hqa, hla, M, K, A);
  dequant(hqb, hlb, N, K, B);
  double err2 = 0.0, ref2 = 0.0;
  long gather_mismatch = 0;
  for (int i = 0; i < M; ++i)
    for (int j = 0; j < N; ++j) {
      double acc = 0.0;
      for (int kk = 0; kk < K; ++kk) acc += A[(size_t)i * K + kk] * B[(size_t)j * K + kk];
      double got = half_to_double(hc[(size_t)i * N + j]);
      err2 += (got - acc) * (got - acc);
      ref2 += acc * acc;
      gather_mismatch += hw[(size_t)i * ldc + col0 + j] != hc[(size_t)i * N + j];
    }
  const double rel = sqrt(err2 / ref2);
  printf("capi_gemm %dx%dx%d: rel_err=%.3e gather_mismatch=%ld status=%d\n", M, N, K, rel, gather_mismatch,
         nvfp4_last_cuda_error());
  return (rel < 1e-3 && gather_mismatch == 0) ? 0 : 4;
}
