/* A plain C host of libemugen (include/emugen.h only, no torch): quantise two fp16 matrices, run the
 * emulated NVFP4 GEMM through emu_gemm and emu_gemm_ws, and check the two agree bit for bit and
 * that emu_compare sees no mismatch.  Built and run by tests/test_c_abi.py. */
#include <cuda_runtime.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "emugen.h"

#define CHECK(x)                                                                            \
  do {                                                                                      \
    emu_status s_ = (x);                                                                    \
    if (s_ != EMU_OK) {                                                                     \
      fprintf(stderr, "%s failed: %s (%s)\n", #x, emu_status_string(s_), emu_last_error()); \
      return 1;                                                                             \
    }                                                                                       \
  } while (0)
#define CUDA(x)                                                                   \
  do {                                                                            \
    cudaError_t e_ = (x);                                                         \
    if (e_ != cudaSuccess) {                                                      \
      fprintf(stderr, "%s failed: %s\n", #x, cudaGetErrorString(e_));             \
      return 1;                                                                   \
    }                                                                             \
  } while (0)

static uint16_t f32_to_f16_bits(float f) { /* small normal values only: enough for this test */
  uint32_t u;
  memcpy(&u, &f, 4);
  uint32_t sign = (u >> 16) & 0x8000u, e = (u >> 23) & 0xFFu, m = u & 0x7FFFFFu;
  if (e == 0) return (uint16_t)sign;
  int ne = (int)e - 127 + 15;
  uint32_t mm = m >> 13, rem = m & 0x1FFFu;
  if (rem > 0x1000u || (rem == 0x1000u && (mm & 1u))) ++mm;
  if (mm == 0x400u) { mm = 0; ++ne; }
  return (uint16_t)(sign | ((uint32_t)ne << 10) | mm);
}

int main(void) {
  if (emu_abi_version() != EMU_ABI_VERSION) { fprintf(stderr, "ABI version mismatch\n"); return 1; }
  const int64_t M = 256, N = 128, K = 512, G = K / 16;
  const int64_t sf_rows_a = 256, sf_rows_b = 128, sf_cols = (G + 3) / 4 * 4;
  uint16_t* ha = (uint16_t*)malloc(sizeof(uint16_t) * M * K);
  uint16_t* hb = (uint16_t*)malloc(sizeof(uint16_t) * N * K);
  uint32_t state = 12345u;
  for (int64_t i = 0; i < M * K; ++i) { state = state * 1664525u + 1013904223u; ha[i] = f32_to_f16_bits(((int)(state >> 9) % 2001 - 1000) / 250.0f); }
  for (int64_t i = 0; i < N * K; ++i) { state = state * 1664525u + 1013904223u; hb[i] = f32_to_f16_bits(((int)(state >> 9) % 2001 - 1000) / 250.0f); }
  void *da, *db, *qa, *qb, *sa, *sb, *out1, *out2, *ws, *stats;
  float *gsa, *gsb, *alpha;
  CUDA(cudaMalloc(&da, 2 * M * K)); CUDA(cudaMalloc(&db, 2 * N * K));
  CUDA(cudaMalloc(&qa, M * K / 2)); CUDA(cudaMalloc(&qb, N * K / 2));
  CUDA(cudaMalloc(&sa, sf_rows_a * sf_cols)); CUDA(cudaMalloc(&sb, sf_rows_b * sf_cols));
  CUDA(cudaMalloc((void**)&gsa, 4)); CUDA(cudaMalloc((void**)&gsb, 4)); CUDA(cudaMalloc((void**)&alpha, 4));
  CUDA(cudaMalloc(&out1, 2 * M * N)); CUDA(cudaMalloc(&out2, 2 * M * N));
  CUDA(cudaMalloc(&stats, sizeof(emu_compare_stats)));
  CUDA(cudaMemcpy(da, ha, 2 * M * K, cudaMemcpyHostToDevice));
  CUDA(cudaMemcpy(db, hb, 2 * N * K, cudaMemcpyHostToDevice));
  CHECK(emu_nvfp4_global_scales(da, M * K, db, N * K, EMU_DTYPE_F16, gsa, gsb, alpha, NULL));
  CHECK(emu_quant_nvfp4(da, EMU_DTYPE_F16, M, K, gsa, (uint8_t*)qa, (uint8_t*)sa, NULL));
  CHECK(emu_quant_nvfp4(db, EMU_DTYPE_F16, N, K, gsb, (uint8_t*)qb, (uint8_t*)sb, NULL));
  emu_gemm_params p = {EMU_FMT_NVFP4, 16, 4, EMU_RZ, EMU_RZ, EMU_OUT_F16};
  CHECK(emu_gemm((const uint8_t*)qa, (const uint8_t*)qb, (const uint8_t*)sa, (const uint8_t*)sb, M, N, K, sf_rows_a,
                 sf_cols, sf_rows_b, sf_cols, alpha, &p, out1, NULL));
  size_t need = emu_gemm_tc_workspace_size(M, N, K, &p);   /* the tensor-core kernel at this small shape */
  if (need == 0) { fprintf(stderr, "expected the tensor-core path at this shape\n"); return 1; }
  CUDA(cudaMalloc(&ws, need + 1024));
  void* ws_al = (void*)(((uintptr_t)ws + 1023) & ~(uintptr_t)1023);
  CHECK(emu_gemm_ws((const uint8_t*)qa, (const uint8_t*)qb, (const uint8_t*)sa, (const uint8_t*)sb, M, N, K, sf_rows_a,
                    sf_cols, sf_rows_b, sf_cols, alpha, &p, out2, ws_al, need, NULL));
  CHECK(emu_compare(out1, out2, EMU_DTYPE_F16, M * N, (emu_compare_stats*)stats, NULL));
  emu_compare_stats hs;
  CUDA(cudaMemcpy(&hs, stats, sizeof(hs), cudaMemcpyDeviceToHost));
  uint16_t* h1 = (uint16_t*)malloc(2 * M * N);
  uint16_t* h2 = (uint16_t*)malloc(2 * M * N);
  CUDA(cudaMemcpy(h1, out1, 2 * M * N, cudaMemcpyDeviceToHost));
  CUDA(cudaMemcpy(h2, out2, 2 * M * N, cudaMemcpyDeviceToHost));
  if (memcmp(h1, h2, 2 * M * N) != 0 || hs.mismatches != 0 || hs.first_index != -1) {
    fprintf(stderr, "mismatch: %lld elements, first %lld\n", (long long)hs.mismatches, (long long)hs.first_index);
    return 1;
  }
  /* an argument the reference rejects comes back as a status with its message */
  emu_gemm_params bad = p;
  bad.group_size = 32;
  emu_status s = emu_gemm((const uint8_t*)qa, (const uint8_t*)qb, (const uint8_t*)sa, (const uint8_t*)sb, M, N, K,
                          sf_rows_a, sf_cols, sf_rows_b, sf_cols, alpha, &bad, out1, NULL);
  if (s != EMU_ERR_GROUP_SIZE || strcmp(emu_last_error(), "only NVFP4 group_size=16 is supported") != 0) {
    fprintf(stderr, "unexpected status %d / message '%s'\n", s, emu_last_error());
    return 1;
  }
  printf("c abi ok: %lld outputs equal\n", (long long)(M * N));
  return 0;
}
