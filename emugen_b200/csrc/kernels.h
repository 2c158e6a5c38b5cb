// Internal launcher declarations shared by the C-ABI layer (capi.cu) and the kernels.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace emu {

// Validated, runtime accumulator parameters passed by value to the GEMM kernels.
struct GemmArgs {
  int format;           // EMU_FMT_*
  int w_reduce;         // groups per stage-3 block
  int stage3_rounding;  // EMU_RZ / EMU_RNE
  int stage4_rounding;
  int out_mode;         // EMU_OUT_*
  // optional comparison of the result with a reference output, fused into the tensor-core epilogue
  const void* cmp_ref = nullptr;          // [M][N], the output's dtype
  emu_compare_stats* cmp_stats = nullptr; // device; initialised by launch_compare_init
  bool write_out = true;                  // false: compare only, `out` is not written
};

// Accumulator model of emu_gemm_model (include/emugen.h emu_accum_model).
struct ModelArgs {
  int align3, align4, align_rounding, order;
};

cudaError_t launch_gemm_model(const uint8_t* A, const uint8_t* B, const uint8_t* SA, const uint8_t* SB, int64_t M,
                              int64_t N, int64_t K, int64_t sa_cols, int64_t sb_cols, const float* alpha,
                              const GemmArgs& args, const ModelArgs& ma, void* out, cudaStream_t stream);

// Skinny problems (M < 128): block sums split over warps, stage-4 chains per output (gemm_skinny.cu).
bool gemm_skinny_supported(int fmt, int w_reduce, int64_t M);
cudaError_t launch_gemm_skinny(const uint8_t* A, const uint8_t* B, const uint8_t* SA, const uint8_t* SB, int64_t M,
                               int64_t N, int64_t K, int64_t sa_cols, int64_t sb_cols, const float* alpha,
                               const GemmArgs& args, void* out, cudaStream_t stream);

cudaError_t launch_gemm_simt(const uint8_t* A, const uint8_t* B, const uint8_t* SA, const uint8_t* SB,
                             int64_t M, int64_t N, int64_t K, int64_t sa_cols, int64_t sb_cols,
                             const float* alpha, const GemmArgs& args, void* out, cudaStream_t stream);

size_t gemm_tc_workspace_size(int fmt, int64_t M, int64_t N, int64_t K);
bool gemm_tc_supported(int fmt, int w_reduce, int64_t M, int64_t N, int64_t K);
cudaError_t launch_gemm_tc(const uint8_t* A, const uint8_t* B, const uint8_t* SA, const uint8_t* SB,
                           int64_t M, int64_t N, int64_t K, int64_t sa_cols, int64_t sb_cols,
                           const float* alpha, const GemmArgs& args, void* out, void* workspace,
                           cudaStream_t stream);

cudaError_t launch_quant(int sf_vec, const void* x, int dtype, int64_t M, int64_t K,
                         const float* global_scale, uint8_t* q, uint8_t* sf, cudaStream_t stream);

// sets emu_last_error() of the calling thread to `message` and returns s (capi.cu)
int32_t record_failure(int32_t s, const char* message);

cudaError_t launch_global_scales(const void* a, int64_t a_numel, const void* b, int64_t b_numel,
                                 int dtype, float* gs_a, float* gs_b, float* alpha,
                                 cudaStream_t stream);

cudaError_t launch_compare_init(emu_compare_stats* stats, int64_t n, cudaStream_t stream);
cudaError_t launch_compare_fini(emu_compare_stats* stats, cudaStream_t stream);
cudaError_t launch_compare(const void* ref, const void* out, int dtype, int64_t n, emu_compare_stats* stats,
                           cudaStream_t stream);
cudaError_t launch_dequant(const uint8_t* q, const uint8_t* sf, int64_t rows, int64_t K, int64_t sf_cols, int fmt,
                           const float* global_scale, float* out, cudaStream_t stream);

}  // namespace emu
