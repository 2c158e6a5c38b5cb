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

// Accumulator-model sweep (gemm_sweep.cu): up to SWEEP_MAX_CONFIGS models of one block size per launch,
// each compared with a reference output; per-model mismatch counts added into `mismatches` (device).
constexpr int SWEEP_MAX_CONFIGS = 24;
struct SweepModel {
  int stage4_rounding, align3, align4, align_rounding, order;
};
bool sweep_supported_w_reduce(int w_reduce);
cudaError_t launch_gemm_sweep(const uint8_t* A, const uint8_t* B, const uint8_t* SA, const uint8_t* SB, int64_t M,
                              int64_t N, int64_t K, int64_t sa_cols, int64_t sb_cols, const float* alpha, int fmt,
                              int w_reduce, int r3, const SweepModel* models, const int* slots, int n,
                              const void* ref, int ref_dtype, unsigned long long* mismatches, cudaStream_t stream);

// Decode shapes (M < 128) on the integer MMA, 16 output columns per warp (gemm_decode.cu).
bool gemm_decode_supported(int fmt, int64_t M, int64_t N, int64_t K, const void* A, const void* B, const void* SB);
cudaError_t launch_gemm_decode(const uint8_t* A, const uint8_t* B, const uint8_t* SA, const uint8_t* SB, int64_t M,
                               int64_t N, int64_t K, int64_t sa_cols, int64_t sb_cols, const float* alpha,
                               const GemmArgs& args, void* out, cudaStream_t stream);

// One row of A on the CUDA cores, one output column per thread (gemm_decode.cu).
bool gemm_gemv_supported(int fmt, int64_t M, int64_t N, int64_t K, const void* A, const void* B, const void* SB);
cudaError_t launch_gemm_gemv(const uint8_t* A, const uint8_t* B, const uint8_t* SA, const uint8_t* SB, int64_t N,
                             int64_t K, int64_t sa_cols, int64_t sb_cols, const float* alpha, const GemmArgs& args,
                             void* out, cudaStream_t stream);

// Skinny problems (M < 128): block sums split over warps, stage-4 chains per output (gemm_skinny.cu).
bool gemm_skinny_supported(int fmt, int w_reduce, int64_t M);
cudaError_t launch_gemm_skinny(const uint8_t* A, const uint8_t* B, const uint8_t* SA, const uint8_t* SB, int64_t M,
                               int64_t N, int64_t K, int64_t sa_cols, int64_t sb_cols, const float* alpha,
                               const GemmArgs& args, void* out, cudaStream_t stream);

cudaError_t launch_gemm_simt(const uint8_t* A, const uint8_t* B, const uint8_t* SA, const uint8_t* SB,
                             int64_t M, int64_t N, int64_t K, int64_t sa_cols, int64_t sb_cols,
                             const float* alpha, const GemmArgs& args, void* out, cudaStream_t stream);

size_t gemm_tc_workspace_size(int fmt, int64_t M, int64_t N, int64_t K);
size_t gemm_tc_path_offset(int fmt, int64_t M, int64_t N, int64_t K);
// pipeline-wait bound of later tensor-core launches (cycles; <= 0 restores 2^31); returns the old one
long long set_wait_limit(long long cycles);
// test hook: later tensor-core launches withhold the first accumulator-ready signal (gemm_tc.cu)
void set_hold_first_ready(int enable);
// this device's first timed-out wait code since the last call (0 = none), then cleared
cudaError_t take_wait_error(int* code);
bool gemm_tc_supported(int fmt, int w_reduce, int64_t M, int64_t N, int64_t K);
cudaError_t launch_gemm_tc(const uint8_t* A, const uint8_t* B, const uint8_t* SA, const uint8_t* SB,
                           int64_t M, int64_t N, int64_t K, int64_t sa_cols, int64_t sb_cols,
                           const float* alpha, const GemmArgs& args, void* out, void* workspace,
                           cudaStream_t stream);

cudaError_t launch_quant(int sf_vec, const void* x, int dtype, int64_t M, int64_t K,
                         const float* global_scale, uint8_t* q, uint8_t* sf, cudaStream_t stream);

// sets emu_last_error() of the calling thread to `message` and returns s (capi.cu)
int32_t record_failure(int32_t s, const char* message);

// the argument checks of emu_gemm_ws before it looks at the workspace (capi.cu); EMU_OK or the
// status emu_gemm_ws would return, with emu_last_error() set
int32_t check_gemm_call(const uint8_t* a_fp4, const uint8_t* b_fp4, const uint8_t* scale_a, const uint8_t* scale_b,
                        int64_t M, int64_t N, int64_t K, int64_t scale_a_rows, int64_t scale_a_cols,
                        int64_t scale_b_rows, int64_t scale_b_cols, const emu_gemm_params* params, const void* out);

cudaError_t launch_amax(const void* a, int64_t a_numel, const void* b, int64_t b_numel, int dtype, unsigned* amax_a,
                        unsigned* amax_b, cudaStream_t stream);
cudaError_t launch_scales_from_amax(const unsigned* amax_a, const unsigned* amax_b, float* gs_a, float* gs_b,
                                    float* alpha, cudaStream_t stream);
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
