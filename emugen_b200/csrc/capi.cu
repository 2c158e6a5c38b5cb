// extern "C" entry points of libemugen.so (declared in include/emugen.h): argument validation with
// the reference's error messages, then dispatch to the kernels.  No allocation, no host sync.
#include <cuda_runtime.h>
#include <stdarg.h>
#include <stdint.h>
#include <stdio.h>

#include <string>

#include "../../include/emugen.h"
#include "kernels.h"

namespace {

thread_local std::string g_last_error;

emu_status fail(emu_status s, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return s;
}

emu_status ok() {
  g_last_error.clear();
  return EMU_OK;
}

emu_status cuda_status(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return ok();
  return fail(EMU_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

bool aligned(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0; }

}  // namespace

emu_status emu::record_failure(emu_status s, const char* message) {
  g_last_error = message;
  return s;
}

extern "C" {

int32_t emu_abi_version(void) { return EMU_ABI_VERSION; }

const char* emu_last_error(void) { return g_last_error.c_str(); }

const char* emu_status_string(emu_status s) {
  switch (s) {
    case EMU_OK: return "EMU_OK";
    case EMU_ERR_INVALID_ARGUMENT: return "EMU_ERR_INVALID_ARGUMENT";
    case EMU_ERR_K_MISMATCH: return "EMU_ERR_K_MISMATCH";
    case EMU_ERR_K_GROUP: return "EMU_ERR_K_GROUP";
    case EMU_ERR_W_REDUCE: return "EMU_ERR_W_REDUCE";
    case EMU_ERR_GROUP_SIZE: return "EMU_ERR_GROUP_SIZE";
    case EMU_ERR_SCALE_SHAPE: return "EMU_ERR_SCALE_SHAPE";
    case EMU_ERR_SCALE_TOO_SMALL: return "EMU_ERR_SCALE_TOO_SMALL";
    case EMU_ERR_UNSUPPORTED: return "EMU_ERR_UNSUPPORTED";
    case EMU_ERR_CUDA: return "EMU_ERR_CUDA";
    case EMU_ERR_TIMEOUT: return "EMU_ERR_TIMEOUT";
    default: return "EMU_ERR_UNKNOWN";
  }
}

static emu_status validate_gemm(int64_t M, int64_t N, int64_t K, int64_t scale_a_rows, int64_t scale_a_cols,
                                int64_t scale_b_rows, int64_t scale_b_cols, const emu_gemm_params* params) {
  if (!params) return fail(EMU_ERR_INVALID_ARGUMENT, "params must not be NULL");
  const emu_gemm_params p = *params;
  if (M < 0 || N < 0 || K < 0) return fail(EMU_ERR_INVALID_ARGUMENT, "negative size");
  if (p.format != EMU_FMT_NVFP4 && p.format != EMU_FMT_MXFP4)
    return fail(EMU_ERR_INVALID_ARGUMENT, "unknown format %d", p.format);
  // reference order of checks: nvfp_emulation.cpp:99-106, mxfp_emulation.cpp:107-118
  if (p.format == EMU_FMT_MXFP4 && p.group_size != 32)
    return fail(EMU_ERR_GROUP_SIZE, "only MXFP4 group_size=32 is supported");
  if (p.format == EMU_FMT_NVFP4 && p.group_size != 16)
    return fail(EMU_ERR_GROUP_SIZE, "only NVFP4 group_size=16 is supported");
  if (K % p.group_size != 0)
    return fail(EMU_ERR_K_GROUP, p.format == EMU_FMT_NVFP4 ? "K must be multiple of 16"
                                                           : "K must be divisible by group_size");
  const int64_t G = K / p.group_size;
  if (p.w_reduce < 1 || p.w_reduce > 64)
    return fail(EMU_ERR_UNSUPPORTED, "w_reduce must be in [1, 64], got %d", p.w_reduce);
  if (G % p.w_reduce != 0) {
    if (p.format == EMU_FMT_NVFP4 && p.w_reduce == 4)
      return fail(EMU_ERR_W_REDUCE, "G = K/16 must be multiple of 4");
    if (p.format == EMU_FMT_MXFP4 && p.w_reduce == 2)
      return fail(EMU_ERR_W_REDUCE,
                  "MXFP emulation (w_reduce=2) requires K/(2*group_size) to be integral (e.g. K divisible by 64)");
    return fail(EMU_ERR_W_REDUCE, "G=K/group_size (%lld) must be divisible by w_reduce (%d)", (long long)G,
                p.w_reduce);
  }
  if (K == 0) return fail(EMU_ERR_INVALID_ARGUMENT, "K must be positive");
  if (scale_a_rows % 128 != 0 || scale_a_cols % 4 != 0 || scale_b_rows % 128 != 0 || scale_b_cols % 4 != 0)
    return fail(EMU_ERR_SCALE_SHAPE, "swizzled scale shape must be divisible by 128 and 4");
  if (scale_a_rows < M || scale_b_rows < N)
    return fail(EMU_ERR_SCALE_TOO_SMALL, "scale rows (%lld, %lld) fewer than M, N (%lld, %lld)",
                (long long)scale_a_rows, (long long)scale_b_rows, (long long)M, (long long)N);
  if (scale_a_cols < G || scale_b_cols < G)
    return fail(EMU_ERR_SCALE_TOO_SMALL, "scale columns (%lld, %lld) fewer than K/group_size (%lld)",
                (long long)scale_a_cols, (long long)scale_b_cols, (long long)G);
  if ((p.stage3_rounding != EMU_RZ && p.stage3_rounding != EMU_RNE) ||
      (p.stage4_rounding != EMU_RZ && p.stage4_rounding != EMU_RNE))
    return fail(EMU_ERR_INVALID_ARGUMENT, "rounding must be EMU_RZ (0) or EMU_RNE (1)");
  if (p.out_mode < EMU_OUT_F16 || p.out_mode > EMU_OUT_F32)
    return fail(EMU_ERR_INVALID_ARGUMENT, "unknown out_mode %d", p.out_mode);
  if ((N + 63) / 64 > 65535) return fail(EMU_ERR_UNSUPPORTED, "N too large for the tensor-core tile index (max 4194240)");
  return EMU_OK;
}

static bool tc_path(const emu_gemm_params& p, int64_t M, int64_t N, int64_t K) {
  return emu::gemm_tc_supported(p.format, p.w_reduce, M, N, K);
}

// Problems below these sizes finish sooner on the CUDA-core kernels than through the tensor-core
// kernel's pre-pass and two launches (B200: NVFP4 128x128x256 30 us vs 95 us, 512x512x1024 101 vs
// 109 us; MXFP4 1024^3 76 vs 133 us, 1024x1024x2048 148 vs 144 us).
static bool tc_preferred(const emu_gemm_params& p, int64_t M, int64_t N, int64_t K) {
  const double macs = (double)M * (double)N * (double)K;
  return tc_path(p, M, N, K) && macs >= (p.format == EMU_FMT_NVFP4 ? 0x1p27 : 0x1p30);
}

static size_t workspace_for(int64_t M, int64_t N, int64_t K, const emu_gemm_params* params, bool prefer) {
  if (!params || M <= 0 || N <= 0 || K <= 0) return 0;
  if (params->group_size <= 0 || K % params->group_size != 0) return 0;
  if (!(prefer ? tc_preferred(*params, M, N, K) : tc_path(*params, M, N, K))) return 0;
  return emu::gemm_tc_workspace_size(params->format, M, N, K);
}

size_t emu_gemm_workspace_size(int64_t M, int64_t N, int64_t K, const emu_gemm_params* params) {
  return workspace_for(M, N, K, params, true);
}

size_t emu_gemm_tc_workspace_size(int64_t M, int64_t N, int64_t K, const emu_gemm_params* params) {
  return workspace_for(M, N, K, params, false);
}

}  // extern "C"

// Every check emu_gemm_ws makes before it looks at the workspace: sizes, parameters, scale shapes
// (validate_gemm), then the tensor pointers.  Sets emu_last_error() on failure.
emu_status emu::check_gemm_call(const uint8_t* a_fp4, const uint8_t* b_fp4, const uint8_t* scale_a,
                                const uint8_t* scale_b, int64_t M, int64_t N, int64_t K, int64_t scale_a_rows,
                                int64_t scale_a_cols, int64_t scale_b_rows, int64_t scale_b_cols,
                                const emu_gemm_params* params, const void* out) {
  emu_status st = validate_gemm(M, N, K, scale_a_rows, scale_a_cols, scale_b_rows, scale_b_cols, params);
  if (st != EMU_OK) return st;
  if (M == 0 || N == 0) return ok();
  if (!a_fp4 || !b_fp4 || !scale_a || !scale_b || !out)
    return fail(EMU_ERR_INVALID_ARGUMENT, "tensor pointers must not be NULL");
  if (!aligned(a_fp4, 16) || !aligned(b_fp4, 16))
    return fail(EMU_ERR_INVALID_ARGUMENT, "a_fp4 / b_fp4 must be 16-byte aligned");
  return ok();
}

extern "C" {

size_t emu_gemm_tc_path_offset(int64_t M, int64_t N, int64_t K, const emu_gemm_params* params) {
  if (workspace_for(M, N, K, params, false) == 0) return (size_t)-1;
  return emu::gemm_tc_path_offset(params->format, M, N, K);
}

emu_status emu_gemm_ws(const uint8_t* a_fp4, const uint8_t* b_fp4, const uint8_t* scale_a, const uint8_t* scale_b,
                       int64_t M, int64_t N, int64_t K, int64_t scale_a_rows, int64_t scale_a_cols,
                       int64_t scale_b_rows, int64_t scale_b_cols, const float* alpha, const emu_gemm_params* params,
                       void* out, void* workspace, size_t workspace_bytes, void* stream) {
  emu_status st = emu::check_gemm_call(a_fp4, b_fp4, scale_a, scale_b, M, N, K, scale_a_rows, scale_a_cols,
                                       scale_b_rows, scale_b_cols, params, out);
  if (st != EMU_OK) return st;
  if (M == 0 || N == 0) return ok();
  const emu_gemm_params p = *params;
  emu::GemmArgs args{p.format, p.w_reduce, p.stage3_rounding, p.stage4_rounding, p.out_mode};
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (workspace && tc_path(p, M, N, K)) {
    if (!aligned(workspace, 1024))
      return fail(EMU_ERR_INVALID_ARGUMENT, "workspace must be 1024-byte aligned");
    if (workspace_bytes < emu::gemm_tc_workspace_size(p.format, M, N, K))
      return fail(EMU_ERR_INVALID_ARGUMENT, "workspace too small: %zu < %zu bytes", workspace_bytes,
                  emu::gemm_tc_workspace_size(p.format, M, N, K));
    return cuda_status(emu::launch_gemm_tc(a_fp4, b_fp4, scale_a, scale_b, M, N, K, scale_a_cols, scale_b_cols, alpha,
                                           args, out, workspace, s),
                       "emu_gemm tensor-core launch");
  }
  if (emu::gemm_skinny_supported(p.format, p.w_reduce, M))
    return cuda_status(emu::launch_gemm_skinny(a_fp4, b_fp4, scale_a, scale_b, M, N, K, scale_a_cols, scale_b_cols,
                                               alpha, args, out, s),
                       "emu_gemm skinny launch");
  return cuda_status(emu::launch_gemm_simt(a_fp4, b_fp4, scale_a, scale_b, M, N, K, scale_a_cols, scale_b_cols, alpha,
                                           args, out, s),
                     "emu_gemm launch");
}

emu_status emu_gemm(const uint8_t* a_fp4, const uint8_t* b_fp4, const uint8_t* scale_a,
                    const uint8_t* scale_b, int64_t M, int64_t N, int64_t K, int64_t scale_a_rows,
                    int64_t scale_a_cols, int64_t scale_b_rows, int64_t scale_b_cols,
                    const float* alpha, const emu_gemm_params* params, void* out, void* stream) {
  return emu_gemm_ws(a_fp4, b_fp4, scale_a, scale_b, M, N, K, scale_a_rows, scale_a_cols, scale_b_rows, scale_b_cols,
                     alpha, params, out, nullptr, 0, stream);
}

emu_status emu_nvfp4_global_scales(const void* a, int64_t a_numel, const void* b, int64_t b_numel,
                                   int32_t dtype, float* gs_a, float* gs_b, float* alpha, void* stream) {
  if (!a || !b || !gs_a || !gs_b) return fail(EMU_ERR_INVALID_ARGUMENT, "pointers must not be NULL");
  if (a_numel < 0 || b_numel < 0) return fail(EMU_ERR_INVALID_ARGUMENT, "negative size");
  if (dtype != EMU_DTYPE_F16 && dtype != EMU_DTYPE_BF16)
    return fail(EMU_ERR_INVALID_ARGUMENT, "dtype must be EMU_DTYPE_F16 or EMU_DTYPE_BF16");
  cudaError_t e = emu::launch_global_scales(a, a_numel, b, b_numel, dtype, gs_a, gs_b, alpha,
                                            static_cast<cudaStream_t>(stream));
  return cuda_status(e, "emu_nvfp4_global_scales launch");
}

emu_status emu_nvfp4_amax(const void* a, int64_t a_numel, const void* b, int64_t b_numel, int32_t dtype,
                          uint32_t* amax_a, uint32_t* amax_b, void* stream) {
  if (!a || !b || !amax_a || !amax_b) return fail(EMU_ERR_INVALID_ARGUMENT, "pointers must not be NULL");
  if (a_numel < 0 || b_numel < 0) return fail(EMU_ERR_INVALID_ARGUMENT, "negative size");
  if (dtype != EMU_DTYPE_F16 && dtype != EMU_DTYPE_BF16)
    return fail(EMU_ERR_INVALID_ARGUMENT, "dtype must be EMU_DTYPE_F16 or EMU_DTYPE_BF16");
  if (!aligned(amax_a, 4) || !aligned(amax_b, 4)) return fail(EMU_ERR_INVALID_ARGUMENT, "amax words must be 4-byte aligned");
  return cuda_status(emu::launch_amax(a, a_numel, b, b_numel, dtype, amax_a, amax_b, static_cast<cudaStream_t>(stream)),
                     "emu_nvfp4_amax launch");
}

emu_status emu_nvfp4_scales_from_amax(const uint32_t* amax_a, const uint32_t* amax_b, float* gs_a, float* gs_b,
                                      float* alpha, void* stream) {
  if (!amax_a || !amax_b || !gs_a || !gs_b) return fail(EMU_ERR_INVALID_ARGUMENT, "pointers must not be NULL");
  return cuda_status(emu::launch_scales_from_amax(amax_a, amax_b, gs_a, gs_b, alpha, static_cast<cudaStream_t>(stream)),
                     "emu_nvfp4_scales_from_amax launch");
}

static emu_status quant_common(int sf_vec, const void* x, int32_t dtype, int64_t M, int64_t K,
                               const float* gs, uint8_t* q, uint8_t* sf, void* stream) {
  if (M < 0 || K < 0) return fail(EMU_ERR_INVALID_ARGUMENT, "negative size");
  if (dtype != EMU_DTYPE_F16 && dtype != EMU_DTYPE_BF16)
    return fail(EMU_ERR_INVALID_ARGUMENT, "dtype must be EMU_DTYPE_F16 or EMU_DTYPE_BF16");
  if (K % sf_vec != 0) return fail(EMU_ERR_K_GROUP, "K must be a multiple of %d", sf_vec);
  if (M == 0 || K == 0) return ok();
  if (!x || !q || !sf) return fail(EMU_ERR_INVALID_ARGUMENT, "pointers must not be NULL");
  if (!aligned(x, 16) || !aligned(q, 8)) return fail(EMU_ERR_INVALID_ARGUMENT, "x must be 16-byte and q 8-byte aligned");
  cudaError_t e = emu::launch_quant(sf_vec, x, dtype, M, K, gs, q, sf, static_cast<cudaStream_t>(stream));
  return cuda_status(e, "quantize launch");
}

emu_status emu_quant_nvfp4(const void* x, int32_t dtype, int64_t M, int64_t K, const float* global_scale,
                           uint8_t* q, uint8_t* sf, void* stream) {
  if (!global_scale) return fail(EMU_ERR_INVALID_ARGUMENT, "global_scale must not be NULL");
  return quant_common(16, x, dtype, M, K, global_scale, q, sf, stream);
}

emu_status emu_quant_mxfp4(const void* x, int32_t dtype, int64_t M, int64_t K, uint8_t* q, uint8_t* sf,
                           void* stream) {
  return quant_common(32, x, dtype, M, K, nullptr, q, sf, stream);
}

emu_status emu_compare(const void* ref, const void* out, int32_t dtype, int64_t n, emu_compare_stats* stats,
                       void* stream) {
  if (n < 0) return fail(EMU_ERR_INVALID_ARGUMENT, "negative size");
  if (!stats || (n > 0 && (!ref || !out))) return fail(EMU_ERR_INVALID_ARGUMENT, "pointers must not be NULL");
  if (dtype != EMU_DTYPE_F16 && dtype != EMU_DTYPE_BF16 && dtype != EMU_DTYPE_F32)
    return fail(EMU_ERR_INVALID_ARGUMENT, "dtype must be EMU_DTYPE_F16, EMU_DTYPE_BF16 or EMU_DTYPE_F32");
  if (!aligned(stats, 8)) return fail(EMU_ERR_INVALID_ARGUMENT, "stats must be 8-byte aligned");
  return cuda_status(emu::launch_compare(ref, out, dtype, n, stats, static_cast<cudaStream_t>(stream)),
                     "emu_compare launch");
}

emu_status emu_gemm_model(const uint8_t* a_fp4, const uint8_t* b_fp4, const uint8_t* scale_a, const uint8_t* scale_b,
                          int64_t M, int64_t N, int64_t K, int64_t scale_a_rows, int64_t scale_a_cols,
                          int64_t scale_b_rows, int64_t scale_b_cols, const float* alpha,
                          const emu_gemm_params* params, const emu_accum_model* model, void* out, void* stream) {
  if (!model) return fail(EMU_ERR_INVALID_ARGUMENT, "model must not be NULL");
  const emu_accum_model md = *model;
  if (md.align3 < 0 || md.align3 > 46) return fail(EMU_ERR_INVALID_ARGUMENT, "align3 must be in [0, 46], got %d", md.align3);
  if (md.align4 < 0 || md.align4 > 52) return fail(EMU_ERR_INVALID_ARGUMENT, "align4 must be in [0, 52], got %d", md.align4);
  if (md.align_rounding != EMU_RZ && md.align_rounding != EMU_RNE)
    return fail(EMU_ERR_INVALID_ARGUMENT, "align_rounding must be EMU_RZ (0) or EMU_RNE (1)");
  if (md.order < 0 || md.order > 2) return fail(EMU_ERR_INVALID_ARGUMENT, "order must be 0, 1 or 2, got %d", md.order);
  if (md.align3 == 0 && md.align4 == 0 && md.order == 0)
    return emu_gemm(a_fp4, b_fp4, scale_a, scale_b, M, N, K, scale_a_rows, scale_a_cols, scale_b_rows, scale_b_cols,
                    alpha, params, out, stream);
  emu_status st = validate_gemm(M, N, K, scale_a_rows, scale_a_cols, scale_b_rows, scale_b_cols, params);
  if (st != EMU_OK) return st;
  if (params->w_reduce > 16) return fail(EMU_ERR_UNSUPPORTED, "a nonzero accumulator model needs w_reduce <= 16");
  if (M == 0 || N == 0) return ok();
  if (!a_fp4 || !b_fp4 || !scale_a || !scale_b || !out)
    return fail(EMU_ERR_INVALID_ARGUMENT, "tensor pointers must not be NULL");
  if (!aligned(a_fp4, 16) || !aligned(b_fp4, 16))
    return fail(EMU_ERR_INVALID_ARGUMENT, "a_fp4 / b_fp4 must be 16-byte aligned");
  const emu_gemm_params p = *params;
  emu::GemmArgs args{p.format, p.w_reduce, p.stage3_rounding, p.stage4_rounding, p.out_mode};
  emu::ModelArgs ma{md.align3, md.align4, md.align_rounding, md.order};
  return cuda_status(emu::launch_gemm_model(a_fp4, b_fp4, scale_a, scale_b, M, N, K, scale_a_cols, scale_b_cols,
                                            alpha, args, ma, out, static_cast<cudaStream_t>(stream)),
                     "emu_gemm_model launch");
}

emu_status emu_gemm_sweep(const uint8_t* a_fp4, const uint8_t* b_fp4, const uint8_t* scale_a, const uint8_t* scale_b,
                          int64_t M, int64_t N, int64_t K, int64_t scale_a_rows, int64_t scale_a_cols,
                          int64_t scale_b_rows, int64_t scale_b_cols, const float* alpha, int32_t format,
                          int32_t stage3_rounding, const emu_sweep_model* models, int32_t n_models, const void* ref,
                          int32_t ref_dtype, int64_t* mismatches, void* stream) {
  if (format != EMU_FMT_NVFP4 && format != EMU_FMT_MXFP4)
    return fail(EMU_ERR_INVALID_ARGUMENT, "unknown format %d", format);
  const emu_gemm_params base{format, format == EMU_FMT_NVFP4 ? 16 : 32, 1, stage3_rounding, EMU_RZ, EMU_OUT_F32};
  emu_status st = emu::check_gemm_call(a_fp4, b_fp4, scale_a, scale_b, M, N, K, scale_a_rows, scale_a_cols,
                                       scale_b_rows, scale_b_cols, &base, ref);
  if (st != EMU_OK) return st;
  if (n_models < 0 || (n_models > 0 && (!models || !mismatches)))
    return fail(EMU_ERR_INVALID_ARGUMENT, "models and mismatches must not be NULL");
  if (ref_dtype != EMU_DTYPE_F16 && ref_dtype != EMU_DTYPE_BF16 && ref_dtype != EMU_DTYPE_F32)
    return fail(EMU_ERR_INVALID_ARGUMENT, "ref_dtype must be EMU_DTYPE_F16, EMU_DTYPE_BF16 or EMU_DTYPE_F32");
  if (!aligned(mismatches, 8)) return fail(EMU_ERR_INVALID_ARGUMENT, "mismatches must be 8-byte aligned");
  const int64_t G = K / base.group_size;
  for (int i = 0; i < n_models; ++i) {
    const emu_sweep_model& m = models[i];
    if (!emu::sweep_supported_w_reduce(m.w_reduce) || G % m.w_reduce != 0)
      return fail(EMU_ERR_UNSUPPORTED, "model %d: w_reduce %d must be 1, 2, 4 or 8 and divide K/group_size (%lld)", i,
                  m.w_reduce, (long long)G);
    if ((m.stage4_rounding != EMU_RZ && m.stage4_rounding != EMU_RNE) ||
        (m.align_rounding != EMU_RZ && m.align_rounding != EMU_RNE))
      return fail(EMU_ERR_INVALID_ARGUMENT, "model %d: roundings must be EMU_RZ (0) or EMU_RNE (1)", i);
    if (m.align3 < 0 || m.align3 > 46 || m.align4 < 0 || m.align4 > 52 || m.order < 0 || m.order > 2)
      return fail(EMU_ERR_INVALID_ARGUMENT, "model %d: align3 in [0, 46], align4 in [0, 52], order in [0, 2]", i);
  }
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (n_models == 0) return ok();
  cudaError_t e = cudaMemsetAsync(mismatches, 0, sizeof(int64_t) * (size_t)n_models, s);
  if (e != cudaSuccess || M == 0 || N == 0) return cuda_status(e, "emu_gemm_sweep");
  // one launch per block size and chunk of up to SWEEP_MAX_CONFIGS models
  for (int wr : {1, 2, 4, 8}) {
    emu::SweepModel chunk[emu::SWEEP_MAX_CONFIGS];
    int slots[emu::SWEEP_MAX_CONFIGS];
    int n = 0;
    for (int i = 0; i <= n_models; ++i) {
      if (i < n_models && models[i].w_reduce == wr) {
        const emu_sweep_model& m = models[i];
        chunk[n] = emu::SweepModel{m.stage4_rounding, m.align3, m.align4, m.align_rounding, m.order};
        slots[n++] = i;
      }
      if (n == emu::SWEEP_MAX_CONFIGS || (i == n_models && n > 0)) {
        e = emu::launch_gemm_sweep(a_fp4, b_fp4, scale_a, scale_b, M, N, K, scale_a_cols, scale_b_cols, alpha, format,
                                   wr, stage3_rounding, chunk, slots, n, ref, ref_dtype,
                                   reinterpret_cast<unsigned long long*>(mismatches), s);
        if (e != cudaSuccess) return cuda_status(e, "emu_gemm_sweep launch");
        n = 0;
      }
    }
  }
  return ok();
}

emu_status emu_gemm_compare(const uint8_t* a_fp4, const uint8_t* b_fp4, const uint8_t* scale_a,
                            const uint8_t* scale_b, int64_t M, int64_t N, int64_t K, int64_t scale_a_rows,
                            int64_t scale_a_cols, int64_t scale_b_rows, int64_t scale_b_cols, const float* alpha,
                            const emu_gemm_params* params, const void* ref, void* out, emu_compare_stats* stats,
                            void* workspace, size_t workspace_bytes, void* stream) {
  emu_status st = validate_gemm(M, N, K, scale_a_rows, scale_a_cols, scale_b_rows, scale_b_cols, params);
  if (st != EMU_OK) return st;
  if (!stats || !aligned(stats, 8)) return fail(EMU_ERR_INVALID_ARGUMENT, "stats must be a non-NULL, 8-byte aligned pointer");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (M == 0 || N == 0) {
    cudaError_t e = emu::launch_compare_init(stats, 0, s);
    if (e == cudaSuccess) e = emu::launch_compare_fini(stats, s);
    return cuda_status(e, "emu_gemm_compare");
  }
  if (!a_fp4 || !b_fp4 || !scale_a || !scale_b || !ref)
    return fail(EMU_ERR_INVALID_ARGUMENT, "tensor pointers must not be NULL");
  if (!aligned(a_fp4, 16) || !aligned(b_fp4, 16))
    return fail(EMU_ERR_INVALID_ARGUMENT, "a_fp4 / b_fp4 must be 16-byte aligned");
  const emu_gemm_params p = *params;
  const int cmp_dtype = p.out_mode == EMU_OUT_F32 ? EMU_DTYPE_F32
                        : p.out_mode == EMU_OUT_BF16_VIA_F16 ? EMU_DTYPE_BF16 : EMU_DTYPE_F16;
  if (workspace && tc_path(p, M, N, K)) {
    if (!aligned(workspace, 1024)) return fail(EMU_ERR_INVALID_ARGUMENT, "workspace must be 1024-byte aligned");
    if (workspace_bytes < emu::gemm_tc_workspace_size(p.format, M, N, K))
      return fail(EMU_ERR_INVALID_ARGUMENT, "workspace too small: %zu < %zu bytes", workspace_bytes,
                  emu::gemm_tc_workspace_size(p.format, M, N, K));
    emu::GemmArgs args{p.format, p.w_reduce, p.stage3_rounding, p.stage4_rounding, p.out_mode};
    args.cmp_ref = ref;
    args.cmp_stats = stats;
    args.write_out = out != nullptr;
    cudaError_t e = emu::launch_compare_init(stats, M * N, s);
    if (e == cudaSuccess)
      e = emu::launch_gemm_tc(a_fp4, b_fp4, scale_a, scale_b, M, N, K, scale_a_cols, scale_b_cols, alpha, args, out,
                              workspace, s);
    if (e == cudaSuccess) e = emu::launch_compare_fini(stats, s);
    return cuda_status(e, "emu_gemm_compare tensor-core launch");
  }
  if (!out)
    return fail(EMU_ERR_INVALID_ARGUMENT,
                "out must not be NULL on the CUDA-core path (no workspace, or a shape the tensor-core path does not take)");
  emu::GemmArgs args{p.format, p.w_reduce, p.stage3_rounding, p.stage4_rounding, p.out_mode};
  cudaError_t e = emu::launch_gemm_simt(a_fp4, b_fp4, scale_a, scale_b, M, N, K, scale_a_cols, scale_b_cols, alpha,
                                        args, out, s);
  if (e == cudaSuccess) e = emu::launch_compare(ref, out, cmp_dtype, M * N, stats, s);
  return cuda_status(e, "emu_gemm_compare launch");
}

emu_status emu_gemm_batch(const uint8_t* a_fp4, const uint8_t* b_fp4, const uint8_t* scale_a,
                          const uint8_t* scale_b, int64_t M, int64_t N, int64_t K, int64_t scale_a_rows,
                          int64_t scale_a_cols, int64_t scale_b_rows, int64_t scale_b_cols, const float* alpha,
                          const emu_gemm_params* params, int32_t n_params, const void* ref, void* out,
                          emu_compare_stats* stats, void* workspace, size_t workspace_bytes, void* stream) {
  if (!params) return fail(EMU_ERR_INVALID_ARGUMENT, "params must not be NULL");
  if (n_params < 1 || n_params > 4096) return fail(EMU_ERR_INVALID_ARGUMENT, "n_params must be in [1, 4096], got %d", n_params);
  if (!out && !ref) return fail(EMU_ERR_INVALID_ARGUMENT, "out and ref are both NULL: nothing to produce");
  if (ref && !stats) return fail(EMU_ERR_INVALID_ARGUMENT, "stats must not be NULL when ref is given");
  for (int32_t i = 0; i < n_params; ++i) {
    const emu_status st = validate_gemm(M, N, K, scale_a_rows, scale_a_cols, scale_b_rows, scale_b_cols, &params[i]);
    if (st != EMU_OK) return st;
    if (params[i].format != params[0].format || params[i].group_size != params[0].group_size ||
        params[i].out_mode != params[0].out_mode)
      return fail(EMU_ERR_INVALID_ARGUMENT, "params[%d]: every set must have params[0]'s format, group_size and out_mode", i);
  }
  const size_t elem = params[0].out_mode == EMU_OUT_F32 ? 4 : 2;
  for (int32_t i = 0; i < n_params; ++i) {
    void* oi = out ? static_cast<void*>(static_cast<char*>(out) + (size_t)i * (size_t)M * (size_t)N * elem) : nullptr;
    const emu_status st =
        ref ? emu_gemm_compare(a_fp4, b_fp4, scale_a, scale_b, M, N, K, scale_a_rows, scale_a_cols, scale_b_rows,
                               scale_b_cols, alpha, &params[i], ref, oi, stats + i, workspace, workspace_bytes, stream)
            : emu_gemm_ws(a_fp4, b_fp4, scale_a, scale_b, M, N, K, scale_a_rows, scale_a_cols, scale_b_rows,
                          scale_b_cols, alpha, &params[i], oi, workspace, workspace_bytes, stream);
    if (st != EMU_OK) return st;
  }
  return ok();
}

int64_t emu_set_wait_limit(int64_t cycles) { return emu::set_wait_limit(cycles); }

emu_status emu_test_hold_first_ready(int32_t enable) {
  emu::set_hold_first_ready(enable);
  return ok();
}

emu_status emu_device_status(void* stream) {
  cudaError_t e = cudaStreamSynchronize(static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_status(e, "emu_device_status: stream");
  int code = 0;
  e = emu::take_wait_error(&code);
  if (e != cudaSuccess) return cuda_status(e, "emu_device_status: error word");
  if (code == 0) return ok();
  static const char* const kSite[] = {"", "producer stage slot", "producer record slot", "MMA accumulator set",
                                      "MMA stage data", "epilogue accumulator", "epilogue records",
                                      "producer drain", "record drain", "MMA drain"};
  return fail(EMU_ERR_TIMEOUT,
              "a tensor-core pipeline wait ran out (code %d: %s); outputs of the calls on this device since the "
              "last emu_device_status are undefined", code, code > 0 && code < 10 ? kSite[code] : "unknown");
}

emu_status emu_dequant_fp4(const uint8_t* q, const uint8_t* sf, int64_t rows, int64_t K, int64_t sf_cols,
                           int32_t format, const float* global_scale, float* out, void* stream) {
  if (rows < 0 || K < 0 || sf_cols < 0) return fail(EMU_ERR_INVALID_ARGUMENT, "negative size");
  if (format != EMU_FMT_NVFP4 && format != EMU_FMT_MXFP4)
    return fail(EMU_ERR_INVALID_ARGUMENT, "unknown format %d", format);
  const int64_t gsz = format == EMU_FMT_NVFP4 ? 16 : 32;
  if (K % gsz != 0) return fail(EMU_ERR_K_GROUP, "K must be a multiple of %lld", (long long)gsz);
  if (rows == 0 || K == 0) return ok();
  if (!q || !sf || !out || (format == EMU_FMT_NVFP4 && !global_scale))
    return fail(EMU_ERR_INVALID_ARGUMENT, "pointers must not be NULL");
  if (sf_cols % 4 != 0 || sf_cols < K / gsz)
    return fail(EMU_ERR_SCALE_SHAPE, "scale columns (%lld) must be a multiple of 4 and at least K/group (%lld)",
                (long long)sf_cols, (long long)(K / gsz));
  if (!aligned(q, 4) || !aligned(out, 16)) return fail(EMU_ERR_INVALID_ARGUMENT, "q must be 4-byte, out 16-byte aligned");
  return cuda_status(emu::launch_dequant(q, sf, rows, K, sf_cols, format, global_scale, out,
                                         static_cast<cudaStream_t>(stream)),
                     "emu_dequant_fp4 launch");
}

}  // extern "C"
