/*
 * emugen.h — C ABI of libemugen.so, the B200 (sm_100a) implementation of EmuGen's emulated
 * NVFP4 / MXFP4 scaled GEMM and of the FP4 quantisation that feeds it.
 *
 * Conventions (every entry point):
 *   - All tensor arguments are DEVICE pointers owned by the caller; nothing is allocated or freed
 *     on the caller's behalf.  Row-major, contiguous.
 *   - Work is enqueued on `stream` (a cudaStream_t passed as void*; NULL = legacy default stream)
 *     and returns without synchronising.  Device-resident scalars (alpha, global scales) are read
 *     on the device, so no host round trip happens (the reference reads alpha with `.item()`).
 *   - The return value is an emu_status; on failure emu_last_error() gives a message (thread-local)
 *     whose text matches the reference's TORCH_CHECK message where the reference has one.
 *   - Calls are reentrant; calls on different streams may overlap.
 *
 * Packed FP4 operands: [rows][K/2] bytes, element 2j in the low nibble of byte j, element 2j+1 in
 * the high nibble; e2m1 codes, bit 3 = sign (reference nvfp_emulation.cpp:7-13, 29-39).
 * Block scales: the 128x4 swizzled layout, a [rows_pad][cols_pad] byte buffer with rows_pad a
 * multiple of 128 and cols_pad a multiple of 4; byte (r, c) sits at
 *   (r/128)*(cols_pad/4)*512 + (c/4)*512 + (r%32)*16 + ((r%128)/32)*4 + c%4
 * (reference nvfp_emulation.cpp:15-27; writer flashinfer quantization_utils.cuh:626-666).
 */
#ifndef EMUGEN_H_
#define EMUGEN_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define EMU_ABI_VERSION 1

#if defined(__GNUC__)
#define EMU_API __attribute__((visibility("default")))
#else
#define EMU_API
#endif

typedef int32_t emu_status;
enum {
  EMU_OK = 0,
  EMU_ERR_INVALID_ARGUMENT = 1,   /* null pointer, negative size, unknown enum value            */
  EMU_ERR_K_MISMATCH = 2,         /* "K mismatch between a and b"                               */
  EMU_ERR_K_GROUP = 3,            /* "K must be multiple of 16" / "K must be divisible by group_size" */
  EMU_ERR_W_REDUCE = 4,           /* "G = K/16 must be multiple of 4" (generic: of w_reduce)     */
  EMU_ERR_GROUP_SIZE = 5,         /* "only MXFP4 group_size=32 is supported" (and NVFP4: 16)     */
  EMU_ERR_SCALE_SHAPE = 6,        /* "swizzled scale shape must be divisible by 128 and 4"        */
  EMU_ERR_SCALE_TOO_SMALL = 7,    /* scale buffer has fewer rows / columns than M,N / K/group     */
  EMU_ERR_UNSUPPORTED = 8,        /* a size beyond what this library supports (message says which) */
  EMU_ERR_CUDA = 9,               /* a CUDA runtime error (message carries cudaGetErrorString)    */
  EMU_ERR_TIMEOUT = 10            /* a tensor-core pipeline wait ran out (emu_device_status)       */
};

/* Element formats. */
enum { EMU_FMT_NVFP4 = 0, /* E4M3 block scales, group 16, stage-2 product in f32 */
       EMU_FMT_MXFP4 = 1  /* UE8M0 block scales, group 32, stage-2 product in f64 */ };
enum { EMU_RZ = 0, EMU_RNE = 1 };   /* same codes as nvfp_cpp_emul.RZ / RNE */
enum { EMU_OUT_F16 = 0,             /* fp16, the C++ emulators' output */
       EMU_OUT_BF16_VIA_F16 = 1,    /* bf16(fp16(x)): reference `.to(out_dtype)` after fp16, gemm.py:69 */
       EMU_OUT_F32 = 2 };           /* the f32 accumulator times alpha, before the fp16 rounding */
enum { EMU_DTYPE_F16 = 0, EMU_DTYPE_BF16 = 1,   /* quantiser input dtypes */
       EMU_DTYPE_F32 = 2 };                      /* also accepted by emu_compare */

/* Accumulator model of one emulated GEMM (search/emulation/config.py:10-81 and the state fields
 * of gemm_compare/backends/nvfp.py:30-44, mxfp.py:27-42).  w_stage3 / w_stage4 / m_chunk_size are
 * absent on purpose: the reference keeps them for API compatibility and they change no result
 * (search/emulation/core.py:31-38). */
typedef struct emu_gemm_params {
  int32_t format;           /* EMU_FMT_NVFP4 or EMU_FMT_MXFP4                                 */
  int32_t group_size;       /* elements per block scale: 16 (NVFP4) or 32 (MXFP4)             */
  int32_t w_reduce;         /* groups summed exactly in stage 3 (reference: 4 NVFP, 2 MXFP), 1..64 */
  int32_t stage3_rounding;  /* EMU_RZ / EMU_RNE, used when K/group == w_reduce (one block)    */
  int32_t stage4_rounding;  /* EMU_RZ / EMU_RNE, the running f32 accumulator                  */
  int32_t out_mode;         /* EMU_OUT_*                                                      */
} emu_gemm_params;

/* ABI version of the loaded library (EMU_ABI_VERSION it was built with). */
EMU_API int32_t emu_abi_version(void);

/* Message of the last failing call on this thread ("" if none). */
EMU_API const char* emu_last_error(void);

/* Name of a status code. */
EMU_API const char* emu_status_string(emu_status s);

/*
 * Emulated scaled FP4 GEMM:  out[M][N] = emul(A[M][K] x B[N][K]^T).
 * Replaces:
 *   nvfp_cpp_emul/nvfp_cpp_emul/csrc/nvfp_emulation.cpp:90-156  emulated_scaled_fp4_mm
 *       (params {NVFP4, 16, 4, r3, r4, EMU_OUT_F16}, alpha = state.alpha)
 *   mxfp_cpp_emul/mxfp_cpp_emul/csrc/mxfp_emulation.cpp:98-166  emulated_mxfp4_mm
 *       (params {MXFP4, 32, 2, r3, r4, EMU_OUT_F16}, alpha = NULL)
 *   search/emulation/core.py:69-148 MMAEngine.emulation_scaled_fp4_mm + gemm.py:35-69
 *       emulate_nvfp_scaled_fp4_mm (generic w_reduce; EMU_OUT_BF16_VIA_F16 for bf16 out_dtype)
 * a_fp4 [M][K/2], b_fp4 [N][K/2]; scale_a [scale_a_rows][scale_a_cols], scale_b likewise (swizzled);
 * alpha: device float[1] multiplied into the f32 result (NULL = no multiply);
 * out: [M][N] uint16 bits (fp16 / bf16) or float (EMU_OUT_F32).
 * M, N >= 1; K >= 1 a multiple of group_size; (K/group_size) a multiple of w_reduce.
 */
EMU_API emu_status emu_gemm(const uint8_t* a_fp4, const uint8_t* b_fp4, const uint8_t* scale_a,
                    const uint8_t* scale_b, int64_t M, int64_t N, int64_t K, int64_t scale_a_rows,
                    int64_t scale_a_cols, int64_t scale_b_rows, int64_t scale_b_cols,
                    const float* alpha, const emu_gemm_params* params, void* out, void* stream);

/*
 * Bytes of device workspace emu_gemm_ws needs to take the tensor-core path for this problem
 * (0 when the problem runs on the CUDA-core path, which needs none).  The tensor-core path covers
 * the reference's accumulator shapes (NVFP4 w_reduce 4, MXFP4 w_reduce 2) with K a multiple of 64;
 * problems below 2^27 (NVFP4) / 2^30 (MXFP4) multiply-accumulates return 0 here because the CUDA-core
 * kernels finish them sooner.
 */
EMU_API size_t emu_gemm_workspace_size(int64_t M, int64_t N, int64_t K, const emu_gemm_params* params);

/*
 * The tensor-core path's workspace for this problem whatever its size (0 where that path does not
 * apply): a workspace of this size passed to emu_gemm_ws selects the tensor-core kernel even for
 * small problems.  No reference counterpart (a kernel choice the reference does not have).
 */
EMU_API size_t emu_gemm_tc_workspace_size(int64_t M, int64_t N, int64_t K, const emu_gemm_params* params);

/*
 * Diagnostic: byte offset, within the tensor-core path's workspace, of its per-block epilogue path
 * codes ((size_t)-1 where that path does not apply).  After a call on that path completes,
 * workspace[offset + (tm * tiles_n + tn) * (K / 64) + kb] holds the code of 128-row tile tm,
 * 64-column tile tn (tiles_n = ceil(N / 64)) and 64-wide K block kb: bits 0-1 = 0 f64, 1 integer,
 * 2 block-sum, 3 mixed (the exactness classes the kernel chose).  No reference counterpart.
 */
EMU_API size_t emu_gemm_tc_path_offset(int64_t M, int64_t N, int64_t K, const emu_gemm_params* params);

/*
 * emu_gemm with caller-provided scratch: `workspace` (1024-byte aligned, at least
 * emu_gemm_workspace_size bytes, contents need not be initialised) enables the tcgen05 path; with
 * workspace == NULL the call is exactly emu_gemm.  Same results bit for bit either way.
 * Replaces the same reference entry points as emu_gemm.  The workspace must not be used by
 * another call until this one has completed on `stream`.
 */
EMU_API emu_status emu_gemm_ws(const uint8_t* a_fp4, const uint8_t* b_fp4, const uint8_t* scale_a,
                       const uint8_t* scale_b, int64_t M, int64_t N, int64_t K, int64_t scale_a_rows,
                       int64_t scale_a_cols, int64_t scale_b_rows, int64_t scale_b_cols,
                       const float* alpha, const emu_gemm_params* params, void* out,
                       void* workspace, size_t workspace_bytes, void* stream);

/*
 * Accumulator model beyond the reference.  The reference keeps w_stage3 / w_stage4 as parameters
 * and ignores them (search/emulation/core.py:31-38, config.py:16-19); this model gives them a
 * definition, for on-device parameter sweeps (no reference oracle exists for nonzero values):
 *   align3 (W3, 0 or 1..46): stage 3 aligns the block's addends to the largest exponent E among the
 *           finite nonzero ones, each rounded (align_rounding: EMU_RZ truncate, EMU_RNE) onto the
 *           grid 2^(E - W3 + 1), then sums them exactly; a non-finite addend leaves the f64 sum.
 *   align4 (W4, 0 or 1..52): stage 4 aligns acc and the block sum the same way before R4.
 *   order (0..2), used when align3 == 0: stage-3 f64 summation order, 0 left to right (the
 *           reference), 1 right to left, 2 pairwise tree.
 * All zero = the reference model.
 */
typedef struct emu_accum_model {
  int32_t align3;
  int32_t align4;
  int32_t align_rounding;
  int32_t order;
} emu_accum_model;

/*
 * emu_gemm under an accumulator model.  A zero model runs emu_gemm itself.  A nonzero model runs a
 * CUDA-core kernel that needs w_reduce <= 16.  Replaces the reference's HardwareConfig-driven
 * MMAEngine.emulation_scaled_fp4_mm (search/emulation/core.py:69-148) for sweeps over the fields
 * the reference leaves unimplemented.
 */
EMU_API emu_status emu_gemm_model(const uint8_t* a_fp4, const uint8_t* b_fp4, const uint8_t* scale_a,
                                  const uint8_t* scale_b, int64_t M, int64_t N, int64_t K,
                                  int64_t scale_a_rows, int64_t scale_a_cols, int64_t scale_b_rows,
                                  int64_t scale_b_cols, const float* alpha, const emu_gemm_params* params,
                                  const emu_accum_model* model, void* out, void* stream);

/*
 * Status of the asynchronous work on this device: synchronises `stream`, then reads and clears the
 * device's record of tensor-core pipeline waits that ran out.  Every wait in that kernel is
 * bounded (emu_set_wait_limit); a wait that runs out makes the kernel stop, drain the copies and
 * MMAs it has in flight, free its tensor memory and return, leaving the outputs of the unfinished
 * tiles undefined.  Returns EMU_OK, EMU_ERR_TIMEOUT (the message names the wait) or EMU_ERR_CUDA.
 * The reference raises synchronously on bad input (nvfp_emulation.cpp:99-106); this is the
 * asynchronous counterpart for failures that only the device can see.
 */
EMU_API emu_status emu_device_status(void* stream);

/*
 * Bound, in SM clock cycles, of each pipeline wait of the tensor-core kernels launched after this
 * call, process-wide (<= 0 restores the default 2^31, about a second); returns the previous bound.
 * Waits for copies or MMAs already in flight at exit always use the default.  No reference
 * counterpart (the reference has no device pipeline).
 */
EMU_API int64_t emu_set_wait_limit(int64_t cycles);

/*
 * Test hook for the failure path, process-wide: while enabled, tensor-core launches withhold their
 * first accumulator-ready signal, so the epilogue's bounded wait runs out (no fault, no hang; the
 * kernel returns and emu_device_status reports EMU_ERR_TIMEOUT).  Never enable it in production.
 */
EMU_API emu_status emu_test_hold_first_ready(int32_t enable);

/*
 * One model of an accumulator-model sweep: the block size and stage-4 rounding it runs with, and the
 * emu_accum_model fields (all zero = the reference model at that block size).
 */
typedef struct emu_sweep_model {
  int32_t w_reduce;         /* groups per stage-3 block: 1, 2, 4 or 8, a divisor of K / group size */
  int32_t stage4_rounding;  /* EMU_RZ / EMU_RNE                                                   */
  int32_t align3;           /* as emu_accum_model                                                 */
  int32_t align4;
  int32_t align_rounding;
  int32_t order;
} emu_sweep_model;

/*
 * Accumulator-model sweep: the emulated GEMM of (a_fp4, b_fp4) under each of n_models models, every
 * result -- the f32 accumulator times alpha, rounded once to ref_dtype (EMU_DTYPE_F16 / BF16 / F32)
 * -- compared element-wise with `ref` ([M][N], device) by gemm_compare's rule (equal, or NaN on both
 * sides, gemm_compare/runner.py:20-55); mismatches[i] (device int64[n_models], overwritten) receives
 * model i's mismatch count.  No output is written.  Stages 1-2 run once per group for all models of
 * one block size.  Replaces the reference's one-emulation-per-candidate loops (search/w3.py:123-158,
 * search/w4.py:60-90) for the models emu_gemm_model defines; bit for bit emu_gemm_model's results.
 * format / stage3_rounding as in emu_gemm_params (stage3_rounding applies when K / group == w_reduce).
 */
EMU_API emu_status emu_gemm_sweep(const uint8_t* a_fp4, const uint8_t* b_fp4, const uint8_t* scale_a,
                                  const uint8_t* scale_b, int64_t M, int64_t N, int64_t K, int64_t scale_a_rows,
                                  int64_t scale_a_cols, int64_t scale_b_rows, int64_t scale_b_cols,
                                  const float* alpha, int32_t format, int32_t stage3_rounding,
                                  const emu_sweep_model* models, int32_t n_models, const void* ref,
                                  int32_t ref_dtype, int64_t* mismatches, void* stream);

/*
 * Bytes of the per-device static scratch behind emu_gemm_static (64 MiB).  The array belongs to the
 * library's device module: every device on which that module is loaded holds it (64 MiB + 1 KiB)
 * until the process exits, whether or not emu_gemm_static is called -- at library load under
 * CUDA_MODULE_LOADING=EAGER, else when the module is first used on the device.
 */
#define EMU_STATIC_SCRATCH_BYTES (64u << 20)

/*
 * emu_gemm that allocates nothing: the tensor-core path with its scratch in a static device array
 * of EMU_STATIC_SCRATCH_BYTES inside the library, for callers that cannot allocate device memory
 * (FFI hosts without a caching allocator, where cudaMalloc/cudaFree would synchronise the device;
 * processes whose memory pools already hold the device).  Problems taking the CUDA-core path run
 * it (it needs no scratch).  No reference counterpart: the reference allocates its outputs and
 * temporaries through torch.
 *   - The arguments are checked first, exactly as emu_gemm checks them (same status codes and
 *     messages); then problems whose emu_gemm_workspace_size exceeds EMU_STATIC_SCRATCH_BYTES fail
 *     with EMU_ERR_UNSUPPORTED (use emu_gemm_ws).
 *   - Every call looks up the scratch's device address on the current device
 *     (cudaGetSymbolAddress; nothing is cached, so a device reset cannot leave a stale address).
 *     The first call on a device may load the library's module: make it before any stream capture.
 *   - One scratch per device: calls whose executions overlap on a device (different streams or
 *     threads) race on it and must be serialised by the caller.
 *   - Nothing needs to be zeroed beforehand: each call clears its own flag words on `stream`.
 * Same arguments, validation and results (bit for bit) as emu_gemm.
 */
EMU_API emu_status emu_gemm_static(const uint8_t* a_fp4, const uint8_t* b_fp4, const uint8_t* scale_a,
                           const uint8_t* scale_b, int64_t M, int64_t N, int64_t K, int64_t scale_a_rows,
                           int64_t scale_a_cols, int64_t scale_b_rows, int64_t scale_b_cols,
                           const float* alpha, const emu_gemm_params* params, void* out, void* stream);

/*
 * NVFP4 global scale and GEMM alpha, on the device, without host synchronisation.
 * Replaces gemm_compare/backends/nvfp.py:24-27 global_scale_nvfp and nvfp.py:174-177:
 *   gs = f32(2688.0 / amax) in double, amax = max|x| (1.0 when amax is 0 or NaN),
 *   alpha = f32(1.0 / max(gs_a * gs_b, 1e-8)) in double.
 * a: [a_numel] fp16/bf16, b: [b_numel]; gs_a, gs_b, alpha: device float[1] outputs.
 */
EMU_API emu_status emu_nvfp4_global_scales(const void* a, int64_t a_numel, const void* b, int64_t b_numel,
                                   int32_t dtype, float* gs_a, float* gs_b, float* alpha,
                                   void* stream);

/*
 * The two halves of emu_nvfp4_global_scales, for operands sharded over several devices.
 * emu_nvfp4_amax writes max|x| of a and of b as the bits of a non-negative f32 (device uint32[1]
 * each; unsigned order is value order, a NaN input gives a NaN pattern above +inf), so the words of
 * several shards combine with an integer MAX (e.g. an NCCL all_reduce MAX) into the amax of the
 * whole operand.  emu_nvfp4_scales_from_amax turns two such words into gs_a, gs_b and alpha exactly
 * as emu_nvfp4_global_scales does (the words may alias gs_a / gs_b).  Together they replace
 * gemm_compare/backends/nvfp.py:24-27 global_scale_nvfp and nvfp.py:174-177 for a sharded caller.
 */
EMU_API emu_status emu_nvfp4_amax(const void* a, int64_t a_numel, const void* b, int64_t b_numel, int32_t dtype,
                                  uint32_t* amax_a, uint32_t* amax_b, void* stream);
EMU_API emu_status emu_nvfp4_scales_from_amax(const uint32_t* amax_a, const uint32_t* amax_b, float* gs_a,
                                              float* gs_b, float* alpha, void* stream);

/*
 * NVFP4 quantisation: x [M][K] fp16/bf16 -> q [M][K/2] packed e2m1, sf [pad128(M)][pad4(K/16)]
 * swizzled E4M3 block scales (padding written as 0).  global_scale: device float[1].
 * Replaces nvfp.ops.scaled_fp4_quant at gemm_compare/backends/nvfp.py:178-179 (third-party,
 * absent); the recipe is flashinfer fp4_quantize(x, gs, 16, sf_use_ue8m0=False, swizzled=True),
 * flashinfer/data/csrc/nv_internal/tensorrt_llm/kernels/quantization_utils.cuh:352-366.
 * K must be a multiple of 16.
 */
EMU_API emu_status emu_quant_nvfp4(const void* x, int32_t dtype, int64_t M, int64_t K,
                           const float* global_scale, uint8_t* q, uint8_t* sf, void* stream);

/*
 * MXFP4 quantisation: x [M][K] fp16/bf16 -> q [M][K/2], sf [pad128(M)][pad4(K/32)] swizzled UE8M0.
 * Replaces flashinfer.mxfp4_quantize at gemm_compare/backends/mxfp.py:199-200
 * (flashinfer/quantization/fp4_quantization.py:1237-1282 -> quantization_utils.cuh:326-333).
 * K must be a multiple of 32.
 */
EMU_API emu_status emu_quant_mxfp4(const void* x, int32_t dtype, int64_t M, int64_t K, uint8_t* q,
                           uint8_t* sf, void* stream);

/*
 * Element-wise comparison of two [n] tensors (fp16 / bf16 / f32, same dtype), on the device.
 * Replaces the torch reductions of gemm_compare/runner.py:20-55 compare_tensors and 58-79
 * compare_mse: an element is a mismatch when it is neither == (so +0 == -0) nor NaN on both sides;
 * max_diff is max |ref - out| (f32) over the mismatches with NaN differences as +inf (0 if none);
 * the squared-error terms are (ref - out)^2 and ref^2 in f32 with non-finite terms dropped, summed
 * in f64 (the reference sums in f32: the sums agree to rounding).  `stats` is DEVICE memory the call
 * overwrites; read it after the stream reaches this point.
 */
typedef struct emu_compare_stats {
  int64_t mismatches;
  int64_t first_index;     /* row-major index of the first mismatch, -1 if none */
  float max_diff;
  float max_sq_error;
  double sq_error_sum;
  double ref_sq_sum;
  int64_t numel;
} emu_compare_stats;

EMU_API emu_status emu_compare(const void* ref, const void* out, int32_t dtype, int64_t n,
                               emu_compare_stats* stats, void* stream);

/*
 * emu_gemm_ws fused with emu_compare: the emulated GEMM's output compared on the device with `ref`
 * ([M][N], the output's dtype), filling `stats` as emu_compare(ref, out) does (the squared-error sums
 * accumulate in another order, so they agree to rounding).  On the tensor-core path (workspace given
 * and the shape taken) the comparison runs in the GEMM epilogue and `out` may be NULL, in which
 * case no output is written; otherwise the CUDA-core GEMM writes `out` (then required) and
 * emu_compare runs after it.  This is the mismatch count of gemm_compare's runner
 * (gemm_compare/runner.py:20-79 applied to emul_fn's output) without the M x N round trip.
 */
EMU_API emu_status emu_gemm_compare(const uint8_t* a_fp4, const uint8_t* b_fp4, const uint8_t* scale_a,
                                    const uint8_t* scale_b, int64_t M, int64_t N, int64_t K,
                                    int64_t scale_a_rows, int64_t scale_a_cols, int64_t scale_b_rows,
                                    int64_t scale_b_cols, const float* alpha, const emu_gemm_params* params,
                                    const void* ref, void* out, emu_compare_stats* stats, void* workspace,
                                    size_t workspace_bytes, void* stream);

/*
 * Several parameter sets on the same operands in one call: for i in [0, n_params), the emulated GEMM of
 * emu_gemm_ws under params[i], written to out + i * M * N elements (all sets' outputs back to back,
 * [n_params][M][N]) when `out` is not NULL, and compared with `ref` ([M][N]) into stats[i] as
 * emu_gemm_compare does when `ref` is not NULL (then `stats` points to n_params structs; with no `out`
 * the comparison runs in the tensor-core epilogue, which needs the workspace and a shape that path
 * takes).  The operands fix the format and group size, and `out` / `ref` one element type, so every
 * set has params[0]'s format, group_size and out_mode; block size and roundings vary per set.  The
 * workspace is sized as for emu_gemm_ws (the size does not depend on the block size or roundings).
 * The batched entry the survey of the reference's callers asks for (one call per sweep of rounding /
 * block-size settings instead of one per setting); no counterpart in the reference, which runs one
 * emulation per call.  n_params <= 4096.
 */
EMU_API emu_status emu_gemm_batch(const uint8_t* a_fp4, const uint8_t* b_fp4, const uint8_t* scale_a,
                                  const uint8_t* scale_b, int64_t M, int64_t N, int64_t K, int64_t scale_a_rows,
                                  int64_t scale_a_cols, int64_t scale_b_rows, int64_t scale_b_cols, const float* alpha,
                                  const emu_gemm_params* params, int32_t n_params, const void* ref, void* out,
                                  emu_compare_stats* stats, void* workspace, size_t workspace_bytes, void* stream);

/*
 * Dequantise packed FP4 to f32: out[r][k] = e2m1(q[r][k]) * scale(r, k / group), scales in the
 * swizzled layout ([pad128(rows)][sf_cols]).  MXFP4: scale = f32 with bits (u << 23) (u = 0 -> 0,
 * u = 255 -> inf), as flashinfer.mxfp4_dequantize, the reference's MXFP4 pseudo_fn operand
 * (gemm_compare/backends/mxfp.py:155-165).  NVFP4: scale = f32(e4m3) / global_scale (device
 * float[1]), the reference's NVFP4 pseudo_fn operand (gemm_compare/backends/nvfp.py:133-146, whose
 * nvfp.pseudo_quant module is absent from the reference tree).  K must be a multiple of the group.
 */
EMU_API emu_status emu_dequant_fp4(const uint8_t* q, const uint8_t* sf, int64_t rows, int64_t K,
                                   int64_t sf_cols, int32_t format, const float* global_scale,
                                   float* out, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* EMUGEN_H_ */
