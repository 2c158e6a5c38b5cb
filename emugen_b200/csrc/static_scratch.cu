// emu_gemm_static: the tensor-core emulated GEMM with its scratch in a file-scope device array
// instead of a caller-provided workspace.  The call allocates nothing.
//
// Who needs it: callers that cannot allocate device memory around the GEMM.  An FFI host (cgo,
// JNI, a ctypes script) driving libemugen directly has no caching allocator, and cudaMalloc /
// cudaFree synchronise the whole device, stalling every other stream on it; a serving process that
// has reserved nearly all of HBM for its own pools up front may have no room left for a
// per-call workspace.  Such callers get the tensor-core path with a fixed footprint, paid once per
// device, instead of falling back to the CUDA-core kernel.
//
// Cost: the array is part of this library's device module, so every device on which the module
// is loaded holds EMU_STATIC_SCRATCH_BYTES (+1 KiB) until the process exits, whether or not
// emu_gemm_static is ever called: at library load under CUDA_MODULE_LOADING=EAGER, otherwise when
// the module is first used on that device.
//
// Address: in host code the array's name stands for a host-side shadow, not device memory, so each
// call asks the runtime for the array's device address on the current device
// (cudaGetSymbolAddress).  Nothing is cached: a cached address would dangle after cudaDeviceReset
// or any re-creation of the primary context, which reloads the module.  The first call on a
// device may load the module; make it before any stream capture begins.
//
// Limits: problems whose tensor-core workspace exceeds EMU_STATIC_SCRATCH_BYTES are rejected with
// EMU_ERR_UNSUPPORTED, after the argument checks emu_gemm_ws makes (so a bad argument reports the
// same status as emu_gemm).  There is one scratch per device, so calls whose executions overlap on
// one device (different streams, or different host threads) race on it; serialise them (one
// stream, or events).  Nothing in the scratch has to start at zero: each call clears its flag words
// on `stream` before its kernels read them and writes every other byte before reading it.
#include <cuda_runtime.h>
#include <stdarg.h>
#include <stdint.h>
#include <stdio.h>

#include "../../include/emugen.h"
#include "kernels.h"

namespace {

constexpr size_t kAlign = 1024;   // the workspace alignment emu_gemm_ws requires

// +kAlign so that a 1024-aligned window of EMU_STATIC_SCRATCH_BYTES always fits
static __device__ __align__(256) uint8_t g_static_scratch[EMU_STATIC_SCRATCH_BYTES + kAlign];

// sets emu_last_error() of this thread and returns s
emu_status reject(emu_status s, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  return emu::record_failure(s, buf);
}

// 1024-aligned start of the scratch on the current device
cudaError_t scratch_base(void** out) {
  void* p = nullptr;
  const cudaError_t e = cudaGetSymbolAddress(&p, g_static_scratch);
  if (e != cudaSuccess) return e;
  const uintptr_t a = (reinterpret_cast<uintptr_t>(p) + kAlign - 1) & ~(uintptr_t)(kAlign - 1);
  *out = reinterpret_cast<void*>(a);
  return cudaSuccess;
}

}  // namespace

extern "C" {

emu_status emu_gemm_static(const uint8_t* a_fp4, const uint8_t* b_fp4, const uint8_t* scale_a,
                           const uint8_t* scale_b, int64_t M, int64_t N, int64_t K, int64_t scale_a_rows,
                           int64_t scale_a_cols, int64_t scale_b_rows, int64_t scale_b_cols, const float* alpha,
                           const emu_gemm_params* params, void* out, void* stream) {
  const emu_status st = emu::check_gemm_call(a_fp4, b_fp4, scale_a, scale_b, M, N, K, scale_a_rows, scale_a_cols,
                                             scale_b_rows, scale_b_cols, params, out);
  if (st != EMU_OK) return st;
  const size_t need = emu_gemm_workspace_size(M, N, K, params);
  if (need == 0)   // the CUDA-core path: no scratch involved
    return emu_gemm(a_fp4, b_fp4, scale_a, scale_b, M, N, K, scale_a_rows, scale_a_cols, scale_b_rows, scale_b_cols,
                    alpha, params, out, stream);
  if (need > (size_t)EMU_STATIC_SCRATCH_BYTES)
    return reject(EMU_ERR_UNSUPPORTED,
                  "emu_gemm_static: M=%lld N=%lld K=%lld needs %zu bytes of scratch, more than the static %zu; "
                  "use emu_gemm_ws with a workspace",
                  (long long)M, (long long)N, (long long)K, need, (size_t)EMU_STATIC_SCRATCH_BYTES);
  void* base = nullptr;
  cudaError_t e = scratch_base(&base);
  if (e != cudaSuccess) return reject(EMU_ERR_CUDA, "emu_gemm_static: scratch address: %s", cudaGetErrorString(e));
  return emu_gemm_ws(a_fp4, b_fp4, scale_a, scale_b, M, N, K, scale_a_rows, scale_a_cols, scale_b_rows, scale_b_cols,
                     alpha, params, out, base, EMU_STATIC_SCRATCH_BYTES, stream);
}

}  // extern "C"
