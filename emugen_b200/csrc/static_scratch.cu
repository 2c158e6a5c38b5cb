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
// Setup: the first call on each device (with that device current) resolves the array's address
// with cudaGetSymbolAddress, which can load this file's module; make that first call before any
// stream capture begins.  Later calls reuse the cached address.
//
// Limits: problems whose tensor-core workspace exceeds EMU_STATIC_SCRATCH_BYTES are rejected with
// EMU_ERR_UNSUPPORTED.  There is one scratch per device, so calls whose executions overlap on one
// device (different streams, or different host threads) race on it; serialise them (one stream,
// or events).  Nothing in the scratch has to start at zero: each call clears its flag words on
// `stream` before its kernels read them and writes every other byte before reading it.
#include <cuda_runtime.h>
#include <stdarg.h>
#include <stdint.h>
#include <stdio.h>

#include <mutex>

#include "../../include/emugen.h"
#include "kernels.h"

namespace {

constexpr size_t kAlign = 1024;   // the workspace alignment emu_gemm_ws requires
constexpr int kMaxDevices = 64;

// +kAlign so that a 1024-aligned window of EMU_STATIC_SCRATCH_BYTES always fits
static __device__ __align__(256) uint8_t g_static_scratch[EMU_STATIC_SCRATCH_BYTES + kAlign];

std::mutex g_mu;
void* g_base[kMaxDevices] = {};

// sets emu_last_error() of this thread and returns s
emu_status reject(emu_status s, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  return emu::record_failure(s, buf);
}

// 1024-aligned start of this device's scratch, resolved once per device with the device current
cudaError_t scratch_base(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lock(g_mu);
  if (!g_base[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_static_scratch);
    if (e != cudaSuccess) return e;
    const uintptr_t a = (reinterpret_cast<uintptr_t>(p) + kAlign - 1) & ~(uintptr_t)(kAlign - 1);
    g_base[dev] = reinterpret_cast<void*>(a);
  }
  *out = g_base[dev];
  return cudaSuccess;
}

}  // namespace

extern "C" {

emu_status emu_gemm_static(const uint8_t* a_fp4, const uint8_t* b_fp4, const uint8_t* scale_a,
                           const uint8_t* scale_b, int64_t M, int64_t N, int64_t K, int64_t scale_a_rows,
                           int64_t scale_a_cols, int64_t scale_b_rows, int64_t scale_b_cols, const float* alpha,
                           const emu_gemm_params* params, void* out, void* stream) {
  const size_t need = emu_gemm_workspace_size(M, N, K, params);
  if (need == 0)   // the CUDA-core path (or an argument error emu_gemm reports): no scratch involved
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
