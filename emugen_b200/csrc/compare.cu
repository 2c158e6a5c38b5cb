// Result checking and the dequantised ("pseudo") operand path, on sm_100a.
//
// compare:  one pass over a pair of [n] fp16 / bf16 / f32 tensors computing, on the device, what the
//           reference's gemm_compare/runner.py:20-79 compare_tensors and compare_mse compute with
//           torch ops: elements that are neither equal (IEEE ==, so +0 == -0) nor both NaN count as
//           mismatches; |a - b| in f32 over the mismatches (NaN -> inf) gives max_diff; (a - b)^2 and
//           a^2 in f32 with non-finite terms dropped give the squared-error sums (accumulated in
//           f64 here; torch accumulates in f32, so sums agree to rounding, not bit for bit).
// dequant:  packed e2m1 x block scale -> f32, the operand the reference's pseudo_fn multiplies
//           (gemm_compare/backends/nvfp.py:133-146, mxfp.py:155-165).  MXFP4 follows flashinfer's
//           e2m1_and_ufp8sf_scale_to_float (fp4Op.cpp:284-337): scale = f32 bits (u << 23), so
//           u = 0 gives 0 and u = 255 gives inf, value = e2m1 * scale in f32.  NVFP4: value =
//           e2m1 * (f32(e4m3) / global_scale), the convention of the pseudo-quant module the
//           reference imports (absent from the reference tree).
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>

#include "common.cuh"
#include "kernels.h"

namespace emu {
namespace {

__device__ __forceinline__ float load_as_f32(const void* p, int64_t i, int dtype) {
  if (dtype == EMU_DTYPE_F16) return __half2float(static_cast<const __half*>(p)[i]);
  if (dtype == EMU_DTYPE_BF16) return __bfloat162float(static_cast<const __nv_bfloat16*>(p)[i]);
  return static_cast<const float*>(p)[i];
}

__device__ __forceinline__ bool finite_f32(float x) { return (__float_as_uint(x) & 0x7F800000u) != 0x7F800000u; }

constexpr int CMP_THREADS = 256;

__global__ void __launch_bounds__(CMP_THREADS)
compare_kernel(const void* __restrict__ ref, const void* __restrict__ out, int dtype, int64_t n,
               emu_compare_stats* __restrict__ st) {
  unsigned long long cnt = 0;
  long long first = 0x7FFFFFFFFFFFFFFFll;
  float maxd = 0.0f, maxsq = 0.0f;
  double sq = 0.0, rsq = 0.0;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const float r = load_as_f32(ref, i, dtype), o = load_as_f32(out, i, dtype);
    const bool both_nan = (r != r) && (o != o);
    const float d = __fsub_rn(r, o);
    if (!(r == o) && !both_nan) {
      ++cnt;
      first = min(first, (long long)i);
      const float ad = (d != d) ? __int_as_float(0x7F800000) : fabsf(d);
      maxd = fmaxf(maxd, ad);
    }
    const float e2 = __fmul_rn(d, d), r2 = __fmul_rn(r, r);
    if (finite_f32(e2)) {   // nan_to_num(nan=0, posinf=0, neginf=0)
      sq += (double)e2;
      maxsq = fmaxf(maxsq, e2);
    }
    if (finite_f32(r2)) rsq += (double)r2;
  }
  // warp, then block reduction, then one set of atomics per block
  for (int o = 16; o > 0; o >>= 1) {
    cnt += __shfl_xor_sync(0xFFFFFFFFu, cnt, o);
    first = min(first, __shfl_xor_sync(0xFFFFFFFFu, first, o));
    maxd = fmaxf(maxd, __shfl_xor_sync(0xFFFFFFFFu, maxd, o));
    maxsq = fmaxf(maxsq, __shfl_xor_sync(0xFFFFFFFFu, maxsq, o));
    sq += __shfl_xor_sync(0xFFFFFFFFu, sq, o);
    rsq += __shfl_xor_sync(0xFFFFFFFFu, rsq, o);
  }
  __shared__ unsigned long long s_cnt[CMP_THREADS / 32];
  __shared__ long long s_first[CMP_THREADS / 32];
  __shared__ float s_maxd[CMP_THREADS / 32], s_maxsq[CMP_THREADS / 32];
  __shared__ double s_sq[CMP_THREADS / 32], s_rsq[CMP_THREADS / 32];
  const int w = threadIdx.x >> 5;
  if ((threadIdx.x & 31) == 0) {
    s_cnt[w] = cnt; s_first[w] = first; s_maxd[w] = maxd; s_maxsq[w] = maxsq; s_sq[w] = sq; s_rsq[w] = rsq;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int k = 1; k < CMP_THREADS / 32; ++k) {
      cnt += s_cnt[k]; first = min(first, s_first[k]); maxd = fmaxf(maxd, s_maxd[k]);
      maxsq = fmaxf(maxsq, s_maxsq[k]); sq += s_sq[k]; rsq += s_rsq[k];
    }
    if (cnt) {
      atomicAdd(reinterpret_cast<unsigned long long*>(&st->mismatches), cnt);
      atomicMin(reinterpret_cast<long long*>(&st->first_index), first);
      atomicMax(reinterpret_cast<unsigned int*>(&st->max_diff), __float_as_uint(maxd));   // >= 0: bit order
    }
    atomicMax(reinterpret_cast<unsigned int*>(&st->max_sq_error), __float_as_uint(maxsq));
    atomicAdd(&st->sq_error_sum, sq);
    atomicAdd(&st->ref_sq_sum, rsq);
  }
}

__global__ void compare_init_kernel(emu_compare_stats* st, int64_t n) {
  st->mismatches = 0;
  st->first_index = 0x7FFFFFFFFFFFFFFFll;
  st->max_diff = 0.0f;
  st->max_sq_error = 0.0f;
  st->sq_error_sum = 0.0;
  st->ref_sq_sum = 0.0;
  st->numel = n;
}

__global__ void compare_fini_kernel(emu_compare_stats* st) {
  if (st->mismatches == 0) st->first_index = -1;
}

__device__ __forceinline__ float e4m3_to_f32(uint32_t b) {
  bool nan;
  const int32_t v = e4m3_times_512(b, &nan);   // exact multiple of 2^-9
  return nan ? __int_as_float(0x7FC00000) : __fmul_rn((float)v, 0x1p-9f);
}

// one thread per 8 elements (4 packed bytes); groups of 16 / 32 never straddle a thread
__global__ void dequant_kernel(const uint8_t* __restrict__ q, const uint8_t* __restrict__ sf, int64_t rows, int64_t K,
                               int64_t sf_cols, int fmt, const float* __restrict__ gs, float* __restrict__ out) {
  const int64_t n8 = rows * (K / 8);
  const int gsz = fmt == EMU_FMT_NVFP4 ? 16 : 32;
  const float g = (fmt == EMU_FMT_NVFP4) ? *gs : 1.0f;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n8; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / (K / 8), k0 = (i % (K / 8)) * 8;
    const uint32_t b = sf[swz_offset(r, k0 / gsz, sf_cols)];
    const float scale = (fmt == EMU_FMT_NVFP4) ? __fdiv_rn(e4m3_to_f32(b), g) : __uint_as_float(b << 23);
    const uint32_t w = reinterpret_cast<const uint32_t*>(q)[i];
    float v[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const uint32_t code = (w >> (4 * e)) & 0xFu;
      const float mag = __fmul_rn((float)e2m1_twice(code & 7u), 0.5f);
      v[e] = __fmul_rn((code & 8u) ? -mag : mag, scale);   // code 8 is -0, as in the e2m1 table
    }
    float4* dst = reinterpret_cast<float4*>(out + r * K + k0);
    dst[0] = make_float4(v[0], v[1], v[2], v[3]);
    dst[1] = make_float4(v[4], v[5], v[6], v[7]);
  }
}

unsigned grid_for(int64_t n, int threads) {
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  return (unsigned)std::max<int64_t>(1, std::min<int64_t>((n + threads - 1) / threads, (int64_t)sms * 8));
}

}  // namespace

cudaError_t launch_compare_init(emu_compare_stats* stats, int64_t n, cudaStream_t stream) {
  compare_init_kernel<<<1, 1, 0, stream>>>(stats, n);
  return cudaGetLastError();
}

cudaError_t launch_compare_fini(emu_compare_stats* stats, cudaStream_t stream) {
  compare_fini_kernel<<<1, 1, 0, stream>>>(stats);
  return cudaGetLastError();
}

cudaError_t launch_compare(const void* ref, const void* out, int dtype, int64_t n, emu_compare_stats* stats,
                           cudaStream_t stream) {
  compare_init_kernel<<<1, 1, 0, stream>>>(stats, n);
  if (n > 0) compare_kernel<<<grid_for(n, CMP_THREADS), CMP_THREADS, 0, stream>>>(ref, out, dtype, n, stats);
  compare_fini_kernel<<<1, 1, 0, stream>>>(stats);
  return cudaGetLastError();
}

cudaError_t launch_dequant(const uint8_t* q, const uint8_t* sf, int64_t rows, int64_t K, int64_t sf_cols, int fmt,
                           const float* global_scale, float* out, cudaStream_t stream) {
  const int64_t n8 = rows * (K / 8);
  if (n8 > 0) dequant_kernel<<<grid_for(n8, 256), 256, 0, stream>>>(q, sf, rows, K, sf_cols, fmt, global_scale, out);
  return cudaGetLastError();
}

}  // namespace emu
