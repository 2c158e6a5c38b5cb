// FP4 quantisers (NVFP4: per-16 E4M3 scale + f32 global scale; MXFP4: per-32 UE8M0 scale) and the
// NVFP4 global-scale / alpha computation, on sm_100a.
//
// The recipe is the one the reference's quant_fn calls (gemm_compare/backends/nvfp.py:173-196,
// mxfp.py:198-217): flashinfer fp4_quantize, whose device arithmetic is in
// flashinfer/data/csrc/nv_internal/tensorrt_llm/kernels/quantization_utils.cuh:294-366:
//   vecMax   = max |x| over the block, taken in the input type (fp16 / bf16) with hmax2,
//   NVFP4:   SF = e4m3_satfinite(gs * (vecMax * rcp(6)));  outScale = rcp(f32(SF) * rcp(gs))
//   MXFP4:   v = vecMax * rcp(6); SF = ue8m0(v) rounded toward +inf, satfinite;
//            outScale = SF==0 ? 1 : 2^(127-SF)
//   q        = cvt.rn.satfinite.e2m1x2(x * outScale), low nibble = even element
// where rcp is the hardware approximate reciprocal rcp.approx.ftz.f32 and outScale is 0 when
// vecMax is 0.  The same PTX instructions are issued here so the bytes match bit for bit.
// flashinfer builds those kernels with fast math, so f32 subnormals are flushed to (signed) zero
// in its comparisons, products and exp2; this library is built without (the emulation kernels need
// subnormals), so the flushes that change a byte are written out (ftz() below): the block maximum
// and its product with rcp(6) (a bf16 block of subnormals: outScale 0, signed-zero codes), bf16
// input elements before scaling, and MXFP4's outScale 2^(127 - SF), subnormal for SF >= 254 (a block
// holding an infinity: outScale 0, so inf * 0 = NaN -> code 0x7 as flashinfer writes).
// Layout: one thread per 16 input elements (32 bytes, two 16-byte loads); for MXFP4 two adjacent
// lanes share a scale and combine their maxima with one shuffle.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>
#include <type_traits>

#include "common.cuh"
#include "kernels.h"

namespace emu {
namespace {

__device__ __forceinline__ float rcp_approx_ftz(float a) {
  float b;
  asm volatile("rcp.approx.ftz.f32 %0, %1;\n" : "=f"(b) : "f"(a));
  return b;
}

// 8 floats -> 8 e2m1 codes in one 32-bit word (element 2i in the low nibble of byte i).
__device__ __forceinline__ uint32_t f32x8_to_e2m1(const float (&v)[8]) {
  uint32_t val;
  asm volatile(
      "{\n"
      ".reg .b8 byte0, byte1, byte2, byte3;\n"
      "cvt.rn.satfinite.e2m1x2.f32 byte0, %2, %1;\n"
      "cvt.rn.satfinite.e2m1x2.f32 byte1, %4, %3;\n"
      "cvt.rn.satfinite.e2m1x2.f32 byte2, %6, %5;\n"
      "cvt.rn.satfinite.e2m1x2.f32 byte3, %8, %7;\n"
      "mov.b32 %0, {byte0, byte1, byte2, byte3};\n"
      "}"
      : "=r"(val)
      : "f"(v[0]), "f"(v[1]), "f"(v[2]), "f"(v[3]), "f"(v[4]), "f"(v[5]), "f"(v[6]), "f"(v[7]));
  return val;
}

template <typename T> struct Vec2;
template <> struct Vec2<__half> {
  using type = __half2;
  static __device__ __forceinline__ float2 to_f2(type v) { return __half22float2(v); }
};
template <> struct Vec2<__nv_bfloat16> {
  using type = __nv_bfloat162;
  static __device__ __forceinline__ float2 to_f2(type v) { return __bfloat1622float2(v); }
};

// 2^(127 - e) as f32 bits for e in [1, 255] (exact, subnormal for e >= 254).
__device__ __forceinline__ float pow2_127_minus(uint32_t e) {
  if (e >= 254u) return 0.0f;   // 2^-127 and below: subnormal, flushed as in flashinfer's build
  return __uint_as_float((254u - e) << 23);
}

// f32 subnormal -> signed zero (fast-math flush-to-zero); NaN and inf pass
__device__ __forceinline__ float ftz(float x) { return fabsf(x) < 1.17549435e-38f ? copysignf(0.0f, x) : x; }

template <typename T, int SF_VEC>
__global__ void __launch_bounds__(256)
quant_fp4_kernel(const T* __restrict__ x, int64_t M, int64_t K, const float* __restrict__ gsp,
                 uint8_t* __restrict__ q, uint8_t* __restrict__ sf) {
  using V2 = typename Vec2<T>::type;
  constexpr int TPS = SF_VEC / 16;               // threads per scale (1 NVFP4, 2 MXFP4)
  const int64_t nchunks = K / 16;                 // 16-element chunks with data
  const int64_t sf_cols = (K / SF_VEC + 3) / 4 * 4;
  const int64_t nchunks_sf = sf_cols * TPS;       // chunks including scale padding
  const int64_t rows_sf = (M + 127) / 128 * 128;
  const int64_t chunk_loop = (nchunks_sf + 31) / 32 * 32;  // whole warps take part in shuffles
  const float gs = (SF_VEC == 16 && gsp) ? *gsp : 1.0f;

  for (int64_t row = blockIdx.x; row < rows_sf; row += gridDim.x) {
    for (int64_t c = threadIdx.x; c < chunk_loop; c += blockDim.x) {
      const bool has_data = row < M && c < nchunks;
      V2 e[8];
      if (has_data) {
        const uint4* src = reinterpret_cast<const uint4*>(x + row * K + c * 16);
        const uint4 w0 = src[0], w1 = src[1];
        const uint32_t w[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
        for (int i = 0; i < 8; ++i) e[i] = *reinterpret_cast<const V2*>(&w[i]);
      } else {
        const uint32_t zero = 0u;
#pragma unroll
        for (int i = 0; i < 8; ++i) e[i] = *reinterpret_cast<const V2*>(&zero);
      }
      V2 local = __habs2(e[0]);
#pragma unroll
      for (int i = 1; i < 8; ++i) local = __hmax2(local, __habs2(e[i]));
      if (TPS == 2) {
        uint32_t lb = *reinterpret_cast<uint32_t*>(&local);
        uint32_t ob = __shfl_xor_sync(0xFFFFFFFFu, lb, 1);
        local = __hmax2(*reinterpret_cast<V2*>(&ob), local);
      }
      float vecMax = ftz((float)((local.x > local.y) ? local.x : local.y));

      uint8_t sfbyte;
      float outScale;
      if (SF_VEC == 16) {
        float sfv = ftz(gs * ftz(vecMax * rcp_approx_ftz(6.0f)));
        __nv_fp8_e4m3 t = __nv_fp8_e4m3(sfv);
        sfbyte = t.__x;
        sfv = static_cast<float>(t);
        outScale = vecMax != 0.0f ? rcp_approx_ftz(sfv * rcp_approx_ftz(gs)) : 0.0f;
      } else {
        vecMax = ftz(vecMax * rcp_approx_ftz(6.0f));
        sfbyte = __nv_cvt_float_to_e8m0(vecMax, __NV_SATFINITE, cudaRoundPosInf);
        outScale = vecMax != 0.0f ? (sfbyte == 0 ? 1.0f : pow2_127_minus(sfbyte)) : 0.0f;
      }

      if (has_data) {
        float f[16];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          float2 p = Vec2<T>::to_f2(e[i]);
          if constexpr (!std::is_same<T, __half>::value) p = make_float2(ftz(p.x), ftz(p.y));   // fp16 has none
          f[2 * i] = __fmul_rn(p.x, outScale);
          f[2 * i + 1] = __fmul_rn(p.y, outScale);
        }
        const float lo8[8] = {f[0], f[1], f[2], f[3], f[4], f[5], f[6], f[7]};
        const float hi8[8] = {f[8], f[9], f[10], f[11], f[12], f[13], f[14], f[15]};
        uint2 packed = make_uint2(f32x8_to_e2m1(lo8), f32x8_to_e2m1(hi8));
        *reinterpret_cast<uint2*>(q + row * (K / 2) + c * 8) = packed;
      }
      if (row < rows_sf && c < nchunks_sf && (c % TPS) == 0) {
        sf[swz_offset(row, c / TPS, sf_cols)] = has_data ? sfbyte : (uint8_t)0;
      }
    }
  }
}

// max |x| as float bits (non-negative floats order like their bit patterns; NaN sorts above inf,
// so a NaN anywhere wins, as torch.max propagates NaN).  The same holds for the 16-bit patterns of
// fp16 / bf16 magnitudes, so the maximum is taken on those, two per 32-bit lane (16-byte loads), and
// converted to float once per thread (the conversion is monotonic, so the result is the same).
template <typename T>
__device__ __forceinline__ unsigned half_bits_to_float_bits(unsigned h) {
  if constexpr (std::is_same<T, __half>::value) return __float_as_uint(__half2float(__ushort_as_half((unsigned short)h)));
  else return h << 16;
}

// amax of A (blockIdx.y == 0) and B (blockIdx.y == 1) in one launch, as the bits of a non-negative
// float (atomicMax on unsigned orders them like the values): 16-bit magnitudes compared two at a time,
// four 16-byte loads in flight per thread, the unaligned remainder element by element.
template <typename T>
__global__ void amax_bits_kernel(const T* __restrict__ xa, int64_t na, const T* __restrict__ xb, int64_t nb,
                                 unsigned* __restrict__ out_a, unsigned* __restrict__ out_b) {
  const T* x = blockIdx.y ? xb : xa;
  const int64_t n = blockIdx.y ? nb : na;
  unsigned* out = blockIdx.y ? out_b : out_a;
  unsigned m2 = 0;   // two 16-bit magnitude maxima
  const int64_t n8 = (reinterpret_cast<uintptr_t>(x) & 15) == 0 ? n / 8 : 0;
  const uint4* x8 = reinterpret_cast<const uint4*>(x);
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  for (; i + 3 * stride < n8; i += 4 * stride) {
    uint4 w[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) w[u] = __ldg(x8 + i + u * stride);
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      m2 = __vmaxu2(m2, w[u].x & 0x7FFF7FFFu);
      m2 = __vmaxu2(m2, w[u].y & 0x7FFF7FFFu);
      m2 = __vmaxu2(m2, w[u].z & 0x7FFF7FFFu);
      m2 = __vmaxu2(m2, w[u].w & 0x7FFF7FFFu);
    }
  }
  for (; i < n8; i += stride) {
    const uint4 w = __ldg(x8 + i);
    m2 = __vmaxu2(m2, w.x & 0x7FFF7FFFu);
    m2 = __vmaxu2(m2, w.y & 0x7FFF7FFFu);
    m2 = __vmaxu2(m2, w.z & 0x7FFF7FFFu);
    m2 = __vmaxu2(m2, w.w & 0x7FFF7FFFu);
  }
  const unsigned short* xs = reinterpret_cast<const unsigned short*>(x);
  for (int64_t j = n8 * 8 + blockIdx.x * (int64_t)blockDim.x + threadIdx.x; j < n; j += stride)
    m2 = __vmaxu2(m2, (unsigned)xs[j] & 0x7FFFu);
  unsigned m = half_bits_to_float_bits<T>(max(m2 & 0xFFFFu, m2 >> 16));
  for (int o = 16; o > 0; o >>= 1) m = max(m, __shfl_xor_sync(0xFFFFFFFFu, m, o));
  if ((threadIdx.x & 31) == 0) atomicMax(out, m);
}

// gs = f32(2688.0 / (amax > 0 ? amax : 1.0)) and alpha = f32(1 / max(gs_a * gs_b, 1e-8)), all in
// double like the reference's Python floats (gemm_compare/backends/nvfp.py:24-27, 176).
// The amax words may be the gs words themselves (read before written).
__global__ void global_scales_finalize(const unsigned* amax_a, const unsigned* amax_b, float* gs_a, float* gs_b,
                                       float* alpha) {
  const float aa = __uint_as_float(*amax_a);
  const float ab = __uint_as_float(*amax_b);
  asm volatile("" ::: "memory");   // both words are read before either output (which may alias them) is written
  const double da = aa > 0.0f ? (double)aa : 1.0;
  const double db = ab > 0.0f ? (double)ab : 1.0;
  const float ga = __double2float_rn(__ddiv_rn(2688.0, da));
  const float gb = __double2float_rn(__ddiv_rn(2688.0, db));
  *gs_a = ga;
  *gs_b = gb;
  if (alpha) {
    const double p = __dmul_rn((double)ga, (double)gb);
    const double mx = (1e-8 > p) ? 1e-8 : p;
    *alpha = __double2float_rn(__ddiv_rn(1.0, mx));
  }
}

template <int SF_VEC>
cudaError_t launch_quant_t(const void* x, int dtype, int64_t M, int64_t K, const float* gs, uint8_t* q,
                           uint8_t* sf, cudaStream_t stream) {
  const int64_t rows_sf = (M + 127) / 128 * 128;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const unsigned grid = (unsigned)(rows_sf < (int64_t)sms * 8 ? rows_sf : (int64_t)sms * 8);
  if (dtype == EMU_DTYPE_F16)
    quant_fp4_kernel<__half, SF_VEC><<<grid, 256, 0, stream>>>(static_cast<const __half*>(x), M, K, gs, q, sf);
  else
    quant_fp4_kernel<__nv_bfloat16, SF_VEC><<<grid, 256, 0, stream>>>(static_cast<const __nv_bfloat16*>(x), M, K, gs, q, sf);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_quant(int sf_vec, const void* x, int dtype, int64_t M, int64_t K, const float* gs,
                         uint8_t* q, uint8_t* sf, cudaStream_t stream) {
  return sf_vec == 16 ? launch_quant_t<16>(x, dtype, M, K, gs, q, sf, stream)
                      : launch_quant_t<32>(x, dtype, M, K, gs, q, sf, stream);
}

cudaError_t launch_amax(const void* a, int64_t a_numel, const void* b, int64_t b_numel, int dtype, unsigned* amax_a,
                        unsigned* amax_b, cudaStream_t stream) {
  cudaError_t err = cudaMemsetAsync(amax_a, 0, sizeof(unsigned), stream);
  if (err == cudaSuccess) err = cudaMemsetAsync(amax_b, 0, sizeof(unsigned), stream);
  if (err != cudaSuccess) return err;
  // one wave: 4 CTAs of 256 threads per SM and tensor, each thread four 16-byte loads per step
  const int64_t n_max = std::max(a_numel, b_numel);
  int sms = 148;
  {
    int dev = 0;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  }
  const dim3 grid((unsigned)std::min<int64_t>(std::max<int64_t>((n_max / 8 + 1023) / 1024, 1), (int64_t)sms * 4), 2);
  if (dtype == EMU_DTYPE_F16) {
    amax_bits_kernel<__half><<<grid, 256, 0, stream>>>(static_cast<const __half*>(a), a_numel, static_cast<const __half*>(b),
                                                      b_numel, amax_a, amax_b);
  } else {
    amax_bits_kernel<__nv_bfloat16><<<grid, 256, 0, stream>>>(
        static_cast<const __nv_bfloat16*>(a), a_numel, static_cast<const __nv_bfloat16*>(b), b_numel, amax_a, amax_b);
  }
  return cudaGetLastError();
}

cudaError_t launch_scales_from_amax(const unsigned* amax_a, const unsigned* amax_b, float* gs_a, float* gs_b,
                                    float* alpha, cudaStream_t stream) {
  global_scales_finalize<<<1, 1, 0, stream>>>(amax_a, amax_b, gs_a, gs_b, alpha);
  return cudaGetLastError();
}

cudaError_t launch_global_scales(const void* a, int64_t a_numel, const void* b, int64_t b_numel, int dtype,
                                 float* gs_a, float* gs_b, float* alpha, cudaStream_t stream) {
  // the amax words live in the gs outputs until the finalize step overwrites them
  unsigned* wa = reinterpret_cast<unsigned*>(gs_a);
  unsigned* wb = reinterpret_cast<unsigned*>(gs_b);
  cudaError_t err = launch_amax(a, a_numel, b, b_numel, dtype, wa, wb, stream);
  return err != cudaSuccess ? err : launch_scales_from_amax(wa, wb, gs_a, gs_b, alpha, stream);
}

}  // namespace emu
