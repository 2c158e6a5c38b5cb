// Shared device helpers for the emulated FP4 GEMM and the FP4 quantisers (sm_100a).
//
// Numerics follow the reference emulators exactly (nvfp_cpp_emul/.../nvfp_emulation.cpp,
// mxfp_cpp_emul/.../mxfp_emulation.cpp, search/emulation/core.py).  This file must be compiled
// without --use_fast_math / -ftz=true: f32/f64 subnormals are significant in the reference (CPU
// PyTorch does not flush them), and every float operation below is an explicitly rounded
// intrinsic so that no FMA contraction can change a result.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include "../../include/emugen.h"

namespace emu {

// e2m1 code (low 3 bits) -> 2*|value| = {0, 1, 2, 3, 4, 6, 8, 12} (values 0, .5, 1, 1.5, 2, 3, 4, 6);
// bit 3 is the sign.  Reference table: nvfp_emulation.cpp:7-13.
__host__ __device__ __forceinline__ int e2m1_twice(uint32_t code) {
  const uint32_t mag = code & 7u;
  // 0,1,2,3,4,6,8,12 packed as nibbles of 0xC8643210
  const int v = (int)((0xC8643210u >> (4u * mag)) & 0xFu);
  return (code & 8u) ? -v : v;
}

// Four e2m1 codes (bits 0-15, code i in bits 4i..4i+3) -> four int8 "2x" values, byte i = code i.
// Two byte permutes look the magnitude up in a positive and a negated table, a third turns each sign
// bit into a byte mask that picks between them (code 8, negative zero, gives 0).
__device__ __forceinline__ uint32_t e2m1x4_to_int8x4(uint32_t codes) {
  const uint32_t sel = codes & 0x7777u;
  const uint32_t sel_sign = (codes >> 3) & 0x1111u;
  uint32_t pos, neg, msk;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(pos) : "r"(0x03020100u), "r"(0x0C080604u), "r"(sel));
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(neg) : "r"(0xFDFEFF00u), "r"(0xF4F8FAFCu), "r"(sel));
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(msk) : "r"(0x0000FF00u), "r"(0u), "r"(sel_sign));
  return (pos & ~msk) | (neg & msk);
}

// Byte offset of scale (row r, scale column c) in a swizzled 128x4 buffer whose column count is
// cols_pad (a multiple of 4).  Reference un-swizzle: nvfp_emulation.cpp:24-26
// (reshape (m_tiles, k_tiles, 32, 4, 4).transpose(1, 3)).
__host__ __device__ __forceinline__ int64_t swz_offset(int64_t r, int64_t c, int64_t cols_pad) {
  return (r >> 7) * (cols_pad >> 2) * 512 + (c >> 2) * 512 + (r & 31) * 16 + ((r & 127) >> 5) * 4 +
         (c & 3);
}

// E4M3 (fn: no inf; 0x7F / 0xFF are NaN) as an exact integer multiple of 2^-9, sign included.
// |value| <= 448 -> |result| <= 229376.  *is_nan set for the NaN codes (result 0).
__host__ __device__ __forceinline__ int32_t e4m3_times_512(uint32_t x, bool* is_nan) {
  const uint32_t e = (x >> 3) & 0xFu, m = x & 7u;
  *is_nan = (e == 15u && m == 7u);
  int32_t mag;
  if (e == 0u) mag = (int32_t)m;                       // subnormal: m * 2^-9
  else mag = (int32_t)((8u + m) << (e - 1u));          // (8+m) * 2^(e-10) * 2^9
  if (*is_nan) mag = 0;
  return (x & 0x80u) ? -mag : mag;
}

// UE8M0 scale u -> exp2(u - 127 - 2) as f64: the reference's f32 exp2(u-127) (mxfp_emulation.cpp:31-33,
// 255 -> +inf, 0 -> 2^-127) with the stage-1 partial's 1/4 unit folded in.  Exact.
__device__ __forceinline__ double ue8m0_quarter_f64(uint32_t u) {
  if (u == 255u) return __longlong_as_double(0x7FF0000000000000ll);
  // 2^(u - 129): f64 exponent field u - 129 + 1023 = u + 894, always a normal f64
  return __longlong_as_double((long long)(u + 894u) << 52);
}

// Stage 1 rounding: p4 = 4 * (exact group dot product), an integer with |p4| <= 4608.  The
// reference rounds the exact sum once to fp16 (einsum in fp16 with f32 accumulation,
// nvfp_emulation.cpp:77-86); fp16 keeps 11 significant bits, so |p4| < 2048 is exact and above
// that the value is rounded to nearest-even on a grid of 2 (|p4| < 4096) or 4 (|p4| < 8192).
__device__ __forceinline__ int round_p4_to_fp16_grid(int p4) {
  const unsigned a = (unsigned)(p4 < 0 ? -p4 : p4);
  if (a < 2048u) return p4;
  const unsigned sh = (a >= 4096u) ? 2u : 1u;
  const unsigned half = 1u << (sh - 1u);
  unsigned q = a >> sh;
  const unsigned r = a & ((1u << sh) - 1u);
  q += (r > half || (r == half && (q & 1u))) ? 1u : 0u;
  const int res = (int)(q << sh);
  return p4 < 0 ? -res : res;
}

// f64 -> f32 with the reference's rounding.  RNE: the plain cast.  RZ: the reference casts with RNE
// and steps one ulp toward zero when the magnitude grew (nvfp_emulation.cpp:42-50); for every f64
// input (subnormal results, overflow to FLT_MAX, inf, NaN included) that equals IEEE round-toward-
// zero, which cvt.rz.f32.f64 computes directly.
__device__ __forceinline__ float round_f64_to_f32(double x, int mode) {
  return mode == EMU_RZ ? __double2float_rz(x) : __double2float_rn(x);
}

// The output element as a float: y after the output dtype's rounding (what store_output stores).
__device__ __forceinline__ float output_value(float y, int out_mode) {
  if (out_mode == EMU_OUT_F32) return y;
  const __half h = __float2half_rn(y);
  if (out_mode == EMU_OUT_BF16_VIA_F16) return __bfloat162float(__float2bfloat16_rn(__half2float(h)));
  return __half2float(h);
}

// An element of a [*] fp16 / bf16 (EMU_OUT_BF16_VIA_F16) / f32 tensor as a float.
__device__ __forceinline__ float load_output(const void* p, int64_t i, int out_mode) {
  if (out_mode == EMU_OUT_F32) return static_cast<const float*>(p)[i];
  const uint16_t b = static_cast<const uint16_t*>(p)[i];
  if (out_mode == EMU_OUT_BF16_VIA_F16) return __uint_as_float((uint32_t)b << 16);
  return __half2float(__ushort_as_half(b));
}

// Final output conversion: y is the f32 result (already multiplied by alpha).
__device__ __forceinline__ void store_output(void* out, int64_t idx, float y, int out_mode) {
  if (out_mode == EMU_OUT_F32) {
    static_cast<float*>(out)[idx] = y;
    return;
  }
  __half h = __float2half_rn(y);
  uint16_t bits = __half_as_ushort(h);
  if (out_mode == EMU_OUT_BF16_VIA_F16) bits = __bfloat16_as_ushort(__float2bfloat16_rn(__half2float(h)));
  static_cast<uint16_t*>(out)[idx] = bits;
}

}  // namespace emu
