// Emulated scaled FP4 GEMM under an accumulator model with alignment widths and summation order
// (the parameters the reference keeps as w_stage3 / w_stage4 without using them,
// search/emulation/core.py:31-38, config.py:16-19).  CUDA cores; for parameter sweeps.
//
// Stages 1-2 are the reference's (exact group dot, fp16 rounding, scale multiply).  Then, with
// W3 = align3, W4 = align4 and rounding RZ (truncate) or RNE for the aligned addends:
//   stage 3  W3 > 0: the block's addends v_g are aligned to the largest exponent E among the finite
//            nonzero ones -- each becomes round(v_g / q) * q, q = 2^(E - W3 + 1) -- and summed
//            exactly; a non-finite addend leaves the plain f64 sum.  W3 = 0: f64 sum from +0.0 in
//            the given order (0 left to right = the reference, 1 right to left, 2 pairwise tree).
//   stage 4  W4 > 0: acc and s_b aligned the same way to the larger exponent and summed exactly
//            (the first block aligns s_0 alone); W4 = 0: f64(acc) + s_b.  Then R4 (cvt.rz/rn) to
//            f32.  A single-block GEMM rounds s_0 with R3, as the reference does.
// With every parameter 0 this is the reference model; the C ABI routes that case to emu_gemm.
// Exactness: |round(v / q)| <= 2^W3 and at most 16 addends (W3 <= 46), two addends for stage 4
// (W4 <= 52), so every aligned sum is an integer below 2^53 and exact in f64.
#include <cuda_runtime.h>
#include <stdint.h>

#include <type_traits>

#include "common.cuh"
#include "kernels.h"

namespace emu {
namespace {

constexpr int MBM = 32, MBN = 32, MKC = 64;        // CTA tile and K chunk (elements)
constexpr int MTHREADS = 256;                       // 16 x 16 threads, 2 x 2 outputs each
constexpr int MROW_WORDS = MKC / 4 + 4;
constexpr int MAX_WR = 16;

__device__ __forceinline__ uint4 unpack16m(uint2 w) {
  return make_uint4(e2m1x4_to_int8x4(w.x & 0xFFFFu), e2m1x4_to_int8x4(w.x >> 16), e2m1x4_to_int8x4(w.y & 0xFFFFu),
                    e2m1x4_to_int8x4(w.y >> 16));
}

__device__ __forceinline__ bool finite_d(double x) {
  return ((__double2hiint(x) >> 20) & 0x7FF) != 0x7FF;
}

// floor(log2 |x|) for a finite nonzero double
__device__ __forceinline__ int exp_of(double x) { return ilogb(x); }

// x / 2^eq rounded to an integer, RZ (truncate) or RNE; the quotient is below 2^62 in magnitude
__device__ __forceinline__ long long to_grid(double x, int eq, int rm) {
  const double y = scalbn(x, -eq);
  return __double2ll_rn(rm == EMU_RZ ? trunc(y) : rint(y));
}

// floor(log2 |x|) for a finite nonzero double from its exponent field (subnormals through ilogb)
__device__ __forceinline__ int exp_bits(double x) {
  const int f = (__double2hiint(x) >> 20) & 0x7FF;
  return f ? f - 1023 : ilogb(x);
}

__device__ __forceinline__ double pow2(int e) {   // exact 2^e for e in [-1022, 1023]
  return __longlong_as_double((long long)(e + 1023) << 52);
}

// x * 2^e exactly as scalbn, by one multiply when 2^e is a normal double
__device__ __forceinline__ double scale2(double x, int e) {
  return (e >= -1022 && e <= 1023) ? x * pow2(e) : scalbn(x, e);
}

// x / 2^eq rounded to an integer, RZ or RNE, by a power-of-two multiply and one conversion (the
// quotient is below 2^62 in magnitude; a quotient too small to be exact rounds to 0 either way)
__device__ __forceinline__ long long to_grid_fast(double x, int eq, int rm) {
  const double y = scale2(x, -eq);
  return rm == EMU_RZ ? __double2ll_rz(y) : __double2ll_rn(y);
}

// stage 3 of the model for a compile-time block of WR (a power of two) addends, held in registers
template <int WR>
__device__ __forceinline__ double stage3_model_t(const double (&v)[WR], const ModelArgs& ma) {
  bool finite = true;
#pragma unroll
  for (int i = 0; i < WR; ++i) finite = finite && finite_d(v[i]);
  if (ma.align3 > 0 && finite) {
    bool have = false;
    int E = 0;
#pragma unroll
    for (int i = 0; i < WR; ++i)
      if (v[i] != 0.0) { const int e = exp_bits(v[i]); E = have ? max(E, e) : e; have = true; }
    if (!have) return 0.0;
    const int eq = E - ma.align3 + 1;
    long long m = 0;
#pragma unroll
    for (int i = 0; i < WR; ++i) m += to_grid_fast(v[i], eq, ma.align_rounding);
    return __dadd_rn(scale2(__ll2double_rn(m), eq), 0.0);
  }
  if (ma.order == 1) {
    double s = 0.0;
#pragma unroll
    for (int i = WR - 1; i >= 0; --i) s = __dadd_rn(s, v[i]);
    return s;
  }
  if (ma.order == 2) {
    double t[WR];
#pragma unroll
    for (int i = 0; i < WR; ++i) t[i] = v[i];
#pragma unroll
    for (int k = WR; k > 1; k >>= 1)
#pragma unroll
      for (int i = 0; i < k / 2; ++i) t[i] = __dadd_rn(t[2 * i], t[2 * i + 1]);
    return __dadd_rn(0.0, t[0]);
  }
  double s = 0.0;
#pragma unroll
  for (int i = 0; i < WR; ++i) s = __dadd_rn(s, v[i]);
  return s;
}

__device__ __forceinline__ double stage4_model_fast(double acc, double s, const ModelArgs& ma) {
  if (ma.align4 <= 0 || !finite_d(acc) || !finite_d(s)) return __dadd_rn(acc, s);
  bool have = false;
  int E = 0;
  if (acc != 0.0) { E = exp_bits(acc); have = true; }
  if (s != 0.0) { const int e = exp_bits(s); E = have ? max(E, e) : e; have = true; }
  if (!have) return __dadd_rn(acc, s);
  const int eq = E - ma.align4 + 1;
  const long long m = to_grid_fast(acc, eq, ma.align_rounding) + to_grid_fast(s, eq, ma.align_rounding);
  return __dadd_rn(scale2(__ll2double_rn(m), eq), 0.0);
}

__device__ double stage3_model(const double* v, int n, const ModelArgs& ma) {
  bool finite = true;
  for (int i = 0; i < n; ++i) finite = finite && finite_d(v[i]);
  if (ma.align3 > 0 && finite) {
    bool have = false;
    int E = 0;
    for (int i = 0; i < n; ++i)
      if (v[i] != 0.0) { const int e = exp_of(v[i]); E = have ? max(E, e) : e; have = true; }
    if (!have) return 0.0;
    const int eq = E - ma.align3 + 1;
    long long m = 0;
    for (int i = 0; i < n; ++i) m += to_grid(v[i], eq, ma.align_rounding);
    return __dadd_rn(scalbn(__ll2double_rn(m), eq), 0.0);
  }
  if (ma.order == 1) {
    double s = 0.0;
    for (int i = n - 1; i >= 0; --i) s = __dadd_rn(s, v[i]);
    return s;
  }
  if (ma.order == 2) {
    double t[MAX_WR];
    int k = n;
    for (int i = 0; i < n; ++i) t[i] = v[i];
    while (k > 1) {
      int h = 0;
      for (int i = 0; i + 1 < k; i += 2) t[h++] = __dadd_rn(t[i], t[i + 1]);
      if (k & 1) t[h++] = t[k - 1];
      k = h;
    }
    return __dadd_rn(0.0, t[0]);
  }
  double s = 0.0;
  for (int i = 0; i < n; ++i) s = __dadd_rn(s, v[i]);
  return s;
}

__device__ double stage4_model_sum(double acc, double s, const ModelArgs& ma) {
  if (ma.align4 <= 0 || !finite_d(acc) || !finite_d(s)) return __dadd_rn(acc, s);
  bool have = false;
  int E = 0;
  if (acc != 0.0) { E = exp_of(acc); have = true; }
  if (s != 0.0) { const int e = exp_of(s); E = have ? max(E, e) : e; have = true; }
  if (!have) return __dadd_rn(acc, s);
  const int eq = E - ma.align4 + 1;
  const long long m = to_grid(acc, eq, ma.align_rounding) + to_grid(s, eq, ma.align_rounding);
  return __dadd_rn(scalbn(__ll2double_rn(m), eq), 0.0);
}

template <int FMT>
__global__ void __launch_bounds__(MTHREADS)
emul_gemm_model_kernel(const uint8_t* __restrict__ A, const uint8_t* __restrict__ B, const uint8_t* __restrict__ SA,
                       const uint8_t* __restrict__ SB, int64_t M, int64_t N, int64_t K, int64_t sa_cols,
                       int64_t sb_cols, const float* __restrict__ alpha, GemmArgs args, ModelArgs ma,
                       void* __restrict__ out) {
  constexpr int GS = (FMT == EMU_FMT_NVFP4) ? 16 : 32;
  constexpr int GPC = MKC / GS;
  constexpr int WPG = GS / 4;
  __shared__ __align__(16) uint32_t As[MBM * MROW_WORDS];
  __shared__ __align__(16) uint32_t Bs[MBN * MROW_WORDS];

  const int tid = threadIdx.x;
  const int tx = tid & 15, ty = tid >> 4;
  const int64_t m0 = (int64_t)blockIdx.x * MBM, n0 = (int64_t)blockIdx.y * MBN;
  const int64_t G = K / GS;
  const int wr = args.w_reduce;
  const int64_t nb = G / wr;
  const int64_t kbytes = K / 2;

  double vbuf[4][MAX_WR];
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
  bool nan_out[4] = {false, false, false, false};
  int gi = 0;
  int64_t blk = 0;

  for (int64_t k0 = 0; k0 < K; k0 += MKC) {
    {
      // 32 rows x 32 bytes per operand: threads 0..127 load A, 128..255 load B, 8 bytes each
      const int t = tid & 127, r = t >> 2, part = t & 3;
      const int64_t kb = k0 / 2 + part * 8;
      uint2 w = make_uint2(0, 0);
      if (tid < 128) {
        if (m0 + r < M && kb < kbytes) w = *reinterpret_cast<const uint2*>(A + (m0 + r) * kbytes + kb);
        *reinterpret_cast<uint4*>(&As[r * MROW_WORDS + part * 4]) = unpack16m(w);
      } else {
        if (n0 + r < N && kb < kbytes) w = *reinterpret_cast<const uint2*>(B + (n0 + r) * kbytes + kb);
        *reinterpret_cast<uint4*>(&Bs[r * MROW_WORDS + part * 4]) = unpack16m(w);
      }
    }
    __syncthreads();
    const int ngroups = (K - k0) / GS < GPC ? (int)((K - k0) / GS) : GPC;
    for (int gl = 0; gl < ngroups; ++gl) {
      const int64_t g = k0 / GS + gl;
#pragma unroll
      for (int o = 0; o < 4; ++o) {
        const int i = o >> 1, j = o & 1;
        const int64_t r = m0 + ty + 16 * i, c = n0 + tx + 16 * j;
        const uint32_t ba = (r < M) ? SA[swz_offset(r, g, sa_cols)] : 0u;
        const uint32_t bb = (c < N) ? SB[swz_offset(c, g, sb_cols)] : 0u;
        int p4 = 0;
#pragma unroll
        for (int w = 0; w < WPG; ++w)
          p4 = __dp4a((int)As[(ty + 16 * i) * MROW_WORDS + gl * WPG + w], (int)Bs[(tx + 16 * j) * MROW_WORDS + gl * WPG + w],
                      p4);
        const int p = round_p4_to_fp16_grid(p4);
        double v;
        if (FMT == EMU_FMT_NVFP4) {
          bool na, nbn;
          const int32_t sa = e4m3_times_512(ba, &na), sb = e4m3_times_512(bb, &nbn);
          nan_out[o] |= na || nbn;
          v = __ll2double_rn((long long)(p * sa) * (long long)sb) * 0x1p-20;   // p * sa * sb, exact
        } else {
          const double c4 = __dmul_rn(ue8m0_quarter_f64(ba), ue8m0_quarter_f64(bb) * 4.0);
          v = __dmul_rn((double)p, c4);
        }
        vbuf[o][gi] = v;
      }
      if (++gi == wr) {
        gi = 0;
#pragma unroll
        for (int o = 0; o < 4; ++o) {
          const double s = stage3_model(vbuf[o], wr, ma);
          if (nb == 1) acc[o] = round_f64_to_f32(s, args.stage3_rounding);
          else acc[o] = round_f64_to_f32(stage4_model_sum(blk == 0 ? 0.0 : (double)acc[o], s, ma),
                                         args.stage4_rounding);
        }
        ++blk;
      }
    }
    __syncthreads();
  }
  const float al = alpha ? *alpha : 1.0f;
#pragma unroll
  for (int o = 0; o < 4; ++o) {
    const int i = o >> 1, j = o & 1;
    const int64_t r = m0 + ty + 16 * i, c = n0 + tx + 16 * j;
    if (r >= M || c >= N) continue;
    float y = alpha ? __fmul_rn(acc[o], al) : acc[o];
    if (FMT == EMU_FMT_NVFP4 && nan_out[o]) y = __int_as_float(0x7FFFFFFF);
    store_output(out, r * N + c, y, args.out_mode);
  }
}

// w_reduce a power of two (WR): K chunks of max(64, WR * GS) elements hold whole blocks, so a block's
// WR addends per output sit in registers (compile-time indices) and the model runs on them there.
// Same arithmetic and order as emul_gemm_model_kernel.
template <int FMT, int WR>
__global__ void __launch_bounds__(MTHREADS)
emul_gemm_model_wr_kernel(const uint8_t* __restrict__ A, const uint8_t* __restrict__ B, const uint8_t* __restrict__ SA,
                          const uint8_t* __restrict__ SB, int64_t M, int64_t N, int64_t K, int64_t sa_cols,
                          int64_t sb_cols, const float* __restrict__ alpha, GemmArgs args, ModelArgs ma,
                          void* __restrict__ out) {
  constexpr int GS = (FMT == EMU_FMT_NVFP4) ? 16 : 32;
  constexpr int KC = WR * GS > MKC ? WR * GS : MKC;      // elements per chunk, a multiple of the block
  constexpr int GPC = KC / GS;
  constexpr int WPG = GS / 4;
  constexpr int ROW_WORDS = KC / 4 + 4;
  constexpr int PARTS = KC / 16;                          // 8-byte pieces per row of a chunk
  __shared__ __align__(16) uint32_t As[MBM * ROW_WORDS];
  __shared__ __align__(16) uint32_t Bs[MBN * ROW_WORDS];

  const int tid = threadIdx.x;
  const int tx = tid & 15, ty = tid >> 4;
  const int64_t m0 = (int64_t)blockIdx.x * MBM, n0 = (int64_t)blockIdx.y * MBN;
  const int64_t G = K / GS;
  const int64_t nb = G / WR;
  const int64_t kbytes = K / 2;

  float acc[4] = {0.f, 0.f, 0.f, 0.f};
  bool nan_out[4] = {false, false, false, false};
  int64_t blk = 0;

  for (int64_t k0 = 0; k0 < K; k0 += KC) {
    // 32 rows x KC/2 bytes per operand: threads 0..127 load A, 128..255 load B, 8 bytes per piece
    for (int piece = tid & 127; piece < MBM * PARTS; piece += 128) {
      const int r = piece / PARTS, part = piece % PARTS;
      const int64_t kb = k0 / 2 + part * 8;
      uint2 w = make_uint2(0, 0);
      if (tid < 128) {
        if (m0 + r < M && kb < kbytes) w = *reinterpret_cast<const uint2*>(A + (m0 + r) * kbytes + kb);
        *reinterpret_cast<uint4*>(&As[r * ROW_WORDS + part * 4]) = unpack16m(w);
      } else {
        if (n0 + r < N && kb < kbytes) w = *reinterpret_cast<const uint2*>(B + (n0 + r) * kbytes + kb);
        *reinterpret_cast<uint4*>(&Bs[r * ROW_WORDS + part * 4]) = unpack16m(w);
      }
    }
    __syncthreads();
    const int ngroups = (K - k0) / GS < GPC ? (int)((K - k0) / GS) : GPC;   // a multiple of WR
    for (int b0 = 0; b0 < ngroups; b0 += WR) {
      double v[4][WR];
#pragma unroll
      for (int gw = 0; gw < WR; ++gw) {
        const int gl = b0 + gw;
        const int64_t g = k0 / GS + gl;
#pragma unroll
        for (int o = 0; o < 4; ++o) {
          const int i = o >> 1, j = o & 1;
          const int64_t r = m0 + ty + 16 * i, c = n0 + tx + 16 * j;
          const uint32_t ba = (r < M) ? SA[swz_offset(r, g, sa_cols)] : 0u;
          const uint32_t bb = (c < N) ? SB[swz_offset(c, g, sb_cols)] : 0u;
          int p4 = 0;
#pragma unroll
          for (int w = 0; w < WPG; ++w)
            p4 = __dp4a((int)As[(ty + 16 * i) * ROW_WORDS + gl * WPG + w], (int)Bs[(tx + 16 * j) * ROW_WORDS + gl * WPG + w],
                        p4);
          const int p = round_p4_to_fp16_grid(p4);
          if (FMT == EMU_FMT_NVFP4) {
            bool na, nbn;
            const int32_t sa = e4m3_times_512(ba, &na), sb = e4m3_times_512(bb, &nbn);
            nan_out[o] |= na || nbn;
            v[o][gw] = __ll2double_rn((long long)(p * sa) * (long long)sb) * 0x1p-20;   // p * sa * sb, exact
          } else {
            const double c4 = __dmul_rn(ue8m0_quarter_f64(ba), ue8m0_quarter_f64(bb) * 4.0);
            v[o][gw] = __dmul_rn((double)p, c4);
          }
        }
      }
#pragma unroll
      for (int o = 0; o < 4; ++o) {
        const double s3 = stage3_model_t<WR>(v[o], ma);
        if (nb == 1) acc[o] = round_f64_to_f32(s3, args.stage3_rounding);
        else acc[o] = round_f64_to_f32(stage4_model_fast(blk == 0 ? 0.0 : (double)acc[o], s3, ma), args.stage4_rounding);
      }
      ++blk;
    }
    __syncthreads();
  }
  const float al = alpha ? *alpha : 1.0f;
#pragma unroll
  for (int o = 0; o < 4; ++o) {
    const int i = o >> 1, j = o & 1;
    const int64_t r = m0 + ty + 16 * i, c = n0 + tx + 16 * j;
    if (r >= M || c >= N) continue;
    float y = alpha ? __fmul_rn(acc[o], al) : acc[o];
    if (FMT == EMU_FMT_NVFP4 && nan_out[o]) y = __int_as_float(0x7FFFFFFF);
    store_output(out, r * N + c, y, args.out_mode);
  }
}

template <int FMT>
cudaError_t launch_model(const uint8_t* A, const uint8_t* B, const uint8_t* SA, const uint8_t* SB, int64_t M,
                         int64_t N, int64_t K, int64_t sa_cols, int64_t sb_cols, const float* alpha,
                         const GemmArgs& args, const ModelArgs& ma, void* out, cudaStream_t stream) {
  dim3 grid((unsigned)((M + MBM - 1) / MBM), (unsigned)((N + MBN - 1) / MBN));
  switch (args.w_reduce) {
    case 1: emul_gemm_model_wr_kernel<FMT, 1><<<grid, MTHREADS, 0, stream>>>(A, B, SA, SB, M, N, K, sa_cols, sb_cols, alpha, args, ma, out); break;
    case 2: emul_gemm_model_wr_kernel<FMT, 2><<<grid, MTHREADS, 0, stream>>>(A, B, SA, SB, M, N, K, sa_cols, sb_cols, alpha, args, ma, out); break;
    case 4: emul_gemm_model_wr_kernel<FMT, 4><<<grid, MTHREADS, 0, stream>>>(A, B, SA, SB, M, N, K, sa_cols, sb_cols, alpha, args, ma, out); break;
    case 8: emul_gemm_model_wr_kernel<FMT, 8><<<grid, MTHREADS, 0, stream>>>(A, B, SA, SB, M, N, K, sa_cols, sb_cols, alpha, args, ma, out); break;
    default:
      emul_gemm_model_kernel<FMT><<<grid, MTHREADS, 0, stream>>>(A, B, SA, SB, M, N, K, sa_cols, sb_cols, alpha, args, ma, out);
  }
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_gemm_model(const uint8_t* A, const uint8_t* B, const uint8_t* SA, const uint8_t* SB, int64_t M,
                              int64_t N, int64_t K, int64_t sa_cols, int64_t sb_cols, const float* alpha,
                              const GemmArgs& args, const ModelArgs& ma, void* out, cudaStream_t stream) {
  if (args.format == EMU_FMT_NVFP4)
    return launch_model<EMU_FMT_NVFP4>(A, B, SA, SB, M, N, K, sa_cols, sb_cols, alpha, args, ma, out, stream);
  return launch_model<EMU_FMT_MXFP4>(A, B, SA, SB, M, N, K, sa_cols, sb_cols, alpha, args, ma, out, stream);
}

}  // namespace emu
