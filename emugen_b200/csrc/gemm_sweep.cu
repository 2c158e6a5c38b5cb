// Accumulator-model sweep: one quantised GEMM evaluated under many accumulator models at once, each
// model's result compared on the device with a reference output; only the per-model mismatch counts
// leave the kernel.  The reference runs such sweeps one model at a time from its search scripts
// (search/w3.py:123-158, search/w4.py:60-90), each a full emulation.
//
// Per output and 32- (MXFP4) / 16-element (NVFP4) group, stages 1-2 run once: the exact group dot
// (DP4A on the "2x" values), the fp16 rounding of stage 1, the block-scale product -- the same
// expressions as emul_gemm_model_wr_kernel (gemm_model.cu).  Up to SWEEP_MAX_CONFIGS models then take their own
// stage 3 (alignment width W3, aligned-addend rounding, summation order) and stage 4 (W4, RZ / RNE
// accumulator) on that value, in registers, with the models of one launch sharing the block size
// (w_reduce).
//
// Alignment without conversions: a value x rounded onto the grid q = 2^eq (eq = E - W + 1, E the
// largest exponent of the aligned addends) is, for |x| < 2^(eq + 51),
//   RNE:  (x + C) - C                      C = 1.5 * 2^(eq + 52): the sum's ulp is q, RN-even at q
//   RZ:   sign(x) * ((|x| +rz C) - C)      the same sum rounded toward zero
// both exact f64 additions, where the sweep kernel of gemm_model.cu converts x / q to an integer
// (quarter-rate conversions).  The aligned addends are multiples of q below 2^(E + 1), so their sums
// are exact while W <= 49 (stage 3, at most 16 addends) / 50 (stage 4, two): the result is bit for
// bit the integer-grid sum m * q of the model's definition.  Wider W take that definition directly.
#include <cuda_runtime.h>
#include <stdint.h>

#include "common.cuh"
#include "kernels.h"

namespace emu {
namespace {

constexpr int OPT = 2;                              // outputs per thread: rows ty and ty + 16 of one column
constexpr int SBN = 16, SBM = 16 * OPT;             // CTA tile: 32 x 16 outputs
constexpr int STHREADS = 256;

struct SweepParams {
  int n;                                  // models in this launch (<= SWEEP_MAX_CONFIGS)
  int align3[SWEEP_MAX_CONFIGS];
  int align4[SWEEP_MAX_CONFIGS];
  int arm[SWEEP_MAX_CONFIGS];             // aligned-addend rounding, EMU_RZ / EMU_RNE
  int order[SWEEP_MAX_CONFIGS];
  int r4[SWEEP_MAX_CONFIGS];              // stage-4 rounding
  int slot[SWEEP_MAX_CONFIGS];            // index into the caller's mismatch array
};

__device__ __forceinline__ int exp_field(double x) { return (__double2hiint(x) >> 20) & 0x7FF; }

// the model's integer-grid rounding by definition (any width): round(x / 2^eq) * 2^eq; out of line, as
// only the rare fallback of aligned_sum reaches it
__device__ __noinline__ double to_grid_def(double x, int eq, int rm) {
  const double y = scalbn(x, -eq);
  return scalbn(rm == EMU_RZ ? trunc(y) : rint(y), eq);
}

// floor(log2 |x|) of a finite nonzero double
__device__ __forceinline__ int exp_of(double x) {
  const int f = exp_field(x);
  return f ? f - 1023 : ilogb(x);
}

// The definition of the aligned sum of n addends at width w (no fast-path preconditions): E the
// largest exponent of the nonzero ones, each rounded onto 2^(E - w + 1), summed exactly, + 0.0.
// Reached only for subnormal addends, widths beyond the fast path's, or grids out of its range.
template <int WR>
__device__ __forceinline__ double aligned_sum_def(const double (&v)[WR], int w, int rm) {
  bool have = false;
  int E = 0;
#pragma unroll
  for (int i = 0; i < WR; ++i)
    if (v[i] != 0.0) { const int e = exp_of(v[i]); E = have ? max(E, e) : e; have = true; }
  if (!have) return 0.0;
  const int eq = E - w + 1;
  double s = 0.0;
#pragma unroll
  for (int i = 0; i < WR; ++i) s = __dadd_rn(s, to_grid_def(v[i], eq, rm));
  return __dadd_rn(s, 0.0);
}

// The aligned sum of WR finite addends at width w (stage 3 of a model, or stage 4 with the addends
// acc and s): the fast path when every nonzero addend is a normal double, w <= 49 and the grid
// 2^eq has a normal magic constant; the definition otherwise.  Uniform branches except for the
// rare fallback.
template <int WR>
__device__ __forceinline__ double aligned_sum(const double (&v)[WR], int w, int rm) {
  int fmax = 0;
  bool sub = false;
#pragma unroll
  for (int i = 0; i < WR; ++i) {
    const int f = exp_field(v[i]);
    fmax = max(fmax, f);
    sub = sub || (f == 0 && v[i] != 0.0);
  }
  if (fmax == 0 && !sub) return 0.0;
  const int eq = fmax - 1023 - w + 1;
  if (sub || w > 49 || eq < -1022 || eq > 971) return aligned_sum_def<WR>(v, w, rm);
  const double c = __hiloint2double((eq + 52 + 1023) << 20 | 0x80000, 0);   // 1.5 * 2^(eq + 52)
  double s = 0.0;
  if (rm == EMU_RNE) {
#pragma unroll
    for (int i = 0; i < WR; ++i) s = __dadd_rn(s, __dadd_rn(__dadd_rn(v[i], c), -c));
  } else {
#pragma unroll
    for (int i = 0; i < WR; ++i) s = __dadd_rn(s, copysign(__dadd_rn(__dadd_rz(fabs(v[i]), c), -c), v[i]));
  }
  return __dadd_rn(s, 0.0);
}

// Stage 3 of one model over WR addends (search/emulation/core.py:37-45 for the reference's order 0;
// the width / order model as defined in include/emugen.h emu_accum_model).
template <int WR>
__device__ __forceinline__ double stage3(const double (&v)[WR], int w3, int rm, int order) {
  if (w3 > 0) {
    bool finite = true;
#pragma unroll
    for (int i = 0; i < WR; ++i) finite = finite && exp_field(v[i]) != 0x7FF;
    if (finite) return aligned_sum<WR>(v, w3, rm);
  }
  if (order == 1) {
    double s = 0.0;
#pragma unroll
    for (int i = WR - 1; i >= 0; --i) s = __dadd_rn(s, v[i]);
    return s;
  }
  if (order == 2) {
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

// Stage 4 of one model: acc (an f32 value held in f64) and the block sum s, aligned to W4 (W4 <= 50
// keeps the two-addend sum exact on the fast path) or added in f64, before the accumulator rounding
__device__ __forceinline__ double stage4(double acc, double s, int w4, int rm) {
  if (w4 <= 0 || exp_field(acc) == 0x7FF || exp_field(s) == 0x7FF) return __dadd_rn(acc, s);
  const double v[2] = {acc, s};
  if (w4 > 49) return aligned_sum_def<2>(v, w4, rm);
  return aligned_sum<2>(v, w4, rm);
}

// What every model of a launch shares about one block's WR addends.
struct BlockFacts {
  int fmax;        // largest exponent field (0: every addend is zero)
  int fmin;        // smallest exponent field among the nonzero addends (2047 if none)
  bool finite;     // no inf / NaN addend
  bool sub;        // some addend is an f64 subnormal
  double plain;    // ((+0 + v0) + v1) + ... in f64
};

template <int WR>
__device__ __forceinline__ BlockFacts block_facts(const double (&v)[WR]) {
  BlockFacts b{0, 2047, true, false, 0.0};
#pragma unroll
  for (int i = 0; i < WR; ++i) {
    const int f = exp_field(v[i]);
    b.finite = b.finite && f != 0x7FF;
    b.fmax = max(b.fmax, f);
    if (f != 0) b.fmin = min(b.fmin, f);
    else b.sub = b.sub || v[i] != 0.0;
    b.plain = __dadd_rn(b.plain, v[i]);
  }
  return b;
}

// Significant bits of one stage-2 addend: MXFP4 p * 2^k with |p| < 2^13 (an fp16-rounded group dot
// of at most 32 products of 2x values up to 12); NVFP4 p * sa * sb * 2^-20 with at most 4 significant
// bits in each E4M3 scale.  An addend's lowest set bit is at least its exponent - (SIG - 1).
template <int FMT> struct AddendBits { static constexpr int SIG = FMT == EMU_FMT_NVFP4 ? 21 : 13; };

// Stage 3 of one model (stage3() above), using the block's shared facts: when the addends' exponent
// spread is at most W3 - SIG, every addend is already a multiple of the alignment grid 2^(E - W3 + 1),
// so the aligned sum is their exact sum -- the shared left-to-right sum, which is exact then (each
// addend a multiple of the grid and the total below 2^(E + 4), W3 + 3 <= 53 bits).  lb receives a
// lower bound on the exponent of the result's lowest set bit (stage 4 uses it).
template <int WR, int FMT>
__device__ __forceinline__ double stage3_shared(const double (&v)[WR], const BlockFacts& bf, int w3, int rm, int order,
                                                int& lb) {
  constexpr int SIG = AddendBits<FMT>::SIG;
  if (w3 > 0 && bf.finite) {
    if (!bf.sub && bf.fmax == 0) { lb = 1 << 20; return 0.0; }
    if (!bf.sub && bf.fmax - bf.fmin <= w3 - SIG) {
      lb = bf.fmin - 1023 - (SIG - 1);
      return __dadd_rn(bf.plain, 0.0);
    }
    lb = bf.fmax - 1023 - w3 + 1;    // every aligned addend is a multiple of the grid
    return aligned_sum<WR>(v, w3, rm);
  }
  // no alignment, or a non-finite addend (which leaves the alignment): the f64 sum in the model's order
  const double s = order == 0 ? bf.plain : stage3<WR>(v, 0, rm, order);
  lb = exp_field(s) - 1023 - 52;     // any double
  return s;
}

// The general stage 3 / stage 4 of a model, out of line: reached only where the fast checks below fail
// (non-finite or all-zero operands, subnormal addends, widths or grids beyond the magic constant's range).
template <int WR> struct Addends { double v[WR]; };

template <int WR, int FMT>
__device__ __noinline__ double stage3_general(const Addends<WR> a, BlockFacts bf, int w3, int rm, int order, int* lb) {
  return stage3_shared<WR, FMT>(a.v, bf, w3, rm, order, *lb);
}

__device__ __noinline__ double stage4_general(double acc, double s, int w4, int rm) {
  return stage4(acc, s, w4, rm);
}

// 1.5 * 2^(eq + 52): added to a value below 2^(eq + 51) in magnitude, its sum's ulp is 2^eq
__device__ __forceinline__ double grid_constant(int eq) {
  return __hiloint2double((eq + 52 + 1023) << 20 | 0x80000, 0);
}

// x rounded onto the grid of c = grid_constant(eq) (RZ: toward zero, RNE: nearest-even), exactly, for
// |x| < 2^(eq + 51); zero stays +0
__device__ __forceinline__ double to_grid_magic(double x, double c, int rm) {
  if (rm == EMU_RNE) return __dadd_rn(__dadd_rn(x, c), -c);
  return copysign(__dadd_rn(__dadd_rz(fabs(x), c), -c), x);
}

// One model's packed parameters: bits 0-7 align3, 8-15 align4, 16 aligned-addend rounding, 17-18
// stage-3 order, 19 stage-4 rounding.
__host__ __device__ __forceinline__ uint32_t pack_model(int w3, int w4, int arm, int order, int r4) {
  return (uint32_t)w3 | (uint32_t)w4 << 8 | (uint32_t)arm << 16 | (uint32_t)order << 17 | (uint32_t)r4 << 19;
}

// f64 -> f32 with rounding mode r, returned as the f64 holding that f32 value: the conversion pair, two
// instructions on the conversion pipes, which this ALU-bound kernel leaves idle (the 24-bit bit rounding
// in f64 takes about seven integer instructions and a branch)
__device__ __forceinline__ double to_f32_in_f64(double x, int r) { return (double)round_f64_to_f32(x, r); }

// A reference element as a float (fp16 / bf16 / f32 storage).
__device__ __forceinline__ float ref_value(const void* ref, int64_t i, int dtype) {
  if (dtype == EMU_DTYPE_F32) return static_cast<const float*>(ref)[i];
  const uint16_t b = static_cast<const uint16_t*>(ref)[i];
  if (dtype == EMU_DTYPE_BF16) return __uint_as_float((uint32_t)b << 16);
  return __half2float(__ushort_as_half(b));
}

// The model's f32 result in the reference's dtype: rounded once (bf16 / fp16), or itself (f32).
__device__ __forceinline__ float in_ref_dtype(float y, int dtype) {
  if (dtype == EMU_DTYPE_F32) return y;
  if (dtype == EMU_DTYPE_BF16) return __bfloat162float(__float2bfloat16_rn(y));
  return __half2float(__float2half_rn(y));
}

// One model's stage 3 and stage 4 for one output and K block: the accumulator after the block.  The
// common path is branch-uniform across a warp: every addend is rounded onto the alignment grid by the
// exact magic-constant additions (an addend already on the grid passes unchanged), so no lane-dependent
// shortcut test splits the warp; only non-finite or all-zero operands and out-of-range grids take the
// general, out-of-line code.
template <int WR, int FMT>
__device__ __forceinline__ double model_block(const double (&v)[WR], const BlockFacts& bf, uint32_t pm, double acc,
                                              bool first, bool single, int r3) {
  const int w3 = pm & 0xFF, w4 = (pm >> 8) & 0xFF, arm = (pm >> 16) & 1;
  const bool blk_ok = bf.finite && !bf.sub && bf.fmax != 0;
  double s3;
  const int eq3 = bf.fmax - 1023 - w3 + 1;
  if (w3 == 0) {
    const int order = (pm >> 17) & 3;
    s3 = order == 0 ? bf.plain : stage3<WR>(v, 0, arm, order);
  } else if (WR == 1 && w3 >= AddendBits<FMT>::SIG && !bf.sub) {
    // one addend of at most SIG significant bits is on any grid of width >= SIG: the aligned "sum" is
    // the addend + 0.0 (and a non-finite addend leaves the alignment, 0.0 + x = x + 0.0)
    s3 = __dadd_rn(bf.plain, 0.0);
  } else if (blk_ok && w3 <= 49 && eq3 >= -1022 && eq3 <= 971) {
    const double c = grid_constant(eq3);
    double t = 0.0;
#pragma unroll
    for (int k = 0; k < WR; ++k) t = __dadd_rn(t, to_grid_magic(v[k], c, arm));
    s3 = __dadd_rn(t, 0.0);
  } else {
    Addends<WR> ad;
#pragma unroll
    for (int k = 0; k < WR; ++k) ad.v[k] = v[k];
    int lb;
    s3 = stage3_general<WR, FMT>(ad, bf, w3, arm, (pm >> 17) & 3, &lb);
  }
  if (single) return to_f32_in_f64(s3, r3);
  const double a = first ? 0.0 : acc;
  double x;
  if (w4 == 0) {
    x = __dadd_rn(a, s3);
  } else {
    const int fa = exp_field(a), fs = exp_field(s3);
    const int eq4 = max(fa, fs) - 1023 - w4 + 1;
    if (fa != 0x7FF && fs != 0x7FF && (fa | fs) != 0 && w4 <= 50 && eq4 >= -1022 && eq4 <= 971) {
      const double c = grid_constant(eq4);
      x = __dadd_rn(__dadd_rn(to_grid_magic(a, c, arm), to_grid_magic(s3, c, arm)), 0.0);
    } else {
      x = stage4_general(a, s3, w4, arm);
    }
  }
  return to_f32_in_f64(x, (pm >> 19) & 1);
}

template <int FMT, int WR>
__global__ void __launch_bounds__(STHREADS)
emul_gemm_sweep_kernel(const uint8_t* __restrict__ A, const uint8_t* __restrict__ B, const uint8_t* __restrict__ SA,
                       const uint8_t* __restrict__ SB, int64_t M, int64_t N, int64_t K, int64_t sa_cols,
                       int64_t sb_cols, const float* __restrict__ alpha, int r3, const SweepParams sp,
                       const void* __restrict__ ref, int ref_dtype, unsigned long long* __restrict__ mismatches) {
  constexpr int GS = (FMT == EMU_FMT_NVFP4) ? 16 : 32;
  constexpr int KC = WR * GS > 64 ? WR * GS : 64;       // elements per chunk: whole blocks
  constexpr int GPC = KC / GS;                           // groups per chunk
  constexpr int WPG = GS / 4;                            // int8x4 words per group
  constexpr int ROW_WORDS = KC / 4 + 4;                  // padded against bank conflicts
  constexpr int PARTS = KC / 16;                         // 8-byte pieces per row of a chunk
  __shared__ __align__(16) uint32_t As[SBM * ROW_WORDS];
  __shared__ __align__(16) uint32_t Bs[SBN * ROW_WORDS];
  __shared__ uint8_t Sa[SBM * GPC], Sb[SBN * GPC];
  __shared__ uint32_t s_models[SWEEP_MAX_CONFIGS];
  if (threadIdx.x < sp.n)
    s_models[threadIdx.x] = pack_model(sp.align3[threadIdx.x], sp.align4[threadIdx.x], sp.arm[threadIdx.x],
                                       sp.order[threadIdx.x], sp.r4[threadIdx.x]);

  const int tid = threadIdx.x;
  const int tx = tid % SBN, ty = tid / SBN;             // outputs (m0 + ty + 16 o, n0 + tx), o < OPT
  const int64_t m0 = (int64_t)blockIdx.y * SBM, n0 = (int64_t)blockIdx.x * SBN;
  const int64_t c = n0 + tx;
  const int64_t G = K / GS, nb = G / WR, kbytes = K / 2;

  double acc[OPT][SWEEP_MAX_CONFIGS];
#pragma unroll 1
  for (int i = 0; i < SWEEP_MAX_CONFIGS; ++i) {
#pragma unroll
    for (int o = 0; o < OPT; ++o) acc[o][i] = 0.0;
  }
  bool nan_out[OPT] = {};
  int64_t blk = 0;

  for (int64_t k0 = 0; k0 < K; k0 += KC) {
    // operands: SBM + SBN rows x KC/2 bytes, unpacked to int8 "2x" values; scale bytes of the chunk
    for (int piece = tid; piece < (SBM + SBN) * PARTS; piece += STHREADS) {
      const int row = piece / PARTS, part = piece % PARTS;
      const int64_t kb = k0 / 2 + part * 8;
      const bool is_a = row < SBM;
      const int64_t gr = is_a ? m0 + row : n0 + row - SBM;
      uint2 w = make_uint2(0, 0);
      if (gr < (is_a ? M : N) && kb < kbytes) w = *reinterpret_cast<const uint2*>((is_a ? A : B) + gr * kbytes + kb);
      uint32_t* dst = is_a ? &As[row * ROW_WORDS + part * 4] : &Bs[(row - SBM) * ROW_WORDS + part * 4];
      *reinterpret_cast<uint4*>(dst) = make_uint4(e2m1x4_to_int8x4(w.x & 0xFFFFu), e2m1x4_to_int8x4(w.x >> 16),
                                                  e2m1x4_to_int8x4(w.y & 0xFFFFu), e2m1x4_to_int8x4(w.y >> 16));
    }
    for (int i = tid; i < (SBM + SBN) * GPC; i += STHREADS) {
      const int row = i / GPC, gl = i % GPC;
      const int64_t g = k0 / GS + gl;
      const bool is_a = row < SBM;
      const int64_t gr = is_a ? m0 + row : n0 + row - SBM;
      uint8_t byte = 0;
      if (gr < (is_a ? M : N) && g < G) byte = (is_a ? SA : SB)[swz_offset(gr, g, is_a ? sa_cols : sb_cols)];
      (is_a ? Sa : Sb)[(is_a ? row : row - SBM) * GPC + gl] = byte;
    }
    __syncthreads();
    const int ngroups = (K - k0) / GS < GPC ? (int)((K - k0) / GS) : GPC;   // a multiple of WR
    for (int b0 = 0; b0 < ngroups; b0 += WR) {
      double v[OPT][WR];
#pragma unroll
      for (int gw = 0; gw < WR; ++gw) {
        const int gl = b0 + gw;
        const uint32_t bb = Sb[tx * GPC + gl];
#pragma unroll
        for (int o = 0; o < OPT; ++o) {
          const int row = ty + 16 * o;
          int p4 = 0;
#pragma unroll
          for (int w = 0; w < WPG; ++w)
            p4 = __dp4a((int)As[row * ROW_WORDS + gl * WPG + w], (int)Bs[tx * ROW_WORDS + gl * WPG + w], p4);
          const int p = round_p4_to_fp16_grid(p4);
          const uint32_t ba = Sa[row * GPC + gl];
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
      // shared by every model of the launch: the addends' largest exponent, finiteness, and their
      // left-to-right f64 sum (the reference's stage 3)
      BlockFacts bf[OPT];
#pragma unroll
      for (int o = 0; o < OPT; ++o) bf[o] = block_facts<WR>(v[o]);
      // one copy of the model code, looped (unrolled, SWEEP_MAX_CONFIGS copies overflow the instruction
      // cache); the accumulators live in local memory, L1-resident; a model's parameters are decoded
      // once for the thread's OPT outputs
#pragma unroll 1
      for (int i = 0; i < sp.n; ++i) {
        const uint32_t pm = s_models[i];
#pragma unroll
        for (int o = 0; o < OPT; ++o)
          acc[o][i] = model_block<WR, FMT>(v[o], bf[o], pm, acc[o][i], blk == 0, nb == 1, r3);
      }
      ++blk;
    }
    __syncthreads();
  }
  // compare each model's result with the reference (gemm_compare/runner.py:20-55: equal, or NaN on both
  // sides); one atomic per warp and model
  bool live[OPT];
  float rv[OPT];
#pragma unroll
  for (int o = 0; o < OPT; ++o) {
    const int64_t r = m0 + ty + 16 * o;
    live[o] = r < M && c < N;
    rv[o] = live[o] ? ref_value(ref, r * N + c, ref_dtype) : 0.0f;
  }
  const float al = alpha ? *alpha : 1.0f;
#pragma unroll 1
  for (int i = 0; i < SWEEP_MAX_CONFIGS; ++i) {
    if (i < sp.n) {
      unsigned n_bad = 0;
#pragma unroll
      for (int o = 0; o < OPT; ++o) {
        float y = (float)acc[o][i];
        if (alpha) y = __fmul_rn(y, al);
        if (FMT == EMU_FMT_NVFP4 && nan_out[o]) y = __int_as_float(0x7FFFFFFF);
        const float q = in_ref_dtype(y, ref_dtype);
        const bool bad = live[o] && !(q == rv[o]) && !(q != q && rv[o] != rv[o]);
        n_bad += __popc(__ballot_sync(0xFFFFFFFFu, bad));
      }
      if ((tid & 31) == 0 && n_bad) atomicAdd(&mismatches[sp.slot[i]], (unsigned long long)n_bad);
    }
  }
}

template <int FMT>
cudaError_t launch_sweep_fmt(const uint8_t* A, const uint8_t* B, const uint8_t* SA, const uint8_t* SB, int64_t M,
                             int64_t N, int64_t K, int64_t sa_cols, int64_t sb_cols, const float* alpha, int w_reduce,
                             int r3, const SweepParams& sp, const void* ref, int ref_dtype,
                             unsigned long long* mismatches, cudaStream_t stream) {
  const dim3 grid((unsigned)((N + SBN - 1) / SBN), (unsigned)((M + SBM - 1) / SBM));
  switch (w_reduce) {
    case 1: emul_gemm_sweep_kernel<FMT, 1><<<grid, STHREADS, 0, stream>>>(A, B, SA, SB, M, N, K, sa_cols, sb_cols, alpha, r3, sp, ref, ref_dtype, mismatches); break;
    case 2: emul_gemm_sweep_kernel<FMT, 2><<<grid, STHREADS, 0, stream>>>(A, B, SA, SB, M, N, K, sa_cols, sb_cols, alpha, r3, sp, ref, ref_dtype, mismatches); break;
    case 4: emul_gemm_sweep_kernel<FMT, 4><<<grid, STHREADS, 0, stream>>>(A, B, SA, SB, M, N, K, sa_cols, sb_cols, alpha, r3, sp, ref, ref_dtype, mismatches); break;
    case 8: emul_gemm_sweep_kernel<FMT, 8><<<grid, STHREADS, 0, stream>>>(A, B, SA, SB, M, N, K, sa_cols, sb_cols, alpha, r3, sp, ref, ref_dtype, mismatches); break;
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

}  // namespace

bool sweep_supported_w_reduce(int w_reduce) { return w_reduce == 1 || w_reduce == 2 || w_reduce == 4 || w_reduce == 8; }

cudaError_t launch_gemm_sweep(const uint8_t* A, const uint8_t* B, const uint8_t* SA, const uint8_t* SB, int64_t M,
                              int64_t N, int64_t K, int64_t sa_cols, int64_t sb_cols, const float* alpha, int fmt,
                              int w_reduce, int r3, const SweepModel* models, const int* slots, int n,
                              const void* ref, int ref_dtype, unsigned long long* mismatches, cudaStream_t stream) {
  SweepParams sp{};
  sp.n = n;
  for (int i = 0; i < n; ++i) {
    sp.align3[i] = models[i].align3;
    sp.align4[i] = models[i].align4;
    sp.arm[i] = models[i].align_rounding;
    sp.order[i] = models[i].order;
    sp.r4[i] = models[i].stage4_rounding;
    sp.slot[i] = slots[i];
  }
  if (fmt == EMU_FMT_NVFP4)
    return launch_sweep_fmt<EMU_FMT_NVFP4>(A, B, SA, SB, M, N, K, sa_cols, sb_cols, alpha, w_reduce, r3, sp, ref,
                                           ref_dtype, mismatches, stream);
  return launch_sweep_fmt<EMU_FMT_MXFP4>(A, B, SA, SB, M, N, K, sa_cols, sb_cols, alpha, w_reduce, r3, sp, ref,
                                         ref_dtype, mismatches, stream);
}

}  // namespace emu
