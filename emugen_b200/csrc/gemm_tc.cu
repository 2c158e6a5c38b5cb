// Emulated scaled FP4 GEMM on the 5th-generation tensor cores (tcgen05 + TMEM + TMA), sm_100a.
//
// Stage 1 (the exact group dot products) runs on the tensor core; stages 2-4 (scale, exact f64
// group sums, RZ/RNE accumulation) run on CUDA cores reading TMEM.  Bit-exact to the reference
// emulators (nvfp_emulation.cpp:90-156, mxfp_emulation.cpp:98-166) for the reference's accumulator
// shapes: NVFP4 w_reduce 4 and MXFP4 w_reduce 2 (one 64-element K block per stage-3 sum).
//
// Pre-pass (one launch per operand):  packed e2m1 -> fp16 "2x" integers (0, +-1 .. +-12, exact),
// and per-row / per-column scale tables in the form the epilogue consumes.
//
// Main kernel: persistent, one CTA per SM, 10 warps:
//   warp 0      TMA producer: A tile [128 x 64] and B tile [64 x 64] fp16 per K block into a
//               6-stage shared-memory ring (128-byte swizzle), B-side scale table [groups x 64]
//               f64 into a 4-stage ring.
//   warp 1      TMEM owner + MMA issuer: per group one tcgen05.mma kind::f16 M128 N64 K16
//               (NVFP4; MXFP4 groups take two, accumulated) into its own TMEM accumulator, so
//               TMEM holds p4 = 4 * (exact group dot) for every (row, column, group) in f32.
//   warps 2-9   epilogue: each thread owns one output row (its TMEM lane) and 32 columns.
// TMEM: 512 columns = ring of accumulator sets, one set per K block (NVFP4: 4 groups x 64 columns,
// two sets; MXFP4: 2 x 64, four sets), so the MMA of block b+1 overlaps the epilogue of block b.
//
// Epilogue arithmetic per group partial (exact; conversions into 64-bit types avoided because
// they run at a quarter of the FP64 rate on B200):
//   NVFP4: bits = FFMA(p4, ma, 1.5*2^23)            (integer p4*ma in the f32 mantissa, exact)
//          d    = double{hi = 2^E exponent word of the row scale, lo = bits}
//          diff = d - double{hi, 0x4B400000}        = p * sa exactly
//          S    = FMA(diff, sb, S)                  (f64; the 4-group sum is exact)
//   MXFP4: diff = double{2^52, FADD(p4, 1.5*2^23)} - (2^52 + 0x4B400000)  = p4 exactly
//          S    = FMA(diff * (2^(ua-127)/4), 2^(ub-127), S)   (inf / NaN follow IEEE as in the reference)
//   block: acc = R4(f64(acc) + S)  (first block: R4(S); single block: R3(S))
// A stage-1 group sum of magnitude >= 512 is rounded to the fp16 grid first; a per-warp max test
// sends those (rare) cases through the rounding routine.
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>

#include "common.cuh"
#include "kernels.h"
#include "tc_ptx.cuh"

namespace emu {
namespace tc {

constexpr int BM = 128, BN = 64, BK = 64;
constexpr int NSTAGE = 6, NSB = 4;
constexpr int NUM_THREADS = 320;                  // 10 warps
constexpr int A_BYTES = BM * BK * 2, B_BYTES = BN * BK * 2;
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;    // 24 KB
constexpr int SB_BYTES = 4 * BN * 8;              // up to 4 groups x 64 columns x f64
constexpr float MAGIC_F = 12582912.0f;            // 1.5 * 2^23
constexpr uint32_t MAGIC_BITS = 0x4B400000u;
constexpr int GROUP_M = 16;                       // tile raster: 16 M-tiles per band
constexpr int SMEM_BYTES = 1024 /*align*/ + NSTAGE * STAGE_BYTES + NSB * SB_BYTES + 256;

// NVFP4 row-scale record, one per (row, group).
struct __align__(16) RowScaleNv {
  float ma;        // signed E4M3 significand (0..15), 0 for NaN
  uint32_t hi;     // exponent word: 2^(sxa + 50) with the low 20 mantissa bits zero
  double d0;       // double{hi, MAGIC_BITS}
};

// ------------------------------------------------------------------------------ pre-pass
__global__ void unpack_fp16x2_kernel(const uint8_t* __restrict__ packed, int64_t rows, int64_t K,
                                     __half* __restrict__ out) {
  const int64_t n8 = rows * (K / 16);               // 8-byte chunks (16 elements)
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n8; i += (int64_t)gridDim.x * blockDim.x) {
    const uint2 w = reinterpret_cast<const uint2*>(packed)[i];
    const uint32_t in[2] = {w.x, w.y};
    uint32_t o[8];
#pragma unroll
    for (int h = 0; h < 2; ++h)
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const uint32_t lo = (in[h] >> (8 * q)) & 0xFu, hi = (in[h] >> (8 * q + 4)) & 0xFu;
        const __half a = __int2half_rn(e2m1_twice(lo)), b = __int2half_rn(e2m1_twice(hi));
        o[4 * h + q] = (uint32_t)__half_as_ushort(a) | ((uint32_t)__half_as_ushort(b) << 16);
      }
    uint4* dst = reinterpret_cast<uint4*>(out) + 2 * i;
    dst[0] = make_uint4(o[0], o[1], o[2], o[3]);
    dst[1] = make_uint4(o[4], o[5], o[6], o[7]);
  }
}

// NVFP4 rows: RowScaleNv[rows][G]; row_nan[rows].  MXFP4 rows: f64 2^(u-129) [rows][G].
template <int FMT>
__global__ void row_scales_kernel(const uint8_t* __restrict__ sf, int64_t rows, int64_t G, int64_t sf_cols,
                                  void* __restrict__ table, uint8_t* __restrict__ row_nan) {
  for (int64_t r = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; r < rows; r += (int64_t)gridDim.x * blockDim.x) {
    bool any_nan = false;
    for (int64_t g = 0; g < G; ++g) {
      const uint32_t byte = sf[swz_offset(r, g, sf_cols)];
      if (FMT == EMU_FMT_NVFP4) {
        const uint32_t e = (byte >> 3) & 0xFu, m = byte & 7u;
        const bool nan = (e == 15u && m == 7u);
        any_nan |= nan;
        int ma = (e == 0u) ? (int)m : (int)(8u + m);
        const int sxa = (e == 0u) ? -9 : (int)e - 10;
        if (byte & 0x80u) ma = -ma;
        if (nan) ma = 0;
        RowScaleNv rec;
        rec.ma = (float)ma;
        rec.hi = (uint32_t)(sxa + 1073) << 20;
        rec.d0 = __hiloint2double((int)rec.hi, (int)MAGIC_BITS);
        static_cast<RowScaleNv*>(table)[r * G + g] = rec;
      } else {
        static_cast<double*>(table)[r * G + g] = ue8m0_quarter_f64(byte);
      }
    }
    if (FMT == EMU_FMT_NVFP4) row_nan[r] = any_nan ? 1 : 0;
  }
}

// Column scales transposed to [G][ncols_pad] f64: NVFP4 sb (signed, 0 for NaN), MXFP4 2^(u-127).
template <int FMT>
__global__ void col_scales_kernel(const uint8_t* __restrict__ sf, int64_t cols, int64_t ncols_pad, int64_t G,
                                  int64_t sf_cols, double* __restrict__ table, uint8_t* __restrict__ col_nan) {
  const int64_t total = G * ncols_pad;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t g = i / ncols_pad, c = i % ncols_pad;
    double v = 0.0;
    if (c < cols) {
      const uint32_t byte = sf[swz_offset(c, g, sf_cols)];
      if (FMT == EMU_FMT_NVFP4) {
        bool nan;
        const int32_t s512 = e4m3_times_512(byte, &nan);
        v = (double)s512 * 0x1p-9;
      } else {
        v = ue8m0_quarter_f64(byte) * 4.0;
      }
    }
    table[i] = v;
  }
  if (FMT == EMU_FMT_NVFP4) {
    for (int64_t c = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; c < cols; c += (int64_t)gridDim.x * blockDim.x) {
      bool any = false;
      for (int64_t g = 0; g < G; ++g) {
        bool nan;
        (void)e4m3_times_512(sf[swz_offset(c, g, sf_cols)], &nan);
        any |= nan;
      }
      col_nan[c] = any ? 1 : 0;
    }
  }
}

// ------------------------------------------------------------------------------ main kernel
struct Params {
  int64_t M, N, K;
  int64_t G, nb, tiles_m, tiles_n;
  const void* row_tab;        // RowScaleNv[M][G] or double[M][G]
  const uint8_t* row_nan;     // NVFP4 only
  const uint8_t* col_nan;     // NVFP4 only
  const float* alpha;         // nullable
  void* out;
  int* err;
  int r3, r4, out_mode;
};

__device__ __forceinline__ void tile_coords(int64_t t, const Params& p, int64_t& tm, int64_t& tn) {
  const int64_t per_band = (int64_t)GROUP_M * p.tiles_n;
  const int64_t band = t / per_band;
  const int64_t first_m = band * GROUP_M;
  const int64_t rem = p.tiles_m - first_m;
  const int64_t gm = rem < GROUP_M ? rem : (int64_t)GROUP_M;
  const int64_t idx = t % per_band;
  tm = first_m + idx % gm;
  tn = idx / gm;
}

// p4 -> nearest fp16 grid value (only called when |p4| >= 2048 somewhere in the warp)
__device__ __forceinline__ float round_p4_f(float p4) {
  return __half2float(__float2half_rn(p4 * 0.25f)) * 4.0f;
}

// NVFP4 f32-range rounding of an f64 that holds a finite value with |x| in [2^-126, 2^128) or 0:
// clear (RZ) or round-to-nearest-even (RNE) the 29 low mantissa bits.  Values here are multiples
// of 2^-20 below 2^64, so they are always in that range.
__device__ __forceinline__ double round24(double x, int mode) {
  long long b = __double_as_longlong(x);
  if (mode == EMU_RNE) b += 0x0FFFFFFFll + ((b >> 29) & 1ll);
  b &= ~0x1FFFFFFFll;
  return __longlong_as_double(b);
}

template <int FMT>
__global__ void __launch_bounds__(NUM_THREADS, 1)
emul_gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                    const __grid_constant__ CUtensorMap tmSB, const Params p) {
  constexpr int GPB = (FMT == EMU_FMT_NVFP4) ? 4 : 2;       // groups per 64-element K block
  constexpr int SET_COLS = GPB * BN;                         // TMEM columns per K block
  constexpr int NSETS = 512 / SET_COLS;                      // 2 (NVFP4) or 4 (MXFP4)
  constexpr uint32_t SB_TX = GPB * BN * 8;

  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  uint8_t* stage_base = smem;
  double* sb_ring = reinterpret_cast<double*>(smem + NSTAGE * STAGE_BYTES);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + NSTAGE * STAGE_BYTES + NSB * SB_BYTES);
  uint64_t* full = bars;                       // [NSTAGE]
  uint64_t* empty = full + NSTAGE;             // [NSTAGE]
  uint64_t* sb_full = empty + NSTAGE;          // [NSB]
  uint64_t* sb_empty = sb_full + NSB;          // [NSB]
  uint64_t* tm_full = sb_empty + NSB;          // [NSETS]
  uint64_t* tm_empty = tm_full + 4;            // [NSETS]
  uint64_t* drain = tm_empty + 4;              // MMA completion before TMEM release
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t total_tiles = p.tiles_m * p.tiles_n;

  if (threadIdx.x == 0) {
    for (int i = 0; i < NSTAGE; ++i) { ptx::mbar_init(&full[i], 1); ptx::mbar_init(&empty[i], 1); }
    for (int i = 0; i < NSB; ++i) { ptx::mbar_init(&sb_full[i], 1); ptx::mbar_init(&sb_empty[i], 8); }
    for (int i = 0; i < NSETS; ++i) { ptx::mbar_init(&tm_full[i], 1); ptx::mbar_init(&tm_empty[i], 8); }
    ptx::mbar_init(drain, 1);
    ptx::fence_mbar_init();
    ptx::prefetch_tmap(&tmA);
    ptx::prefetch_tmap(&tmB);
    ptx::prefetch_tmap(&tmSB);
  }
  if (warp == 1) {
    ptx::tmem_alloc(tmem_slot, 512);
    ptx::tmem_relinquish();
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ---------------------------------------------------------------- TMA producer
    if (lane == 0) {
      int64_t it = 0;
      bool ok = true;
      for (int64_t t = blockIdx.x; t < total_tiles && ok; t += gridDim.x) {
        int64_t tm, tn;
        tile_coords(t, p, tm, tn);
        for (int64_t kb = 0; kb < p.nb && ok; ++kb, ++it) {
          const int s = (int)(it % NSTAGE);
          const uint32_t ph = (uint32_t)((it / NSTAGE) & 1);
          ok = ptx::mbar_wait(&empty[s], ph ^ 1u, p.err, 1);
          if (!ok) break;
          uint8_t* sa = stage_base + s * STAGE_BYTES;
          ptx::mbar_arrive_expect_tx(&full[s], STAGE_BYTES);
          ptx::tma_load_2d(sa, &tmA, &full[s], (int)(kb * BK), (int)(tm * BM));
          ptx::tma_load_2d(sa + A_BYTES, &tmB, &full[s], (int)(kb * BK), (int)(tn * BN));
          const int q = (int)(it % NSB);
          const uint32_t qph = (uint32_t)((it / NSB) & 1);
          ok = ptx::mbar_wait(&sb_empty[q], qph ^ 1u, p.err, 2);
          if (!ok) break;
          ptx::mbar_arrive_expect_tx(&sb_full[q], SB_TX);
          ptx::tma_load_2d(sb_ring + q * (SB_BYTES / 8), &tmSB, &sb_full[q], (int)(tn * BN), (int)(kb * GPB));
        }
      }
      // drain: every issued TMA copy must have landed before the CTA may exit (bounded waits)
      for (int64_t j = (it > NSTAGE ? it - NSTAGE : 0); j < it; ++j)
        ptx::mbar_wait(&full[j % NSTAGE], (uint32_t)((j / NSTAGE) & 1), p.err, 7);
      for (int64_t j = (it > NSB ? it - NSB : 0); j < it; ++j)
        ptx::mbar_wait(&sb_full[j % NSB], (uint32_t)((j / NSB) & 1), p.err, 8);
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t IDESC = ptx::idesc_f16_f32(BM, BN);
      int64_t it = 0;
      bool ok = true;
      for (int64_t t = blockIdx.x; t < total_tiles && ok; t += gridDim.x) {
        for (int64_t kb = 0; kb < p.nb && ok; ++kb, ++it) {
          const int s = (int)(it % NSTAGE);
          const uint32_t ph = (uint32_t)((it / NSTAGE) & 1);
          const int set = (int)(it % NSETS);
          const uint32_t tph = (uint32_t)((it / NSETS) & 1);
          ok = ptx::mbar_wait(&tm_empty[set], tph ^ 1u, p.err, 3);
          if (!ok) break;
          ok = ptx::mbar_wait(&full[s], ph, p.err, 4);
          if (!ok) break;
          ptx::tc_fence_after();
          const uint32_t a_addr = ptx::smem_u32(stage_base + s * STAGE_BYTES);
          const uint32_t b_addr = a_addr + A_BYTES;
          const uint32_t d_col = tmem_base + (uint32_t)(set * SET_COLS);
#pragma unroll
          for (int g = 0; g < GPB; ++g) {
            const uint32_t d = d_col + (uint32_t)(g * BN);
            if (FMT == EMU_FMT_NVFP4) {
              // group g = K elements [16g, 16g+16) = bytes [32g, 32g+32) of each 128-byte row
              ptx::mma_f16(d, ptx::smem_desc_sw128(a_addr + 32 * g), ptx::smem_desc_sw128(b_addr + 32 * g), IDESC, 0);
            } else {
              ptx::mma_f16(d, ptx::smem_desc_sw128(a_addr + 64 * g), ptx::smem_desc_sw128(b_addr + 64 * g), IDESC, 0);
              ptx::mma_f16(d, ptx::smem_desc_sw128(a_addr + 64 * g + 32), ptx::smem_desc_sw128(b_addr + 64 * g + 32),
                           IDESC, 1);
            }
          }
          ptx::mma_commit(&empty[s]);
          ptx::mma_commit(&tm_full[set]);
        }
      }
      // drain: all issued MMAs complete before TMEM is released
      ptx::mma_commit(drain);
      ptx::mbar_wait(drain, 0, p.err, 9);
    }
  } else {
    // ---------------------------------------------------------------- epilogue (warps 2..9)
    const int ew = warp - 2;                 // 0..7
    const int quarter = warp & 3;            // TMEM lane quarter this warp may access
    const int half = ew >> 2;                // column half: 0 -> 0..31, 1 -> 32..63
    const uint32_t lane_base = (uint32_t)(quarter * 32) << 16;
    int64_t it = 0;
    bool ok = true;
    for (int64_t t = blockIdx.x; t < total_tiles && ok; t += gridDim.x) {
      int64_t tm, tn;
      tile_coords(t, p, tm, tn);
      const int64_t m = tm * BM + quarter * 32 + lane;
      const bool row_ok = m < p.M;
      const int64_t mr = row_ok ? m : (p.M - 1);
      double acc[32];
#pragma unroll
      for (int j = 0; j < 32; ++j) acc[j] = 0.0;

      for (int64_t kb = 0; kb < p.nb && ok; ++kb, ++it) {
        const int set = (int)(it % NSETS);
        const uint32_t tph = (uint32_t)((it / NSETS) & 1);
        const int q = (int)(it % NSB);
        const uint32_t qph = (uint32_t)((it / NSB) & 1);
        // per-row scale constants for this block's groups
        float ma[GPB];
        uint32_t hi[GPB];
        double d0[GPB], sa[GPB];
        if (FMT == EMU_FMT_NVFP4) {
          const RowScaleNv* rs = static_cast<const RowScaleNv*>(p.row_tab) + mr * p.G + kb * GPB;
#pragma unroll
          for (int g = 0; g < GPB; ++g) { const RowScaleNv r = rs[g]; ma[g] = r.ma; hi[g] = r.hi; d0[g] = r.d0; }
        } else {
          const double* rs = static_cast<const double*>(p.row_tab) + mr * p.G + kb * GPB;
#pragma unroll
          for (int g = 0; g < GPB; ++g) sa[g] = rs[g];
        }
        ok = __all_sync(0xFFFFFFFFu, ptx::mbar_wait(&tm_full[set], tph, p.err, 5));
        if (!ok) break;
        ok = __all_sync(0xFFFFFFFFu, ptx::mbar_wait(&sb_full[q], qph, p.err, 6));
        if (!ok) break;
        ptx::tc_fence_after();
        const double* sbs = sb_ring + q * (SB_BYTES / 8);

#pragma unroll
        for (int h16 = 0; h16 < 2; ++h16) {
          float v[GPB][16];
#pragma unroll
          for (int g = 0; g < GPB; ++g)
            ptx::tmem_ld16(tmem_base + lane_base + (uint32_t)(set * SET_COLS + g * BN + half * 32 + h16 * 16), v[g]);
          ptx::tmem_wait_ld();
          if (h16 == 1) {
            ptx::tc_fence_before();
            __syncwarp();
            if (lane == 0) ptx::mbar_arrive(&tm_empty[set]);
          }
          // stage-1 fp16 rounding only matters for |p4| >= 2048 (|p| >= 512)
          float mx = 0.0f;
#pragma unroll
          for (int g = 0; g < GPB; ++g)
#pragma unroll
            for (int j = 0; j < 16; ++j) mx = fmaxf(mx, fabsf(v[g][j]));
          if (__any_sync(0xFFFFFFFFu, mx >= 2048.0f)) {
#pragma unroll
            for (int g = 0; g < GPB; ++g)
#pragma unroll
              for (int j = 0; j < 16; ++j) v[g][j] = round_p4_f(v[g][j]);
          }
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const int col = half * 32 + h16 * 16 + j;
            double S = 0.0;
#pragma unroll
            for (int g = 0; g < GPB; ++g) {
              const double sb = sbs[g * BN + col];
              if (FMT == EMU_FMT_NVFP4) {
                const float bits = __fmaf_rn(v[g][j], ma[g], MAGIC_F);
                const double dd = __hiloint2double((int)hi[g], __float_as_int(bits));
                const double diff = __dadd_rn(dd, -d0[g]);
                S = __fma_rn(diff, sb, S);
              } else {
                const float bits = __fadd_rn(v[g][j], MAGIC_F);
                const double dd = __hiloint2double(0x43300000, __float_as_int(bits));
                const double p4 = __dadd_rn(dd, -(4503599627370496.0 + (double)MAGIC_BITS));
                S = __fma_rn(__dmul_rn(p4, sa[g]), sb, S);
              }
            }
            const int jj = h16 * 16 + j;
            if (FMT == EMU_FMT_NVFP4) {
              if (p.nb == 1) acc[jj] = round24(S, p.r3);
              else acc[jj] = round24(kb == 0 ? S : __dadd_rn(acc[jj], S), p.r4);
            } else {
              float a;
              if (p.nb == 1) a = round_f64_to_f32(S, p.r3);
              else a = round_f64_to_f32(kb == 0 ? S : __dadd_rn(acc[jj], S), p.r4);
              acc[jj] = (double)a;
            }
          }
        }
        __syncwarp();
        if (lane == 0) ptx::mbar_arrive(&sb_empty[q]);
      }
      if (!ok) break;
      // ---- output
      if (row_ok) {
        const float al = p.alpha ? *p.alpha : 1.0f;
        const bool rnan = (FMT == EMU_FMT_NVFP4) && p.row_nan[m];
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          const int64_t n = tn * BN + half * 32 + j;
          if (n < p.N) {
            float y = (float)acc[j];
            if (p.alpha) y = __fmul_rn(y, al);
            if (FMT == EMU_FMT_NVFP4 && (rnan || p.col_nan[n])) y = __int_as_float(0x7FFFFFFF);
            store_output(p.out, m * p.N + n, y, p.out_mode);
          }
        }
      }
    }
  }

  ptx::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    ptx::tc_fence_after();
    ptx::tmem_dealloc(tmem_base, 512);
  }
}

// ------------------------------------------------------------------------------ host side
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn get_encode() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(ptr);
  }
  return fn;
}

static bool make_map_2d(CUtensorMap* m, CUtensorMapDataType dt, void* base, uint64_t inner, uint64_t outer,
                        uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer, CUtensorMapSwizzle sw) {
  EncodeTiledFn enc = get_encode();
  if (!enc) return false;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t es[2] = {1, 1};
  return enc(m, dt, 2, base, dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

static size_t align_up(size_t x) { return (x + 1023) & ~(size_t)1023; }

struct WsLayout {
  size_t a16, b16, row_tab, sb_tab, row_nan, col_nan, err, total;
};

static WsLayout layout(int fmt, int64_t M, int64_t N, int64_t K) {
  const int gs = fmt == EMU_FMT_NVFP4 ? 16 : 32;
  const int64_t G = K / gs;
  const int64_t Np = (N + BN - 1) / BN * BN;
  WsLayout L{};
  size_t off = 0;
  L.a16 = off; off = align_up(off + (size_t)M * K * 2);
  L.b16 = off; off = align_up(off + (size_t)N * K * 2);
  L.row_tab = off; off = align_up(off + (size_t)M * G * (fmt == EMU_FMT_NVFP4 ? sizeof(RowScaleNv) : 8));
  L.sb_tab = off; off = align_up(off + (size_t)G * Np * 8);
  L.row_nan = off; off = align_up(off + (size_t)M);
  L.col_nan = off; off = align_up(off + (size_t)N);
  L.err = off; off = align_up(off + 16);
  L.total = off;
  return L;
}

}  // namespace tc

size_t gemm_tc_workspace_size(int fmt, int64_t M, int64_t N, int64_t K) { return tc::layout(fmt, M, N, K).total; }

bool gemm_tc_supported(int fmt, int w_reduce, int64_t M, int64_t N, int64_t K) {
  using tc::BM;
  using tc::BN;
  if (fmt == EMU_FMT_NVFP4 && w_reduce != 4) return false;
  if (fmt == EMU_FMT_MXFP4 && w_reduce != 2) return false;
  if (K % 64 != 0 || M < BM || N < BN) return false;   // every TMA box lies within its tensor
  if (K > (int64_t)1 << 30 || M > ((int64_t)1 << 31) - 1 || N > ((int64_t)1 << 31) - 1) return false;
  return true;
}

cudaError_t launch_gemm_tc(const uint8_t* A, const uint8_t* B, const uint8_t* SA, const uint8_t* SB, int64_t M,
                           int64_t N, int64_t K, int64_t sa_cols, int64_t sb_cols, const float* alpha,
                           const GemmArgs& args, void* out, void* workspace, cudaStream_t stream) {
  using namespace tc;
  const int fmt = args.format;
  const int gs = fmt == EMU_FMT_NVFP4 ? 16 : 32;
  const int64_t G = K / gs;
  const int64_t Np = (N + BN - 1) / BN * BN;
  const WsLayout L = layout(fmt, M, N, K);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  __half* a16 = reinterpret_cast<__half*>(ws + L.a16);
  __half* b16 = reinterpret_cast<__half*>(ws + L.b16);
  int* err = reinterpret_cast<int*>(ws + L.err);

  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  cudaError_t e = cudaMemsetAsync(err, 0, 16, stream);
  if (e != cudaSuccess) return e;

  auto grid_for = [&](int64_t n) { return (unsigned)std::max<int64_t>(1, std::min<int64_t>((n + 255) / 256, (int64_t)sms * 16)); };
  unpack_fp16x2_kernel<<<grid_for(M * K / 16), 256, 0, stream>>>(A, M, K, a16);
  unpack_fp16x2_kernel<<<grid_for(N * K / 16), 256, 0, stream>>>(B, N, K, b16);
  if (fmt == EMU_FMT_NVFP4) {
    row_scales_kernel<EMU_FMT_NVFP4><<<grid_for(M), 256, 0, stream>>>(SA, M, G, sa_cols, ws + L.row_tab, ws + L.row_nan);
    col_scales_kernel<EMU_FMT_NVFP4><<<grid_for(G * Np), 256, 0, stream>>>(SB, N, Np, G, sb_cols,
                                                                          reinterpret_cast<double*>(ws + L.sb_tab), ws + L.col_nan);
  } else {
    row_scales_kernel<EMU_FMT_MXFP4><<<grid_for(M), 256, 0, stream>>>(SA, M, G, sa_cols, ws + L.row_tab, nullptr);
    col_scales_kernel<EMU_FMT_MXFP4><<<grid_for(G * Np), 256, 0, stream>>>(SB, N, Np, G, sb_cols,
                                                                          reinterpret_cast<double*>(ws + L.sb_tab), nullptr);
  }
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;

  CUtensorMap tmA, tmB, tmSB;
  const int gpb = fmt == EMU_FMT_NVFP4 ? 4 : 2;
  if (!make_map_2d(&tmA, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, a16, K, M, K * 2, BK, BM, CU_TENSOR_MAP_SWIZZLE_128B) ||
      !make_map_2d(&tmB, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, b16, K, N, K * 2, BK, BN, CU_TENSOR_MAP_SWIZZLE_128B) ||
      !make_map_2d(&tmSB, CU_TENSOR_MAP_DATA_TYPE_FLOAT64, ws + L.sb_tab, Np, G, Np * 8, BN, gpb,
                   CU_TENSOR_MAP_SWIZZLE_NONE))
    return cudaErrorInvalidValue;

  Params prm;
  prm.M = M; prm.N = N; prm.K = K; prm.G = G; prm.nb = K / BK;
  prm.tiles_m = (M + BM - 1) / BM; prm.tiles_n = (N + BN - 1) / BN;
  prm.row_tab = ws + L.row_tab;
  prm.row_nan = ws + L.row_nan;
  prm.col_nan = ws + L.col_nan;
  prm.alpha = alpha;
  prm.out = out;
  prm.err = err;
  prm.r3 = args.stage3_rounding;
  prm.r4 = args.stage4_rounding;
  prm.out_mode = args.out_mode;

  const int64_t tiles = prm.tiles_m * prm.tiles_n;
  const unsigned grid = (unsigned)std::min<int64_t>(tiles, sms);
  if (fmt == EMU_FMT_NVFP4) {
    cudaFuncSetAttribute(emul_gemm_tc_kernel<EMU_FMT_NVFP4>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
    emul_gemm_tc_kernel<EMU_FMT_NVFP4><<<grid, NUM_THREADS, SMEM_BYTES, stream>>>(tmA, tmB, tmSB, prm);
  } else {
    cudaFuncSetAttribute(emul_gemm_tc_kernel<EMU_FMT_MXFP4>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
    emul_gemm_tc_kernel<EMU_FMT_MXFP4><<<grid, NUM_THREADS, SMEM_BYTES, stream>>>(tmA, tmB, tmSB, prm);
  }
  return cudaGetLastError();
}

}  // namespace emu
