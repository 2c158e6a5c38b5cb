// Emulated scaled FP4 GEMM on the 5th-generation tensor cores (tcgen05 + TMEM + TMA), sm_100a.
//
// Stage 1 (the exact group dot products) runs on the tensor core; stages 2-4 (scale, exact group sums,
// RZ/RNE accumulation) run on CUDA cores reading TMEM.  Bit-exact to the reference emulators
// (nvfp_emulation.cpp:90-156, mxfp_emulation.cpp:98-166) for the reference's accumulator shapes:
// NVFP4 w_reduce 4 and MXFP4 w_reduce 2 (one 64-element K block per stage-3 sum).
//
// Pre-pass kernels (per call):
//   unpack_stats    packed e2m1 -> fp16 "2x" integers (exact), plus per (row, group) the L1, max and
//                   squared L2 norms of the 2x values, which bound |p4| = |4 * group dot| from above.
//   row / col       scale tables for the epilogue paths (below) and per-(row|col, block) exponent
//                   bases; row and column records are laid out per (block, tile) so one bulk copy
//                   each brings a block's row and column data into shared memory.
//   tile stats      per (128-row | 64-column tile, group) maxima of the norms and multipliers.
//   decide          per (row tile, column tile, block): block-sum, mixed, integer or f64 path (below).
//   tile f32/lists  per tile pair: may its block-sum updates run in f32 (exactness bound, share of
//                   blocks off the block-sum path); the tile pairs split into two lists by that flag.
//   fold            the operands times their group multipliers, for the block-sum / mixed / integer
//                   paths: A within its unpack pass, B after the tile stats (twice: every group
//                   folded, and all but the mixed path's separate group).
//
// Main kernel: persistent, one CTA per SM, 12 warps, launched once per tile list (F32 = 0 / 1):
//   warp 0      producer: TMA A [128 x 64] and B [64 x 64] fp16 tiles (128-byte swizzle; the folded
//               or raw operand per the block's path) into a 6-stage ring, the block's path code in a
//               shared byte per stage; bulk copies of the block's column and row records into an
//               8-slot ring.
//   warp 1      TMEM owner + MMA issuer (tcgen05.mma kind::f16 M128 N64 K16): the block-sum path
//               into one accumulator, the other paths one accumulator per group.  512 columns = a
//               ring of K-block sets (NVFP4: 2 sets of 4 x 64; MXFP4: 4 sets of 2 x 64).
//   warps 4-11  epilogue: a thread owns one output row (its TMEM lane) and 32 columns.
//
// Block-sum path (tile bounds prove it exact): operands pre-multiplied by the group multipliers
//     x' = 2a * ma * 2^(ea_g - ea), y' = 2b * mb * 2^(eb_g - eb) (exact fp16 integers), one bias MMA
//     writing 1.5*2^23 and the block's four K16 MMAs into ONE accumulator: its f32 word is exactly
//     0x4B400000 + T, T = sum_g p4_g * ma'_g * mb'_g.  Epilogue per output and block:
//     Tf = double{2^(52+e_row), T + 2^31} - (2^52 + 2^31) * 2^e_row = T * 2^e_row,
//     acc = R4(FMA(Tf, 2^e_col, acc));  in the F32 launch acc = R4(FFMA(T * 2^e_row, 2^e_col, acc)) in f32.
// Mixed path (NVFP4): the block-sum path over all groups but one, that group's B left unscaled in its
//     own accumulator (an integer-path word): T = (w0 - bias) + (w1 - bias) * mb'.  Then as above.
// Integer path: A folded, B raw, one accumulator per group started from the 1.5*2^23 bias, so each
//     word is 0x4B400000 + p4 * ma'; S32 = sum_g word * mb'_g wraps in int32 and a per-column
//     constant removes the bias terms: S32 + K_col = T + 2^31.  Then as above.
// f64 path (any other block):  per group partial
//     NVFP4: diff = double{2^E(sa), FFMA(p4, ma, 1.5*2^23)} - double{2^E(sa), 2^23 bias} = p*sa
//            S = FMA(diff, sb, S)
//     MXFP4: p4 exactly as f64 by the same construction; S = FMA(p4 * sa/4, sb, S)  (inf/NaN as IEEE)
//   with stage-1 fp16 rounding applied when a warp sees |p4| >= 2048.
// Conversions into 64-bit types are never used per partial: they run at a quarter of the FP64 rate.
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <stdlib.h>

#include <algorithm>
#include <atomic>
#include <type_traits>

#include "common.cuh"
#include "kernels.h"
#include "tc_ptx.cuh"

namespace emu {
namespace tc {

constexpr int BM = 128, BN = 64, BK = 64;
constexpr int NSTAGE = 6, NCR = 8;
constexpr int A_BYTES = BM * BK * 2, B_BYTES = BN * BK * 2;
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;          // 24 KB
constexpr float MAGIC_F = 12582912.0f;                  // 1.5 * 2^23
constexpr uint32_t MAGIC_BITS = 0x4B400000u;
constexpr double TWO52 = 4503599627370496.0;
constexpr int GROUP_M = 16;                             // tile raster: 16 M-tiles per band

// Column record of one (K block, 64-column tile), GPB groups:
//   int32  sbq[4][64]   mb * 2^(eb_g - eb)                       (integer / mixed path)
//   uint32 kc[64]       2^31 - 2^23-bias * sum_g sbq   (mod 2^32)  (integer path)
//   double cs[64]       2^eb * unit                               (integer / mixed / block-sum path)
//   float  csf[64]      the same in f32                           (block-sum path, f32 update)
//   double sbw[4][64]   sb as f64                                 (f64 path)
constexpr int CR_SBQ = 0, CR_KC = 1024, CR_CS = 1280, CR_CSF = 1792, CR_SBW = 2048, CR_BYTES = 4096;
// Row record of one (K block, 128-row tile):
//   double2 rs[128]      row base {exponent word of 2^(52+e) (high half), (2^52 + 2^31) * 2^e}
constexpr int RR_RS = 0, RR_BYTES = 2048;
// Per-block path code (decide kernel): bits 0-1 the epilogue path, bit 2 set when the accumulator
// provably stays in the f32 normal range (always for NVFP4), so 24-bit rounding in f64 is exact;
// bits 3-4 the group the mixed path keeps apart.
constexpr uint8_t PATH_F64 = 0, PATH_INT = 1, PATH_SUM = 2, PATH_MIXED = 3, PATH_NORMAL = 4;
constexpr int PATH_GROUP_SHIFT = 3;
// Constant bias tiles for the block-sum path: A row r = {3072, 0, ...}, B row n = {4096, 0, ...} in
// the 128-byte-swizzled K-major layout, so one K=16 MMA writes 3072 * 4096 = 1.5 * 2^23 everywhere.
constexpr int BIAS_BYTES = A_BYTES + B_BYTES;
// mbarriers (full/empty per stage, cr_full/cr_empty per record slot, 4 + 4 TMEM-set barriers, drain)
// the TMEM address word and one path byte per stage, after the rings; the leading 1024 bytes cover
// aligning the base to 1024
constexpr int BAR_BYTES = (2 * NSTAGE + 2 * NCR + 9) * 8 + 8 + 8;
static_assert(NSTAGE <= 8, "one path byte per stage after the TMEM address word");
constexpr int SMEM_BYTES = 1024 + NSTAGE * STAGE_BYTES + BIAS_BYTES + NCR * (CR_BYTES + RR_BYTES) + BAR_BYTES;
static_assert(SMEM_BYTES <= 232448, "shared memory per CTA");
constexpr uint32_t F_TO_T31 = 0x80000000u - MAGIC_BITS;   // (T + 0x4B400000) + this = T + 2^31 (mod 2^32)

// NVFP4 f64-path row record, one per (row, group).
struct __align__(16) RowScaleNv {
  float ma;        // signed E4M3 significand (0..15), 0 for NaN / zero
  uint32_t hi;     // exponent word of 2^(sxa + 50), low 20 mantissa bits zero
  double d0;       // double{hi, MAGIC_BITS}
};

template <int FMT> struct Fmt;
template <> struct Fmt<EMU_FMT_NVFP4> { static constexpr int GS = 16, GPB = 4; };
template <> struct Fmt<EMU_FMT_MXFP4> { static constexpr int GS = 32, GPB = 2; };

// ------------------------------------------------------------------------------ pre-pass
// One thread per 16 elements.  For 32-element groups the two halves sit in adjacent lanes.  FOLD
// (the A operand): also writes the block-sum / mixed / integer paths' operand, the "2x" values times
// their row-group multiplier `mult` (ma * 2^(e_g - e)) in fp16 -- exact wherever a block passes the
// decide test (|product| <= 65504, at most 6 significant bits); other values are never read.
template <int GS, bool FOLD = false>
__global__ void unpack_stats_kernel(const uint8_t* __restrict__ packed, int64_t rows, int64_t K,
                                    __half* __restrict__ out, uint32_t* __restrict__ stats,
                                    const float* __restrict__ mult = nullptr, __half* __restrict__ folded = nullptr) {
  const int64_t n8 = rows * (K / 16);
  const int64_t G = K / GS;
  const int64_t loop = (n8 + 31) / 32 * 32;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < loop; i += (int64_t)gridDim.x * blockDim.x) {
    uint32_t l1 = 0, li = 0, l2 = 0;
    const bool live = i < n8;
    if (live) {
      const uint2 w = reinterpret_cast<const uint2*>(packed)[i];
      const uint32_t in[2] = {w.x, w.y};
      uint32_t o[8];
#pragma unroll
      for (int h = 0; h < 2; ++h)
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int lo = e2m1_twice((in[h] >> (8 * q)) & 0xFu), hi = e2m1_twice((in[h] >> (8 * q + 4)) & 0xFu);
          const uint32_t alo = (uint32_t)abs(lo), ahi = (uint32_t)abs(hi);
          l1 += alo + ahi;
          li = max(li, max(alo, ahi));
          l2 += alo * alo + ahi * ahi;
          o[4 * h + q] =
              (uint32_t)__half_as_ushort(__int2half_rn(lo)) | ((uint32_t)__half_as_ushort(__int2half_rn(hi)) << 16);
        }
      uint4* dst = reinterpret_cast<uint4*>(out) + 2 * i;
      dst[0] = make_uint4(o[0], o[1], o[2], o[3]);
      dst[1] = make_uint4(o[4], o[5], o[6], o[7]);
      if (FOLD) {
        const int64_t r = i / (K / 16), k0 = (i % (K / 16)) * 16;
        const float m = mult[r * G + k0 / GS];
        uint32_t f[8];
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          const float2 v = __half22float2(*reinterpret_cast<const __half2*>(&o[q]));
          const __half2 h = __floats2half2_rn(v.x * m, v.y * m);
          f[q] = *reinterpret_cast<const uint32_t*>(&h);
        }
        uint4* fd = reinterpret_cast<uint4*>(folded) + 2 * i;
        fd[0] = make_uint4(f[0], f[1], f[2], f[3]);
        fd[1] = make_uint4(f[4], f[5], f[6], f[7]);
      }
    }
    if (GS == 32) {
      l1 += __shfl_xor_sync(0xFFFFFFFFu, l1, 1);
      li = max(li, __shfl_xor_sync(0xFFFFFFFFu, li, 1));
      l2 += __shfl_xor_sync(0xFFFFFFFFu, l2, 1);
    }
    if (live && (GS == 16 || (i & 1) == 0)) {
      const int64_t r = i / (K / 16), c = i % (K / 16);
      stats[r * G + c / (GS / 16)] = l1 | (li << 10) | (l2 << 14);   // <= 384 | <= 12 | <= 4608
    }
  }
}

struct PrepTables {
  float* rmaq;          // [M][G]    integer-path row multipliers
  uint8_t* rowrec;      // [nb][tiles_m][RR_BYTES]
  void* rw;             // [M][G]    f64-path rows: RowScaleNv (NVFP4) / double sa/4 (MXFP4)
  uint32_t* row_nan;    // [M]       NVFP4: any NaN scale in the row
  uint8_t* rinf;        // [M][nb]   MXFP4: a 255 scale in the block
  uint8_t* colrec;      // [nb][tiles_n][CR_BYTES]
  uint32_t* col_nan;    // [Np]
  uint8_t* cinf;        // [Np][nb]
  uint32_t* ast;        // [M][G]    L1 | Linf << 10 | L2^2 << 14 of the 2x values
  uint32_t* bst;        // [N][G]
  uint2* rts;           // [tiles_m][G]   {max L1 | max Linf << 16, max L2^2} over the tile's rows
  float4* rtm;          // [tiles_m][G]   max of L1 * |mult|, Linf * |mult|, L2^2 * mult^2 over the rows
  uint8_t* rtinf;       // [tiles_m][nb]
  uint2* cts;           // [tiles_n][G]
  float4* ctm;          // [tiles_n][G]
  uint8_t* ctinf;       // [tiles_n][nb]
  uint8_t* path;        // [tiles_m][tiles_n][nb]  path code
  uint32_t* rng_r;      // [tiles_m][2]  MXFP4: max scale byte, 255 - min scale byte (zeroed per call)
  uint32_t* rng_c;      // [tiles_n][2]
  uint32_t* rbmax;      // [tiles_m][nb] NVFP4: 512 + max row base exponent over the tile (zeroed per call)
  uint32_t* cbmax;      // [tiles_n][nb]
  uint32_t* rbmin;      // [tiles_m]     NVFP4: 512 - min row base exponent over the tile and all blocks
  uint32_t* cbmin;      // [tiles_n]
  float* tile_bound;    // [tiles_m][tiles_n] NVFP4: bound on sum_b max |s_b| (zeroed per call)
  uint32_t* tile_other; // [tiles_m][tiles_n] blocks off the block-sum path (zeroed per call)
  uint8_t* tile_f32;    // [tiles_m][tiles_n] 1: the tile pair goes to the launch with f32 block-sum updates
};

// E4M3 -> (signed significand, exponent) with value = ma * 2^sx; NaN -> ma 0.
__device__ __forceinline__ void e4m3_split(uint32_t byte, int& ma, int& sx, bool& nan) {
  const uint32_t e = (byte >> 3) & 0xFu, m = byte & 7u;
  nan = (e == 15u && m == 7u);
  ma = (e == 0u) ? (int)m : (int)(8u + m);
  sx = (e == 0u) ? -9 : (int)e - 10;
  if (byte & 0x80u) ma = -ma;
  if (nan) ma = 0;
}

__device__ __forceinline__ double pow2d(int e) {   // exact 2^e for e in [-1022, 1023]
  return __longlong_as_double((long long)(e + 1023) << 52);
}

__device__ __forceinline__ float pow2f(int e) {    // exact 2^e for e in [-149, 127]
  return e >= -126 ? __int_as_float((e + 127) << 23) : __int_as_float(1 << (e + 149));
}

// atomicMax of v into *slot, reduced first over the active lanes of the warp that target the same slot
__device__ __forceinline__ void warp_atomic_max(uint32_t* slot, uint32_t v) {
  const unsigned peers = __match_any_sync(__activemask(), reinterpret_cast<unsigned long long>(slot));
  v = __reduce_max_sync(peers, v);
  if ((threadIdx.x & 31) == __ffs(peers) - 1) atomicMax(slot, v);
}

// Row base record for exponent e: x = double{hi = exponent word of 2^(52+e), lo = T + 2^31} is
// 2^(52+e) + (T + 2^31) * 2^e, so x - (2^52 + 2^31) * 2^e = T * 2^e exactly.
__device__ __forceinline__ double2 row_base(int e) {
  double2 r;
  r.x = __longlong_as_double((long long)(52 + e + 1023) << 52);   // bits; only the high word is used
  r.y = (4503599627370496.0 + 2147483648.0) * pow2d(e);
  return r;
}

// MXFP4: fold this thread's scale bytes into its tile's {max byte, 255 - min byte}
__device__ __forceinline__ void scale_range(const uint32_t* byte, int n, uint32_t* rng) {
  uint32_t mx = 0, mn = 255;
  for (int g = 0; g < n; ++g) { mx = max(mx, byte[g]); mn = min(mn, byte[g]); }
  warp_atomic_max(&rng[0], mx);
  warp_atomic_max(&rng[1], 255u - mn);
}

// one thread per (row, block)
template <int FMT>
__global__ void row_tables_kernel(const uint8_t* __restrict__ sf, int64_t M, int64_t Mp, int64_t G, int64_t nb,
                                  int64_t sf_cols, PrepTables t) {
  constexpr int GPB = Fmt<FMT>::GPB;
  const int64_t tiles_m = Mp / BM;
  // the block index runs fastest, so a warp's per-(row, group) table writes are contiguous
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < Mp * nb; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / nb, kb = i % nb;
    uint8_t* rec = t.rowrec + (kb * tiles_m + r / BM) * RR_BYTES;
    double2* rs = reinterpret_cast<double2*>(rec + RR_RS) + r % BM;
    if (r >= M) {   // rows of the last tile beyond M: finite, discarded by the epilogue
      *rs = row_base(0);
      continue;
    }
    uint32_t byte[GPB];
#pragma unroll
    for (int g = 0; g < GPB; ++g) byte[g] = sf[swz_offset(r, kb * GPB + g, sf_cols)];
    if (FMT == EMU_FMT_NVFP4) {
      int ma[GPB], sx[GPB];
      bool nan[GPB], any_nan = false;
      int base = 1 << 30;
#pragma unroll
      for (int g = 0; g < GPB; ++g) {
        e4m3_split(byte[g], ma[g], sx[g], nan[g]);
        any_nan |= nan[g];
        if (ma[g] != 0) base = min(base, sx[g]);
      }
      if (base == (1 << 30)) base = 0;
#pragma unroll
      for (int g = 0; g < GPB; ++g) {
        t.rmaq[r * G + kb * GPB + g] = ma[g] == 0 ? 0.0f : (float)ma[g] * (float)(1 << (sx[g] - base));
        RowScaleNv rec;
        rec.ma = (float)ma[g];
        rec.hi = (uint32_t)(sx[g] + 1073) << 20;
        rec.d0 = __hiloint2double((int)rec.hi, (int)MAGIC_BITS);
        static_cast<RowScaleNv*>(t.rw)[r * G + kb * GPB + g] = rec;
      }
      *rs = row_base(base - 1);     // v = p4*ma*mb*2^(sxa+sxb-2)
      if (any_nan) atomicOr(&t.row_nan[r], 1u);
      warp_atomic_max(&t.rbmax[(r / BM) * nb + kb], (uint32_t)(base + 512));
      warp_atomic_max(&t.rbmin[r / BM], (uint32_t)(512 - base));
    } else {
      int base = 1 << 30;
      bool inf = false;
#pragma unroll
      for (int g = 0; g < GPB; ++g) {
        if (byte[g] == 255u) inf = true;
        else base = min(base, (int)byte[g]);
      }
      if (base == (1 << 30)) base = 0;
#pragma unroll
      for (int g = 0; g < GPB; ++g) {
        const int d = (int)byte[g] - base;
        // 2^126 sentinel: finite, and fails the bounds unless the data is 0
        t.rmaq[r * G + kb * GPB + g] = (byte[g] == 255u) ? 0.0f : __int_as_float((min(d, 126) + 127) << 23);
        static_cast<double*>(t.rw)[r * G + kb * GPB + g] = ue8m0_quarter_f64(byte[g]);
      }
      *rs = row_base(base - 128);  // v = p4 * 2^(ua+ub-256)
      t.rinf[r * nb + kb] = inf ? 1 : 0;
      scale_range(byte, GPB, t.rng_r + 2 * (r / BM));
    }
  }
}

// one thread per (column, block), columns padded to the tile
template <int FMT>
__global__ void col_tables_kernel(const uint8_t* __restrict__ sf, int64_t N, int64_t Np, int64_t G, int64_t nb,
                                  int64_t sf_cols, PrepTables t) {
  constexpr int GPB = Fmt<FMT>::GPB;
  const int64_t tiles_n = Np / BN;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < Np * nb; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t kb = i / Np, n = i % Np;
    const int64_t tn = n / BN, c = n % BN;
    uint8_t* rec = t.colrec + (kb * tiles_n + tn) * CR_BYTES;
    int32_t* sbq = reinterpret_cast<int32_t*>(rec + CR_SBQ);
    uint32_t* kc = reinterpret_cast<uint32_t*>(rec + CR_KC);
    double* cs = reinterpret_cast<double*>(rec + CR_CS);
    float* csf = reinterpret_cast<float*>(rec + CR_CSF);
    double* sbw = reinterpret_cast<double*>(rec + CR_SBW);
    uint32_t sum = 0;
    if (n >= N) {
#pragma unroll
      for (int g = 0; g < GPB; ++g) { sbq[g * BN + c] = 0; sbw[g * BN + c] = 0.0; }
      kc[c] = 0x80000000u;
      cs[c] = 0.0;
      csf[c] = 0.0f;
      t.cinf[n * nb + kb] = 0;
      continue;
    }
    uint32_t byte[GPB];
#pragma unroll
    for (int g = 0; g < GPB; ++g) byte[g] = sf[swz_offset(n, kb * GPB + g, sf_cols)];
    if (FMT == EMU_FMT_NVFP4) {
      int mb[GPB], sx[GPB];
      bool nan[GPB], any_nan = false;
      int base = 1 << 30;
#pragma unroll
      for (int g = 0; g < GPB; ++g) {
        e4m3_split(byte[g], mb[g], sx[g], nan[g]);
        any_nan |= nan[g];
        if (mb[g] != 0) base = min(base, sx[g]);
      }
      if (base == (1 << 30)) base = 0;
#pragma unroll
      for (int g = 0; g < GPB; ++g) {
        const int32_t q = mb[g] == 0 ? 0 : mb[g] * (1 << (sx[g] - base));
        sbq[g * BN + c] = q;
        sum += (uint32_t)q;
        sbw[g * BN + c] = (double)mb[g] * pow2d(sx[g]);
      }
      cs[c] = pow2d(base - 1);
      csf[c] = pow2f(base - 1);
      if (any_nan) atomicOr(&t.col_nan[n], 1u);
      warp_atomic_max(&t.cbmax[tn * nb + kb], (uint32_t)(base + 512));
      warp_atomic_max(&t.cbmin[tn], (uint32_t)(512 - base));
      t.cinf[n * nb + kb] = 0;
    } else {
      int base = 1 << 30;
      bool inf = false;
#pragma unroll
      for (int g = 0; g < GPB; ++g) {
        if (byte[g] == 255u) inf = true;
        else base = min(base, (int)byte[g]);
      }
      if (base == (1 << 30)) base = 0;
#pragma unroll
      for (int g = 0; g < GPB; ++g) {
        const int d = (int)byte[g] - base;
        // exponent spreads beyond 2^30 cannot pass the integer-path bounds: record a value that fails them
        const int32_t q = (byte[g] == 255u) ? 0 : (d <= 30 ? (1 << d) : 0x7FFFFFFF);
        sbq[g * BN + c] = q;
        sum += (uint32_t)q;
        sbw[g * BN + c] = ue8m0_quarter_f64(byte[g]) * 4.0;
      }
      cs[c] = pow2d(base - 128);
      csf[c] = pow2f(base - 128);
      t.cinf[n * nb + kb] = inf ? 1 : 0;
      scale_range(byte, GPB, t.rng_c + 2 * tn);
    }
    kc[c] = 0x80000000u - MAGIC_BITS * sum;
  }
}

// The group the mixed path keeps apart in a (column tile, K block): the one with the largest
// max |2b| * |mb'| over the tile's columns (first on ties).  The fold kernel and the decide kernel both
// derive it from the same table.
template <int GPB>
__device__ __forceinline__ int mixed_group(const float4* __restrict__ ctm, int64_t tn, int64_t kb, int64_t G) {
  int gx = 0;
  float best = ctm[tn * G + kb * GPB].y;
#pragma unroll
  for (int g = 1; g < GPB; ++g) {
    const float v = ctm[tn * G + kb * GPB + g].y;
    if (v > best) { best = v; gx = g; }
  }
  return gx;
}


// B operands, the "2x" values times their column-group multiplier (mb * 2^(e_g - e)) in fp16, exact
// wherever a block passes the decide test: `out` every group folded (block-sum path); `out_mixed`
// (NVFP4) the same except the mixed path's separate group of the (column tile, block), which keeps
// the plain "2x" values.
template <int FMT>
__global__ void fold_cols_kernel(const __half* __restrict__ x16, int64_t N, int64_t K, int64_t tiles_n,
                                 const uint8_t* __restrict__ colrec, const float4* __restrict__ ctm,
                                 __half* __restrict__ out, __half* __restrict__ out_mixed) {
  constexpr int GS = Fmt<FMT>::GS, GPB = Fmt<FMT>::GPB;
  const int64_t n8 = N * (K / 8);
  const int64_t G = K / GS;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n8; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t n = i / (K / 8), k0 = (i % (K / 8)) * 8;
    const int64_t g = k0 / GS, kb = g / GPB;
    const uint8_t* rec = colrec + (kb * tiles_n + n / BN) * CR_BYTES;
    const float m = (float)reinterpret_cast<const int32_t*>(rec + CR_SBQ)[(g % GPB) * BN + n % BN];
    const bool apart = FMT == EMU_FMT_NVFP4 && (int)(g % GPB) == mixed_group<GPB>(ctm, n / BN, kb, G);
    const uint4 w = reinterpret_cast<const uint4*>(x16)[i];
    uint32_t in[4] = {w.x, w.y, w.z, w.w}, o[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&in[q]));
      const __half2 h = __floats2half2_rn(f.x * m, f.y * m);
      o[q] = *reinterpret_cast<const uint32_t*>(&h);
    }
    reinterpret_cast<uint4*>(out)[i] = make_uint4(o[0], o[1], o[2], o[3]);
    if (FMT == EMU_FMT_NVFP4) reinterpret_cast<uint4*>(out_mixed)[i] = apart ? w : make_uint4(o[0], o[1], o[2], o[3]);
  }
}

// per (tile, group) maxima over the tile's rows (A) or columns (B) of the norms and of norm x
// integer multiplier; per (tile, block) inf flags
template <int FMT>
__global__ void tile_stats_kernel(int64_t rows, int64_t tile, int64_t ntiles, int64_t G, int64_t nb, int is_col,
                                  PrepTables t) {
  constexpr int GPB = Fmt<FMT>::GPB;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < ntiles * G; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t tl = i / G, g = i % G;
    const int64_t kb = g / GPB;
    const int64_t r0 = tl * tile, r1 = min(rows, r0 + tile);
    uint32_t l1 = 0, li = 0, l2 = 0;
    float m1 = 0.0f, mi = 0.0f, m2 = 0.0f;
    bool inf = false;
    for (int64_t r = r0; r < r1; ++r) {
      const uint32_t s = (is_col ? t.bst : t.ast)[r * G + g];
      const uint32_t sl1 = s & 0x3FFu, sli = (s >> 10) & 0xFu, sl2 = s >> 14;
      l1 = max(l1, sl1);
      li = max(li, sli);
      l2 = max(l2, sl2);
      float mult;
      if (is_col) {
        const uint8_t* rec = t.colrec + (kb * ntiles + tl) * CR_BYTES;
        mult = fabsf((float)reinterpret_cast<const int32_t*>(rec + CR_SBQ)[(g % GPB) * BN + (r - r0)]);
        inf |= t.cinf[r * nb + kb] != 0;
      } else {
        mult = fabsf(t.rmaq[r * G + g]);
        if (FMT == EMU_FMT_MXFP4) inf |= t.rinf[r * nb + kb] != 0;
      }
      m1 = fmaxf(m1, (float)sl1 * mult);    // rounded f32 maxima (inf when out of range): the decide
      mi = fmaxf(mi, (float)sli * mult);    // kernel compares them with a 2^-20 safety margin
      m2 = fmaxf(m2, (float)sl2 * mult * mult);
    }
    (is_col ? t.cts : t.rts)[tl * G + g] = make_uint2(l1 | (li << 16), l2);
    (is_col ? t.ctm : t.rtm)[tl * G + g] = make_float4(m1, mi, m2, 0.0f);
    if (g % GPB == 0) (is_col ? t.ctinf : t.rtinf)[tl * nb + kb] = inf ? 1 : 0;
  }
}

// Path code per (row tile, column tile, block).  With x = 2a, y = 2b the 2x values of one group and
// L1, Linf, L2 their norms, |p4| = |sum x y| <= min(L1(x) Linf(y), Linf(x) L1(y), L2(x) L2(y)) for
// every (row, column), and the same holds with the multipliers ma', mb' folded in.  Evaluated on
// tile maxima of the norms and of the norms times the multipliers:
//   integer path    no stage-1 fp16 rounding (|p4| < 2048); every per-group word 1.5*2^23 + p4*ma'
//                   exact in f32 (sum |x ma'| |y| < 2^22); the folded A operand exact in fp16
//                   (max |x ma'| <= 65504); |T| < 2^31 for the int32 sum;
//   block-sum path  additionally the folded B operand exact in fp16 and sum |x ma'| |y mb'| < 2^22
//                   over the whole block, so the f32 accumulation of 1.5*2^23 + T is exact;
//   mixed path      (NVFP4) the integer-path conditions, and the block-sum conditions over every group but
//                   one (the column tile's group with the largest B multiplier), which gets its own
//                   integer-path word;
//   f64 path        every other block.
template <int FMT>
__global__ void decide_kernel(int64_t tiles_m, int64_t tiles_n, int64_t nb, int64_t G, PrepTables t) {
  constexpr int GPB = Fmt<FMT>::GPB;
  const double margin = 1.0 + 0x1p-20;   // covers the f32 rounding of the stored maxima
  int lg_nb = 0;
  while ((1ll << lg_nb) < nb) ++lg_nb;
  const int64_t total = tiles_m * tiles_n * nb;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t kb = i % nb, tn = (i / nb) % tiles_n, tm = i / (nb * tiles_n);
    bool ok = !t.rtinf[tm * nb + kb] && !t.ctinf[tn * nb + kb];
    bool fold_a = true, fold_b = true;
    double s1 = 0.0, s2 = 0.0, s3 = 0.0;
    // the same sums without the mixed path's separate group
    const int gx = mixed_group<GPB>(t.ctm, tn, kb, G);
    bool fold_rest = true;
    double r1 = 0.0, r2 = 0.0, r3 = 0.0;
#pragma unroll
    for (int g = 0; g < GPB; ++g) {
      const int64_t gg = kb * GPB + g;
      const uint2 ra = t.rts[tm * G + gg], cb = t.cts[tn * G + gg];
      const double l1a = ra.x & 0xFFFFu, lia = ra.x >> 16, l1b = cb.x & 0xFFFFu, lib = cb.x >> 16;
      const double l2a = ra.y, l2b = cb.y;   // squared L2 norms, exact integers
      const float4 am = t.rtm[tm * G + gg], bm = t.ctm[tn * G + gg];
      // |sum_k x_k y_k| <= min(L1(x) Linf(y), Linf(x) L1(y), L2(x) L2(y)) per (row, column)
      const bool p_small = fmin(l1a * lib, lia * l1b) < 2048.0 || l2a * l2b < 2048.0 * 2048.0;
      const double tmax = fmin(fmin((double)am.x * lib, (double)am.y * l1b), sqrt((double)am.z * l2b) * margin) * margin;
      ok = ok && p_small && (tmax < 4194304.0);
      // folded operands: max |2a * ma'| = max Linf * |ma'| (and the B side) must be exact fp16 values
      fold_a = fold_a && ((double)am.y * margin <= 65504.0);
      const bool fb = (double)bm.y * margin <= 65504.0;
      fold_b = fold_b && fb;
      const double t1 = (double)am.x * (double)bm.y * margin, t2 = (double)am.y * (double)bm.x * margin,
                   t3 = sqrt((double)am.z * (double)bm.z) * margin * margin;
      s1 += t1;
      s2 += t2;
      s3 += t3;
      if (g != gx) {
        fold_rest = fold_rest && fb;
        r1 += t1;
        r2 += t2;
        r3 += t3;
      }
    }
    const double tb = fmin(fmin(s1, s2), s3);
    ok = ok && fold_a && (tb < 2147483648.0);
    // the block sum accumulates 1.5*2^23 + T in f32 on the tensor core: exact while every partial sum
    // stays in (2^23, 2^24), i.e. |partial sums of T| < 2^22, which tb bounds
    const bool sum = ok && fold_b && (tb < 4194304.0);
    // mixed path: the block sum of the other groups on the tensor core as above (word 0), the separate
    // group as an integer-path word (word 1, whose bound tmax already holds); |T| < 2^31 as above
    // (NVFP4 only: MXFP4 blocks rarely miss the block-sum path and its epilogue keeps one path less)
    const bool mixed = FMT == EMU_FMT_NVFP4 && ok && fold_rest && (fmin(fmin(r1, r2), r3) < 4194304.0);
    uint8_t code = sum ? PATH_SUM : mixed ? (uint8_t)(PATH_MIXED | (gx << PATH_GROUP_SHIFT)) : (ok ? PATH_INT : PATH_F64);
    float sabs = 0.0f;
    if (FMT == EMU_FMT_NVFP4) {
      code |= PATH_NORMAL;   // |acc| < 2^40 and every term a multiple of 2^-20: always in range
      // |s_b| <= tb * 2^(row base + column base - 2) for every output of the tile pair
      const int eb = (int)t.rbmax[tm * nb + kb] + (int)t.cbmax[tn * nb + kb] - 1024 - 2;
      sabs = ok ? (float)(tb * margin * pow2d(eb)) : __int_as_float(0x7F800000);
    } else {
      // every block term is a multiple of 2^(minA + minB - 256) and at most 9216 * 2^(maxA + maxB - 256):
      // no accumulator value is subnormal or reaches 2^127 when these hold for the whole tile pair
      const uint32_t maxa = t.rng_r[2 * tm], mina = 255u - t.rng_r[2 * tm + 1];
      const uint32_t maxb = t.rng_c[2 * tn], minb = 255u - t.rng_c[2 * tn + 1];
      if (maxa < 255u && maxb < 255u && mina + minb >= 130u && (int)(maxa + maxb) + 14 + lg_nb <= 382)
        code |= PATH_NORMAL;
    }
    t.path[i] = code;
    // per tile pair: the sum of the block bounds and the count of blocks off the block-sum path.  When
    // nb is a multiple of 32 every warp (32-aligned, every lane active) covers blocks of one tile pair
    // and reduces before its single pair of atomics.
    const bool other = (code & 3) != PATH_SUM;
    if ((nb & 31) == 0) {
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) sabs += __shfl_xor_sync(0xFFFFFFFFu, sabs, o);
      const unsigned n_other = __popc(__ballot_sync(0xFFFFFFFFu, other));
      if ((threadIdx.x & 31) == 0) {
        if (FMT == EMU_FMT_NVFP4) atomicAdd(&t.tile_bound[tm * tiles_n + tn], sabs);
        if (n_other) atomicAdd(&t.tile_other[tm * tiles_n + tn], n_other);
      }
    } else {
      if (FMT == EMU_FMT_NVFP4) atomicAdd(&t.tile_bound[tm * tiles_n + tn], sabs);
      if (other) atomicAdd(&t.tile_other[tm * tiles_n + tn], 1u);
    }
  }
}

// Per tile pair: may the block-sum path update the accumulator in f32 under RZ rounding?  The f32
// update computes RZ32(acc + s) in one FMA; the reference computes RZ32(RN64(acc + s)).  They agree
// whenever acc + s is exact in f64, i.e. below 2^53 quanta.  NVFP4: every term of the tile pair is a
// multiple of 2^(min row base + min column base - 2), so is the accumulator (rounding a multiple of a
// power of two to f32 keeps it one), and |acc + s| <= sum_b max |s_b| (RZ never grows a magnitude
// while every sum is exact), bounded by the decide kernel's per-block bounds (2^-16 of margin for
// their f32 summation).  MXFP4: the terms are multiples of 2^(minA + minB - 256), the accumulator
// below nb * 9216 * 2^(maxA + maxB - 256).
// (RNE needs no bound: with both addends 24-bit numbers, rounding to f64 first never changes the
// f32 result.)  Tile pairs where more than a quarter of the blocks leave the block-sum path stay in
// f64 throughout: every switch of representation costs about as much as the f32 update saves.
template <int FMT>
__global__ void tile_f32_kernel(int64_t tiles_m, int64_t tiles_n, int64_t nb, int rm, PrepTables t) {
  int lg_nb = 0;
  while ((1ll << lg_nb) < nb) ++lg_nb;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < tiles_m * tiles_n; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t tm = i / tiles_n, tn = i % tiles_n;
    bool ok;
    if (FMT == EMU_FMT_NVFP4) {
      const int qe = (512 - (int)t.rbmin[tm]) + (512 - (int)t.cbmin[tn]) - 2;
      ok = (double)t.tile_bound[i] < (1.0 - 0x1p-16) * pow2d(53 + qe);
    } else {
      const int maxa = (int)t.rng_r[2 * tm], mina = 255 - (int)t.rng_r[2 * tm + 1];
      const int maxb = (int)t.rng_c[2 * tn], minb = 255 - (int)t.rng_c[2 * tn + 1];
      ok = maxa < 255 && maxb < 255 && (maxa + maxb) - (mina + minb) + 14 + lg_nb <= 52;
    }
    t.tile_f32[i] = ((rm == EMU_RNE || ok) && 4 * (int64_t)t.tile_other[i] <= nb) ? 1 : 0;
  }
}

// ------------------------------------------------------------------------------ main kernel
struct Params {
  const void* cmp_ref;           // optional reference output to compare with (fused check)
  emu_compare_stats* cmp_stats;
  int write_out;
  int64_t M, N, K;
  int64_t G, nb, tiles_m, tiles_n;
  const uint8_t* rowrec;
  const void* rw;
  const uint32_t* row_nan;
  const uint32_t* col_nan;
  const uint8_t* colrec;
  const uint8_t* path;
  const uint32_t* tile_list;     // tile pairs (tm << 16 | tn) this launch processes, raster order
  const uint32_t* tile_count;    // their number (device memory)
  const float* alpha;
  void* out;
  int* err;
  long long wait_limit;          // cycles a pipeline wait may take before the kernel gives up
  int hold_first_ready;          // test hook: the MMA warp withholds block 0's accumulator-ready signal
  int r3, r4, out_mode;
};

// Per device: the code of the first pipeline wait that ran out since the last emu_device_status
// (0 = none).  Codes: 1 producer stage slot, 2 producer record slot, 3 MMA accumulator set, 4 MMA
// stage data, 5 epilogue accumulator, 6 epilogue records, 7-9 drains at exit.
__device__ int g_wait_error;
constexpr long long DRAIN_LIMIT = 1ll << 31;   // waits for copies / MMAs already in flight

// A pipeline wait bounded by the launch's limit (drains by DRAIN_LIMIT, so that every copy and MMA
// the CTA issued has landed before it exits); on expiry records `code` in the workspace's error
// word and the device's sticky word (first error wins in each) and returns false.
__device__ __forceinline__ bool wait_or_record(uint64_t* bar, uint32_t parity, const Params& p, int code,
                                               bool drain = false) {
  if (ptx::mbar_wait(bar, parity, drain ? DRAIN_LIMIT : p.wait_limit)) return true;
  atomicCAS(p.err, 0, code);
  atomicCAS(&g_wait_error, 0, code);
  return false;
}

__device__ __forceinline__ void tile_coords(int64_t t, int64_t tiles_m, int64_t tiles_n, int64_t& tm, int64_t& tn) {
  const int64_t per_band = (int64_t)GROUP_M * tiles_n;
  const int64_t band = t / per_band;
  const int64_t first_m = band * GROUP_M;
  const int64_t rem = tiles_m - first_m;
  const int64_t gm = rem < GROUP_M ? rem : (int64_t)GROUP_M;
  const int64_t idx = t % per_band;
  tm = first_m + idx % gm;
  tn = idx / gm;
}

// Splits the tile pairs, in raster order (bands of GROUP_M row tiles), into the list of the launch
// without f32 updates (counts[0] of them) and the list of the f32 launch (counts[1]), by the tile flag.
// One CTA of 1024 threads, a block-wide scan per chunk of 1024 tile pairs.  Entries are tm << 16 | tn,
// so the producer and MMA warps, which run with few registers, decode them with a shift and a mask.
__global__ void __launch_bounds__(1024) tile_lists_kernel(int64_t tiles_m, int64_t tiles_n,
                                                           const uint8_t* __restrict__ flag, uint32_t* __restrict__ list64,
                                                           uint32_t* __restrict__ list32, uint32_t* __restrict__ counts) {
  __shared__ uint32_t warp_sums[32];
  const int64_t total = tiles_m * tiles_n;
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  int64_t done32 = 0;                      // tile pairs placed in list32 by earlier chunks
  for (int64_t c0 = 0; c0 < total; c0 += 1024) {
    const int64_t t = c0 + threadIdx.x;
    uint32_t id = 0;
    bool f = false;
    if (t < total) {
      int64_t tm, tn;
      tile_coords(t, tiles_m, tiles_n, tm, tn);
      id = (uint32_t)(tm << 16 | tn);
      f = flag[tm * tiles_n + tn] != 0;
    }
    const unsigned ballot = __ballot_sync(0xFFFFFFFFu, f);
    if (lane == 0) warp_sums[w] = __popc(ballot);
    __syncthreads();
    if (w == 0) {
      uint32_t v = warp_sums[lane];
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const uint32_t n = __shfl_up_sync(0xFFFFFFFFu, v, o);
        if (lane >= o) v += n;
      }
      warp_sums[lane] = v;                   // inclusive prefix over warps
    }
    __syncthreads();
    const int64_t before = (w ? warp_sums[w - 1] : 0) + __popc(ballot & ((1u << lane) - 1));   // flagged, this chunk
    if (t < total) {
      if (f) list32[done32 + before] = id;
      else list64[(c0 - done32) + (threadIdx.x - before)] = id;
    }
    done32 += warp_sums[31];
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    counts[0] = (uint32_t)(total - done32);
    counts[1] = (uint32_t)done32;
  }
}

// p4 -> nearest fp16-grid value of p = p4/4, times 4
__device__ __forceinline__ float round_p4_f(float p4) {
  return __half2float(__float2half_rn(p4 * 0.25f)) * 4.0f;
}

// f64 holding a finite value with |x| in [2^-126, 2^128) or 0 -> the same rounded to 24 significant
// bits (RZ: clear, RNE: round-half-even on the 29 dropped bits): exact f32 rounding in that range.
template <int RM>
__device__ __forceinline__ double round24(double x) {
  long long b = __double_as_longlong(x);
  if (RM == EMU_RNE) b += 0x0FFFFFFFll + ((b >> 29) & 1ll);
  b &= ~0x1FFFFFFFll;
  return __longlong_as_double(b);
}

// general f64 -> f32 rounding kept in f64: bit path in the f32 normal range, cvt otherwise
template <int RM>
__device__ __forceinline__ double round_to_f32_in_f64(double x) {
  const uint32_t e = ((uint32_t)__double2hiint(x) >> 20) & 0x7FFu;
  if ((e - 897u) < 254u || x == 0.0) return round24<RM>(x);
  return (double)round_f64_to_f32(x, RM);
}

template <int RM, bool FAST>
__device__ __forceinline__ double round_acc(double x) {
  return FAST ? round24<RM>(x) : round_to_f32_in_f64<RM>(x);
}

// Block-sum update of 16 accumulators acc[OFF .. OFF+15] from TMEM words 0x4B400000 + T: the word
// as the low half under the row's exponent word, minus rs_c = (2^52 + 0x4B400000) * 2^e_row, is
// T * 2^e_row exactly; one FMA with the column factor 2^e_col adds it with one rounding.
template <int RM, bool FAST, int OFF, int CPT>
__device__ __forceinline__ void sum_update16(double (&acc)[CPT], const float (&v)[16], const double* cs,
                                             uint32_t rs_hi, double rs_c) {
#pragma unroll
  for (int j = 0; j < 16; j += 2) {
    const double2 c = *reinterpret_cast<const double2*>(&cs[OFF + j]);
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const double tf = __dadd_rn(__hiloint2double((int)rs_hi, (int)__float_as_uint(v[j + h])), -rs_c);
      acc[OFF + j + h] = round_acc<RM, FAST>(__fma_rn(tf, h ? c.y : c.x, acc[OFF + j + h]));
    }
  }
}

// f32 form of the block-sum update, the accumulator's f32 value kept in the low half of acc[]:
// s = T * 2^e_row * 2^e_col with T = word - 1.5*2^23 (|T| < 2^22), acc = R4(acc + s) in one FMA.
// T * 2^e_row = FMA(word, 2^e_row, -1.5*2^23 * 2^e_row) exactly while -1.5*2^23 * 2^e_row is finite
// (e_row <= 104) -- always for NVFP4 (e_row >= -10); T * 2^e_row is a multiple of 2^e_row >= 2^-149,
// so it is representable even when subnormal.  Otherwise (MXFP4 rows with e_row > 104) T exactly as
// word - 1.5*2^23 and the factor 2^e_row * 2^e_col, exact for a normal product (the tile pair's
// range test).
template <bool ROW_FOLD, int RM, int OFF, int CPT>
__device__ __forceinline__ void sum_update16_f32(double (&acc)[CPT], const float (&v)[16], const float* csf, float cr) {
  const float ncr = -MAGIC_F * cr;
#pragma unroll
  for (int j = 0; j < 16; j += 4) {
    const float4 c4 = *reinterpret_cast<const float4*>(&csf[OFF + j]);
#pragma unroll
    for (int h = 0; h < 4; ++h) {
      const float c = h == 0 ? c4.x : h == 1 ? c4.y : h == 2 ? c4.z : c4.w;
      const float a = __int_as_float(__double2loint(acc[OFF + j + h]));
      float r;
      if (ROW_FOLD) {
        const float t = __fmaf_rn(v[j + h], cr, ncr);
        r = RM == EMU_RZ ? __fmaf_rz(t, c, a) : __fmaf_rn(t, c, a);
      } else {
        const float t = __fadd_rn(v[j + h], -MAGIC_F);
        const float crc = __fmul_rn(cr, c);
        r = RM == EMU_RZ ? __fmaf_rz(t, crc, a) : __fmaf_rn(t, crc, a);
      }
      acc[OFF + j + h] = __hiloint2double(__double2hiint(acc[OFF + j + h]), __float_as_int(r));
    }
  }
}

// Warpgroup 0 = producer (warp 0), MMA issuer and TMEM owner (warp 1), two idle warps; then EPI
// epilogue warps, each thread owning one row and CPT = 64 / (EPI / 4) columns of the 64-column tile.
// Registers move from warpgroup 0 to the epilogue (setmaxnreg); the split never exceeds what the CTA
// is launched with (LAUNCH_REGS per thread, the largest multiple of 8 that fits the register file).
// RM: the rounding mode in effect (stage-3 mode for a single K block, else the stage-4 mode).
constexpr int EPI = 8, NUM_WARPS = 4 + EPI;
constexpr int LAUNCH_REGS = (65536 / (32 * NUM_WARPS)) / 8 * 8;
constexpr int REG_LOW = 56;
constexpr int REG_HIGH = ((32 * NUM_WARPS * LAUNCH_REGS - 128 * REG_LOW) / (32 * EPI)) / 8 * 8 > 232
                             ? 232 : ((32 * NUM_WARPS * LAUNCH_REGS - 128 * REG_LOW) / (32 * EPI)) / 8 * 8;
static_assert(128 * REG_LOW + 32 * EPI * REG_HIGH <= 32 * NUM_WARPS * LAUNCH_REGS, "register split exceeds the launch");
// CMP: the comparison with a reference output is compiled in (a separate instantiation, so the plain
// GEMM's register allocation is not affected by it).
// F32: the launch for the tile pairs whose block-sum updates run in f32 (see tile_f32_kernel); the
// other tile pairs go to the launch without that code, whose register allocation it would disturb.
template <int FMT, int RM, bool CMP, bool F32>
__global__ void __launch_bounds__(32 * NUM_WARPS, 1)
emul_gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                    const __grid_constant__ CUtensorMap tmAF, const __grid_constant__ CUtensorMap tmBF,
                    const __grid_constant__ CUtensorMap tmBM, const Params p) {
  constexpr int NUM_EPI_WARPS = EPI;
  constexpr int CPT = BN / (EPI / 4);                         // columns per epilogue thread (16 or 32)
  // integer / f64 path: columns per TMEM trip (NVFP4: 8, its four words per column keep 32 registers)
  constexpr int CW = FMT == EMU_FMT_NVFP4 ? 8 : (CPT == 32 ? 16 : 8);
  constexpr int GPB = Fmt<FMT>::GPB;
  constexpr int SET_COLS = GPB * BN;                         // TMEM columns per K block
  constexpr int NSETS = 512 / SET_COLS;                      // 2 (NVFP4) or 4 (MXFP4)
  constexpr uint32_t CR_TX = (FMT == EMU_FMT_NVFP4) ? CR_BYTES : (uint32_t)(CR_SBW + 2 * BN * 8);

  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  uint8_t* stage_base = smem;
  uint8_t* bias_tile = smem + NSTAGE * STAGE_BYTES;
  uint8_t* cr_ring = bias_tile + BIAS_BYTES;
  uint8_t* rr_ring = cr_ring + NCR * CR_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(rr_ring + NCR * RR_BYTES);
  uint64_t* full = bars;                       // [NSTAGE]
  uint64_t* empty = full + NSTAGE;             // [NSTAGE]
  uint64_t* cr_full = empty + NSTAGE;          // [NCR]
  uint64_t* cr_empty = cr_full + NCR;          // [NCR]
  uint64_t* tm_full = cr_empty + NCR;          // [NSETS]
  uint64_t* tm_empty = tm_full + 4;            // [NSETS]
  uint64_t* drain = tm_empty + 4;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  uint8_t* stage_path = reinterpret_cast<uint8_t*>(drain + 2);   // [NSTAGE] path code of the block in each stage

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int i = 0; i < NSTAGE; ++i) { ptx::mbar_init(&full[i], 1); ptx::mbar_init(&empty[i], 1); }
    for (int i = 0; i < NCR; ++i) { ptx::mbar_init(&cr_full[i], 1); ptx::mbar_init(&cr_empty[i], NUM_EPI_WARPS); }
    for (int i = 0; i < NSETS; ++i) { ptx::mbar_init(&tm_full[i], 1); ptx::mbar_init(&tm_empty[i], NUM_EPI_WARPS); }
    ptx::mbar_init(drain, 1);
    ptx::fence_mbar_init();
    ptx::prefetch_tmap(&tmA);
    ptx::prefetch_tmap(&tmB);
    ptx::prefetch_tmap(&tmAF);
    ptx::prefetch_tmap(&tmBF);
    ptx::prefetch_tmap(&tmBM);
  }
  if (warp == 1) {
    ptx::tmem_alloc(tmem_slot, 512);
    ptx::tmem_relinquish();
  }
  // bias tiles: zero, then element k = 0 of every row (its 16-byte chunk sits at chunk index r % 8)
  for (int i = threadIdx.x; i < BIAS_BYTES / 16; i += blockDim.x)
    reinterpret_cast<uint4*>(bias_tile)[i] = make_uint4(0, 0, 0, 0);
  __syncthreads();
  for (int r = threadIdx.x; r < BM + BN; r += blockDim.x) {
    const int rr = r < BM ? r : r - BM;
    uint8_t* base = bias_tile + (r < BM ? 0 : A_BYTES);
    *reinterpret_cast<uint16_t*>(base + rr * 128 + (rr & 7) * 16) = r < BM ? (uint16_t)0x6A00u   // 3072
                                                                           : (uint16_t)0x6C00u;  // 4096
  }
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");   // generic-proxy writes -> tensor core
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  // the register limits hold for the code each call dominates, so they sit inside the role branches
  if (warp < 4) {
    ptx::setmaxnreg_dec<REG_LOW>();
    // loaded after the register split: a loaded value held across setmaxnreg.dec may sit in a register
    // above the new limit and be lost
    const int64_t total_tiles = (int64_t)*p.tile_count < p.tiles_m * p.tiles_n ? (int64_t)*p.tile_count : p.tiles_m * p.tiles_n;
    const uint32_t tmem_base = *tmem_slot;
    if (warp == 0) {
      // ---------------------------------------------------------------- producer
      if (lane == 0) {
        int64_t it = 0;
        bool ok = true;
        for (int64_t t = blockIdx.x; t < total_tiles && ok; t += gridDim.x) {
          int64_t tm, tn;
          const uint32_t tid = p.tile_list[t];
          tm = tid >> 16;
          tn = tid & 0xFFFFu;
          for (int64_t kb = 0; kb < p.nb && ok; ++kb, ++it) {
            const int s = (int)(it % NSTAGE);
            ok = wait_or_record(&empty[s], (uint32_t)((it / NSTAGE) & 1) ^ 1u, p, 1);
            if (!ok) break;
            uint8_t* sa = stage_base + s * STAGE_BYTES;
            // block-sum blocks read both folded operands, mixed blocks the folded A and the mixed B,
            // integer blocks the folded A, f64 blocks neither
            const int pcode = p.path[(tm * p.tiles_n + tn) * p.nb + kb];
            const int path = pcode & 3;
            // the MMA warp reads the block's path code here after its wait on full[s] (the arrive
            // below releases this store)
            stage_path[s] = (uint8_t)pcode;
            ptx::mbar_arrive_expect_tx(&full[s], STAGE_BYTES);
            ptx::tma_load_2d(sa, path != PATH_F64 ? &tmAF : &tmA, &full[s], (int)(kb * BK), (int)(tm * BM));
            ptx::tma_load_2d(sa + A_BYTES, path == PATH_SUM ? &tmBF : path == PATH_MIXED ? &tmBM : &tmB, &full[s],
                             (int)(kb * BK), (int)(tn * BN));
            const int q = (int)(it % NCR);
            ok = wait_or_record(&cr_empty[q], (uint32_t)((it / NCR) & 1) ^ 1u, p, 2);
            if (!ok) break;
            // column record bytes each path reads: block-sum the column factors, integer also the
            // multipliers and bias constants, f64 the f64 scales as well
            const uint32_t c_off = path == PATH_SUM ? (uint32_t)CR_CS : 0u;
            const uint32_t c_len = path == PATH_SUM                          ? (uint32_t)(BN * 12)
                                   : (path == PATH_INT || path == PATH_MIXED) ? (uint32_t)(CR_CS + BN * 8)
                                                                              : CR_TX;
            ptx::mbar_arrive_expect_tx(&cr_full[q], c_len + RR_BYTES);
            ptx::bulk_load(cr_ring + q * CR_BYTES + c_off, p.colrec + (kb * p.tiles_n + tn) * CR_BYTES + c_off, c_len,
                           &cr_full[q]);
            ptx::bulk_load(rr_ring + q * RR_BYTES, p.rowrec + (kb * p.tiles_m + tm) * RR_BYTES, RR_BYTES, &cr_full[q]);
          }
        }
        // drain: every issued copy must have landed before the CTA may exit (bounded waits)
        for (int64_t j = (it > NSTAGE ? it - NSTAGE : 0); j < it; ++j)
          wait_or_record(&full[j % NSTAGE], (uint32_t)((j / NSTAGE) & 1), p, 7, true);
        for (int64_t j = (it > NCR ? it - NCR : 0); j < it; ++j)
          wait_or_record(&cr_full[j % NCR], (uint32_t)((j / NCR) & 1), p, 8, true);
      }
    } else if (warp == 1) {
      // ---------------------------------------------------------------- MMA issuer
      if (lane == 0) {
        constexpr uint32_t IDESC = ptx::idesc_f16_f32(BM, BN);
        int64_t it = 0;
        bool ok = true;
        // the same blocks as the producer, in the same order; each block's path code comes with its stage
        for (int64_t t = blockIdx.x; t < total_tiles && ok; t += gridDim.x) {
          for (int64_t kb = 0; kb < p.nb && ok; ++kb, ++it) {
            const int s = (int)(it % NSTAGE);
            const int set = (int)(it % NSETS);
            ok = wait_or_record(&tm_empty[set], (uint32_t)((it / NSETS) & 1) ^ 1u, p, 3);
            if (!ok) break;
            ok = wait_or_record(&full[s], (uint32_t)((it / NSTAGE) & 1), p, 4);
            if (!ok) break;
            ptx::tc_fence_after();
            const int pcode = stage_path[s];
            const int path = pcode & 3;
            const uint32_t a_addr = ptx::smem_u32(stage_base + s * STAGE_BYTES);
            const uint32_t b_addr = a_addr + A_BYTES;
            const uint32_t d_col = tmem_base + (uint32_t)(set * SET_COLS);
            const uint64_t bias_a = ptx::smem_desc_sw128(ptx::smem_u32(bias_tile));
            const uint64_t bias_b = ptx::smem_desc_sw128(ptx::smem_u32(bias_tile) + A_BYTES);
            if (path == PATH_SUM) {
              // block sum: bias 1.5*2^23, then every group accumulated into one accumulator
              ptx::mma_f16(d_col, bias_a, bias_b, IDESC, 0);
#pragma unroll
              for (int kk = 0; kk < BK / 16; ++kk)
                ptx::mma_f16(d_col, ptx::smem_desc_sw128(a_addr + 32 * kk), ptx::smem_desc_sw128(b_addr + 32 * kk), IDESC, 1);
            } else if (FMT == EMU_FMT_NVFP4 && path == PATH_MIXED) {
              // word 0: bias + every group but gx; word 1: bias + group gx (plain B values)
              const int gx = (pcode >> PATH_GROUP_SHIFT) & 3;
              constexpr int KPG = Fmt<FMT>::GS / 16;
              ptx::mma_f16(d_col, bias_a, bias_b, IDESC, 0);
              ptx::mma_f16(d_col + BN, bias_a, bias_b, IDESC, 0);
#pragma unroll
              for (int kk = 0; kk < BK / 16; ++kk) {
                const uint32_t d = kk / KPG == gx ? d_col + BN : d_col;
                ptx::mma_f16(d, ptx::smem_desc_sw128(a_addr + 32 * kk), ptx::smem_desc_sw128(b_addr + 32 * kk), IDESC, 1);
              }
            } else {
              // one accumulator per group; integer blocks start each from the 1.5*2^23 bias
              constexpr int KPG = Fmt<FMT>::GS / 16;   // K16 steps per group
#pragma unroll
              for (int g = 0; g < GPB; ++g) {
                const uint32_t d = d_col + (uint32_t)(g * BN);
                if (path == PATH_INT) ptx::mma_f16(d, bias_a, bias_b, IDESC, 0);
#pragma unroll
                for (int kk = 0; kk < KPG; ++kk) {
                  // K elements [GS*g + 16*kk, +16) = bytes [2*GS*g + 32*kk, +32) of each 128-byte row
                  const uint32_t off = (uint32_t)(2 * Fmt<FMT>::GS * g + 32 * kk);
                  ptx::mma_f16(d, ptx::smem_desc_sw128(a_addr + off), ptx::smem_desc_sw128(b_addr + off), IDESC,
                               (path == PATH_INT || kk > 0) ? 1u : 0u);
                }
              }
            }
            ptx::mma_commit(&empty[s]);
            if (!(p.hold_first_ready && it == 0)) ptx::mma_commit(&tm_full[set]);
          }
        }
        // drain: all issued MMAs complete before TMEM is released
        ptx::mma_commit(drain);
        wait_or_record(drain, 0, p, 9, true);
      }
    }
  } else {
    ptx::setmaxnreg_inc<REG_HIGH>();
    const int64_t total_tiles = (int64_t)*p.tile_count < p.tiles_m * p.tiles_n ? (int64_t)*p.tile_count : p.tiles_m * p.tiles_n;
    const uint32_t tmem_base = *tmem_slot;
    // ---------------------------------------------------------------- epilogue (warps 4..11)
    const int ew = warp - 4;                 // 0..7
    const int quarter = warp & 3;            // TMEM lane quarter this warp may access
    const int col0 = (ew >> 2) * CPT;        // CPT columns of the 64-column tile
    const uint32_t lane_base = (uint32_t)(quarter * 32) << 16;
    int64_t it = 0;
    bool ok = true;
    for (int64_t t = blockIdx.x; t < total_tiles && ok; t += gridDim.x) {
      int64_t tm, tn;
      const uint32_t tid = p.tile_list[t];
      tm = tid >> 16;
      tn = tid & 0xFFFFu;
      const int64_t m = tm * BM + quarter * 32 + lane;
      const bool row_ok = m < p.M;
      const int64_t mr = row_ok ? m : (p.M - 1);
      double acc[CPT];
#pragma unroll
      for (int j = 0; j < CPT; ++j) acc[j] = 0.0;
      bool in32 = false;                       // acc[] holds f32 values in its low halves
      const uint8_t* path_row = p.path + (tm * p.tiles_n + tn) * p.nb;
      const int rl = quarter * 32 + lane;      // row within the tile
      int nx_path = path_row[0];
      for (int64_t kb = 0; kb < p.nb && ok; ++kb, ++it) {
        const int set = (int)(it % NSETS);
        const int q = (int)(it % NCR);
        const int pcode = nx_path;
        const int path = pcode & 3;
        const bool ipath = path == PATH_INT;
        // 24-bit rounding in f64 is exact when the accumulator provably stays in the f32 normal range
        const bool fast = (FMT == EMU_FMT_NVFP4) || (pcode & PATH_NORMAL);
        if (kb + 1 < p.nb) nx_path = path_row[kb + 1];
        // MXFP4: records first (usually long in place), so the row record's shared-memory read
        // overlaps the wait for the block's MMAs (NVFP4's register allocation does worse with it)
        double2 rsv_early = make_double2(0.0, 0.0);
        if constexpr (FMT == EMU_FMT_MXFP4) {
          ok = __all_sync(0xFFFFFFFFu, wait_or_record(&cr_full[q], (uint32_t)((it / NCR) & 1), p, 6));
          if (!ok) break;
          rsv_early = reinterpret_cast<const double2*>(rr_ring + q * RR_BYTES + RR_RS)[rl];
        }
        ok = __all_sync(0xFFFFFFFFu, wait_or_record(&tm_full[set], (uint32_t)((it / NSETS) & 1), p, 5));
        if (!ok) break;
        if constexpr (FMT != EMU_FMT_MXFP4) {
          ok = __all_sync(0xFFFFFFFFu, wait_or_record(&cr_full[q], (uint32_t)((it / NCR) & 1), p, 6));
          if (!ok) break;
        }
        ptx::tc_fence_after();
        const uint8_t* cr = cr_ring + q * CR_BYTES;
        const int32_t* sbq = reinterpret_cast<const int32_t*>(cr + CR_SBQ);
        const uint32_t* kc = reinterpret_cast<const uint32_t*>(cr + CR_KC);
        const double* cs = reinterpret_cast<const double*>(cr + CR_CS);
        const double* sbw = reinterpret_cast<const double*>(cr + CR_SBW);
        const double2 rsv =
            FMT == EMU_FMT_MXFP4 ? rsv_early : reinterpret_cast<const double2*>(rr_ring + q * RR_BYTES + RR_RS)[rl];
        const uint32_t rs_hi = (uint32_t)__double2hiint(rsv.x);
        const double rs_c = rsv.y;
        const bool use32 = F32 && path == PATH_SUM && fast;
        if (use32 != in32) {
          // switch the accumulator's representation (exact both ways: acc holds f32 values)
#pragma unroll
          for (int j = 0; j < CPT; ++j)
            acc[j] = use32 ? __hiloint2double(0, __float_as_int(__double2float_rn(acc[j])))
                           : (double)__int_as_float(__double2loint(acc[j]));
          in32 = use32;
        }

        if (use32) {
          float v0[16], v1[16];
          ptx::tmem_ld16(tmem_base + lane_base + (uint32_t)(set * SET_COLS + col0), v0);
          if constexpr (CPT == 32) ptx::tmem_ld16(tmem_base + lane_base + (uint32_t)(set * SET_COLS + col0 + 16), v1);
          ptx::tmem_wait_ld();
          ptx::tc_fence_before();
          __syncwarp();
          if (lane == 0) ptx::mbar_arrive(&tm_empty[set]);
          const float* csf = reinterpret_cast<const float*>(cr + CR_CSF) + col0;
          const int e_row = (int)(rs_hi >> 20) - 1075;
          const float crf = pow2f(e_row);
          if (FMT == EMU_FMT_NVFP4 || e_row <= 104) {
            sum_update16_f32<true, RM, 0>(acc, v0, csf, crf);
            if constexpr (CPT == 32) sum_update16_f32<true, RM, 16>(acc, v1, csf, crf);
          } else {
            sum_update16_f32<false, RM, 0>(acc, v0, csf, crf);
            if constexpr (CPT == 32) sum_update16_f32<false, RM, 16>(acc, v1, csf, crf);
          }
        } else if (path == PATH_SUM) {
          // the row constant for words 0x4B400000 + T instead of T + 2^31 (exact: multiples of 2^e)
          const double rs_c_sum = __fma_rn(-(double)F_TO_T31 * 0x1p-52, __hiloint2double((int)rs_hi, 0), rs_c);
          // block-sum path: one TMEM word per output; all CPT are loaded before a single wait, so the
          // TMEM set goes back to the MMA warp after one round trip
          static_assert(CPT == 16 || CPT == 32, "one or two 16-column halves");
          float v0[16], v1[16];
          ptx::tmem_ld16(tmem_base + lane_base + (uint32_t)(set * SET_COLS + col0), v0);
          if constexpr (CPT == 32) ptx::tmem_ld16(tmem_base + lane_base + (uint32_t)(set * SET_COLS + col0 + 16), v1);
          ptx::tmem_wait_ld();
          ptx::tc_fence_before();
          __syncwarp();
          if (lane == 0) ptx::mbar_arrive(&tm_empty[set]);
          if (FMT == EMU_FMT_NVFP4 || fast) {
            sum_update16<RM, true, 0>(acc, v0, cs + col0, rs_hi, rs_c_sum);
            if constexpr (CPT == 32) sum_update16<RM, true, 16>(acc, v1, cs + col0, rs_hi, rs_c_sum);
          } else {
            sum_update16<RM, false, 0>(acc, v0, cs + col0, rs_hi, rs_c_sum);
            if constexpr (CPT == 32) sum_update16<RM, false, 16>(acc, v1, cs + col0, rs_hi, rs_c_sum);
          }
        } else if (FMT == EMU_FMT_NVFP4 && path == PATH_MIXED) {
          // word 0 = 1.5*2^23 + the other groups' block sum, word 1 = 1.5*2^23 + group gx with the plain B
          // values: T = (w0 - bias) + (w1 - bias) * sbq_gx, formed mod 2^32 as T + 2^31 like the integer path
          const int gx = (pcode >> PATH_GROUP_SHIFT) & 3;
          float w0[CPT / 16][16], w1[CPT / 16][16];
#pragma unroll
          for (int h = 0; h < CPT / 16; ++h) {
            ptx::tmem_ld16(tmem_base + lane_base + (uint32_t)(set * SET_COLS + col0 + 16 * h), w0[h]);
            ptx::tmem_ld16(tmem_base + lane_base + (uint32_t)(set * SET_COLS + BN + col0 + 16 * h), w1[h]);
          }
          ptx::tmem_wait_ld();
          ptx::tc_fence_before();
          __syncwarp();
          if (lane == 0) ptx::mbar_arrive(&tm_empty[set]);
#pragma unroll
          for (int j4 = 0; j4 < CPT / 4; ++j4) {
            const int cb = col0 + j4 * 4;
            const int4 q4 = *reinterpret_cast<const int4*>(&sbq[gx * BN + cb]);
            const double2 c01 = *reinterpret_cast<const double2*>(&cs[cb]);
            const double2 c23 = *reinterpret_cast<const double2*>(&cs[cb + 2]);
#pragma unroll
            for (int jj = 0; jj < 4; ++jj) {
              const int j = j4 * 4 + jj;
              const uint32_t q = (uint32_t)(jj == 0 ? q4.x : jj == 1 ? q4.y : jj == 2 ? q4.z : q4.w);
              const uint32_t s32 = __float_as_uint(w0[j / 16][j % 16]) + __float_as_uint(w1[j / 16][j % 16]) * q +
                                   (F_TO_T31 - MAGIC_BITS * q);
              const double cv = jj == 0 ? c01.x : jj == 1 ? c01.y : jj == 2 ? c23.x : c23.y;
              const double tf = __dadd_rn(__hiloint2double((int)rs_hi, (int)s32), -rs_c);
              const double x = __fma_rn(tf, cv, acc[j]);
              acc[j] = fast ? round24<RM>(x) : round_to_f32_in_f64<RM>(x);
            }
          }
        } else
#pragma unroll
        for (int c16 = 0; c16 < CPT / CW; ++c16) {
          // integer and f64 paths: per group CW columns per round trip (two per block)
          float v[GPB][CW];
#pragma unroll
          for (int g = 0; g < GPB; ++g) {
            const uint32_t ta = tmem_base + lane_base + (uint32_t)(set * SET_COLS + g * BN + col0 + c16 * CW);
            if constexpr (CW == 16) ptx::tmem_ld16(ta, v[g]);
            else ptx::tmem_ld8(ta, v[g]);
          }
          ptx::tmem_wait_ld();
          if (c16 == CPT / CW - 1) {
            ptx::tc_fence_before();
            __syncwarp();
            if (lane == 0) ptx::mbar_arrive(&tm_empty[set]);
          }
          if (ipath) {
#pragma unroll
            for (int j4 = 0; j4 < CW / 4; ++j4) {
              const int cb = col0 + c16 * CW + j4 * 4;
              int4 sq[GPB];
#pragma unroll
              for (int g = 0; g < GPB; ++g) sq[g] = *reinterpret_cast<const int4*>(&sbq[g * BN + cb]);
              const uint4 k4 = *reinterpret_cast<const uint4*>(&kc[cb]);
              const double2 c01 = *reinterpret_cast<const double2*>(&cs[cb]);
              const double2 c23 = *reinterpret_cast<const double2*>(&cs[cb + 2]);
#pragma unroll
              for (int jj = 0; jj < 4; ++jj) {
                const int j = c16 * CW + j4 * 4 + jj;
                uint32_t s32 = jj == 0 ? k4.x : jj == 1 ? k4.y : jj == 2 ? k4.z : k4.w;
#pragma unroll
                for (int g = 0; g < GPB; ++g) {
                  const int qv = jj == 0 ? sq[g].x : jj == 1 ? sq[g].y : jj == 2 ? sq[g].z : sq[g].w;
                  s32 += __float_as_uint(v[g][j4 * 4 + jj]) * (uint32_t)qv;
                }
                const double cv = jj == 0 ? c01.x : jj == 1 ? c01.y : jj == 2 ? c23.x : c23.y;
                const double tf = __dadd_rn(__hiloint2double((int)rs_hi, (int)s32), -rs_c);
                const double x = __fma_rn(tf, cv, acc[j]);
                acc[j] = fast ? round24<RM>(x) : round_to_f32_in_f64<RM>(x);
              }
            }
          } else {
            float wma[GPB];
            uint32_t whi[GPB];
            double wd0[GPB], wsa[GPB];
            if (FMT == EMU_FMT_NVFP4) {
              const RowScaleNv* rw = static_cast<const RowScaleNv*>(p.rw) + mr * p.G + kb * GPB;
#pragma unroll
              for (int g = 0; g < GPB; ++g) { const RowScaleNv r = rw[g]; wma[g] = r.ma; whi[g] = r.hi; wd0[g] = r.d0; }
            } else {
              const double* rw = static_cast<const double*>(p.rw) + mr * p.G + kb * GPB;
#pragma unroll
              for (int g = 0; g < GPB; ++g) wsa[g] = rw[g];
            }
            float mx = 0.0f;
#pragma unroll
            for (int g = 0; g < GPB; ++g)
#pragma unroll
              for (int j = 0; j < CW; ++j) mx = fmaxf(mx, fabsf(v[g][j]));
            if (__any_sync(0xFFFFFFFFu, mx >= 2048.0f)) {
#pragma unroll
              for (int g = 0; g < GPB; ++g)
#pragma unroll
                for (int j = 0; j < CW; ++j) v[g][j] = round_p4_f(v[g][j]);
            }
#pragma unroll
            for (int jj = 0; jj < CW; ++jj) {
              const int col = col0 + c16 * CW + jj;
              double S = 0.0;
#pragma unroll
              for (int g = 0; g < GPB; ++g) {
                const double sb = sbw[g * BN + col];
                if (FMT == EMU_FMT_NVFP4) {
                  const float bits = __fmaf_rn(v[g][jj], wma[g], MAGIC_F);
                  const double diff = __dadd_rn(__hiloint2double((int)whi[g], __float_as_int(bits)), -wd0[g]);
                  S = __fma_rn(diff, sb, S);
                } else {
                  const float bits = __fadd_rn(v[g][jj], MAGIC_F);
                  const double p4 = __dadd_rn(__hiloint2double(0x43300000, __float_as_int(bits)),
                                              -(TWO52 + (double)MAGIC_BITS));
                  S = __fma_rn(__dmul_rn(p4, wsa[g]), sb, S);
                }
              }
              const int j = c16 * CW + jj;
              if (FMT == EMU_FMT_NVFP4) {
                acc[j] = round24<RM>(kb == 0 ? S : __dadd_rn(acc[j], S));
              } else {
                const double x = kb == 0 ? S : __dadd_rn(acc[j], S);
                acc[j] = (double)round_f64_to_f32(x, RM);
              }
            }
          }
        }
        __syncwarp();
        if (lane == 0) ptx::mbar_arrive(&cr_empty[q]);
      }
      if (!ok) break;
      if (in32) {
#pragma unroll
        for (int j = 0; j < CPT; ++j) acc[j] = (double)__int_as_float(__double2loint(acc[j]));
      }
      // ---- output (and the optional fused comparison with a reference output, emu_compare's rules)
      unsigned long long c_cnt = 0;
      long long c_first = 0x7FFFFFFFFFFFFFFFll;
      float c_maxd = 0.0f, c_maxsq = 0.0f;
      double c_sq = 0.0, c_rsq = 0.0;
      if (row_ok) {
        const float al = p.alpha ? *p.alpha : 1.0f;
        const bool rnan = (FMT == EMU_FMT_NVFP4) && p.row_nan[m];
#pragma unroll
        for (int j = 0; j < CPT; ++j) {
          const int64_t n = tn * BN + col0 + j;
          if (n < p.N) {
            float y = (float)acc[j];
            if (p.alpha) y = __fmul_rn(y, al);
            if (FMT == EMU_FMT_NVFP4 && (rnan || p.col_nan[n])) y = __int_as_float(0x7FFFFFFF);
            if (!CMP || p.write_out) store_output(p.out, m * p.N + n, y, p.out_mode);
            if (CMP) {
              const float o = output_value(y, p.out_mode), r = load_output(p.cmp_ref, m * p.N + n, p.out_mode);
              const float d = __fsub_rn(r, o);
              if (!(r == o) && !((r != r) && (o != o))) {
                ++c_cnt;
                c_first = min(c_first, (long long)(m * p.N + n));
                c_maxd = fmaxf(c_maxd, (d != d) ? __int_as_float(0x7F800000) : fabsf(d));
              }
              const float e2 = __fmul_rn(d, d), r2 = __fmul_rn(r, r);
              if ((__float_as_uint(e2) & 0x7F800000u) != 0x7F800000u) { c_sq += (double)e2; c_maxsq = fmaxf(c_maxsq, e2); }
              if ((__float_as_uint(r2) & 0x7F800000u) != 0x7F800000u) c_rsq += (double)r2;
            }
          }
        }
      }
      if (CMP) {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
          c_cnt += __shfl_xor_sync(0xFFFFFFFFu, c_cnt, o);
          c_first = min(c_first, __shfl_xor_sync(0xFFFFFFFFu, c_first, o));
          c_maxd = fmaxf(c_maxd, __shfl_xor_sync(0xFFFFFFFFu, c_maxd, o));
          c_maxsq = fmaxf(c_maxsq, __shfl_xor_sync(0xFFFFFFFFu, c_maxsq, o));
          c_sq += __shfl_xor_sync(0xFFFFFFFFu, c_sq, o);
          c_rsq += __shfl_xor_sync(0xFFFFFFFFu, c_rsq, o);
        }
        if (lane == 0) {
          emu_compare_stats* st = p.cmp_stats;
          if (c_cnt) {
            atomicAdd(reinterpret_cast<unsigned long long*>(&st->mismatches), c_cnt);
            atomicMin(reinterpret_cast<long long*>(&st->first_index), c_first);
            atomicMax(reinterpret_cast<unsigned int*>(&st->max_diff), __float_as_uint(c_maxd));
          }
          atomicMax(reinterpret_cast<unsigned int*>(&st->max_sq_error), __float_as_uint(c_maxsq));
          atomicAdd(&st->sq_error_sum, c_sq);
          atomicAdd(&st->ref_sq_sum, c_rsq);
        }
      }
    }
  }

  ptx::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    ptx::tc_fence_after();
    ptx::tmem_dealloc(*tmem_slot, 512);
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
  size_t a16, b16, af16, bf16, bm16, rmaq, rowrec, rw, row_nan, rinf, colrec, col_nan, cinf, ast, bst, rts, rtm, rtinf, cts, ctm, ctinf,
      path, tile_f32, tile_list, tile_count, rng_r, rng_c, rbmax, cbmax, tile_bound, tile_other, rbmin, cbmin, err, zero_begin, zero_end, total;
};

static WsLayout layout(int fmt, int64_t M, int64_t N, int64_t K) {
  const int gs = fmt == EMU_FMT_NVFP4 ? 16 : 32;
  const int64_t G = K / gs, nb = K / BK;
  const int64_t Np = (N + BN - 1) / BN * BN, tiles_n = Np / BN, tiles_m = (M + BM - 1) / BM;
  WsLayout L{};
  size_t off = 0;
  auto take = [&](size_t bytes) { size_t o = off; off = align_up(off + bytes); return o; };
  L.a16 = take((size_t)M * K * 2);
  L.b16 = take((size_t)N * K * 2);
  L.af16 = take((size_t)M * K * 2);
  L.bf16 = take((size_t)N * K * 2);
  L.bm16 = take(fmt == EMU_FMT_NVFP4 ? (size_t)N * K * 2 : 0);
  L.rmaq = take((size_t)M * G * 4);
  L.rowrec = take((size_t)nb * tiles_m * RR_BYTES);
  L.rw = take((size_t)M * G * 16);
  L.rinf = take((size_t)M * nb);
  L.colrec = take((size_t)nb * tiles_n * CR_BYTES);
  L.cinf = take((size_t)Np * nb);
  L.ast = take((size_t)M * G * 4);
  L.bst = take((size_t)N * G * 4);
  L.rts = take((size_t)tiles_m * G * 8);
  L.rtm = take((size_t)tiles_m * G * 16);
  L.rtinf = take((size_t)tiles_m * nb);
  L.cts = take((size_t)tiles_n * G * 8);
  L.ctm = take((size_t)tiles_n * G * 16);
  L.ctinf = take((size_t)tiles_n * nb);
  L.path = take((size_t)tiles_m * tiles_n * nb);
  L.tile_f32 = take((size_t)tiles_m * tiles_n);
  L.tile_list = take((size_t)tiles_m * tiles_n * 8);
  L.tile_count = take(8);
  L.zero_begin = off;                       // regions cleared before every call
  L.row_nan = take((size_t)M * 4);
  L.col_nan = take((size_t)Np * 4);
  L.rng_r = take((size_t)tiles_m * 8);
  L.rng_c = take((size_t)tiles_n * 8);
  L.rbmax = take((size_t)tiles_m * nb * 4);
  L.cbmax = take((size_t)tiles_n * nb * 4);
  L.tile_bound = take((size_t)tiles_m * tiles_n * 4);
  L.tile_other = take((size_t)tiles_m * tiles_n * 4);
  L.rbmin = take((size_t)tiles_m * 4);
  L.cbmin = take((size_t)tiles_n * 4);
  L.err = take(16);
  L.zero_end = off;
  L.total = off;
  return L;
}

std::atomic<long long> g_wait_limit{DRAIN_LIMIT};
std::atomic<int> g_hold_first_ready{0};

}  // namespace tc

size_t gemm_tc_workspace_size(int fmt, int64_t M, int64_t N, int64_t K) { return tc::layout(fmt, M, N, K).total; }

size_t gemm_tc_path_offset(int fmt, int64_t M, int64_t N, int64_t K) { return tc::layout(fmt, M, N, K).path; }

long long set_wait_limit(long long cycles) {
  return tc::g_wait_limit.exchange(cycles > 0 ? cycles : tc::DRAIN_LIMIT);
}

void set_hold_first_ready(int enable) { tc::g_hold_first_ready.store(enable ? 1 : 0); }

cudaError_t take_wait_error(int* code) {
  *code = 0;
  cudaError_t e = cudaMemcpyFromSymbol(code, tc::g_wait_error, sizeof(int));
  if (e != cudaSuccess || *code == 0) return e;
  const int zero = 0;
  return cudaMemcpyToSymbol(tc::g_wait_error, &zero, sizeof(int));
}

bool gemm_tc_supported(int fmt, int w_reduce, int64_t M, int64_t N, int64_t K) {
  using tc::BM;
  using tc::BN;
  if (fmt == EMU_FMT_NVFP4 && w_reduce != 4) return false;
  if (fmt == EMU_FMT_MXFP4 && w_reduce != 2) return false;
  if (K % 64 != 0 || M < BM || N < BN) return false;   // every TMA box lies within its tensor
  if (K > (int64_t)1 << 30 || M > ((int64_t)1 << 31) - 1 || N > ((int64_t)1 << 31) - 1) return false;
  if ((M + BM - 1) / BM > 0xFFFF || (N + BN - 1) / BN > 0xFFFF) return false;   // 16-bit tile coordinates
  return true;
}

template <int FMT>
static cudaError_t run_tc(const uint8_t* A, const uint8_t* B, const uint8_t* SA, const uint8_t* SB, int64_t M,
                          int64_t N, int64_t K, int64_t sa_cols, int64_t sb_cols, const float* alpha,
                          const GemmArgs& args, void* out, void* workspace, cudaStream_t stream) {
  using namespace tc;
  constexpr int GS = Fmt<FMT>::GS;
  const int64_t G = K / GS, nb = K / BK;
  const int64_t Np = (N + BN - 1) / BN * BN, tiles_n = Np / BN, tiles_m = (M + BM - 1) / BM;
  const WsLayout L = layout(FMT, M, N, K);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  __half* a16 = reinterpret_cast<__half*>(ws + L.a16);
  __half* b16 = reinterpret_cast<__half*>(ws + L.b16);

  PrepTables T;
  T.rmaq = reinterpret_cast<float*>(ws + L.rmaq);
  T.rowrec = ws + L.rowrec;
  T.rw = ws + L.rw;
  T.row_nan = reinterpret_cast<uint32_t*>(ws + L.row_nan);
  T.rinf = ws + L.rinf;
  T.colrec = ws + L.colrec;
  T.col_nan = reinterpret_cast<uint32_t*>(ws + L.col_nan);
  T.cinf = ws + L.cinf;
  T.ast = reinterpret_cast<uint32_t*>(ws + L.ast);
  T.bst = reinterpret_cast<uint32_t*>(ws + L.bst);
  T.rts = reinterpret_cast<uint2*>(ws + L.rts);
  T.rtm = reinterpret_cast<float4*>(ws + L.rtm);
  T.rtinf = ws + L.rtinf;
  T.cts = reinterpret_cast<uint2*>(ws + L.cts);
  T.ctm = reinterpret_cast<float4*>(ws + L.ctm);
  T.ctinf = ws + L.ctinf;
  T.path = ws + L.path;
  T.rng_r = reinterpret_cast<uint32_t*>(ws + L.rng_r);
  T.rng_c = reinterpret_cast<uint32_t*>(ws + L.rng_c);
  T.rbmax = reinterpret_cast<uint32_t*>(ws + L.rbmax);
  T.cbmax = reinterpret_cast<uint32_t*>(ws + L.cbmax);
  T.tile_bound = reinterpret_cast<float*>(ws + L.tile_bound);
  T.tile_other = reinterpret_cast<uint32_t*>(ws + L.tile_other);
  T.rbmin = reinterpret_cast<uint32_t*>(ws + L.rbmin);
  T.cbmin = reinterpret_cast<uint32_t*>(ws + L.cbmin);
  T.tile_f32 = ws + L.tile_f32;

  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  cudaError_t e = cudaMemsetAsync(ws + L.zero_begin, 0, L.zero_end - L.zero_begin, stream);
  if (e != cudaSuccess) return e;

  auto grid_for = [&](int64_t n) {
    return (unsigned)std::max<int64_t>(1, std::min<int64_t>((n + 255) / 256, (int64_t)sms * 16));
  };
  __half* af16 = reinterpret_cast<__half*>(ws + L.af16);
  __half* bf16 = reinterpret_cast<__half*>(ws + L.bf16);
  // row tables first: the A unpack writes the folded A operand (row multipliers) in the same pass
  row_tables_kernel<FMT><<<grid_for(tiles_m * BM * nb), 256, 0, stream>>>(SA, M, tiles_m * BM, G, nb, sa_cols, T);
  unpack_stats_kernel<GS, true><<<grid_for(M * K / 16), 256, 0, stream>>>(A, M, K, a16, T.ast, T.rmaq, af16);
  unpack_stats_kernel<GS><<<grid_for(N * K / 16), 256, 0, stream>>>(B, N, K, b16, T.bst);
  col_tables_kernel<FMT><<<grid_for(Np * nb), 256, 0, stream>>>(SB, N, Np, G, nb, sb_cols, T);
  tile_stats_kernel<FMT><<<grid_for(tiles_m * G), 256, 0, stream>>>(M, BM, tiles_m, G, nb, 0, T);
  tile_stats_kernel<FMT><<<grid_for(tiles_n * G), 256, 0, stream>>>(N, BN, tiles_n, G, nb, 1, T);
  decide_kernel<FMT><<<grid_for(tiles_m * tiles_n * nb), 256, 0, stream>>>(tiles_m, tiles_n, nb, G, T);
  tile_f32_kernel<FMT><<<grid_for(tiles_m * tiles_n), 256, 0, stream>>>(
      tiles_m, tiles_n, nb, nb == 1 ? args.stage3_rounding : args.stage4_rounding, T);
  uint32_t* list64 = reinterpret_cast<uint32_t*>(ws + L.tile_list);
  uint32_t* list32 = list64 + tiles_m * tiles_n;
  uint32_t* counts = reinterpret_cast<uint32_t*>(ws + L.tile_count);
  tile_lists_kernel<<<1, 1024, 0, stream>>>(tiles_m, tiles_n, T.tile_f32, list64, list32, counts);

  __half* bm16 = reinterpret_cast<__half*>(ws + L.bm16);
  fold_cols_kernel<FMT><<<grid_for(N * K / 8), 256, 0, stream>>>(b16, N, K, tiles_n, T.colrec, T.ctm, bf16, bm16);
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;

  CUtensorMap tmA, tmB, tmAF, tmBF, tmBM;
  if (!make_map_2d(&tmA, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, a16, K, M, K * 2, BK, BM, CU_TENSOR_MAP_SWIZZLE_128B) ||
      !make_map_2d(&tmB, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, b16, K, N, K * 2, BK, BN, CU_TENSOR_MAP_SWIZZLE_128B) ||
      !make_map_2d(&tmAF, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, af16, K, M, K * 2, BK, BM, CU_TENSOR_MAP_SWIZZLE_128B) ||
      !make_map_2d(&tmBF, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, bf16, K, N, K * 2, BK, BN, CU_TENSOR_MAP_SWIZZLE_128B) ||
      !make_map_2d(&tmBM, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, FMT == EMU_FMT_NVFP4 ? bm16 : bf16, K, N, K * 2, BK, BN,
                   CU_TENSOR_MAP_SWIZZLE_128B))
    return cudaErrorInvalidValue;

  Params prm;
  prm.M = M; prm.N = N; prm.K = K; prm.G = G; prm.nb = nb;
  prm.tiles_m = tiles_m; prm.tiles_n = tiles_n;
  prm.rowrec = T.rowrec;
  prm.rw = T.rw;
  prm.row_nan = T.row_nan;
  prm.col_nan = T.col_nan;
  prm.colrec = T.colrec;
  prm.path = T.path;

  prm.alpha = alpha;
  prm.out = out;
  prm.err = reinterpret_cast<int*>(ws + L.err);
  prm.wait_limit = g_wait_limit.load();
  prm.hold_first_ready = g_hold_first_ready.load();
  prm.r3 = args.stage3_rounding;
  prm.r4 = args.stage4_rounding;
  prm.out_mode = args.out_mode;
  prm.cmp_ref = args.cmp_ref;
  prm.cmp_stats = args.cmp_stats;
  prm.write_out = args.write_out ? 1 : 0;

  const unsigned grid = (unsigned)std::min<int64_t>(tiles_m * tiles_n, sms);
  const int rm = nb == 1 ? args.stage3_rounding : args.stage4_rounding;
  // two launches over the two tile lists; a launch whose list is empty exits after its setup
  auto launch = [&](auto kern, int which) -> cudaError_t {
    cudaError_t err = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
    if (err != cudaSuccess) return err;
    Params pl = prm;
    pl.tile_list = which ? list32 : list64;
    pl.tile_count = counts + which;
    kern<<<grid, 32 * NUM_WARPS, SMEM_BYTES, stream>>>(tmA, tmB, tmAF, tmBF, tmBM, pl);
    return cudaGetLastError();
  };
  auto launch_pair = [&](auto k64, auto k32) -> cudaError_t {
    cudaError_t err = launch(k64, 0);
    return err != cudaSuccess ? err : launch(k32, 1);
  };
  if (args.cmp_ref)
    e = rm == EMU_RNE ? launch_pair(emul_gemm_tc_kernel<FMT, EMU_RNE, true, false>, emul_gemm_tc_kernel<FMT, EMU_RNE, true, true>)
                      : launch_pair(emul_gemm_tc_kernel<FMT, EMU_RZ, true, false>, emul_gemm_tc_kernel<FMT, EMU_RZ, true, true>);
  else
    e = rm == EMU_RNE ? launch_pair(emul_gemm_tc_kernel<FMT, EMU_RNE, false, false>, emul_gemm_tc_kernel<FMT, EMU_RNE, false, true>)
                      : launch_pair(emul_gemm_tc_kernel<FMT, EMU_RZ, false, false>, emul_gemm_tc_kernel<FMT, EMU_RZ, false, true>);
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

cudaError_t launch_gemm_tc(const uint8_t* A, const uint8_t* B, const uint8_t* SA, const uint8_t* SB, int64_t M,
                           int64_t N, int64_t K, int64_t sa_cols, int64_t sb_cols, const float* alpha,
                           const GemmArgs& args, void* out, void* workspace, cudaStream_t stream) {
  if (args.format == EMU_FMT_NVFP4)
    return run_tc<EMU_FMT_NVFP4>(A, B, SA, SB, M, N, K, sa_cols, sb_cols, alpha, args, out, workspace, stream);
  return run_tc<EMU_FMT_MXFP4>(A, B, SA, SB, M, N, K, sa_cols, sb_cols, alpha, args, out, workspace, stream);
}

}  // namespace emu
