// Emulated scaled FP4 GEMM for decode shapes (few rows of A) on the integer MMA of the tensor cores
// (mma.sync m16n8k16 / m16n8k32, s8 x s8 -> s32).
//
// Stage 1 of the reference is an fp16-rounded dot product per scale group of the e2m1 values
// (nvfp_emulation.cpp:77-86, mxfp_emulation.cpp:80-96).  On the "2x" values (integers -12..12, int8)
// that dot product is an integer, so an s8 MMA whose K is exactly one scale group (16 elements NVFP4,
// 32 MXFP4) returns p4 = 4 x the group dot product for a whole tile at once, exactly.  The MMA's M side
// is 16 columns of the output (rows of B, the large operand) and its N side is 8 rows of A, so a decode
// batch of 8 rows fills a tile without padding; 8 x NT rows of A per pass (NT = 1, 2).
//
// Each warp owns 16 output columns and walks K in order, so the stage-3 block sums and the stage-4
// chain stay in registers (no second phase, no barrier per K block).  Per chunk of 64 packed bytes per
// column (8 NVFP4 / 4 MXFP4 groups):
//   B    lane (c, q) = (lane / 4, lane % 4) loads 16 bytes of each of its columns c and c + 8 (bytes
//        16q..16q+15 of the chunk: NVFP4 groups 2q, 2q+1, MXFP4 group q); a byte permute regroups them
//        into one word per destination lane, and an exchange through shared memory hands lane
//        (c, q) the two packed bytes of every group that its MMA k slots 4q..4q+3 take (and 16+4q..,
//        bytes 8+2q.., for the second half of an MXFP4 group).  B enters the MMA as two non-negative
//        operands, P (magnitudes of the positive elements, 0 elsewhere) and N (of the negative ones):
//        one byte permute each, because the permute returns 0 for a selector whose sign bit is set;
//        p4 = A.P + (-A).N, two MMAs chained through the accumulator;
//   A    staged per window of 1024 K elements in shared memory, in MMA fragment order as A and -A, with
//        its scales and one flag per (tile, group) that says whether any |p4| of the group can reach
//        2048;
//   MMA  two per group and 8-row tile; p4 is rounded onto the fp16 grid only for flagged groups (for
//        the rest |p4| <= 12 * sum|2a| < 2048 and fp16 holds it exactly);
//   stages 2-4 bit for bit the reference's: NVFP4 S = sum of p4 * sa512 * sb512, an exact integer (int64;
//        the reference's f64 sum of the same products is exact too), MXFP4 S = fma(p4, sa * sb, S) from +0;
//        per block acc = R4(f64(acc) + s) with s = S * 2^-20 (NVFP4) or S, acc an f32 starting at -0
//        (-0 + s = s, so the first block is R4(s) as in the reference); R3 instead of R4 when K is one
//        block.
// A scale code that is NaN (E4M3 0x7F / 0xFF) makes its row / column NaN, as in the reference, through a
// flag per row (A) and per column (B).
#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>
#include <type_traits>

#include "common.cuh"
#include "kernels.h"

namespace emu {
namespace {

constexpr int DC_THREADS = 256;                    // 8 warps
constexpr int DC_WARPS = DC_THREADS / 32;
constexpr int DC_COLS = 16;                        // output columns per warp (the MMA's M)
constexpr int DC_CTA_COLS = DC_COLS * DC_WARPS;    // 128
constexpr int DC_WIN = 1024;                       // K elements of A per staged window
constexpr int DC_CHUNK = 64;                       // packed bytes of one column per chunk (128 elements)
constexpr int DC_SCS = 80;                         // bytes per column of a chunk's converted B scales (8 f64 + pad)
constexpr int DC_XBUF = DC_COLS * DC_CHUNK + DC_COLS * DC_SCS;   // one exchange buffer of a warp

template <int FMT> struct DcFmt {
  static constexpr int GS = FMT == EMU_FMT_NVFP4 ? 16 : 32;     // elements per scale group
  static constexpr int CG = 2 * DC_CHUNK / GS;                  // groups per chunk: 8 / 4
};

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t s) {
  uint32_t r;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(s));
  return r;
}

// e2m1 magnitudes x 2 by 3-bit index: 0 1 2 3 | 4 6 8 12
constexpr uint32_t MAG_LO = 0x03020100u, MAG_HI = 0x0C080604u;
constexpr uint32_t NEG_LO = 0xFDFEFF00u, NEG_HI = 0xF4F8FAFCu;   // their negatives

// Four e2m1 codes (the low 16 bits of `codes`) -> P: the magnitudes of the non-negative codes, 0 for
// the negative ones (the permute's sign-replicate mode on a byte below 0x80 gives 0); N: the other way.
__device__ __forceinline__ uint32_t pos4(uint32_t codes) { return prmt(MAG_LO, MAG_HI, codes); }
__device__ __forceinline__ uint32_t neg4(uint32_t flipped) { return prmt(MAG_LO, MAG_HI, flipped); }

// Four e2m1 codes -> int8 values v and -v; `mag` gets the magnitudes.
__device__ __forceinline__ void signed4(uint32_t codes, uint32_t& v, uint32_t& nv, uint32_t& mag) {
  const uint32_t sel = codes & 0x7777u;
  mag = prmt(MAG_LO, MAG_HI, sel);
  const uint32_t neg = prmt(NEG_LO, NEG_HI, sel);
  const uint32_t pick = ((codes >> 1) & 0x4444u) | 0x3210u;   // byte k from the second word when sign k is set
  v = prmt(mag, neg, pick);
  nv = prmt(neg, mag, pick);
}

// An int32 held with its top bit flipped (x + 2^31 mod 2^32) as an exact double: the magic-number
// construction, one DADD (the conversion instruction runs at a quarter of the FP64 rate).
__device__ __forceinline__ double flipped_i2d(uint32_t xf) {
  return __dadd_rn(__hiloint2double(0x43300000, (int)xf), -(4503599627370496.0 + 2147483648.0));
}

// d = a.b (zero accumulator), then d += a2.b2
template <int FMT>
__device__ __forceinline__ void mma_first(const uint32_t (&a)[4], const uint32_t (&b)[2], int (&d)[4]) {
  const int z = 0;
  if constexpr (FMT == EMU_FMT_NVFP4) {
    asm volatile("mma.sync.aligned.m16n8k16.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5}, {%6}, {%7,%7,%7,%7};"
                 : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
                 : "r"(a[0]), "r"(a[1]), "r"(b[0]), "r"(z));
  } else {
    asm volatile("mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
                 "{%10,%10,%10,%10};"
                 : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
                 : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]), "r"(z));
  }
}
template <int FMT>
__device__ __forceinline__ void mma_group(const uint32_t (&a)[4], const uint32_t (&b)[2], int (&d)[4]) {
  if constexpr (FMT == EMU_FMT_NVFP4) {
    asm volatile("mma.sync.aligned.m16n8k16.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5}, {%6}, {%0,%1,%2,%3};"
                 : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
                 : "r"(a[0]), "r"(a[1]), "r"(b[0]));
  } else {
    asm volatile("mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
                 "{%0,%1,%2,%3};"
                 : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
                 : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
  }
}

// Shared-memory accesses by 32-bit shared-window address (ld/st.shared), for the kernel's hot loop.
__device__ __forceinline__ uint32_t smem_addr(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }
__device__ __forceinline__ double lds_f64(uint32_t a) {
  double v;
  asm volatile("ld.shared.f64 %0, [%1];" : "=d"(v) : "r"(a));
  return v;
}
__device__ __forceinline__ double2 lds_f64x2(uint32_t a) {
  double2 v;
  asm volatile("ld.shared.v2.f64 {%0, %1}, [%2];" : "=d"(v.x), "=d"(v.y) : "r"(a));
  return v;
}
__device__ __forceinline__ uint32_t lds_u32(uint32_t a) {
  uint32_t v;
  asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(a));
  return v;
}
__device__ __forceinline__ uint32_t lds_u8(uint32_t a) {
  uint16_t v;
  asm volatile("ld.shared.u8 %0, [%1];" : "=h"(v) : "r"(a));
  return v;
}
__device__ __forceinline__ uint32_t lds_u16(uint32_t a) {   // a even
  uint16_t v;
  asm volatile("ld.shared.u16 %0, [%1];" : "=h"(v) : "r"(a));
  return v;
}
__device__ __forceinline__ uint4 lds_v4(uint32_t a) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(a));
  return v;
}
__device__ __forceinline__ void sts_f64x2(uint32_t a, double x, double y) {
  asm volatile("st.shared.v2.f64 [%0], {%1, %2};" ::"r"(a), "d"(x), "d"(y) : "memory");
}
__device__ __forceinline__ void sts_v4(uint32_t a, uint4 v) {
  asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(a), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w) : "memory");
}

// 1 when some byte of w is 0x7F or 0xFF (an E4M3 NaN code).
__device__ __forceinline__ uint32_t has_nan_byte(uint32_t w) {
  return (((w & 0x7F7F7F7Fu) + 0x01010101u) & 0x80808080u) != 0u;
}

// Byte offset of the scale row r in a swizzled 128x4 scale buffer; scale column g adds (g / 4) * 512 + g % 4.
__device__ __forceinline__ int64_t swz_row_base(int64_t r, int64_t cols_pad) {
  return (r >> 7) * (cols_pad >> 2) * 512 + (r & 31) * 16 + ((r & 127) >> 5) * 4;
}

// Shared memory of one CTA (dynamic part):
//   lut   [256]                     scale byte -> NVFP4 int32 sb * 2^9 (0 for the NaN codes) / MXFP4 f64 2^(ub - 127)
//   afr   [NT][16][32 lanes][4]x2   A window in MMA B-fragment order, int8 x 4 words, A then -A:
//                                   NVFP4 [group / 2][lane][group % 2][A, -A]
//                                   MXFP4 [group][lane][A lo, A hi, -A lo, -A hi]
//   asc   [NT] 2 KB                 A scales: NVFP4 int32 sa * 2^9 [group / 2][row][group % 2],
//                                   MXFP4 f64 2^(ua - 129) [group][row]
//   flg   [NT][16]                  per group quad, bit i: some |p4| of the (tile, group 4 quad + i) may reach 2048
//   xch   [8 warps]                 B exchange buffer: [column half][source lane][8 cols][dest lane] words of
//                                   packed codes (1 KB), then [16 cols][80 B] the chunk's column scales (NVFP4
//                                   8 groups as int32, MXFP4 4 as f64; the pad spreads the columns over the
//                                   banks, so the quad-broadcast 16-byte reads of 8 columns are conflict-free)
template <int NT>
struct DcSmem {
  static constexpr size_t LUT = 0, AFR = 2048, ASC = AFR + (size_t)NT * 16384, FLG = ASC + (size_t)NT * 2048,
                          XCH = FLG + (size_t)NT * 64, BYTES = XCH + (size_t)DC_WARPS * DC_XBUF;
};

// WRC: the block size (w_reduce) when it is fixed at compile time (it divides the chunk's groups, so
// blocks open and close at fixed group positions), 0 for a block size read from args.
template <int FMT, int NT, int WRC>
__global__ void __launch_bounds__(DC_THREADS, NT == 1 ? 4 : 3)
emul_gemm_decode_kernel(const uint8_t* __restrict__ A, const uint8_t* __restrict__ B, const uint8_t* __restrict__ SA,
                        const uint8_t* __restrict__ SB, int64_t M, int64_t N, int64_t K, int64_t sa_cols,
                        int64_t sb_cols, const float* __restrict__ alpha, GemmArgs args, void* __restrict__ out) {
  using F = DcFmt<FMT>;
  constexpr int GS = F::GS, CG = F::CG;
  constexpr bool NV = FMT == EMU_FMT_NVFP4;
  static_assert(WRC == 0 || CG % (WRC ? WRC : 1) == 0, "a fixed block size divides the chunk");
  using L = DcSmem<NT>;
  extern __shared__ __align__(16) uint8_t dc_smem[];
  double* lut = reinterpret_cast<double*>(dc_smem + L::LUT);
  uint32_t* afr = reinterpret_cast<uint32_t*>(dc_smem + L::AFR);
  uint8_t* asc = dc_smem + L::ASC;
  uint8_t* flg = dc_smem + L::FLG;
  __shared__ uint32_t row_nan[8 * NT];

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int c = lane >> 2, q = lane & 3;
  const int64_t r0 = (int64_t)blockIdx.y * (8 * NT);
  const int rows = (int)std::min<int64_t>(M - r0, 8 * NT);
  const int64_t kbytes = K / 2, G = K / GS;
  const int wr = WRC ? WRC : args.w_reduce;
  const int64_t nb = G / wr;
  const int rmode = nb == 1 ? args.stage3_rounding : args.stage4_rounding;

  for (int i = tid; i < 256; i += DC_THREADS) {
    if constexpr (NV) {
      bool nan;
      reinterpret_cast<int32_t*>(lut)[i] = e4m3_times_512((uint32_t)i, &nan);   // NaN codes: 0 (flagged per column)
    } else {
      lut[i] = ue8m0_quarter_f64((uint32_t)i) * 4.0;   // 2^(ub - 127), 255 -> inf
    }
  }
  if (tid < 8 * NT) row_nan[tid] = 0u;

  // this lane's two columns: B row pointers (at this lane's 16 bytes of a chunk) and scale rows
  const int64_t col0 = (int64_t)blockIdx.x * DC_CTA_COLS + warp * DC_COLS + c, col1 = col0 + 8;
  const bool ok0 = col0 < N, ok1 = col1 < N;
  const uint8_t* b0p = B + (ok0 ? col0 : 0) * kbytes + 16 * q;
  const uint8_t* b1p = B + (ok1 ? col1 : 0) * kbytes + 16 * q;
  const uint8_t* s0p = SB + swz_row_base(ok0 ? col0 : 0, sb_cols);
  const uint8_t* s1p = SB + swz_row_base(ok1 ? col1 : 0, sb_cols);
  const uint32_t sm0 = smem_addr(dc_smem);
  const uint32_t lut_a = sm0 + L::LUT, afr_a = sm0 + L::AFR, asc_a = sm0 + L::ASC, flg_a = sm0 + L::FLG;
  const uint32_t xch_a = sm0 + L::XCH + warp * DC_XBUF;
  // exchange addresses: lane (c, q) writes its words for the quad at [half][q][c][*] and reads the word
  // source lane m wrote for it at [half][m][c][q] (16-byte rows of 8 columns per plane of 128 bytes: the
  // stores fill whole 128-byte rows and the reads of one m cover 32 consecutive words -- conflict-free
  // both ways, and every read is the base plus a constant)
  const uint32_t xw_a = xch_a + q * 128 + c * 16, xr_a = xch_a + c * 16 + q * 4;

  // chunk loads: 16 bytes per column and lane, the chunk's scale words (NVFP4 two, MXFP4 one per column)
  const int64_t nchunks = (kbytes + DC_CHUNK - 1) / DC_CHUNK;
  constexpr int SWN = NV ? 2 : 1;                      // scale words per column and chunk
  // the quad's four lanes share the scales of columns c and c + 8: lane q loads and converts one word of
  // them, column q / 2, NVFP4 word q % 2 (groups 4 (q % 2) ..), MXFP4 bytes 2 (q % 2) .. of the one word
  const bool okq = (q >> 1) ? ok1 : ok0;
  const uint8_t* sqp = (q >> 1) ? s1p : s0p;
  const int hq = NV ? (q & 1) : 0;
  auto load_chunk = [&](int64_t k, uint4& w0, uint4& w1, uint32_t& swd) {
    const bool in = k * DC_CHUNK + 16 * q < kbytes;
    w0 = (ok0 && in) ? __ldg(reinterpret_cast<const uint4*>(b0p + k * DC_CHUNK)) : make_uint4(0u, 0u, 0u, 0u);
    w1 = (ok1 && in) ? __ldg(reinterpret_cast<const uint4*>(b1p + k * DC_CHUNK)) : make_uint4(0u, 0u, 0u, 0u);
    const int64_t g4 = k * SWN + hq;                   // scale word: groups 4 g4 .. 4 g4 + 3
    swd = (okq && 4 * g4 < G) ? __ldg(reinterpret_cast<const uint32_t*>(sqp + g4 * 512)) : 0u;
  };

  // stage-3 block sums.  NVFP4: the exact integer sum of p4 * sa512 * sb512 (below 2^46.8 per group, so
  // below 2^51 for up to 16 groups and 2^53 for up to 64), held as an int64; with a fixed block size of at
  // most 16 groups it starts from the bits of 1.5 * 2^52, so that its bits are the double 1.5 * 2^52 + S and
  // one DADD gives S.  MXFP4: an f64 sum.
  using SType = typename std::conditional<NV, long long, double>::type;
  constexpr bool SBIAS = NV && WRC != 0 && WRC <= 16;
  constexpr long long S0 = SBIAS ? 0x4338000000000000ll : 0ll;
  SType S[NT][4];
  float acc[NT][4];
#pragma unroll
  for (int t = 0; t < NT; ++t)
#pragma unroll
    for (int e = 0; e < 4; ++e) S[t][e] = 0, acc[t][e] = -0.0f;
  int gi = 0;           // groups of the current block so far (block size read from args)
  uint32_t cnan = 0u;   // NVFP4: a NaN scale code among the words this lane converted

  uint4 nw0, nw1;
  uint32_t nsw;
  load_chunk(0, nw0, nw1, nsw);
  int64_t k = 0;        // next chunk to process

  for (int64_t e0 = 0; e0 < K; e0 += DC_WIN) {
    const int welems = (int)std::min<int64_t>(DC_WIN, K - e0);
    const int wg = welems / GS;
    __syncthreads();    // previous window consumed (and the table / flags initialised)
    // ---- stage the window of A: warp task (tile t, group quad), lane (row n, group 4 quad + i) ----
    {
      const int n = lane >> 2, i = lane & 3;
      const int nquads = (wg + 3) / 4;
      for (int task = warp; task < NT * nquads; task += DC_WARPS) {
        const int t = task / nquads, gw = (task % nquads) * 4 + i;   // tile, group within the window
        const int row = 8 * t + n;
        const bool gok = gw < wg, rok = row < rows && gok;
        const int64_t gg = e0 / GS + gw;                             // group within K
        uint32_t sum = 0u;
        if constexpr (NV) {
          uint2 w = make_uint2(0u, 0u);
          if (rok) w = __ldg(reinterpret_cast<const uint2*>(A + (r0 + row) * kbytes + gg * 8));
          const uint32_t ww[2] = {w.x, w.y};
          uint32_t* dst = afr + ((t * 32 + (gw >> 1)) * 32 + n * 4) * 4 + (gw & 1) * 2;
#pragma unroll
          for (int u = 0; u < 4; ++u) {                              // unit u: elements 4u..4u+3 -> lane (n, u)
            uint32_t v, nv, mag;
            signed4(ww[u >> 1] >> (16 * (u & 1)), v, nv, mag);
            sum = __dp4a(mag, 0x01010101u, sum);
            if (gok) dst[u * 4] = v, dst[u * 4 + 1] = nv;
          }
          if (gok) {
            bool nan = false;
            int32_t s = 0;
            if (rok) s = e4m3_times_512(SA[swz_offset(r0 + row, gg, sa_cols)], &nan);
            if (nan) atomicOr(&row_nan[row], 1u);
            reinterpret_cast<int32_t*>(asc)[(t * 32 + (gw >> 1)) * 16 + n * 2 + (gw & 1)] = s;
          }
        } else {
          uint4 w = make_uint4(0u, 0u, 0u, 0u);
          if (rok) w = __ldg(reinterpret_cast<const uint4*>(A + (r0 + row) * kbytes + gg * 16));
          const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
          uint32_t* dst = afr + ((t * 32 + gw) * 32 + n * 4) * 4;
#pragma unroll
          for (int u = 0; u < 8; ++u) {                              // unit u -> lane (n, u % 4), half u / 4
            uint32_t v, nv, mag;
            signed4(ww[u >> 1] >> (16 * (u & 1)), v, nv, mag);
            sum = __dp4a(mag, 0x01010101u, sum);
            if (gok) dst[(u & 3) * 4 + (u >> 2)] = v, dst[(u & 3) * 4 + 2 + (u >> 2)] = nv;
          }
          if (gok) {
            const uint32_t byte = rok ? (uint32_t)SA[swz_offset(r0 + row, gg, sa_cols)] : 0u;
            reinterpret_cast<double*>(asc)[(t * 32 + gw) * 8 + n] = ue8m0_quarter_f64(byte);
          }
        }
        // |p4| <= 12 * sum|2a| over the group: fp16 rounding is needed only when that bound reaches 2048
        const uint32_t big = __ballot_sync(0xFFFFFFFFu, rok && sum >= 171u);
        if (lane == 0) {
          uint32_t bits = 0u;
#pragma unroll
          for (int b = 0; b < 4; ++b) bits |= (((big >> b) & 0x11111111u) != 0u) << b;
          flg[t * 16 + (task % nquads)] = (uint8_t)bits;
        }
      }
    }
    __syncthreads();
    // ---- the window's chunks ----
    const int64_t kend = (e0 + welems + 127) / 128;   // chunks of 128 elements; a 64-element tail is a half chunk
    for (; k < kend; ++k) {
      const uint4 w0 = nw0, w1 = nw1;
      const uint32_t sw_own = nsw;
      if (k + 1 < nchunks) load_chunk(k + 1, nw0, nw1, nsw);
      // regroup: word p' (for lane p' of the quad) = unit p' of the first 8 bytes | unit p' of the second 8
      // bytes << 16 (NVFP4: groups 2q, 2q+1; MXFP4: units p' and p' + 4 of group q)
      const uint32_t scb = xch_a + DC_COLS * DC_CHUNK;
      __syncwarp();   // every lane has read the previous chunk's exchange buffer
      {   // this lane's scale word through the table (NVFP4 int32 sb * 2^9, MXFP4 f64), into [column][group]
        const uint32_t cc = c + 8 * (q >> 1);
        if constexpr (NV) {
          sts_v4(scb + cc * DC_SCS + hq * 16,
                 make_uint4(lds_u32(lut_a + (sw_own & 0xFFu) * 4), lds_u32(lut_a + ((sw_own >> 8) & 0xFFu) * 4),
                            lds_u32(lut_a + ((sw_own >> 16) & 0xFFu) * 4), lds_u32(lut_a + (sw_own >> 24) * 4)));
          cnan |= has_nan_byte(sw_own);
        } else {
          const uint32_t w = sw_own >> (16 * (q & 1));
          sts_f64x2(scb + cc * DC_SCS + (q & 1) * 16, lds_f64(lut_a + (w & 0xFFu) * 8),
                    lds_f64(lut_a + ((w >> 8) & 0xFFu) * 8));
        }
      }
      sts_v4(xw_a, make_uint4(prmt(w0.x, w0.z, 0x5410u), prmt(w0.x, w0.z, 0x7632u), prmt(w0.y, w0.w, 0x5410u),
                              prmt(w0.y, w0.w, 0x7632u)));
      sts_v4(xw_a + 512, make_uint4(prmt(w1.x, w1.z, 0x5410u), prmt(w1.x, w1.z, 0x7632u), prmt(w1.y, w1.w, 0x5410u),
                                    prmt(w1.y, w1.w, 0x7632u)));
      __syncwarp();
      uint32_t R0[4], R1[4];   // from source lane m: this lane's units of groups 2m, 2m+1 (NVFP4) / of group m (MXFP4)
#pragma unroll
      for (int m = 0; m < 4; ++m) {
        R0[m] = lds_u32(xr_a + m * 128);
        R1[m] = lds_u32(xr_a + 512 + m * 128);
      }

      const int gwc = (int)(k * CG - e0 / GS);        // window group of the chunk's first group (a multiple of CG)
      uint32_t fl[NT];                                // stage-1 rounding flags of the chunk's groups, a bit each
#pragma unroll
      for (int t = 0; t < NT; ++t) {
        if constexpr (NV) {
          const uint32_t w = lds_u16(flg_a + t * 16 + gwc / 4);   // two quads (gwc a multiple of 8: an even offset)
          fl[t] = (w & 0xFu) | ((w >> 4) & 0xF0u);
        } else {
          fl[t] = lds_u8(flg_a + t * 16 + gwc / 4);   // one quad (gwc a multiple of 4: any offset)
        }
      }
      // groups of this chunk: CG, or CG / 2 for a 64-element chunk at the end of K
      const bool half_chunk = G - k * CG < CG;
      // chunk bases of the A fragments and scales: a group's address is base + a compile-time offset
      const uint32_t afr_c = afr_a + ((NV ? gwc >> 1 : gwc) * 32 + lane) * 16;
      const uint32_t asc_c = asc_a + (NV ? ((gwc >> 1) * 16 + 4 * q) * 4 : (gwc * 8 + 2 * q) * 8);
      const uint32_t scb0 = scb + c * DC_SCS, scb1 = scb + (c + 8) * DC_SCS;
      double2 sbp0, sbp1;                             // MXFP4: column scales of two groups, columns c and c + 8
      int4 sbq0, sbq1;                                // NVFP4: column scales of four groups
      uint4 apair[NT];                                // NVFP4: A and -A of two groups
      int4 spair[NT];                                 // NVFP4: sa of rows 2q, 2q+1 for two groups
#pragma unroll
      for (int j = 0; j < CG; ++j) {
        if (j == CG / 2 && half_chunk) break;
        uint32_t P[4], Q[4];                          // B operand: positive / negative magnitudes
        if constexpr (NV) {
          const uint32_t x0 = R0[j >> 1] >> (16 * (j & 1)), x1 = R1[j >> 1] >> (16 * (j & 1));
          P[0] = pos4(x0), P[1] = pos4(x1), Q[0] = neg4(x0 ^ 0x8888u), Q[1] = neg4(x1 ^ 0x8888u);
          P[2] = P[3] = Q[2] = Q[3] = 0u;
        } else {
          const uint32_t f0 = R0[j] ^ 0x88888888u, f1 = R1[j] ^ 0x88888888u;
          P[0] = pos4(R0[j]), P[1] = pos4(R1[j]), P[2] = pos4(R0[j] >> 16), P[3] = pos4(R1[j] >> 16);
          Q[0] = neg4(f0), Q[1] = neg4(f1), Q[2] = neg4(f0 >> 16), Q[3] = neg4(f1 >> 16);
        }
        double sb0 = 0.0, sb1 = 0.0;
        int sbi0 = 0, sbi1 = 0;
        if constexpr (NV) {
          if ((j & 3) == 0) {   // the column scales of groups j .. j + 3
            const uint4 u0 = lds_v4(scb0 + j * 4), u1 = lds_v4(scb1 + j * 4);
            sbq0 = make_int4((int)u0.x, (int)u0.y, (int)u0.z, (int)u0.w);
            sbq1 = make_int4((int)u1.x, (int)u1.y, (int)u1.z, (int)u1.w);
          }
          sbi0 = (j & 3) == 0 ? sbq0.x : (j & 3) == 1 ? sbq0.y : (j & 3) == 2 ? sbq0.z : sbq0.w;
          sbi1 = (j & 3) == 0 ? sbq1.x : (j & 3) == 1 ? sbq1.y : (j & 3) == 2 ? sbq1.z : sbq1.w;
        } else {
          if ((j & 1) == 0) {   // the column scales of groups j, j + 1
            sbp0 = lds_f64x2(scb0 + j * 8);
            sbp1 = lds_f64x2(scb1 + j * 8);
          }
          sb0 = (j & 1) ? sbp0.y : sbp0.x, sb1 = (j & 1) ? sbp1.y : sbp1.x;
        }
        const bool first = WRC ? (j % (WRC ? WRC : 1)) == 0 : gi == 0;
#pragma unroll
        for (int t = 0; t < NT; ++t) {
          uint32_t bp[2], bn[2];
          if constexpr (NV) {
            if ((j & 1) == 0) {
              apair[t] = lds_v4(afr_c + (t * 32 + (j >> 1)) * 32 * 16);
              const uint4 sv = lds_v4(asc_c + (t * 32 + (j >> 1)) * 16 * 4);
              spair[t] = make_int4((int)sv.x, (int)sv.y, (int)sv.z, (int)sv.w);
            }
            bp[0] = (j & 1) ? apair[t].z : apair[t].x;
            bn[0] = (j & 1) ? apair[t].w : apair[t].y;
            bp[1] = bn[1] = 0u;
          } else {
            const uint4 av = lds_v4(afr_c + (t * 32 + j) * 32 * 16);
            bp[0] = av.x, bp[1] = av.y, bn[0] = av.z, bn[1] = av.w;
          }
          int d[4];
          mma_first<FMT>(P, bp, d);
          mma_group<FMT>(Q, bn, d);
          if ((fl[t] >> j) & 1u) {
#pragma unroll
            for (int e = 0; e < 4; ++e) d[e] = round_p4_to_fp16_grid(d[e]);
          }
          // d: (column c, row 2q), (c, 2q + 1), (c + 8, 2q), (c + 8, 2q + 1)
          if constexpr (NV) {
            // p4 * sa512 is below 2^31 (2304 * 229376); its product with sb512 one wide multiply-add
            const int sa0 = (j & 1) ? spair[t].y : spair[t].x;
            const int sa1 = (j & 1) ? spair[t].w : spair[t].z;
            S[t][0] = (first ? S0 : S[t][0]) + (long long)(d[0] * sa0) * (long long)sbi0;
            S[t][1] = (first ? S0 : S[t][1]) + (long long)(d[1] * sa1) * (long long)sbi0;
            S[t][2] = (first ? S0 : S[t][2]) + (long long)(d[2] * sa0) * (long long)sbi1;
            S[t][3] = (first ? S0 : S[t][3]) + (long long)(d[3] * sa1) * (long long)sbi1;
          } else {
            const double2 sa = lds_f64x2(asc_c + (t * 32 + j) * 8 * 8);
            S[t][0] = __fma_rn(flipped_i2d((uint32_t)d[0] + 0x80000000u), __dmul_rn(sa.x, sb0), first ? 0.0 : S[t][0]);
            S[t][1] = __fma_rn(flipped_i2d((uint32_t)d[1] + 0x80000000u), __dmul_rn(sa.y, sb0), first ? 0.0 : S[t][1]);
            S[t][2] = __fma_rn(flipped_i2d((uint32_t)d[2] + 0x80000000u), __dmul_rn(sa.x, sb1), first ? 0.0 : S[t][2]);
            S[t][3] = __fma_rn(flipped_i2d((uint32_t)d[3] + 0x80000000u), __dmul_rn(sa.y, sb1), first ? 0.0 : S[t][3]);
          }
        }
        bool last;
        if constexpr (WRC != 0) {
          last = j % (WRC ? WRC : 1) == (WRC ? WRC : 1) - 1;
        } else {
          last = ++gi == wr;
          if (last) gi = 0;
        }
        if (last) {   // end of a stage-3 block: the stage-4 chain (one uniform branch on the rounding mode)
          double sd[NT][4];   // f64(acc) + s, s = S * 2^-20 (NVFP4, exact) or S
#pragma unroll
          for (int t = 0; t < NT; ++t)
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              if constexpr (NV) {
                const double sv = SBIAS ? __dadd_rn(__longlong_as_double((long long)S[t][e]), -6755399441055744.0)
                                        : __ll2double_rn((long long)S[t][e]);
                sd[t][e] = __fma_rn(sv, 0x1p-20, (double)acc[t][e]);
              } else {
                sd[t][e] = __dadd_rn((double)acc[t][e], (double)S[t][e]);
              }
            }
          if (rmode == EMU_RZ) {
#pragma unroll
            for (int t = 0; t < NT; ++t)
#pragma unroll
              for (int e = 0; e < 4; ++e) acc[t][e] = __double2float_rz(sd[t][e]);
          } else {
#pragma unroll
            for (int t = 0; t < NT; ++t)
#pragma unroll
              for (int e = 0; e < 4; ++e) acc[t][e] = __double2float_rn(sd[t][e]);
          }
        }
      }
    }
  }
  // NaN scale codes of columns c (converted by lanes q = 0, 1 of the quad) and c + 8 (q = 2, 3)
  uint32_t cn0 = 0u, cn1 = 0u;
  if constexpr (NV) {
    const uint32_t cn = cnan | __shfl_xor_sync(0xFFFFFFFFu, cnan, 1);
    cn0 = __shfl_sync(0xFFFFFFFFu, cn, lane & ~3);
    cn1 = __shfl_sync(0xFFFFFFFFu, cn, (lane & ~3) | 2);
  }
  const float al = alpha ? *alpha : 1.0f;
#pragma unroll
  for (int t = 0; t < NT; ++t)
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int row = 8 * t + 2 * q + (e & 1);
      const int64_t col = (e & 2) ? col1 : col0;
      if (row < rows && col < N) {
        float y = nb == 0 ? 0.0f : acc[t][e];
        if (alpha) y = __fmul_rn(y, al);
        if (NV && (row_nan[row] || ((e & 2) ? cn1 : cn0))) y = __int_as_float(0x7FFFFFFF);
        store_output(out, (r0 + row) * N + col, y, args.out_mode);
      }
    }
}

template <int FMT, int NT, int WRC>
static cudaError_t launch_one(const uint8_t* A, const uint8_t* B, const uint8_t* SA, const uint8_t* SB, int64_t M,
                              int64_t N, int64_t K, int64_t sa_cols, int64_t sb_cols, const float* alpha,
                              const GemmArgs& args, void* out, cudaStream_t stream) {
  const size_t smem = DcSmem<NT>::BYTES;
  auto kern = emul_gemm_decode_kernel<FMT, NT, WRC>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  dim3 grid((unsigned)((N + DC_CTA_COLS - 1) / DC_CTA_COLS), (unsigned)((M + 8 * NT - 1) / (8 * NT)));
  kern<<<grid, DC_THREADS, smem, stream>>>(A, B, SA, SB, M, N, K, sa_cols, sb_cols, alpha, args, out);
  return cudaGetLastError();
}

// the reference's block size (NVFP4 4 groups, MXFP4 2) fixed at compile time, any other read from args
template <int FMT, int NT>
static cudaError_t launch_nt(const uint8_t* A, const uint8_t* B, const uint8_t* SA, const uint8_t* SB, int64_t M,
                             int64_t N, int64_t K, int64_t sa_cols, int64_t sb_cols, const float* alpha,
                             const GemmArgs& args, void* out, cudaStream_t stream) {
  constexpr int WDEF = FMT == EMU_FMT_NVFP4 ? 4 : 2;
  if (args.w_reduce == WDEF)
    return launch_one<FMT, NT, WDEF>(A, B, SA, SB, M, N, K, sa_cols, sb_cols, alpha, args, out, stream);
  return launch_one<FMT, NT, 0>(A, B, SA, SB, M, N, K, sa_cols, sb_cols, alpha, args, out, stream);
}

template <int FMT>
static cudaError_t launch_fmt(const uint8_t* A, const uint8_t* B, const uint8_t* SA, const uint8_t* SB, int64_t M,
                              int64_t N, int64_t K, int64_t sa_cols, int64_t sb_cols, const float* alpha,
                              const GemmArgs& args, void* out, cudaStream_t stream) {
  // 8 rows of A per pass up to M = 8, else 16 (two 8-row tiles; 32 rows in one pass take 128 registers and
  // measured slower than two 16-row passes: M = 32 x (128256, 4096) 679 against 654 us)
  if (M <= 8) return launch_nt<FMT, 1>(A, B, SA, SB, M, N, K, sa_cols, sb_cols, alpha, args, out, stream);
  return launch_nt<FMT, 2>(A, B, SA, SB, M, N, K, sa_cols, sb_cols, alpha, args, out, stream);
}

// ---------------------------------------------------------------------------------------------------------
// One row of A (M = 1): emul_gemm_gemv_kernel.  An MMA tile would be 7/8 empty, so stage 1 stays on DP4A,
// with the decode kernel's cheaper operands: each lane owns one output column and walks all of K in order
// (stage-3 sums and the stage-4 chain in registers); B's packed bytes become positive / negative magnitude
// bytes (one byte permute each) multiplied against A and -A staged in shared memory (the same for every
// lane: broadcast reads); B's scales come one word per four groups through a 256-entry table; the stage-1
// fp16 rounding runs only for groups flagged at staging; NVFP4's exact block sum is an int64 (p4 * sa512
// * sb512 < 2^49 per group).
constexpr int GV_THREADS = 256;                    // one output column per thread
constexpr int GV_WIN = 4096;                       // K elements of A per staged window

// Shared memory (dynamic): lut [256] (NVFP4 int32 sb * 2^9, MXFP4 f64 2^(ub - 127)) 2 KB; aw [group][A words,
// -A words] (NVFP4 4 + 4, MXFP4 8 + 8 int8x4 words per group) 8 KB; asc [group] (NVFP4 int32 sa * 2^9,
// MXFP4 f64 2^(ua - 129)) 1 KB; flags, a bit per group (|p4| of the group may reach 2048).
struct GvSmem {
  static constexpr size_t LUT = 0, AW = 2048, ASC = AW + 2 * GV_WIN, FLG = ASC + 1024, BYTES = FLG + 64;
};

template <int FMT, int WRC>
__global__ void __launch_bounds__(GV_THREADS, 4)
emul_gemm_gemv_kernel(const uint8_t* __restrict__ A, const uint8_t* __restrict__ B, const uint8_t* __restrict__ SA,
                      const uint8_t* __restrict__ SB, int64_t N, int64_t K, int64_t sa_cols, int64_t sb_cols,
                      const float* __restrict__ alpha, GemmArgs args, void* __restrict__ out) {
  constexpr bool NV = FMT == EMU_FMT_NVFP4;
  constexpr int GS = NV ? 16 : 32, CG = 2 * DC_CHUNK / GS, WPG = GS / 4, WGW = GV_WIN / GS;
  static_assert(WRC == 0 || CG % (WRC ? WRC : 1) == 0, "a fixed block size divides the chunk");
  extern __shared__ __align__(16) uint8_t gv_smem[];
  __shared__ uint32_t row_nan;
  const int tid = threadIdx.x, lane = tid & 31;
  const int64_t kbytes = K / 2, G = K / GS;
  const int wr = WRC ? WRC : args.w_reduce;
  const int64_t nb = G / wr;
  const int rmode = nb == 1 ? args.stage3_rounding : args.stage4_rounding;
  const uint32_t sm0 = smem_addr(gv_smem);
  const uint32_t lut_a = sm0 + GvSmem::LUT, aw_a = sm0 + GvSmem::AW, asc_a = sm0 + GvSmem::ASC,
                 flg_a = sm0 + GvSmem::FLG;

  {
    bool nan;
    const int32_t v = e4m3_times_512((uint32_t)tid, &nan);
    if constexpr (NV) reinterpret_cast<int32_t*>(gv_smem + GvSmem::LUT)[tid] = v;   // NaN codes: 0 (flagged)
    else reinterpret_cast<double*>(gv_smem + GvSmem::LUT)[tid] = ue8m0_quarter_f64((uint32_t)tid) * 4.0;
  }
  if (tid == 0) row_nan = 0u;

  const int64_t col = (int64_t)blockIdx.x * GV_THREADS + tid;
  const bool ok = col < N;
  const uint8_t* bp = B + (ok ? col : 0) * kbytes;
  const uint8_t* sp = SB + swz_row_base(ok ? col : 0, sb_cols);
  const int64_t nchunks = (kbytes + DC_CHUNK - 1) / DC_CHUNK;
  constexpr int SWN = NV ? 2 : 1;                  // scale words per chunk
  // chunk k: bytes 64k .. of the column (32-bit offsets: a column holds under 2^31 bytes), the scale words of
  // groups 4 (SWN k + h) ..; a 64-element tail chunk holds two 16-byte pieces
  auto load_chunk = [&](int64_t k, uint4 (&w)[4], uint32_t (&s)[SWN]) {
    const int rem = ok ? (int)(kbytes - k * DC_CHUNK) : 0;   // bytes of the column from this chunk on
    const uint8_t* cp = bp + k * DC_CHUNK;
#pragma unroll
    for (int i = 0; i < 4; ++i)
      w[i] = 16 * i < rem ? __ldg(reinterpret_cast<const uint4*>(cp + 16 * i)) : make_uint4(0u, 0u, 0u, 0u);
    const uint8_t* scp = sp + k * SWN * 512;
#pragma unroll
    for (int h = 0; h < SWN; ++h)
      s[h] = 32 * h < rem ? __ldg(reinterpret_cast<const uint32_t*>(scp + h * 512)) : 0u;   // word h: bytes 32h .. of the chunk
  };

  using SType = typename std::conditional<NV, long long, double>::type;
  SType S = 0;
  float acc = G > 0 ? -0.0f : 0.0f;
  uint32_t cnan = 0u;
  int gi = 0;
  uint4 nw[4];
  uint32_t ns[SWN];
  load_chunk(0, nw, ns);
  int64_t k = 0;

  for (int64_t e0 = 0; e0 < K; e0 += GV_WIN) {
    const int welems = (int)std::min<int64_t>(GV_WIN, K - e0), wg = welems / GS;
    __syncthreads();   // the previous window consumed (and the table initialised)
    // stage the window of A: thread t takes group t (a warp 32 consecutive groups, so one ballot gives
    // the window's flag word)
    for (int gw0 = 0; gw0 < WGW; gw0 += GV_THREADS) {
      const int gw = gw0 + tid;
      if (gw0 + (tid & ~31) >= wg) break;                 // whole warps past the window's groups
      const bool gok = gw < wg;
      const int64_t gg = e0 / GS + gw;
      uint32_t ww[WPG / 2] = {};
      if (gok) {
        if constexpr (NV) {
          const uint2 v = __ldg(reinterpret_cast<const uint2*>(A + gg * 8));
          ww[0] = v.x, ww[1] = v.y;
        } else {
          const uint4 v = __ldg(reinterpret_cast<const uint4*>(A + gg * 16));
          ww[0] = v.x, ww[1] = v.y, ww[2] = v.z, ww[3] = v.w;
        }
      }
      uint32_t* dst = reinterpret_cast<uint32_t*>(gv_smem + GvSmem::AW) + gw * 2 * WPG;
      uint32_t sum = 0u;
#pragma unroll
      for (int u = 0; u < WPG; ++u) {                     // unit u: elements 4u .. 4u + 3
        uint32_t v, nv, mag;
        signed4(ww[u >> 1] >> (16 * (u & 1)), v, nv, mag);
        sum = __dp4a(mag, 0x01010101u, sum);
        if (gok) dst[u] = v, dst[WPG + u] = nv;
      }
      const uint32_t big = __ballot_sync(0xFFFFFFFFu, gok && sum >= 171u);   // |p4| <= 12 sum|2a|
      if (lane == 0) reinterpret_cast<uint32_t*>(gv_smem + GvSmem::FLG)[gw >> 5] = big;
      if (gok) {
        const uint32_t byte = SA[swz_offset(0, gg, sa_cols)];
        if constexpr (NV) {
          bool nan;
          reinterpret_cast<int32_t*>(gv_smem + GvSmem::ASC)[gw] = e4m3_times_512(byte, &nan);
          if (nan) row_nan = 1u;
        } else {
          reinterpret_cast<double*>(gv_smem + GvSmem::ASC)[gw] = ue8m0_quarter_f64(byte);
        }
      }
    }
    __syncthreads();
    const int64_t kend = (e0 + welems + 127) / 128;
    for (; k < kend; ++k) {
      uint4 w[4];
      uint32_t s[SWN];
#pragma unroll
      for (int i = 0; i < 4; ++i) w[i] = nw[i];
#pragma unroll
      for (int h = 0; h < SWN; ++h) s[h] = ns[h];
      if (k + 1 < nchunks) load_chunk(k + 1, nw, ns);
      if constexpr (NV) {
#pragma unroll
        for (int h = 0; h < SWN; ++h) cnan |= has_nan_byte(s[h]);
      }
      const uint32_t wd[16] = {w[0].x, w[0].y, w[0].z, w[0].w, w[1].x, w[1].y, w[1].z, w[1].w,
                               w[2].x, w[2].y, w[2].z, w[2].w, w[3].x, w[3].y, w[3].z, w[3].w};
      const int gwc = (int)(k * CG - e0 / GS);      // window group of the chunk's first group
      const int jn = (int)std::min<int64_t>(CG, G - k * CG);
      const uint32_t fl = lds_u32(flg_a + (gwc >> 5) * 4) >> (gwc & 31);   // the chunk's groups: bits 0 .. CG - 1
      int4 sa4;                                      // NVFP4: sa of four groups
#pragma unroll
      for (int j = 0; j < CG; ++j) {
        if (j >= jn) break;
        const int gw = gwc + j;
        int p4 = 0, p4n = 0;                          // two independent DP4A chains: positive / negative parts
#pragma unroll
        for (int h = 0; h < WPG / 4; ++h) {          // 16 elements (four units) per step
          const uint4 av = lds_v4(aw_a + (gw * 2 * WPG + 4 * h) * 4);
          const uint4 nav = lds_v4(aw_a + (gw * 2 * WPG + WPG + 4 * h) * 4);
          const uint32_t x0 = wd[j * (WPG / 2) + 2 * h], x1 = wd[j * (WPG / 2) + 2 * h + 1];
          const uint32_t f0 = x0 ^ 0x88888888u, f1 = x1 ^ 0x88888888u;
          p4 = __dp4a((int)pos4(x0), (int)av.x, p4);
          p4n = __dp4a((int)neg4(f0), (int)nav.x, p4n);
          p4 = __dp4a((int)pos4(x0 >> 16), (int)av.y, p4);
          p4n = __dp4a((int)neg4(f0 >> 16), (int)nav.y, p4n);
          p4 = __dp4a((int)pos4(x1), (int)av.z, p4);
          p4n = __dp4a((int)neg4(f1), (int)nav.z, p4n);
          p4 = __dp4a((int)pos4(x1 >> 16), (int)av.w, p4);
          p4n = __dp4a((int)neg4(f1 >> 16), (int)nav.w, p4n);
        }
        p4 += p4n;
        if ((fl >> j) & 1u) p4 = round_p4_to_fp16_grid(p4);
        const uint32_t sbyte = (s[j >> 2] >> (8 * (j & 3))) & 0xFFu;
        const bool first = WRC ? (j % (WRC ? WRC : 1)) == 0 : gi == 0;
        if constexpr (NV) {
          if ((j & 3) == 0) {
            const uint4 v = lds_v4(asc_a + gw * 4);
            sa4 = make_int4((int)v.x, (int)v.y, (int)v.z, (int)v.w);
          }
          const int sa = (j & 3) == 0 ? sa4.x : (j & 3) == 1 ? sa4.y : (j & 3) == 2 ? sa4.z : sa4.w;
          const int sb = (int)lds_u32(lut_a + sbyte * 4);
          S = (first ? 0ll : S) + (long long)(p4 * sa) * (long long)sb;   // exact: below 2^49 per group
        } else {
          const double sbd = lds_f64(lut_a + sbyte * 8);
          const double sad = lds_f64(asc_a + gw * 8);
          S = __fma_rn(flipped_i2d((uint32_t)p4 + 0x80000000u), __dmul_rn(sad, sbd), first ? 0.0 : S);
        }
        bool last;
        if constexpr (WRC != 0) {
          last = j % (WRC ? WRC : 1) == (WRC ? WRC : 1) - 1;
        } else {
          last = ++gi == wr;
          if (last) gi = 0;
        }
        if (last) {   // stage 4: acc = R(f64(acc) + s), s = S * 2^-20 (NVFP4, exact) or S
          const double sd = NV ? __fma_rn(__ll2double_rn((long long)S), 0x1p-20, (double)acc)
                               : __dadd_rn((double)acc, (double)S);
          acc = rmode == EMU_RZ ? __double2float_rz(sd) : __double2float_rn(sd);
        }
      }
    }
  }
  if (ok) {
    float y = acc;
    if (alpha) y = __fmul_rn(y, *alpha);
    if (NV && (row_nan || cnan)) y = __int_as_float(0x7FFFFFFF);
    store_output(out, col, y, args.out_mode);
  }
}

template <int FMT, int WRC>
static cudaError_t launch_gv(const uint8_t* A, const uint8_t* B, const uint8_t* SA, const uint8_t* SB, int64_t N,
                             int64_t K, int64_t sa_cols, int64_t sb_cols, const float* alpha, const GemmArgs& args,
                             void* out, cudaStream_t stream) {
  auto kern = emul_gemm_gemv_kernel<FMT, WRC>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)GvSmem::BYTES);
  if (e != cudaSuccess) return e;
  kern<<<(unsigned)((N + GV_THREADS - 1) / GV_THREADS), GV_THREADS, GvSmem::BYTES, stream>>>(A, B, SA, SB, N, K, sa_cols,
                                                                                           sb_cols, alpha, args, out);
  return cudaGetLastError();
}

}  // namespace

// Rows of A from 2 to 127 in passes of 8 / 16; K a multiple of 64 (whole swizzled scale words); B and A
// 16-byte aligned (vector loads), the scales of B 4-byte aligned (one word per four groups); N of at least
// 8192 (64 CTAs of 128 columns: with fewer the kernel leaves SMs idle and the skinny kernel, which splits
// K over its warps, is faster: 8 x (4096, 4096) 34 against 53 us).  One row of A goes to the one-row kernel
// below or the skinny row kernel (an MMA tile would be 7/8 empty).
bool gemm_decode_supported(int fmt, int64_t M, int64_t N, int64_t K, const void* A, const void* B, const void* SB) {
  (void)fmt;
  return M >= 2 && M < 128 && N >= 8192 && K % 64 == 0 && (reinterpret_cast<uintptr_t>(A) & 15) == 0 &&
         (reinterpret_cast<uintptr_t>(B) & 15) == 0 && (reinterpret_cast<uintptr_t>(SB) & 3) == 0;
}

// One row of A, N of at least 32768 (128 CTAs of 256 columns; each warp walks all of K, so with fewer
// columns the skinny row kernel, which splits K over its warps, is faster: 1 x (16384, 4096) 33 against 41
// us, 1 x (32768, 4096) 46 against 41, 1 x (128256, 4096) 156 against 107), K a multiple of 64, the same
// alignment as the decode kernel.
bool gemm_gemv_supported(int fmt, int64_t M, int64_t N, int64_t K, const void* A, const void* B, const void* SB) {
  (void)fmt;
  return M == 1 && N >= 32768 && K % 64 == 0 && (reinterpret_cast<uintptr_t>(A) & 15) == 0 &&
         (reinterpret_cast<uintptr_t>(B) & 15) == 0 && (reinterpret_cast<uintptr_t>(SB) & 3) == 0;
}

cudaError_t launch_gemm_gemv(const uint8_t* A, const uint8_t* B, const uint8_t* SA, const uint8_t* SB, int64_t N,
                             int64_t K, int64_t sa_cols, int64_t sb_cols, const float* alpha, const GemmArgs& args,
                             void* out, cudaStream_t stream) {
  if (args.format == EMU_FMT_NVFP4) {
    if (args.w_reduce == 4)
      return launch_gv<EMU_FMT_NVFP4, 4>(A, B, SA, SB, N, K, sa_cols, sb_cols, alpha, args, out, stream);
    return launch_gv<EMU_FMT_NVFP4, 0>(A, B, SA, SB, N, K, sa_cols, sb_cols, alpha, args, out, stream);
  }
  if (args.w_reduce == 2) return launch_gv<EMU_FMT_MXFP4, 2>(A, B, SA, SB, N, K, sa_cols, sb_cols, alpha, args, out, stream);
  return launch_gv<EMU_FMT_MXFP4, 0>(A, B, SA, SB, N, K, sa_cols, sb_cols, alpha, args, out, stream);
}

cudaError_t launch_gemm_decode(const uint8_t* A, const uint8_t* B, const uint8_t* SA, const uint8_t* SB, int64_t M,
                               int64_t N, int64_t K, int64_t sa_cols, int64_t sb_cols, const float* alpha,
                               const GemmArgs& args, void* out, cudaStream_t stream) {
  if (args.format == EMU_FMT_NVFP4)
    return launch_fmt<EMU_FMT_NVFP4>(A, B, SA, SB, M, N, K, sa_cols, sb_cols, alpha, args, out, stream);
  return launch_fmt<EMU_FMT_MXFP4>(A, B, SA, SB, M, N, K, sa_cols, sb_cols, alpha, args, out, stream);
}

}  // namespace emu
