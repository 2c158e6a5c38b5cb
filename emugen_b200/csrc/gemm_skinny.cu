// Emulated scaled FP4 GEMM for skinny problems (few rows of A: decode shapes, M < 128), CUDA cores.
//
// The bytes of B (N x K/2, read once) dominate, and the reference's stage 4 is a sequential chain
// over the K blocks of each output, so the work is split in two phases per window of K blocks:
//   1. the 8 warps of a CTA compute the stage-3 block sums s_b of a window in parallel (warp w takes
//      blocks w, w+8, ...; lane = one of the CTA's 32 output columns, which streams its row of B
//      32 bytes at a time; the window of every A row and its scales sits in shared memory);
//   2. one thread per (row, column) runs the stage-4 chain acc = R4(f64(acc) + s_b) over the
//      window's blocks in order.
// Arithmetic is the general kernel's (gemm_simt.cu), bit for bit the reference's
// (nvfp_emulation.cpp:90-156, mxfp_emulation.cpp:98-166, core.py:69-148):
//   stage 1  p4 = 4 * group dot, exact in int32 (DP4A on 2a, 2b), rounded once onto the fp16 grid;
//   stage 2  NVFP4 p4 * (sa*2^9) * (sb*2^9) exact in int64 (units of 2^-20); MXFP4 p * 2^.. in f64;
//   stage 3  exact int64 sum (NVFP4) / ((+0 + v0) + v1) ... in f64 (MXFP4);
//   stage 4  acc = R4(s0); acc = R4(f64(acc) + s_b); output (acc * alpha) -> fp16 [-> bf16].
#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>
#include <type_traits>

#include "common.cuh"
#include "kernels.h"

namespace emu {
namespace {

constexpr int SK_THREADS = 256;     // 8 warps
constexpr int SK_COLS = 32;         // output columns per CTA (one per lane)
constexpr int SK_WIN_ELEMS = 1024;  // K elements per window (at most; a stage-3 block fits one)
// one row of A: a window of 4096 elements (A and its scales staged once for K <= 4096, fewer barriers)
template <int ROWS> struct SkWin { static constexpr int ELEMS = ROWS == 1 ? 4096 : SK_WIN_ELEMS; };


// Dynamic shared memory of one CTA (ROWS rows of A per pass, a window of WB blocks):
//   a8    [ROWS][WIN / 4]            A window, int8 x 4 per word (WIN = SkWin<ROWS>::ELEMS)
//   scale [ROWS][GMAX] x 8 bytes     NVFP4 scale * 2^9 (int32) / MXFP4 2^(ua - 129) (f64) per group
//   sbuf  [ROWS][WB][32]             block sums of the window (f64)
template <int FMT, int ROWS>
__device__ __forceinline__ void skinny_body(const uint8_t* __restrict__ A, const uint8_t* __restrict__ B,
                                            const uint8_t* __restrict__ SA, const uint8_t* __restrict__ SB, int64_t M,
                                            int64_t N, int64_t K, int64_t sa_cols, int64_t sb_cols,
                                            const float* __restrict__ alpha, const GemmArgs& args, int WB,
                                            void* __restrict__ out) {
  constexpr int GS = (FMT == EMU_FMT_NVFP4) ? 16 : 32;
  constexpr int WPG = GS / 4;                     // int8 x 4 words per group
  constexpr int WIN = SkWin<ROWS>::ELEMS;
  constexpr int GMAX = WIN / GS;                  // groups per window (at most)
  extern __shared__ __align__(16) uint8_t sk_smem[];
  uint32_t* a8 = reinterpret_cast<uint32_t*>(sk_smem);
  int32_t* sai = reinterpret_cast<int32_t*>(sk_smem + ROWS * WIN);
  double* sad = reinterpret_cast<double*>(sk_smem + ROWS * WIN);
  double* sbuf = reinterpret_cast<double*>(sk_smem + ROWS * WIN + ROWS * GMAX * 8);
  __shared__ uint32_t row_nan[ROWS], col_nan[SK_COLS];

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int64_t n0 = (int64_t)blockIdx.x * SK_COLS, r0 = (int64_t)blockIdx.y * ROWS;
  const int rows = (int)std::min<int64_t>(M - r0, ROWS);
  const int64_t n = n0 + lane;
  const bool col_ok = n < N;
  const int wr = args.w_reduce;
  const int BKE = wr * GS;                        // elements per stage-3 block
  const int64_t G = K / GS, nb = G / wr, kbytes = K / 2;
  if (tid < ROWS) row_nan[tid] = 0;
  if (tid < SK_COLS) col_nan[tid] = 0;

  // phase-2 ownership: thread -> (row, column) of one stage-4 chain (rows beyond 8 take a second chain)
  const int cr = tid / SK_COLS, cc = tid % SK_COLS;
  float acc = 0.0f, acc2 = 0.0f;

  for (int64_t b0 = 0; b0 < nb; b0 += WB) {
    const int wblocks = (int)std::min<int64_t>(WB, nb - b0);
    const int64_t e0 = b0 * BKE;                  // first K element of the window
    const int welems = wblocks * BKE, wgroups = welems / GS;
    __syncthreads();                              // previous window consumed, flags initialised
    // stage the window of A (4 bytes = 8 elements per step) and the A scales
    for (int t = tid; t < ROWS * (welems / 8); t += SK_THREADS) {
      const int r = t / (welems / 8), q = t % (welems / 8);
      uint32_t w = 0;
      if (r < rows) w = *reinterpret_cast<const uint32_t*>(A + (r0 + r) * kbytes + e0 / 2 + q * 4);
      a8[r * (WIN / 4) + 2 * q] = e2m1x4_to_int8x4(w & 0xFFFFu);
      a8[r * (WIN / 4) + 2 * q + 1] = e2m1x4_to_int8x4(w >> 16);
    }
    for (int t = tid; t < ROWS * wgroups; t += SK_THREADS) {
      const int r = t / wgroups, gl = t % wgroups;
      const uint32_t byte = r < rows ? SA[swz_offset(r0 + r, e0 / GS + gl, sa_cols)] : 0u;
      if (FMT == EMU_FMT_NVFP4) {
        bool nan;
        sai[r * (GMAX * 2) + gl] = e4m3_times_512(byte, &nan);
        if (nan) atomicOr(&row_nan[r], 1u);
      } else {
        sad[r * GMAX + gl] = ue8m0_quarter_f64(byte);
      }
    }
    __syncthreads();
    // phase 1: block sums, warp w takes blocks w, w + 8, ...
    using SType = typename std::conditional<FMT == EMU_FMT_NVFP4, long long, double>::type;
    constexpr int CH = 32 / (GS / 2);             // groups per chunk of 32 bytes of B: 4 (NVFP4) / 2 (MXFP4)
    const bool b_al16 = (reinterpret_cast<uintptr_t>(B) & 15) == 0;
    // loads of one chunk (groups gq0 .. gq0 + CH - 1 of block j): 32 bytes of B per lane, issued together,
    // and the groups' scale bytes
    auto load_chunk = [&](int j, int gq0, uint32_t (&raw)[CH][WPG / 2], uint32_t (&bbyte)[CH]) {
      if constexpr (GS == 16) {
#pragma unroll
        for (int q = 0; q < CH; q += 2) {
          const int64_t g = e0 / GS + j * wr + gq0 + q;
          const bool in0 = col_ok && gq0 + q < wr, in1 = col_ok && gq0 + q + 1 < wr;
          const uint8_t* src = B + n * kbytes + g * (GS / 2);
          if (in1 && b_al16 && (g & 1) == 0) {    // two groups, one 16-byte load
            const uint4 w = __ldg(reinterpret_cast<const uint4*>(src));
            raw[q][0] = w.x;
            raw[q][1] = w.y;
            raw[q + 1][0] = w.z;
            raw[q + 1][1] = w.w;
          } else {
            uint2 w0 = make_uint2(0u, 0u), w1 = make_uint2(0u, 0u);
            if (in0) w0 = __ldg(reinterpret_cast<const uint2*>(src));
            if (in1) w1 = __ldg(reinterpret_cast<const uint2*>(src + GS / 2));
            raw[q][0] = w0.x;
            raw[q][1] = w0.y;
            raw[q + 1][0] = w1.x;
            raw[q + 1][1] = w1.y;
          }
          bbyte[q] = in0 ? (uint32_t)SB[swz_offset(n, g, sb_cols)] : 0u;
          bbyte[q + 1] = in1 ? (uint32_t)SB[swz_offset(n, g + 1, sb_cols)] : 0u;
        }
      } else {
#pragma unroll
        for (int q = 0; q < CH; ++q) {
          const int64_t g = e0 / GS + j * wr + gq0 + q;
          if (col_ok && gq0 + q < wr) {
            const uint4 w = __ldg(reinterpret_cast<const uint4*>(B + n * kbytes + g * (GS / 2)));
            raw[q][0] = w.x;
            raw[q][1] = w.y;
            raw[q][2] = w.z;
            raw[q][3] = w.w;
            bbyte[q] = SB[swz_offset(n, g, sb_cols)];
          } else {
#pragma unroll
            for (int w = 0; w < WPG / 2; ++w) raw[q][w] = 0;
            bbyte[q] = 0;
          }
        }
      }
    };
    // stage 1-3 of one chunk into the block sums S (one per row of A)
    auto sum_chunk = [&](int j, int gq0, const uint32_t (&raw)[CH][WPG / 2], const uint32_t (&bbyte)[CH],
                         SType (&S)[ROWS], bool& cnan) {
#pragma unroll
      for (int q = 0; q < CH; ++q) {
        if (gq0 + q >= wr) break;
        const int gl = j * wr + gq0 + q;          // group within the window
        uint32_t bw[WPG];
#pragma unroll
        for (int w = 0; w < WPG / 2; ++w) {
          bw[2 * w] = e2m1x4_to_int8x4(raw[q][w] & 0xFFFFu);
          bw[2 * w + 1] = e2m1x4_to_int8x4(raw[q][w] >> 16);
        }
        int32_t sbi = 0;
        double sbd = 0.0;
        if (FMT == EMU_FMT_NVFP4) {
          bool nan;
          sbi = e4m3_times_512(bbyte[q], &nan);
          cnan |= nan;
        } else {
          sbd = ue8m0_quarter_f64(bbyte[q]) * 4.0;   // 2^(ub-127); the 1/4 is in the A scale
        }
#pragma unroll
        for (int i = 0; i < ROWS; ++i) {
          int p4 = 0;
#pragma unroll
          for (int w = 0; w < WPG; ++w) p4 = __dp4a((int)a8[i * (WIN / 4) + gl * WPG + w], (int)bw[w], p4);
          const int p = round_p4_to_fp16_grid(p4);
          if (FMT == EMU_FMT_NVFP4) S[i] += (long long)(p * sai[i * (GMAX * 2) + gl]) * (long long)sbi;
          else S[i] = __dadd_rn(S[i], __dmul_rn((double)p, __dmul_rn(sad[i * GMAX + gl], sbd)));
        }
      }
    };
    auto store_block = [&](int j, const SType (&S)[ROWS], bool cnan) {
      if (cnan) atomicOr(&col_nan[lane], 1u);
#pragma unroll
      for (int i = 0; i < ROWS; ++i) {
        double s;
        if (FMT == EMU_FMT_NVFP4) s = __ll2double_rn(S[i]) * 0x1p-20;   // exact
        else s = S[i];
        sbuf[(i * WB + j) * SK_COLS + lane] = s;
      }
    };
    if constexpr (ROWS == 1) {
      for (int j = warp; j < wblocks; j += SK_THREADS / 32) {
        SType S[ROWS];
        bool cnan = false;
        S[0] = 0;
        for (int gq0 = 0; gq0 < wr; gq0 += CH) {
          uint32_t raw[CH][WPG / 2], bbyte[CH];
          load_chunk(j, gq0, raw, bbyte);
          sum_chunk(j, gq0, raw, bbyte, S, cnan);
        }
        store_block(j, S, cnan);
      }
    } else {
      // more rows: the same arithmetic with the loads of each chunk written in place (the helpers above
      // cost these instantiations registers and occupancy)
      for (int j = warp; j < wblocks; j += SK_THREADS / 32) {
        SType S[ROWS];
#pragma unroll
        for (int i = 0; i < ROWS; ++i) S[i] = 0;
        bool cnan = false;
        // groups in chunks of 32 bytes of B per lane: the chunk's loads are issued together
        for (int gq0 = 0; gq0 < wr; gq0 += CH) {
          uint32_t raw[CH][WPG / 2];                // packed e2m1, 8 per word
          uint32_t bbyte[CH];
#pragma unroll
          for (int q = 0; q < CH; ++q) {
            const int64_t g = e0 / GS + j * wr + gq0 + q;
            if (col_ok && gq0 + q < wr) {
              const uint8_t* src = B + n * kbytes + g * (GS / 2);
              if constexpr (GS == 16) {
                const uint2 w = __ldg(reinterpret_cast<const uint2*>(src));
                raw[q][0] = w.x;
                raw[q][1] = w.y;
              } else {
                const uint4 w = __ldg(reinterpret_cast<const uint4*>(src));
                raw[q][0] = w.x;
                raw[q][1] = w.y;
                raw[q][2] = w.z;
                raw[q][3] = w.w;
              }
              bbyte[q] = SB[swz_offset(n, g, sb_cols)];
            } else {
#pragma unroll
              for (int w = 0; w < WPG / 2; ++w) raw[q][w] = 0;
              bbyte[q] = 0;
            }
          }
#pragma unroll
          for (int q = 0; q < CH; ++q) {
            if (gq0 + q >= wr) break;
            const int gl = j * wr + gq0 + q;        // group within the window
            uint32_t bw[WPG];
#pragma unroll
            for (int w = 0; w < WPG / 2; ++w) {
              bw[2 * w] = e2m1x4_to_int8x4(raw[q][w] & 0xFFFFu);
              bw[2 * w + 1] = e2m1x4_to_int8x4(raw[q][w] >> 16);
            }
            int32_t sbi = 0;
            double sbd = 0.0;
            if (FMT == EMU_FMT_NVFP4) {
              bool nan;
              sbi = e4m3_times_512(bbyte[q], &nan);
              cnan |= nan;
            } else {
              sbd = ue8m0_quarter_f64(bbyte[q]) * 4.0;   // 2^(ub-127); the 1/4 is in the A scale
            }
#pragma unroll
            for (int i = 0; i < ROWS; ++i) {
              int p4 = 0;
#pragma unroll
              for (int w = 0; w < WPG; ++w)
                p4 = __dp4a((int)a8[i * (WIN / 4) + gl * WPG + w], (int)bw[w], p4);
              const int p = round_p4_to_fp16_grid(p4);
              if (FMT == EMU_FMT_NVFP4) S[i] += (long long)(p * sai[i * (GMAX * 2) + gl]) * (long long)sbi;
              else S[i] = __dadd_rn(S[i], __dmul_rn((double)p, __dmul_rn(sad[i * GMAX + gl], sbd)));
            }
          }
        }
        if (cnan) atomicOr(&col_nan[lane], 1u);
#pragma unroll
        for (int i = 0; i < ROWS; ++i) {
          double s;
          if (FMT == EMU_FMT_NVFP4) s = __ll2double_rn(S[i]) * 0x1p-20;   // exact
          else s = S[i];
          sbuf[(i * WB + j) * SK_COLS + lane] = s;
        }
      }
    }
    __syncthreads();
    // phase 2: the stage-4 chain of (row cr, column cc) over the window's blocks, in order
    auto chain = [&](int row, float& a) {
      for (int j = 0; j < wblocks; ++j) {
        const double s = sbuf[(row * WB + j) * SK_COLS + cc];
        const int64_t blk = b0 + j;
        if (nb == 1) a = round_f64_to_f32(s, args.stage3_rounding);
        else if (blk == 0) a = round_f64_to_f32(s, args.stage4_rounding);
        else a = round_f64_to_f32(__dadd_rn((double)a, s), args.stage4_rounding);
      }
    };
    if (cr < ROWS) chain(cr, acc);
    if (ROWS > 8 && cr + 8 < ROWS) chain(cr + 8, acc2);
  }
  __syncthreads();
  const float al = alpha ? *alpha : 1.0f;
#pragma unroll
  for (int h = 0; h < (ROWS > 8 ? 2 : 1); ++h) {
    const int row = cr + 8 * h;
    if (row < rows && n0 + cc < N) {
      const float a = h ? acc2 : acc;
      float y = alpha ? __fmul_rn(a, al) : a;
      if (FMT == EMU_FMT_NVFP4 && (row_nan[row] || col_nan[cc])) y = __int_as_float(0x7FFFFFFF);
      store_output(out, (r0 + row) * N + n0 + cc, y, args.out_mode);
    }
  }
}

template <int FMT, int ROWS>
__global__ void __launch_bounds__(SK_THREADS)
emul_gemm_skinny_kernel(const uint8_t* __restrict__ A, const uint8_t* __restrict__ B,
                        const uint8_t* __restrict__ SA, const uint8_t* __restrict__ SB, int64_t M, int64_t N,
                        int64_t K, int64_t sa_cols, int64_t sb_cols, const float* __restrict__ alpha, GemmArgs args,
                        int WB, void* __restrict__ out) {
  skinny_body<FMT, ROWS>(A, B, SA, SB, M, N, K, sa_cols, sb_cols, alpha, args, WB, out);
}

// One row of A: at most 51 registers, so five CTAs share an SM (the kernel waits on B's loads; 4 CTAs
// with the default register allocation).
template <int FMT>
__global__ void __launch_bounds__(SK_THREADS, 5)
emul_gemm_skinny_row_kernel(const uint8_t* __restrict__ A, const uint8_t* __restrict__ B,
                            const uint8_t* __restrict__ SA, const uint8_t* __restrict__ SB, int64_t M, int64_t N,
                            int64_t K, int64_t sa_cols, int64_t sb_cols, const float* __restrict__ alpha, GemmArgs args,
                            int WB, void* __restrict__ out) {
  skinny_body<FMT, 1>(A, B, SA, SB, M, N, K, sa_cols, sb_cols, alpha, args, WB, out);
}

template <int FMT, int ROWS>
static auto skinny_kernel_for() {
  if constexpr (ROWS == 1) return emul_gemm_skinny_row_kernel<FMT>;
  else return emul_gemm_skinny_kernel<FMT, ROWS>;
}

template <int ROWS>
static size_t smem_bytes(int fmt, int WB) {
  const int gmax = SkWin<ROWS>::ELEMS / (fmt == EMU_FMT_NVFP4 ? 16 : 32);
  return (size_t)ROWS * SkWin<ROWS>::ELEMS + (size_t)ROWS * gmax * 8 + (size_t)ROWS * WB * SK_COLS * 8;
}

template <int ROWS>
static cudaError_t launch_rows(const uint8_t* A, const uint8_t* B, const uint8_t* SA, const uint8_t* SB, int64_t M,
                               int64_t N, int64_t K, int64_t sa_cols, int64_t sb_cols, const float* alpha,
                               const GemmArgs& args, void* out, cudaStream_t stream) {
  const int gs = args.format == EMU_FMT_NVFP4 ? 16 : 32;
  // blocks per window: sums of at most 64 KB (16 x 16 rows), 16 KB for one row
  const int WB = std::min(SkWin<ROWS>::ELEMS / (args.w_reduce * gs), ROWS == 1 ? 64 : 16);
  const size_t smem = smem_bytes<ROWS>(args.format, WB);
  dim3 grid((unsigned)((N + SK_COLS - 1) / SK_COLS), (unsigned)((M + ROWS - 1) / ROWS));
  cudaError_t e;
  if (args.format == EMU_FMT_NVFP4) {
    auto k = skinny_kernel_for<EMU_FMT_NVFP4, ROWS>();
    e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    k<<<grid, SK_THREADS, smem, stream>>>(A, B, SA, SB, M, N, K, sa_cols, sb_cols, alpha, args, WB, out);
  } else {
    auto k = skinny_kernel_for<EMU_FMT_MXFP4, ROWS>();
    e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    k<<<grid, SK_THREADS, smem, stream>>>(A, B, SA, SB, M, N, K, sa_cols, sb_cols, alpha, args, WB, out);
  }
  return cudaGetLastError();
}

}  // namespace

// Rows of A up to 127; a stage-3 block (w_reduce groups) fits one window.
bool gemm_skinny_supported(int fmt, int w_reduce, int64_t M) {
  const int gs = fmt == EMU_FMT_NVFP4 ? 16 : 32;
  return M >= 1 && M < 128 && w_reduce >= 1 && (int64_t)w_reduce * gs <= SK_WIN_ELEMS;
}

cudaError_t launch_gemm_skinny(const uint8_t* A, const uint8_t* B, const uint8_t* SA, const uint8_t* SB, int64_t M,
                               int64_t N, int64_t K, int64_t sa_cols, int64_t sb_cols, const float* alpha,
                               const GemmArgs& args, void* out, cudaStream_t stream) {
  if (gemm_gemv_supported(args.format, M, N, K, A, B, SB))
    return launch_gemm_gemv(A, B, SA, SB, N, K, sa_cols, sb_cols, alpha, args, out, stream);
  if (gemm_decode_supported(args.format, M, N, K, A, B, SB))
    return launch_gemm_decode(A, B, SA, SB, M, N, K, sa_cols, sb_cols, alpha, args, out, stream);
  if (M == 1) return launch_rows<1>(A, B, SA, SB, M, N, K, sa_cols, sb_cols, alpha, args, out, stream);
  if (M <= 4) return launch_rows<4>(A, B, SA, SB, M, N, K, sa_cols, sb_cols, alpha, args, out, stream);
  if (M <= 8) return launch_rows<8>(A, B, SA, SB, M, N, K, sa_cols, sb_cols, alpha, args, out, stream);
  return launch_rows<16>(A, B, SA, SB, M, N, K, sa_cols, sb_cols, alpha, args, out, stream);
}

}  // namespace emu
