// Emulated scaled FP4 GEMM for skinny problems (few rows of A: decode-shaped M <= 16 per pass),
// CUDA cores.  The bytes of B (N x K/2, read once) dominate, so the kernel is built to stream B:
// one thread per output column, B read straight from global memory 32 bytes per K chunk per
// thread, the chunk of all A rows (and their scales) staged in shared memory and read as
// broadcasts.  Each thread carries the emulation state of its column for every row of the pass.
//
// Arithmetic is the general kernel's (gemm_simt.cu), bit for bit the reference's
// (nvfp_emulation.cpp:90-156, mxfp_emulation.cpp:98-166, core.py:69-148):
//   stage 1  p4 = 4 * group dot, exact in int32 (DP4A on 2a, 2b), rounded once onto the fp16 grid;
//   stage 2  NVFP4 p4 * (sa*2^9) * (sb*2^9) exact in int64 (units of 2^-20); MXFP4 p * 2^.. in f64;
//   stage 3  exact int64 sum (NVFP4) / ((+0 + v0) + v1) ... in f64 (MXFP4);
//   stage 4  acc = R4(s0); acc = R4(f64(acc) + s_b); output (acc * alpha) -> fp16 [-> bf16].
#include <cuda_runtime.h>
#include <stdint.h>

#include <type_traits>

#include "common.cuh"
#include "kernels.h"

namespace emu {
namespace {

constexpr int SK_THREADS = 128;   // output columns per CTA
constexpr int SK_KC = 64;         // K elements per chunk

__device__ __forceinline__ uint32_t unpack4(uint32_t nibbles) {   // 4 e2m1 codes -> 4 int8 (2x values)
  uint32_t packed = 0;
#pragma unroll
  for (int e = 0; e < 4; ++e)
    packed |= ((uint32_t)(uint8_t)(int8_t)e2m1_twice((nibbles >> (4 * e)) & 0xFu)) << (8 * e);
  return packed;
}

// ROWS: rows of A per pass (1, 4 or 16; grid.y covers the rest)
template <int FMT, int SK_ROWS>
__global__ void __launch_bounds__(SK_THREADS)
emul_gemm_skinny_kernel(const uint8_t* __restrict__ A, const uint8_t* __restrict__ B,
                        const uint8_t* __restrict__ SA, const uint8_t* __restrict__ SB, int64_t M, int64_t N,
                        int64_t K, int64_t sa_cols, int64_t sb_cols, const float* __restrict__ alpha, GemmArgs args,
                        void* __restrict__ out) {
  constexpr int GS = (FMT == EMU_FMT_NVFP4) ? 16 : 32;
  constexpr int GPC = SK_KC / GS;             // groups per chunk
  constexpr int WPG = GS / 4;                 // int8x4 words per group
  __shared__ __align__(16) uint32_t As[SK_ROWS][SK_KC / 4];
  __shared__ int32_t Si[SK_ROWS][GPC];        // NVFP4: E4M3 * 2^9 (0 for NaN)
  __shared__ double Sd[SK_ROWS][GPC];         // MXFP4: 2^(ua-129)
  __shared__ uint8_t Sn[SK_ROWS];             // NVFP4: the row has a NaN scale

  const int tid = threadIdx.x;
  const int64_t n = (int64_t)blockIdx.x * SK_THREADS + tid;
  const int64_t r0 = (int64_t)blockIdx.y * SK_ROWS;
  const int rows = (int)((M - r0) < SK_ROWS ? (M - r0) : SK_ROWS);
  const bool col_ok = n < N;
  const int64_t G = K / GS;
  const int wr = args.w_reduce;
  const int64_t nb = G / wr;
  const int64_t kbytes = K / 2;

  using SType = typename std::conditional<FMT == EMU_FMT_NVFP4, long long, double>::type;
  SType S[SK_ROWS];
  float acc[SK_ROWS];
#pragma unroll
  for (int i = 0; i < SK_ROWS; ++i) { S[i] = 0; acc[i] = 0.f; }
  bool col_nan = false;
  for (int t = tid; t < SK_ROWS; t += SK_THREADS) Sn[t] = 0;

  int gi = 0;
  int64_t blk = 0;
  for (int64_t k0 = 0; k0 < K; k0 += SK_KC) {
    __syncthreads();   // K is a multiple of the chunk: every chunk holds GPC whole groups
    // A chunk: rows x 32 bytes, 4 bytes (8 elements -> 2 words) per thread
    for (int t = tid; t < SK_ROWS * 8; t += SK_THREADS) {
      const int r = t >> 3, part = t & 7;
      uint32_t w = 0;
      const int64_t kb = k0 / 2 + part * 4;
      if (r < rows) w = *reinterpret_cast<const uint32_t*>(A + (r0 + r) * kbytes + kb);
      As[r][2 * part] = unpack4(w & 0xFFFFu);
      As[r][2 * part + 1] = unpack4(w >> 16);
    }
    for (int t = tid; t < SK_ROWS * GPC; t += SK_THREADS) {
      const int r = t / GPC, gl = t % GPC;
      const uint32_t byte = r < rows ? SA[swz_offset(r0 + r, k0 / GS + gl, sa_cols)] : 0u;
      if (FMT == EMU_FMT_NVFP4) {
        bool nan;
        Si[r][gl] = e4m3_times_512(byte, &nan);
        if (nan) Sn[r] = 1;
      } else {
        Sd[r][gl] = ue8m0_quarter_f64(byte);
      }
    }
    __syncthreads();
    // this column's chunk of B: 32 bytes -> 16 words of int8 pairs
    uint32_t bw[SK_KC / 4];
    {
      uint4 lo = make_uint4(0, 0, 0, 0), hi = make_uint4(0, 0, 0, 0);
      const int64_t kb = k0 / 2;
      if (col_ok) {
        const uint8_t* src = B + n * kbytes + kb;
        lo = __ldg(reinterpret_cast<const uint4*>(src));
        hi = __ldg(reinterpret_cast<const uint4*>(src + 16));
      }
      const uint32_t in[8] = {lo.x, lo.y, lo.z, lo.w, hi.x, hi.y, hi.z, hi.w};
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        bw[2 * q] = unpack4(in[q] & 0xFFFFu);
        bw[2 * q + 1] = unpack4(in[q] >> 16);
      }
    }
#pragma unroll
    for (int gl = 0; gl < GPC; ++gl) {
      const int64_t g = k0 / GS + gl;
      const uint32_t bbyte = col_ok ? SB[swz_offset(n, g, sb_cols)] : 0u;
      int32_t sbi = 0;
      double sbd = 0.0;
      if (FMT == EMU_FMT_NVFP4) {
        bool nan;
        sbi = e4m3_times_512(bbyte, &nan);
        col_nan |= nan;
      } else {
        sbd = ue8m0_quarter_f64(bbyte) * 4.0;   // 2^(ub-127); the 1/4 is in Sd
      }
#pragma unroll
      for (int i = 0; i < SK_ROWS; ++i) {
        int p4 = 0;
#pragma unroll
        for (int w = 0; w < WPG; ++w) p4 = __dp4a((int)As[i][gl * WPG + w], (int)bw[gl * WPG + w], p4);
        const int p = round_p4_to_fp16_grid(p4);
        if (FMT == EMU_FMT_NVFP4) {
          S[i] += (long long)(p * Si[i][gl]) * (long long)sbi;
        } else {
          S[i] = __dadd_rn(S[i], __dmul_rn((double)p, __dmul_rn(Sd[i][gl], sbd)));
        }
      }
      if (++gi == wr) {
        gi = 0;
#pragma unroll
        for (int i = 0; i < SK_ROWS; ++i) {
          double s;
          if (FMT == EMU_FMT_NVFP4) s = __ll2double_rn(S[i]) * 0x1p-20;
          else s = S[i];
          if (nb == 1) acc[i] = round_f64_to_f32(s, args.stage3_rounding);
          else if (blk == 0) acc[i] = round_f64_to_f32(s, args.stage4_rounding);
          else acc[i] = round_f64_to_f32(__dadd_rn((double)acc[i], s), args.stage4_rounding);
          S[i] = 0;
        }
        ++blk;
      }
    }
  }
  if (!col_ok) return;
  const float al = alpha ? *alpha : 1.0f;
#pragma unroll
  for (int i = 0; i < SK_ROWS; ++i) {
    if (i >= rows) break;
    float y = alpha ? __fmul_rn(acc[i], al) : acc[i];
    if (FMT == EMU_FMT_NVFP4 && (Sn[i] || col_nan)) y = __int_as_float(0x7FFFFFFF);
    store_output(out, (r0 + i) * N + n, y, args.out_mode);
  }
}

}  // namespace

bool gemm_skinny_supported(int64_t M, int64_t K) { return M >= 1 && M <= 64 && K % SK_KC == 0; }

template <int ROWS>
static void launch_rows(const uint8_t* A, const uint8_t* B, const uint8_t* SA, const uint8_t* SB, int64_t M, int64_t N,
                        int64_t K, int64_t sa_cols, int64_t sb_cols, const float* alpha, const GemmArgs& args,
                        void* out, cudaStream_t stream) {
  dim3 grid((unsigned)((N + SK_THREADS - 1) / SK_THREADS), (unsigned)((M + ROWS - 1) / ROWS));
  if (args.format == EMU_FMT_NVFP4)
    emul_gemm_skinny_kernel<EMU_FMT_NVFP4, ROWS><<<grid, SK_THREADS, 0, stream>>>(A, B, SA, SB, M, N, K, sa_cols,
                                                                                 sb_cols, alpha, args, out);
  else
    emul_gemm_skinny_kernel<EMU_FMT_MXFP4, ROWS><<<grid, SK_THREADS, 0, stream>>>(A, B, SA, SB, M, N, K, sa_cols,
                                                                                 sb_cols, alpha, args, out);
}

cudaError_t launch_gemm_skinny(const uint8_t* A, const uint8_t* B, const uint8_t* SA, const uint8_t* SB, int64_t M,
                               int64_t N, int64_t K, int64_t sa_cols, int64_t sb_cols, const float* alpha,
                               const GemmArgs& args, void* out, cudaStream_t stream) {
  if (M == 1) launch_rows<1>(A, B, SA, SB, M, N, K, sa_cols, sb_cols, alpha, args, out, stream);
  else if (M <= 4) launch_rows<4>(A, B, SA, SB, M, N, K, sa_cols, sb_cols, alpha, args, out, stream);
  else launch_rows<16>(A, B, SA, SB, M, N, K, sa_cols, sb_cols, alpha, args, out, stream);
  return cudaGetLastError();
}

}  // namespace emu
