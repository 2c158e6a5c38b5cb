// Emulated scaled FP4 GEMM on CUDA cores (DP4A stage 1 + exact integer / f64 epilogue).
//
// This is the general path: any w_reduce, any M/N/K the C ABI accepts, both formats.  The
// tensor-core kernel (gemm_tc.cu) handles the common shapes faster and falls back to this one.
//
// Arithmetic (reference nvfp_emulation.cpp:90-156, mxfp_emulation.cpp:98-166, core.py:69-148):
//   stage 1  p4 = 4 * sum_{k in group} a_k b_k, exact in int32 via DP4A on 2a, 2b in [-12, 12];
//            then rounded once onto the fp16 grid (round_p4_to_fp16_grid).
//   stage 2  NVFP4: v = p * sa * sb is exact in f32 (<= 20 significant bits), so it is kept as the
//            exact integer p4 * (sa*2^9) * (sb*2^9) in units of 2^-20 (int64).
//            MXFP4: v = p * 2^(ua-127) * 2^(ub-127) in f64, exact (or inf / NaN like the reference).
//   stage 3  NVFP4: the f64 sum of w_reduce exact terms is exact (|sum| < 2^53 units of 2^-20 for
//            w_reduce <= 64), so the int64 sum converted once to f64 equals the reference's sum.
//            MXFP4: ((+0.0 + v0) + v1) + ... with f64 adds, as the reference.
//   stage 4  acc = R4(s0); acc = R4(f64(acc) + s_b), R = cvt.{rz,rn}.f32.f64.
//   output   (acc * alpha) in f32 -> fp16 RNE [-> bf16 RNE].
// A NaN E4M3 scale makes every output of its row (A) or column (B) NaN, as NaN propagates through
// all later stages of the reference; those outputs are written as NaN directly.
#include <cuda_runtime.h>
#include <stdint.h>

#include <type_traits>

#include "common.cuh"
#include "kernels.h"

namespace emu {
namespace {

constexpr int BM = 64, BN = 64, KC = 64;      // CTA tile and K chunk (elements)
constexpr int THREADS = 256;                  // 16 x 16 threads, 4 x 4 outputs each
constexpr int ROW_WORDS = KC / 4 + 4;         // int8 row of the chunk + 16 bytes padding

// Expand 16 packed e2m1 nibbles (8 bytes) into 16 int8 values 2*x.
__device__ __forceinline__ uint4 unpack16(uint2 w) {
  return make_uint4(e2m1x4_to_int8x4(w.x & 0xFFFFu), e2m1x4_to_int8x4(w.x >> 16), e2m1x4_to_int8x4(w.y & 0xFFFFu),
                    e2m1x4_to_int8x4(w.y >> 16));
}

template <int FMT>
__global__ void __launch_bounds__(THREADS)
emul_gemm_simt_kernel(const uint8_t* __restrict__ A, const uint8_t* __restrict__ B,
                      const uint8_t* __restrict__ SA, const uint8_t* __restrict__ SB, int64_t M,
                      int64_t N, int64_t K, int64_t sa_cols, int64_t sb_cols,
                      const float* __restrict__ alpha, GemmArgs args, void* __restrict__ out) {
  constexpr int GS = (FMT == EMU_FMT_NVFP4) ? 16 : 32;
  constexpr int GPC = KC / GS;                // groups per chunk
  constexpr int WPG = GS / 4;                 // 32-bit words per group
  __shared__ __align__(16) uint32_t As[BM * ROW_WORDS];
  __shared__ __align__(16) uint32_t Bs[BN * ROW_WORDS];

  const int tid = threadIdx.x;
  const int tx = tid & 15, ty = tid >> 4;
  const int64_t m0 = (int64_t)blockIdx.x * BM, n0 = (int64_t)blockIdx.y * BN;
  const int64_t G = K / GS;
  const int wr = args.w_reduce;
  const int64_t nb = G / wr;
  const int64_t kbytes = K / 2;

  // per-output state
  using SType = typename std::conditional<FMT == EMU_FMT_NVFP4, long long, double>::type;
  SType S[4][4];
  float acc[4][4];
  bool row_nan[4] = {false, false, false, false}, col_nan[4] = {false, false, false, false};
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) { S[i][j] = 0; acc[i][j] = 0.f; }

  int gi = 0;        // group index inside the current stage-3 block
  int64_t blk = 0;   // stage-3 block index

  for (int64_t k0 = 0; k0 < K; k0 += KC) {
    // ---- load + unpack the chunk: 64 rows x 32 bytes per operand, 8 bytes per thread
    {
      const int r = tid >> 2, part = tid & 3;           // row, 8-byte part of the 32-byte row
      const int64_t kb = k0 / 2 + part * 8;              // byte offset in the packed row
      uint2 wa = make_uint2(0, 0), wb = make_uint2(0, 0);
      if (m0 + r < M && kb < kbytes) wa = *reinterpret_cast<const uint2*>(A + (m0 + r) * kbytes + kb);
      if (n0 + r < N && kb < kbytes) wb = *reinterpret_cast<const uint2*>(B + (n0 + r) * kbytes + kb);
      *reinterpret_cast<uint4*>(&As[r * ROW_WORDS + part * 4]) = unpack16(wa);
      *reinterpret_cast<uint4*>(&Bs[r * ROW_WORDS + part * 4]) = unpack16(wb);
    }
    __syncthreads();

    const int ngroups = (K - k0) / GS < GPC ? (int)((K - k0) / GS) : GPC;
    for (int gl = 0; gl < ngroups; ++gl) {
      const int64_t g = k0 / GS + gl;
      // scales of this thread's rows / cols for group g
      int32_t sa_i[4], sb_i[4];
      double sa_d[4], sb_d[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int64_t r = m0 + ty + 16 * i, c = n0 + tx + 16 * i;
        const uint32_t ba = (r < M) ? SA[swz_offset(r, g, sa_cols)] : 0u;
        const uint32_t bb = (c < N) ? SB[swz_offset(c, g, sb_cols)] : 0u;
        if (FMT == EMU_FMT_NVFP4) {
          bool na, nbn;
          sa_i[i] = e4m3_times_512(ba, &na);
          sb_i[i] = e4m3_times_512(bb, &nbn);
          row_nan[i] |= na;
          col_nan[i] |= nbn;
        } else {
          sa_d[i] = ue8m0_quarter_f64(ba);
          sb_d[i] = ue8m0_quarter_f64(bb) * 4.0;      // 2^(ub-127); the 1/4 is folded into sa_d
        }
      }
      // stage 1: exact integer dot products
      int p4[4][4];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) p4[i][j] = 0;
#pragma unroll
      for (int w = 0; w < WPG; w += 4) {
        uint4 av[4], bv[4];
#pragma unroll
        for (int i = 0; i < 4; ++i)
          av[i] = *reinterpret_cast<const uint4*>(&As[(ty + 16 * i) * ROW_WORDS + gl * WPG + w]);
#pragma unroll
        for (int j = 0; j < 4; ++j)
          bv[j] = *reinterpret_cast<const uint4*>(&Bs[(tx + 16 * j) * ROW_WORDS + gl * WPG + w]);
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            int s = p4[i][j];
            s = __dp4a((int)av[i].x, (int)bv[j].x, s);
            s = __dp4a((int)av[i].y, (int)bv[j].y, s);
            s = __dp4a((int)av[i].z, (int)bv[j].z, s);
            s = __dp4a((int)av[i].w, (int)bv[j].w, s);
            p4[i][j] = s;
          }
      }
      // stages 1-3
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int p = round_p4_to_fp16_grid(p4[i][j]);
          if (FMT == EMU_FMT_NVFP4) {
            const int t = p * sa_i[i];                               // |t| < 2^30
            S[i][j] += (long long)t * (long long)sb_i[j];            // units of 2^-20
          } else {
            const double c = __dmul_rn(sa_d[i], sb_d[j]);           // 2^(ua+ub-256) or inf
            S[i][j] = __dadd_rn(S[i][j], __dmul_rn((double)p, c));  // (+0 + v0) + v1 ...
          }
        }
      // stage 4 at the end of a block
      if (++gi == wr) {
        gi = 0;
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            double s;
            if (FMT == EMU_FMT_NVFP4) s = __ll2double_rn(S[i][j]) * 0x1p-20;  // exact
            else s = S[i][j];
            float a;
            if (nb == 1) a = round_f64_to_f32(s, args.stage3_rounding);
            else if (blk == 0) a = round_f64_to_f32(s, args.stage4_rounding);
            else a = round_f64_to_f32(__dadd_rn((double)acc[i][j], s), args.stage4_rounding);
            acc[i][j] = a;
            S[i][j] = 0;
          }
        ++blk;
      }
    }
    __syncthreads();
  }

  const float al = alpha ? *alpha : 1.0f;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int64_t r = m0 + ty + 16 * i;
    if (r >= M) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int64_t c = n0 + tx + 16 * j;
      if (c >= N) continue;
      float y = alpha ? __fmul_rn(acc[i][j], al) : acc[i][j];
      if (FMT == EMU_FMT_NVFP4 && (row_nan[i] || col_nan[j])) y = __int_as_float(0x7FFFFFFF);
      store_output(out, r * N + c, y, args.out_mode);
    }
  }
}

}  // namespace

cudaError_t launch_gemm_simt(const uint8_t* A, const uint8_t* B, const uint8_t* SA,
                             const uint8_t* SB, int64_t M, int64_t N, int64_t K, int64_t sa_cols,
                             int64_t sb_cols, const float* alpha, const GemmArgs& args, void* out,
                             cudaStream_t stream) {
  dim3 grid((unsigned)((M + BM - 1) / BM), (unsigned)((N + BN - 1) / BN));
  if (args.format == EMU_FMT_NVFP4)
    emul_gemm_simt_kernel<EMU_FMT_NVFP4><<<grid, THREADS, 0, stream>>>(A, B, SA, SB, M, N, K, sa_cols,
                                                                      sb_cols, alpha, args, out);
  else
    emul_gemm_simt_kernel<EMU_FMT_MXFP4><<<grid, THREADS, 0, stream>>>(A, B, SA, SB, M, N, K, sa_cols,
                                                                      sb_cols, alpha, args, out);
  return cudaGetLastError();
}

}  // namespace emu
