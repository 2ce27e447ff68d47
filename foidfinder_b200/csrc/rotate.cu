// Per-token activation quantisation for the W8A8 GEMMs, with the LayerNorm in front of it fused in:
//   x fp16 -> [LayerNorm over the valid columns, f32 statistics] -> block-diagonal Sylvester Hadamard
//   (normalised) -> per-row scale s = max(amax, 1e-12) / 127 -> codes clamp(rint(v / s), +-127).
// Follows rot_q8_1024 (foidfinder/backends/cuda/csrc/kernels.cu:49-108) and rot_q8_h128
// (kernels.cu:112-160); quantiser semantics from common.cuh:45-48; the EVA02 LayerNorm eps and the
// SwiGLU hidden norm from foidfinder/backends/mlx/haruka.py:19,97-98.
//
// One warp per row, kRotWarps rows per CTA; the whole row stays in registers. Lane l holds 8
// consecutive columns of every 256-column chunk i (columns i*256 + l*8 + e), loaded as 16-byte vectors,
// so a row costs one coalesced read of 2 B/column and one write of 1 B/column plus the 4-byte scale.
//
// The Hadamard butterflies over column bits 0-2 (e) and 8+ (chunk) run in registers in that layout. The
// butterflies over bits 3..7 (the lane index) do not use shuffles: a group of UNIT chunks is written to a
// per-warp shared-memory buffer and read back transposed — lane (e, q) then holds the G = 2^TB values
// whose columns differ only in bits 3..3+TB-1 — the butterflies run in registers, and the values go back
// through the same buffer into the load layout. Two shared-memory round trips per element replace one
// shuffle + select + add per element per lane-bit stage. The buffer is padded by 8 floats every 8*G
// columns so the transposed accesses hit 32 distinct banks. Arithmetic is packed f32x2 wherever both
// halves of a register pair take the same operation (exactly rounded per lane, like scalar FADD/FFMA).
//
// The LayerNorm runs over the first valid_cols columns: columns past it are zeroed at load, their
// (0 - mean)^2 terms are taken back out of the variance, and they are zeroed again after the affine step.
#include <algorithm>

#include "common.h"
#include "kernels.h"
#include "ptx.cuh"

namespace ff {

constexpr int kRotWarps = 4;  // per-row grid: small CTAs (the 2816-column rows need ~134 registers per thread)

template <int NCH, int BLOCK>
struct RotShape {
  static constexpr int LB = BLOCK == 128 ? 7 : BLOCK == 256 ? 8 : BLOCK == 512 ? 9 : 10;
  static constexpr int TB = LB - 3 < 5 ? LB - 3 : 5;  // column bits 3..3+TB-1 run in the transposed layout
  static constexpr int G = 1 << TB;                   // values per lane in the transposed layout
  static constexpr int UNIT = G / 8;                  // 256-column chunks per transpose
  static constexpr int NCHP = (NCH + UNIT - 1) / UNIT * UNIT;
  static constexpr int COLS = NCH * 256;
  static constexpr int QB = 8 * G;  // columns per transposed lane group (padding period)
  static constexpr int SW = UNIT * 256 + 8 * (UNIT * 256 / QB);  // floats of one warp's transpose buffer
  static_assert((1 << LB) == BLOCK && BLOCK / 256 <= UNIT, "unsupported Hadamard block");
};

// One row by one warp; xr is the row's fp16 input (global memory, or shared memory when SRC_SMEM).
// gb(i, g, b) supplies this lane's 8 gamma and 8 beta values of chunk i.
template <int NCH, int BLOCK, bool NORM, bool SRC_SMEM, class GammaBeta>
__device__ __forceinline__ void rot_row(const __half* __restrict__ xr, float eps, int row, int valid_cols,
                                        int8_t* __restrict__ out, float* __restrict__ row_scale, float* sw, int lane,
                                        GammaBeta gb) {
  using S = RotShape<NCH, BLOCK>;
  constexpr int G = S::G, UNIT = S::UNIT, NCHP = S::NCHP, COLS = S::COLS, QB = S::QB;

  float2 v[NCHP][4];
#pragma unroll
  for (int i = 0; i < NCHP; ++i) {
    if (i < NCH) {
      const uint4* src = reinterpret_cast<const uint4*>(xr + i * 256 + lane * 8);
      const uint4 u = SRC_SMEM ? *src : __ldg(src);
      v[i][0] = unpack_half2(u.x);
      v[i][1] = unpack_half2(u.y);
      v[i][2] = unpack_half2(u.z);
      v[i][3] = unpack_half2(u.w);
    } else {
#pragma unroll
      for (int k = 0; k < 4; ++k) v[i][k] = make_float2(0.f, 0.f);
    }
  }
  // Columns >= valid_cols: only chunks that reach past the boundary take this (warp-uniform) branch.
  auto zero_ragged = [&](int i) {
    if (i < NCH && (i + 1) * 256 > valid_cols) {
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const int c = i * 256 + lane * 8 + 2 * k;
        if (c >= valid_cols) v[i][k].x = 0.f;
        if (c + 1 >= valid_cols) v[i][k].y = 0.f;
      }
    }
  };
#pragma unroll
  for (int i = 0; i < NCH; ++i) zero_ragged(i);

  float rstd = 0.f;
  if constexpr (NORM) {
    // Four partial sums per statistic (one per register pair k): with only a few warps per scheduler, one
    // chain of 4 NCH dependent adds per row left the warps waiting on its latency.
    float2 s2[4], q2[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) s2[k] = q2[k] = make_float2(0.f, 0.f);
#pragma unroll
    for (int i = 0; i < NCH; ++i)
#pragma unroll
      for (int k = 0; k < 4; ++k) s2[k] = add2(s2[k], v[i][k]);
    const float2 st = add2(add2(s2[0], s2[1]), add2(s2[2], s2[3]));
    const float inv_n = 1.f / static_cast<float>(valid_cols);
    const float mean = warp_sum(st.x + st.y) * inv_n;
    const float2 m2 = make_float2(mean, mean);
#pragma unroll
    for (int i = 0; i < NCH; ++i)
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        v[i][k] = sub2(v[i][k], m2);
        q2[k] = fma2(v[i][k], v[i][k], q2[k]);
      }
    const float2 qt = add2(add2(q2[0], q2[1]), add2(q2[2], q2[3]));
    const float q = warp_sum(qt.x + qt.y) - static_cast<float>(COLS - valid_cols) * mean * mean;
    rstd = rsqrtf(fmaxf(q, 0.f) * inv_n + eps);
  }

#pragma unroll
  for (int c0 = 0; c0 < NCHP; c0 += UNIT) {
    if constexpr (NORM) {
      const float2 r2 = make_float2(rstd, rstd);
#pragma unroll
      for (int i = c0; i < c0 + UNIT; ++i) {
        if (i < NCH) {
          float g[8], b[8];
          gb(i, g, b);
#pragma unroll
          for (int k = 0; k < 4; ++k)
            v[i][k] = fma2(v[i][k], mul2(r2, make_float2(g[2 * k], g[2 * k + 1])), make_float2(b[2 * k], b[2 * k + 1]));
          zero_ragged(i);
        }
      }
    }
    // Column bit 0 (inside a register pair), bits 1-2 (across pairs), then chunk bits 8.. (across chunks).
#pragma unroll
    for (int i = c0; i < c0 + UNIT; ++i) {
#pragma unroll
      for (int k = 0; k < 4; ++k) v[i][k] = make_float2(v[i][k].x + v[i][k].y, v[i][k].x - v[i][k].y);
#pragma unroll
      for (int h = 1; h < 4; h <<= 1)
#pragma unroll
        for (int k = 0; k < 4; ++k)
          if (!(k & h)) {
            const float2 a = v[i][k], b = v[i][k + h];
            v[i][k] = add2(a, b);
            v[i][k + h] = sub2(a, b);
          }
    }
#pragma unroll
    for (int h = 1; h * 256 < BLOCK; h <<= 1)
#pragma unroll
      for (int i = c0; i < c0 + UNIT; ++i)
        if (!((i - c0) & h))
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const float2 a = v[i][k], b = v[i + h][k];
            v[i][k] = add2(a, b);
            v[i + h][k] = sub2(a, b);
          }

    // Transpose through shared memory. Writer lane l stores its 8 columns of a chunk as two 16-byte halves
    // at c + 8 (c / QB) (c = chunk offset + 8 l), the halves swapped in place (low half at +4) when bit 2 of
    // l is set: each quarter-warp phase of a 16-byte store then covers all 32 banks once. The swap is in
    // the addresses only (no per-lane data selects); a reader of element t of writer l = t finds column
    // e at offset e when bit 2 of t is clear and at e ^ 4 when it is set.
    const int half_sw = (lane & 4) ? 4 : 0;
#pragma unroll
    for (int i = c0; i < c0 + UNIT; ++i) {
      const int c = (i - c0) * 256 + lane * 8;
      float* d = sw + c + 8 * (c / QB);
      *reinterpret_cast<float4*>(d + half_sw) = make_float4(v[i][0].x, v[i][0].y, v[i][1].x, v[i][1].y);
      *reinterpret_cast<float4*>(d + 4 - half_sw) = make_float4(v[i][2].x, v[i][2].y, v[i][3].x, v[i][3].y);
    }
    __syncwarp();
    const int e = lane & 7, q = lane >> 3;
    // transposed element t at tp[8 t], tp = tp_a when bit 2 of t is clear, tp_b when it is set
    float* const tp_a = sw + e + q * (QB + 8);
    float* const tp_b = sw + (e ^ 4) + q * (QB + 8);
    float2 tv[G / 2];
#pragma unroll
    for (int j = 0; j < G / 2; ++j) {
      const float* tp = ((j >> 1) & 1) ? tp_b : tp_a;  // elements 2j, 2j + 1 share bit 2 (compile-time choice)
      tv[j] = make_float2(tp[16 * j], tp[16 * j + 8]);
    }
#pragma unroll
    for (int j = 0; j < G / 2; ++j) tv[j] = make_float2(tv[j].x + tv[j].y, tv[j].x - tv[j].y);
#pragma unroll
    for (int h = 1; h < G / 2; h <<= 1)
#pragma unroll
      for (int j = 0; j < G / 2; ++j)
        if (!(j & h)) {
          const float2 a = tv[j], b = tv[j + h];
          tv[j] = add2(a, b);
          tv[j + h] = sub2(a, b);
        }
#pragma unroll
    for (int j = 0; j < G / 2; ++j) {
      float* tp = ((j >> 1) & 1) ? tp_b : tp_a;
      tp[16 * j] = tv[j].x;
      tp[16 * j + 8] = tv[j].y;
    }
    __syncwarp();
#pragma unroll
    for (int i = c0; i < c0 + UNIT; ++i) {
      const int c = (i - c0) * 256 + lane * 8;
      const float* d = sw + c + 8 * (c / QB);
      const float4 a = *reinterpret_cast<const float4*>(d + half_sw);
      const float4 b = *reinterpret_cast<const float4*>(d + 4 - half_sw);
      v[i][0] = make_float2(a.x, a.y);
      v[i][1] = make_float2(a.z, a.w);
      v[i][2] = make_float2(b.x, b.y);
      v[i][3] = make_float2(b.z, b.w);
    }
    __syncwarp();
  }

  constexpr float kNorm = BLOCK == 128   ? 0.08838834764831845f
                          : BLOCK == 256 ? 0.0625f
                          : BLOCK == 512 ? 0.04419417382415922f
                                         : 0.03125f;  // 1 / sqrt(BLOCK)
  // For power-of-two blocks (1/sqrt(BLOCK) = 2^-k) the normalisation is folded into the row maximum and
  // the quantisation multiplier: scaling by a power of two is exact, so scale and codes are bit-identical
  // to normalising first.
  constexpr bool kPow2Norm = BLOCK == 256 || BLOCK == 1024;
  const float2 n2 = make_float2(kNorm, kNorm);
  float am[4] = {0.f, 0.f, 0.f, 0.f};  // independent running maxima (max is exact in any order)
#pragma unroll
  for (int i = 0; i < NCH; ++i)
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      if constexpr (!kPow2Norm) v[i][k] = mul2(v[i][k], n2);
      am[k] = max3(am[k], fabsf(v[i][k].x), fabsf(v[i][k].y));
    }
  float amax = warp_max(max3(am[0], am[1], fmaxf(am[2], am[3])));
  if constexpr (kPow2Norm) amax *= kNorm;
  const float scale = fmaxf(amax, 1e-12f) / 127.f;
  const float inv = kPow2Norm ? (1.f / scale) * kNorm : 1.f / scale;
  const float2 inv2 = make_float2(inv, inv), magic2 = make_float2(12582912.f, 12582912.f);
  int8_t* orow = out + static_cast<size_t>(row) * COLS;
#pragma unroll
  for (int i = 0; i < NCH; ++i) {
    // rint(v * inv) (round half to even, as __float2int_rn) without the XU conversion: adding 1.5 * 2^23
    // to the f32 product leaves the rounded integer in the low mantissa bits, whose low byte is the
    // two's-complement int8 code. |v * inv| <= 127 by construction of the scale, so no clamp is needed.
    uint32_t t[8];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float2 r = add2(mul2(v[i][k], inv2), magic2);
      t[2 * k] = __float_as_uint(r.x);
      t[2 * k + 1] = __float_as_uint(r.y);
    }
    const uint32_t w0 = __byte_perm(__byte_perm(t[0], t[1], 0x0040), __byte_perm(t[2], t[3], 0x0040), 0x5410);
    const uint32_t w1 = __byte_perm(__byte_perm(t[4], t[5], 0x0040), __byte_perm(t[6], t[7], 0x0040), 0x5410);
    *reinterpret_cast<uint2*>(orow + i * 256 + lane * 8) = make_uint2(w0, w1);
  }
  if (lane == 0) row_scale[row] = scale;
}

// Per-row grid (one warp per row); gamma/beta, when used, come through L1 for every row.
template <int NCH, int BLOCK, bool NORM>
__global__ void __launch_bounds__(kRotWarps * 32)
    rot_q8_kernel(const __half* __restrict__ x, const float* __restrict__ gamma, const float* __restrict__ beta,
                  float eps, int rows, int valid_cols, int8_t* __restrict__ out, float* __restrict__ row_scale) {
  using S = RotShape<NCH, BLOCK>;
  __shared__ __align__(16) float smem[kRotWarps][S::SW];
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  const int row = blockIdx.x * kRotWarps + wid;
  pdl_wait();
  pdl_trigger();
  if (row >= rows) return;
  rot_row<NCH, BLOCK, NORM, false>(x + static_cast<size_t>(row) * S::COLS, eps, row, valid_cols, out, row_scale,
                                   smem[wid], lane,
                            [&](int i, float (&g)[8], float (&b)[8]) {
                              const int c = i * 256 + lane * 8;
                              const float4 g0 = __ldg(reinterpret_cast<const float4*>(gamma + c));
                              const float4 g1 = __ldg(reinterpret_cast<const float4*>(gamma + c + 4));
                              const float4 b0 = __ldg(reinterpret_cast<const float4*>(beta + c));
                              const float4 b1 = __ldg(reinterpret_cast<const float4*>(beta + c + 4));
                              g[0] = g0.x, g[1] = g0.y, g[2] = g0.z, g[3] = g0.w;
                              g[4] = g1.x, g[5] = g1.y, g[6] = g1.z, g[7] = g1.w;
                              b[0] = b0.x, b[1] = b0.y, b[2] = b0.z, b[3] = b0.w;
                              b[4] = b1.x, b[5] = b1.y, b[6] = b1.z, b[7] = b1.w;
                            });
}

// Persistent grid, one CTA per SM, each warp walking rows with a grid stride. Two things the per-row grid
// pays for every row are moved off the L1 data pipe (the limiter, see above) and off the critical path:
//  - the row itself arrives by a bulk asynchronous copy (cp.async.bulk, no multicast) into a per-warp
//    double buffer in shared memory, issued one row ahead, so HBM latency overlaps the previous row;
//  - with the LayerNorm, gamma and beta live in TMEM: each CTA writes every lane's 8 + 8 values per
//    chunk once (16 columns per chunk, one copy per TMEM sub-partition, so warp w reads lane quarter
//    w % 4 as any tcgen05.ld does) and each row reads them back with tcgen05.ld instead of reloading
//    them through L1, where they cost twice the wavefronts of the row's own input.
// Every wait is bounded; on a timeout the warp records kDevTimeoutRotate, drains its copy and stops.
template <int NCH, int BLOCK, int WARPS, bool NORM>
__global__ void __launch_bounds__(WARPS * 32, 1)
    rot_q8_persistent_kernel(const __half* __restrict__ x, const float* __restrict__ gamma,
                             const float* __restrict__ beta, float eps, int rows, int valid_cols,
                             int8_t* __restrict__ out, float* __restrict__ row_scale, int* err) {
  using S = RotShape<NCH, BLOCK>;
  constexpr uint32_t kRowBytes = S::COLS * 2;
  constexpr uint32_t kCols = NCH * 16 <= 32 ? 32 : NCH * 16 <= 64 ? 64 : NCH * 16 <= 128 ? 128 : 256;
  static_assert(NCH * 16 <= 256, "gamma/beta do not fit the TMEM allocation");
  extern __shared__ float4 rot_dyn[];
  __shared__ uint32_t tmem_slot;
  __shared__ uint64_t bars[WARPS][2];
  __shared__ int abort_flag;
  // [WARPS][2] row buffers, then [WARPS] transpose buffers
  uint8_t* rowbuf = reinterpret_cast<uint8_t*>(rot_dyn);
  float* tbuf = reinterpret_cast<float*>(rowbuf + static_cast<size_t>(WARPS) * 2 * kRowBytes);
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  if (threadIdx.x == 0) {
    for (int w = 0; w < WARPS; ++w) {
      mbar_init(&bars[w][0], 1);
      mbar_init(&bars[w][1], 1);
    }
    abort_flag = 0;
    fence_mbar_init();
  }
  if constexpr (NORM) {
    if (wid == 0) {
      tmem_alloc(&tmem_slot, kCols);
      tmem_relinquish();
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  pdl_wait();
  pdl_trigger();
  uint32_t tmem = 0;
  if constexpr (NORM) {
    tmem = tmem_slot + (static_cast<uint32_t>(32 * (wid & 3)) << 16);
    if (wid < 4) {
#pragma unroll 1
      for (int i = 0; i < NCH; ++i) {
        const int c = i * 256 + lane * 8;
        uint32_t r[16];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          r[e] = __float_as_uint(__ldg(gamma + c + e));
          r[8 + e] = __float_as_uint(__ldg(beta + c + e));
        }
        tmem_st16(tmem + 16 * i, r);
      }
      tmem_st_wait();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
  }
  volatile int* abort_v = &abort_flag;
  const int stride = gridDim.x * WARPS;
  auto buf = [&](int b) { return reinterpret_cast<const __half*>(rowbuf + (2 * wid + b) * kRowBytes); };
  auto issue = [&](int r, int b) {  // lane 0: bring row r into buffer b
    mbar_arrive_expect_tx(&bars[wid][b], kRowBytes);
    bulk_load(buf(b), x + static_cast<size_t>(r) * S::COLS, kRowBytes, &bars[wid][b]);
  };
  int row = blockIdx.x * WARPS + wid;
  int issued = 0, waited = 0;  // copies issued / waited for (buffer of copy n: n & 1)
  if (row < rows) {
    if (lane == 0) issue(row, 0);
    issued = 1;
  }
  for (int k = 0; row < rows; ++k, row += stride) {
    const int b = k & 1;
    const int next = row + stride;
    if (next < rows) {
      fence_async_smem();  // this warp's reads of the buffer being refilled (two rows ago) come first
      __syncwarp();
      if (lane == 0) issue(next, b ^ 1);
      ++issued;
    }
    if (!mbar_wait<true>(&bars[wid][b], static_cast<uint32_t>(k >> 1) & 1u, abort_v, err, kDevTimeoutRotate)) break;
    ++waited;
    // Chunk i's gamma/beta come from a TMEM load issued at chunk i - 1 (chunks are taken in order 0, 1, ...),
    // so each load's latency overlaps the previous chunk's affine step instead of stalling it.
    uint32_t gbr[16];
    rot_row<NCH, BLOCK, NORM, true>(buf(b), eps, row, valid_cols, out, row_scale, tbuf + wid * S::SW, lane,
                                    [&](int i, float (&g)[8], float (&bb)[8]) {
                                      if (i == 0) tmem_ld16(tmem, gbr);
                                      tmem_ld_wait();
#pragma unroll
                                      for (int e = 0; e < 8; ++e) {
                                        g[e] = __uint_as_float(gbr[e]);
                                        bb[e] = __uint_as_float(gbr[8 + e]);
                                      }
                                      if (i + 1 < NCH) tmem_ld16(tmem + 16 * (i + 1), gbr);
                                    });
    __syncwarp();
  }
  // Copies can only still be in flight after a timeout: let them land (bounded) before the CTA exits.
  // Copy n goes to buffer n & 1 and completes that barrier's phase (n >> 1).
  if (lane == 0) {
    const unsigned long long t0 = globaltimer();
    for (int n = waited; n < issued; ++n)
      while (!mbar_try_wait(smem_u32(&bars[wid][n & 1]), static_cast<uint32_t>(n >> 1) & 1u) &&
             globaltimer() - t0 < kWaitLimitNs) {
      }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if constexpr (NORM)
    if (wid == 0) tmem_dealloc(tmem_slot, kCols);
}

namespace {

// Below this many rows of at most 1024 columns the per-row grid wins (a few rows per warp leave the
// persistent kernel's prologue and TMEM fill unamortised; measured at 8,200 x 1024: 15.3 vs 17.4 us, at
// 65,600 x 1024: 79 vs 72 us).
constexpr int kPersistMinRows1024 = 32768;
#ifndef FF_ROT_PWARPS
#define FF_ROT_PWARPS 24
#endif

template <int NCH, int BLOCK, bool NORM>
int launch_persistent(const __half* x, const float* g, const float* b, float eps, int rows, int valid, int8_t* out,
                      float* rs, int* err, cudaStream_t s) {
  // One CTA per SM: 12 warps for the wide rows (registers), 16 for 2048, FF_ROT_PWARPS (24) for 768/1024
  // (measured at 82,944 x 1024: 16 warps 94 us, 20 warps 90, 24 warps 88; a per-row grid holding gamma/beta
  // in registers instead of TMEM measured 107).
  constexpr int WARPS = NCH > 8 ? 12 : NCH > 4 ? 16 : FF_ROT_PWARPS;
  constexpr size_t smem = static_cast<size_t>(WARPS) * (2 * NCH * 256 * 2 + sizeof(float) * RotShape<NCH, BLOCK>::SW);
  static_assert(smem <= 200 * 1024, "rotation staging does not fit shared memory");
  auto kernel = rot_q8_persistent_kernel<NCH, BLOCK, WARPS, NORM>;
  static bool configured[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64 || !configured[dev]) {
    if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)) !=
        cudaSuccess)
      return check_launch("rot_q8: cudaFuncSetAttribute");
    if (dev >= 0 && dev < 64) configured[dev] = true;
  }
  const int ctas = std::min(sm_count(), (rows + WARPS - 1) / WARPS);
  launch(kernel, dim3(ctas), dim3(WARPS * 32), smem, s, x, g, b, eps, rows, valid, out, rs, err);
  return check_launch("rot_q8_persistent_kernel");
}

template <int NCH, int BLOCK>
int launch_rot(const __half* x, const float* g, const float* b, float eps, int rows, int valid, int8_t* out,
               float* rs, int* err, cudaStream_t s) {
  // LayerNorm rows take the persistent kernel (gamma/beta in TMEM) unless there are few of them. Rows
  // without a norm need no per-row
  // constants and run faster on the per-row grid, whose higher occupancy hides the HBM latency (measured:
  // 48 vs 64 us for 65,600 x 1024). The widest rows (4096) do not fit the persistent kernel's staging.
  if constexpr (NCH <= 11) {
    if (g != nullptr && (NCH > 4 || rows >= kPersistMinRows1024))
      return launch_persistent<NCH, BLOCK, true>(x, g, b, eps, rows, valid, out, rs, err, s);
  }
  const dim3 grid((rows + kRotWarps - 1) / kRotWarps);
  if (g != nullptr)
    launch(rot_q8_kernel<NCH, BLOCK, true>, dim3(grid), dim3(kRotWarps * 32), 0, s, x, g, b, eps, rows, valid, out, rs);
  else
    launch(rot_q8_kernel<NCH, BLOCK, false>, dim3(grid), dim3(kRotWarps * 32), 0, s, x, g, b, eps, rows, valid, out, rs);
  return check_launch("rot_q8_kernel");
}

template <int NCH>
int dispatch_block(int block, const __half* x, const float* g, const float* b, float eps, int rows, int valid,
                   int8_t* out, float* rs, int* err, cudaStream_t s) {
  switch (block) {
    case 128: return launch_rot<NCH, 128>(x, g, b, eps, rows, valid, out, rs, err, s);
    case 256: return launch_rot<NCH, 256>(x, g, b, eps, rows, valid, out, rs, err, s);
    case 512:
      if constexpr (NCH % 2 == 0) return launch_rot<NCH, 512>(x, g, b, eps, rows, valid, out, rs, err, s);
      break;
    case 1024:
      if constexpr (NCH % 4 == 0) return launch_rot<NCH, 1024>(x, g, b, eps, rows, valid, out, rs, err, s);
      break;
  }
  set_error("ff_rot_q8: block %d does not divide %d columns", block, NCH * 256);
  return FF_ERR_INVALID_ARGUMENT;
}

}  // namespace

int rot_q8(const void* x, const float* g, const float* b, float eps, int rows, int cols, int valid, int block,
           int8_t* out, float* rs, cudaStream_t s, int* err) {
  FF_REQUIRE(x && out && rs, "ff_rot_q8: NULL pointer");
  FF_REQUIRE(rows >= 0, "ff_rot_q8: rows %d", rows);
  FF_REQUIRE(valid >= 1 && valid <= cols, "ff_rot_q8: valid_cols %d not in [1, %d]", valid, cols);
  FF_REQUIRE((g == nullptr) == (b == nullptr), "ff_rot_q8: gamma and beta must both be given or both NULL");
  FF_REQUIRE(aligned16(x) && (g == nullptr || (aligned16(g) && aligned16(b))), "ff_rot_q8: pointers must be 16-byte aligned");
  FF_REQUIRE((reinterpret_cast<uintptr_t>(out) & 7u) == 0, "ff_rot_q8: out must be 8-byte aligned");
  if (rows == 0) return FF_OK;
  const bool standard = cols == 768 || cols == 1024 || cols == 2048 || cols == 2816 || cols == 4096;
  if (!standard && g == nullptr && block == 128 && valid == cols && cols % 128 == 0)
    return rot_q8_h128_wide(x, rows, cols, out, rs, s);  // e.g. PixAI's 4736-wide GELU hidden
  FF_REQUIRE(standard, "ff_rot_q8: %d columns is not one of 768, 1024, 2048, 2816, 4096 (or, for H128 without a "
             "LayerNorm, a multiple of 128)", cols);
  if (err == nullptr && g != nullptr) err = device_error_word();  // the LayerNorm kernel's bounded waits
  FF_REQUIRE(err != nullptr || g == nullptr, "ff_rot_q8: no device error word");
  const __half* xh = static_cast<const __half*>(x);
  switch (cols) {
    case 768: return dispatch_block<3>(block, xh, g, b, eps, rows, valid, out, rs, err, s);
    case 1024: return dispatch_block<4>(block, xh, g, b, eps, rows, valid, out, rs, err, s);
    case 2048: return dispatch_block<8>(block, xh, g, b, eps, rows, valid, out, rs, err, s);
    case 2816: return dispatch_block<11>(block, xh, g, b, eps, rows, valid, out, rs, err, s);
    case 4096: return dispatch_block<16>(block, xh, g, b, eps, rows, valid, out, rs, err, s);
  }
  set_error("ff_rot_q8: %d columns is not one of 768, 1024, 2048, 2816, 4096", cols);
  return FF_ERR_INVALID_ARGUMENT;
}

// H128 rotation + per-row int8 for rows of any multiple of 128 columns without a LayerNorm (the PixAI GELU
// hidden, 4736 padded to 4864 = 19 x 256, foidfinder/backends/cuda/engine.py:158-159). A row is split over
// WPR warps of the CTA, each holding CPW 256-column chunks of it in registers (4864 columns = 5 warps x 4
// chunks, the last warp 3), so it is read once and never re-read. Small CPW keeps registers low (~55) and
// so many rows in flight per SM, which the memory latency needs (measured at 82,944 x 4864: CPW 10 ->
// 2.5 TB/s, 6 -> 3.6, 4 -> 4.4). Each H128 block lies inside one chunk half (lanes 0-15 or 16-31), so the
// warps transform independently: column bits 0-2 in registers, bits 3-6 through a per-warp shared-memory
// transpose (rot_row's layout for BLOCK 128: two chunks per transpose, 8 floats of padding every 128
// columns). Only the row maximum crosses warps, through shared memory. Chunk columns at or past `cols` load
// as zero and are not stored.
template <int CPW, int WPR>
__global__ void __launch_bounds__((WPR >= 8 ? 1 : 8 / WPR) * WPR * 32)
    rot_q8_h128_split_kernel(const __half* __restrict__ x, int rows, int cols, int8_t* __restrict__ out,
                             float* __restrict__ row_scale) {
  static_assert(CPW % 2 == 0, "chunks are transposed in pairs");
  constexpr int ROWS = WPR >= 8 ? 1 : 8 / WPR;  // rows per CTA
  constexpr int QB = 128;             // columns per transposed lane group
  constexpr int SW = 512 + 8 * 4;     // floats of one warp's transpose buffer (two chunks + padding)
  __shared__ __align__(16) float tbuf[ROWS * WPR][SW];
  __shared__ float part[ROWS][WPR];
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  pdl_wait();
  pdl_trigger();
  const int rloc = wid / WPR, wpart = wid % WPR;
  const int row = blockIdx.x * ROWS + rloc;
  const bool live = row < rows;  // dead warps still reach the barrier below
  const int nch = (cols + 255) / 256;
  const int first = wpart * CPW;  // this warp's first chunk
  const __half* xr = x + static_cast<size_t>(live ? row : 0) * cols;
  float* sw = tbuf[wid];

  float2 v[CPW][4];
#pragma unroll
  for (int i = 0; i < CPW; ++i) {
    const int c = (first + i) * 256 + lane * 8;
    if (live && c < cols) {
      const uint4 u = __ldg(reinterpret_cast<const uint4*>(xr + c));
      v[i][0] = unpack_half2(u.x);
      v[i][1] = unpack_half2(u.y);
      v[i][2] = unpack_half2(u.z);
      v[i][3] = unpack_half2(u.w);
    } else {
#pragma unroll
      for (int k = 0; k < 4; ++k) v[i][k] = make_float2(0.f, 0.f);
    }
  }

  // Transposes as in rot_row: writer lane l stores the low half of its 8 columns at +4 when bit 2 of l is
  // set (the swap is in the addresses only), so a reader of element t finds column e at offset e ^ 4 when
  // bit 2 of t is set.
  const int half_sw = (lane & 4) ? 4 : 0;
  const int e = lane & 7, q = lane >> 3;
  float* const tp_a = sw + e + q * (QB + 8);        // transposed element t at tp[8 t], bit 2 of t clear
  float* const tp_b = sw + (e ^ 4) + q * (QB + 8);  // bit 2 of t set
#pragma unroll
  for (int c0 = 0; c0 < CPW; c0 += 2) {
    if (first + c0 >= nch) break;  // warp-uniform: the rest of this warp's chunks are past the row
#pragma unroll
    for (int i = c0; i < c0 + 2; ++i) {
#pragma unroll
      for (int k = 0; k < 4; ++k) v[i][k] = make_float2(v[i][k].x + v[i][k].y, v[i][k].x - v[i][k].y);
#pragma unroll
      for (int h = 1; h < 4; h <<= 1)
#pragma unroll
        for (int k = 0; k < 4; ++k)
          if (!(k & h)) {
            const float2 a = v[i][k], b = v[i][k + h];
            v[i][k] = add2(a, b);
            v[i][k + h] = sub2(a, b);
          }
    }
#pragma unroll
    for (int i = c0; i < c0 + 2; ++i) {
      const int c = (i - c0) * 256 + lane * 8;
      float* d = sw + c + 8 * (c / QB);
      *reinterpret_cast<float4*>(d + half_sw) = make_float4(v[i][0].x, v[i][0].y, v[i][1].x, v[i][1].y);
      *reinterpret_cast<float4*>(d + 4 - half_sw) = make_float4(v[i][2].x, v[i][2].y, v[i][3].x, v[i][3].y);
    }
    __syncwarp();
    float2 tv[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float* tp = ((j >> 1) & 1) ? tp_b : tp_a;  // elements 2j, 2j + 1 share bit 2 (compile-time choice)
      tv[j] = make_float2(tp[16 * j], tp[16 * j + 8]);
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) tv[j] = make_float2(tv[j].x + tv[j].y, tv[j].x - tv[j].y);
#pragma unroll
    for (int h = 1; h < 8; h <<= 1)
#pragma unroll
      for (int j = 0; j < 8; ++j)
        if (!(j & h)) {
          const float2 a = tv[j], b = tv[j + h];
          tv[j] = add2(a, b);
          tv[j + h] = sub2(a, b);
        }
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      float* tp = ((j >> 1) & 1) ? tp_b : tp_a;
      tp[16 * j] = tv[j].x;
      tp[16 * j + 8] = tv[j].y;
    }
    __syncwarp();
#pragma unroll
    for (int i = c0; i < c0 + 2; ++i) {
      const int c = (i - c0) * 256 + lane * 8;
      const float* d = sw + c + 8 * (c / QB);
      const float4 a = *reinterpret_cast<const float4*>(d + half_sw);
      const float4 b = *reinterpret_cast<const float4*>(d + 4 - half_sw);
      v[i][0] = make_float2(a.x, a.y);
      v[i][1] = make_float2(a.z, a.w);
      v[i][2] = make_float2(b.x, b.y);
      v[i][3] = make_float2(b.z, b.w);
    }
    __syncwarp();
  }

  const float2 n2 = make_float2(0.08838834764831845f, 0.08838834764831845f);  // 1 / sqrt(128)
  float amax = 0.f;
#pragma unroll
  for (int i = 0; i < CPW; ++i)
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      v[i][k] = mul2(v[i][k], n2);
      amax = max3(amax, fabsf(v[i][k].x), fabsf(v[i][k].y));
    }
  amax = warp_max(amax);
  if (lane == 0) part[rloc][wpart] = amax;
  __syncthreads();
#pragma unroll
  for (int w = 0; w < WPR; ++w) amax = fmaxf(amax, part[rloc][w]);
  if (!live) return;
  const float scale = fmaxf(amax, 1e-12f) / 127.f;
  const float inv = 1.f / scale;
  const float2 inv2 = make_float2(inv, inv), magic2 = make_float2(12582912.f, 12582912.f);
  int8_t* orow = out + static_cast<size_t>(row) * cols;
#pragma unroll
  for (int i = 0; i < CPW; ++i) {
    const int c = (first + i) * 256 + lane * 8;
    if (c >= cols) continue;
    uint32_t t[8];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float2 r = add2(mul2(v[i][k], inv2), magic2);
      t[2 * k] = __float_as_uint(r.x);
      t[2 * k + 1] = __float_as_uint(r.y);
    }
    const uint32_t w0 = __byte_perm(__byte_perm(t[0], t[1], 0x0040), __byte_perm(t[2], t[3], 0x0040), 0x5410);
    const uint32_t w1 = __byte_perm(__byte_perm(t[4], t[5], 0x0040), __byte_perm(t[6], t[7], 0x0040), 0x5410);
    *reinterpret_cast<uint2*>(orow + c) = make_uint2(w0, w1);
  }
  if (lane == 0 && wpart == 0) row_scale[row] = scale;
}

#ifndef FF_ROTW_CPW
#define FF_ROTW_CPW 4
#endif
constexpr int kSplitCpw = FF_ROTW_CPW;  // 256-column chunks per warp
constexpr int kSplitMaxWarps = 8;       // warps per row: rows up to 8 x kSplitCpw x 256 columns

template <int WPR>
int launch_split(const __half* x, int rows, int cols, int8_t* out, float* rs, cudaStream_t s) {
  constexpr int ROWS = WPR >= 8 ? 1 : 8 / WPR;
  launch(rot_q8_h128_split_kernel<kSplitCpw, WPR>, dim3((rows + ROWS - 1) / ROWS), dim3(ROWS * WPR * 32), 0, s, x, rows, cols, out, rs);
  return check_launch("rot_q8_h128_split_kernel");
}

int rot_q8_h128_wide(const void* x, int rows, int cols, int8_t* out, float* rs, cudaStream_t s) {
  FF_REQUIRE(x && out && rs, "rot_q8 (wide): NULL pointer");
  FF_REQUIRE(cols >= 128 && cols % 128 == 0, "rot_q8 (wide): %d columns is not a multiple of 128", cols);
  const int wpr = ((cols + 255) / 256 + kSplitCpw - 1) / kSplitCpw;
  FF_REQUIRE(wpr <= kSplitMaxWarps, "rot_q8 (wide): %d columns (at most %d)", cols, kSplitMaxWarps * kSplitCpw * 256);
  FF_REQUIRE(aligned16(x) && (reinterpret_cast<uintptr_t>(out) & 7u) == 0, "rot_q8 (wide): alignment");
  if (rows == 0) return FF_OK;
  const __half* xh = static_cast<const __half*>(x);
  switch (wpr) {
    case 1: return launch_split<1>(xh, rows, cols, out, rs, s);
    case 2: return launch_split<2>(xh, rows, cols, out, rs, s);
    case 3: return launch_split<3>(xh, rows, cols, out, rs, s);
    case 4: return launch_split<4>(xh, rows, cols, out, rs, s);
    case 5: return launch_split<5>(xh, rows, cols, out, rs, s);
    case 6: return launch_split<6>(xh, rows, cols, out, rs, s);
    case 7: return launch_split<7>(xh, rows, cols, out, rs, s);
    default: return launch_split<8>(xh, rows, cols, out, rs, s);
  }
}

}  // namespace ff

extern "C" int ff_rot_q8(const uint16_t* x, const float* gamma, const float* beta, float eps, int rows, int cols,
                         int valid_cols, int block, int8_t* out, float* row_scale, void* stream) {
  return ff::rot_q8(x, gamma, beta, eps, rows, cols, valid_cols, block, out, row_scale,
                    static_cast<cudaStream_t>(stream));
}

extern "C" int ff_rot_q8_1024(const uint16_t* x, const float* gamma, const float* beta, int rows, int8_t* out,
                              float* row_scale, void* stream) {
  return ff::rot_q8(x, gamma, beta, 1e-5f, rows, 1024, 1024, 1024, out, row_scale, static_cast<cudaStream_t>(stream));
}

extern "C" int ff_rot_q8_h128(const uint16_t* x, int rows, int cols, int8_t* out, float* row_scale, void* stream) {
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (cols == 768 || cols == 1024 || cols == 2048 || cols == 2816 || cols == 4096)
    return ff::rot_q8(x, nullptr, nullptr, 0.f, rows, cols, cols, 128, out, row_scale, s);
  return ff::rot_q8_h128_wide(x, rows, cols, out, row_scale, s);  // e.g. PixAI's 4736
}
