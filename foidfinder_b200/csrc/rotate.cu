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
#include "common.h"
#include "ptx.cuh"

namespace ff {

constexpr int kRotWarps = 4;  // small CTAs: the 2816-column rows need ~134 registers per thread

template <int NCH, int BLOCK, bool NORM>
__global__ void __launch_bounds__(kRotWarps * 32)
    rot_q8_kernel(const __half* __restrict__ x, const float* __restrict__ gamma, const float* __restrict__ beta,
                  float eps, int rows, int valid_cols, int8_t* __restrict__ out, float* __restrict__ row_scale) {
  constexpr int LB = BLOCK == 128 ? 7 : BLOCK == 256 ? 8 : BLOCK == 512 ? 9 : 10;
  constexpr int TB = LB - 3 < 5 ? LB - 3 : 5;  // column bits 3..3+TB-1 run in the transposed layout
  constexpr int G = 1 << TB;                   // values per lane in the transposed layout
  constexpr int UNIT = G / 8;                  // 256-column chunks per transpose
  constexpr int NCHP = (NCH + UNIT - 1) / UNIT * UNIT;
  constexpr int COLS = NCH * 256;
  constexpr int QB = 8 * G;  // columns per transposed lane group (padding period)
  constexpr int SW = UNIT * 256 + 8 * (UNIT * 256 / QB);
  static_assert((1 << LB) == BLOCK && BLOCK / 256 <= UNIT, "unsupported Hadamard block");
  __shared__ __align__(16) float smem[kRotWarps][SW];

  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  const int row = blockIdx.x * kRotWarps + wid;
  if (row >= rows) return;
  float* sw = smem[wid];
  const __half* xr = x + static_cast<size_t>(row) * COLS;

  float2 v[NCHP][4];
#pragma unroll
  for (int i = 0; i < NCHP; ++i) {
    if (i < NCH) {
      const uint4 u = __ldg(reinterpret_cast<const uint4*>(xr + i * 256 + lane * 8));
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
    float2 s2 = make_float2(0.f, 0.f);
#pragma unroll
    for (int i = 0; i < NCH; ++i)
#pragma unroll
      for (int k = 0; k < 4; ++k) s2 = add2(s2, v[i][k]);
    const float inv_n = 1.f / static_cast<float>(valid_cols);
    const float mean = warp_sum(s2.x + s2.y) * inv_n;
    const float2 m2 = make_float2(mean, mean);
    float2 q2 = make_float2(0.f, 0.f);
#pragma unroll
    for (int i = 0; i < NCH; ++i)
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        v[i][k] = sub2(v[i][k], m2);
        q2 = fma2(v[i][k], v[i][k], q2);
      }
    const float q = warp_sum(q2.x + q2.y) - static_cast<float>(COLS - valid_cols) * mean * mean;
    rstd = rsqrtf(fmaxf(q, 0.f) * inv_n + eps);
  }

#pragma unroll
  for (int c0 = 0; c0 < NCHP; c0 += UNIT) {
    if constexpr (NORM) {
      const float2 r2 = make_float2(rstd, rstd);
#pragma unroll
      for (int i = c0; i < c0 + UNIT; ++i) {
        if (i < NCH) {
          const int c = i * 256 + lane * 8;
          const float4 g0 = __ldg(reinterpret_cast<const float4*>(gamma + c));
          const float4 g1 = __ldg(reinterpret_cast<const float4*>(gamma + c + 4));
          const float4 b0 = __ldg(reinterpret_cast<const float4*>(beta + c));
          const float4 b1 = __ldg(reinterpret_cast<const float4*>(beta + c + 4));
          v[i][0] = fma2(v[i][0], mul2(r2, make_float2(g0.x, g0.y)), make_float2(b0.x, b0.y));
          v[i][1] = fma2(v[i][1], mul2(r2, make_float2(g0.z, g0.w)), make_float2(b0.z, b0.w));
          v[i][2] = fma2(v[i][2], mul2(r2, make_float2(g1.x, g1.y)), make_float2(b1.x, b1.y));
          v[i][3] = fma2(v[i][3], mul2(r2, make_float2(g1.z, g1.w)), make_float2(b1.z, b1.w));
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

    // Transpose through shared memory: column c of the group sits at c + 8 * (c / QB). Lanes with bit 2
    // set move their two 16-byte halves in the opposite order, so each quarter-warp phase of a 16-byte
    // access covers all 32 banks once.
    const bool swap_halves = lane & 4;
#pragma unroll
    for (int i = c0; i < c0 + UNIT; ++i) {
      const int c = (i - c0) * 256 + lane * 8;
      float* d = sw + c + 8 * (c / QB);
      const float4 lo = make_float4(v[i][0].x, v[i][0].y, v[i][1].x, v[i][1].y);
      const float4 hi = make_float4(v[i][2].x, v[i][2].y, v[i][3].x, v[i][3].y);
      *reinterpret_cast<float4*>(d + (swap_halves ? 4 : 0)) = swap_halves ? hi : lo;
      *reinterpret_cast<float4*>(d + (swap_halves ? 0 : 4)) = swap_halves ? lo : hi;
    }
    __syncwarp();
    const int e = lane & 7, q = lane >> 3;
    float* tp = sw + e + q * (QB + 8);  // transposed element t at tp[8 t]
    float2 tv[G / 2];
#pragma unroll
    for (int j = 0; j < G / 2; ++j) tv[j] = make_float2(tp[16 * j], tp[16 * j + 8]);
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
      tp[16 * j] = tv[j].x;
      tp[16 * j + 8] = tv[j].y;
    }
    __syncwarp();
#pragma unroll
    for (int i = c0; i < c0 + UNIT; ++i) {
      const int c = (i - c0) * 256 + lane * 8;
      const float* d = sw + c + 8 * (c / QB);
      const float4 first = *reinterpret_cast<const float4*>(d + (swap_halves ? 4 : 0));
      const float4 second = *reinterpret_cast<const float4*>(d + (swap_halves ? 0 : 4));
      const float4 a = swap_halves ? second : first;
      const float4 b = swap_halves ? first : second;
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
  const float2 n2 = make_float2(kNorm, kNorm);
  float amax = 0.f;
#pragma unroll
  for (int i = 0; i < NCH; ++i)
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      v[i][k] = mul2(v[i][k], n2);
      amax = max3(amax, fabsf(v[i][k].x), fabsf(v[i][k].y));
    }
  amax = warp_max(amax);
  const float scale = fmaxf(amax, 1e-12f) / 127.f;
  const float inv = 1.f / scale;
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

namespace {

template <int NCH, int BLOCK>
int launch_rot(const __half* x, const float* g, const float* b, float eps, int rows, int valid, int8_t* out,
               float* rs, cudaStream_t s) {
  const dim3 grid((rows + kRotWarps - 1) / kRotWarps);
  if (g != nullptr)
    rot_q8_kernel<NCH, BLOCK, true><<<grid, kRotWarps * 32, 0, s>>>(x, g, b, eps, rows, valid, out, rs);
  else
    rot_q8_kernel<NCH, BLOCK, false><<<grid, kRotWarps * 32, 0, s>>>(x, g, b, eps, rows, valid, out, rs);
  return check_launch("rot_q8_kernel");
}

template <int NCH>
int dispatch_block(int block, const __half* x, const float* g, const float* b, float eps, int rows, int valid,
                   int8_t* out, float* rs, cudaStream_t s) {
  switch (block) {
    case 128: return launch_rot<NCH, 128>(x, g, b, eps, rows, valid, out, rs, s);
    case 256: return launch_rot<NCH, 256>(x, g, b, eps, rows, valid, out, rs, s);
    case 512:
      if constexpr (NCH % 2 == 0) return launch_rot<NCH, 512>(x, g, b, eps, rows, valid, out, rs, s);
      break;
    case 1024:
      if constexpr (NCH % 4 == 0) return launch_rot<NCH, 1024>(x, g, b, eps, rows, valid, out, rs, s);
      break;
  }
  set_error("ff_rot_q8: block %d does not divide %d columns", block, NCH * 256);
  return FF_ERR_INVALID_ARGUMENT;
}

}  // namespace

int rot_q8(const void* x, const float* g, const float* b, float eps, int rows, int cols, int valid, int block,
           int8_t* out, float* rs, cudaStream_t s) {
  FF_REQUIRE(x && out && rs, "ff_rot_q8: NULL pointer");
  FF_REQUIRE(rows >= 0, "ff_rot_q8: rows %d", rows);
  FF_REQUIRE(valid >= 1 && valid <= cols, "ff_rot_q8: valid_cols %d not in [1, %d]", valid, cols);
  FF_REQUIRE((g == nullptr) == (b == nullptr), "ff_rot_q8: gamma and beta must both be given or both NULL");
  FF_REQUIRE(aligned16(x) && (g == nullptr || (aligned16(g) && aligned16(b))), "ff_rot_q8: pointers must be 16-byte aligned");
  FF_REQUIRE((reinterpret_cast<uintptr_t>(out) & 7u) == 0, "ff_rot_q8: out must be 8-byte aligned");
  if (rows == 0) return FF_OK;
  const __half* xh = static_cast<const __half*>(x);
  switch (cols) {
    case 768: return dispatch_block<3>(block, xh, g, b, eps, rows, valid, out, rs, s);
    case 1024: return dispatch_block<4>(block, xh, g, b, eps, rows, valid, out, rs, s);
    case 2048: return dispatch_block<8>(block, xh, g, b, eps, rows, valid, out, rs, s);
    case 2816: return dispatch_block<11>(block, xh, g, b, eps, rows, valid, out, rs, s);
    case 4096: return dispatch_block<16>(block, xh, g, b, eps, rows, valid, out, rs, s);
  }
  set_error("ff_rot_q8: %d columns is not one of 768, 1024, 2048, 2816, 4096", cols);
  return FF_ERR_INVALID_ARGUMENT;
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
  return ff::rot_q8(x, nullptr, nullptr, 0.f, rows, cols, cols, 128, out, row_scale, static_cast<cudaStream_t>(stream));
}
