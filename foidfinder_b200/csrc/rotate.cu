// Per-token activation quantisation for the W8A8 GEMMs, with the LayerNorm in front of it fused in:
//   x fp16 -> [LayerNorm over the valid columns, f32 statistics] -> block-diagonal Sylvester Hadamard
//   (normalised) -> per-row scale s = max(amax, 1e-12) / 127 -> codes clamp(rint(v / s), +-127).
// Follows rot_q8_1024 (foidfinder/backends/cuda/csrc/kernels.cu:49-108) and rot_q8_h128
// (kernels.cu:112-160); quantiser semantics from common.cuh:45-48; the EVA02 LayerNorm eps and the
// SwiGLU hidden norm from foidfinder/backends/mlx/haruka.py:19,97-98.
//
// One warp per row, 8 rows per 256-thread CTA. Lane l owns 8 consecutive columns of every 256-column
// chunk i (columns i*256 + l*8 + e), loaded as 16-byte vectors, so a row costs one coalesced read of
// 2 B/column and one write of 1 B/column plus the 4-byte scale: the kernel is HBM-bound. The
// Hadamard butterflies over column bits 0-2 run in registers, bits 3-7 across lanes (shuffles), bits 8+
// across the lane's chunks (registers).
#include "common.h"
#include "ptx.cuh"

namespace ff {

template <int NCH, int BLOCK, bool NORM>
__global__ void __launch_bounds__(256) rot_q8_kernel(const __half* __restrict__ x, const float* __restrict__ gamma,
                                                     const float* __restrict__ beta, float eps, int rows,
                                                     int valid_cols, int8_t* __restrict__ out,
                                                     float* __restrict__ row_scale) {
  constexpr int COLS = NCH * 256;
  const int lane = threadIdx.x & 31;
  const int row = blockIdx.x * 8 + (threadIdx.x >> 5);
  if (row >= rows) return;
  const __half* xr = x + static_cast<size_t>(row) * COLS;
  float v[NCH][8];
#pragma unroll
  for (int i = 0; i < NCH; ++i) {
    const uint4 u = __ldg(reinterpret_cast<const uint4*>(xr + i * 256 + lane * 8));
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 f = unpack_half2(w[e]);
      v[i][2 * e] = f.x;
      v[i][2 * e + 1] = f.y;
    }
  }
  if constexpr (NORM) {
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < NCH; ++i)
#pragma unroll
      for (int e = 0; e < 8; ++e)
        if (i * 256 + lane * 8 + e < valid_cols) s += v[i][e];
    const float inv_n = 1.f / static_cast<float>(valid_cols);
    const float mean = warp_sum(s) * inv_n;
    float q = 0.f;
#pragma unroll
    for (int i = 0; i < NCH; ++i)
#pragma unroll
      for (int e = 0; e < 8; ++e)
        if (i * 256 + lane * 8 + e < valid_cols) {
          const float d = v[i][e] - mean;
          q += d * d;
        }
    const float rstd = rsqrtf(warp_sum(q) * inv_n + eps);
#pragma unroll
    for (int i = 0; i < NCH; ++i) {
      const int c = i * 256 + lane * 8;
      const float4 g0 = __ldg(reinterpret_cast<const float4*>(gamma + c));
      const float4 g1 = __ldg(reinterpret_cast<const float4*>(gamma + c + 4));
      const float4 b0 = __ldg(reinterpret_cast<const float4*>(beta + c));
      const float4 b1 = __ldg(reinterpret_cast<const float4*>(beta + c + 4));
      const float g[8] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z, g1.w};
      const float b[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
      for (int e = 0; e < 8; ++e) v[i][e] = c + e < valid_cols ? (v[i][e] - mean) * rstd * g[e] + b[e] : 0.f;
    }
  } else {
#pragma unroll
    for (int i = 0; i < NCH; ++i)
#pragma unroll
      for (int e = 0; e < 8; ++e)
        if (i * 256 + lane * 8 + e >= valid_cols) v[i][e] = 0.f;
  }

  // Column bits 0-2: inside the lane's 8-element group.
#pragma unroll
  for (int h = 1; h < 8; h <<= 1)
#pragma unroll
    for (int i = 0; i < NCH; ++i)
#pragma unroll
      for (int e = 0; e < 8; ++e)
        if (!(e & h)) {
          const float a = v[i][e], b = v[i][e + h];
          v[i][e] = a + b;
          v[i][e + h] = a - b;
        }
  // Column bits 3..min(7, log2(BLOCK)-1): across lanes.
#pragma unroll
  for (int m = 1; m < 32 && m * 8 < BLOCK; m <<= 1) {
    const bool upper = lane & m;
#pragma unroll
    for (int i = 0; i < NCH; ++i)
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const float o = __shfl_xor_sync(0xffffffffu, v[i][e], m);
        v[i][e] = upper ? o - v[i][e] : v[i][e] + o;
      }
  }
  // Column bits 8..log2(BLOCK)-1: across the lane's chunks.
#pragma unroll
  for (int h = 1; h * 256 < BLOCK; h <<= 1)
#pragma unroll
    for (int i = 0; i < NCH; ++i)
      if (!(i & h))
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const float a = v[i][e], b = v[i + h][e];
          v[i][e] = a + b;
          v[i + h][e] = a - b;
        }
  constexpr float kNorm = BLOCK == 128   ? 0.08838834764831845f
                          : BLOCK == 256 ? 0.0625f
                          : BLOCK == 512 ? 0.04419417382415922f
                                         : 0.03125f;  // 1 / sqrt(BLOCK)
  float amax = 0.f;
#pragma unroll
  for (int i = 0; i < NCH; ++i)
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      v[i][e] *= kNorm;
      amax = fmaxf(amax, fabsf(v[i][e]));
    }
  amax = warp_max(amax);
  const float scale = fmaxf(amax, 1e-12f) / 127.f;
  const float inv = 1.f / scale;
  int8_t* orow = out + static_cast<size_t>(row) * COLS;
#pragma unroll
  for (int i = 0; i < NCH; ++i) {
    // rint(v * inv) (round half to even, as __float2int_rn) without the XU conversion: adding 1.5 * 2^23
    // to the f32 product leaves the rounded integer in the low mantissa bits, whose low byte is the
    // two's-complement int8 code. |v * inv| <= 127 by construction of the scale, so no clamp is needed.
    uint32_t t[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) t[e] = __float_as_uint(__fadd_rn(__fmul_rn(v[i][e], inv), 12582912.f));
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
  const dim3 grid((rows + 7) / 8);
  if (g != nullptr)
    rot_q8_kernel<NCH, BLOCK, true><<<grid, 256, 0, s>>>(x, g, b, eps, rows, valid, out, rs);
  else
    rot_q8_kernel<NCH, BLOCK, false><<<grid, 256, 0, s>>>(x, g, b, eps, rows, valid, out, rs);
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
