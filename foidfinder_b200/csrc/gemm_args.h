// Arguments of the tcgen05 GEMM kernel (plain data, passed by value as a kernel parameter).
#pragma once
#include <cstdint>

namespace ff {

// Epilogues. The first three keep the numbering of the reference's Epi enum
// (foidfinder/backends/cuda/csrc/gemm.cuh:8-12) so callers that pass the integer keep working.
enum Epi : int {
  EPI_QKV_ROPE = 0,  // s8: fp16 out; 2-D RoPE on the q and k column ranges (columns < rope_cols)
  EPI_RESIDUAL = 1,  // s8: fp16 out[m, n] = fp16(float(out[m, n]) + y)
  EPI_GELU_F16 = 2,  // s8: fp16 out = gelu_tanh(y)   (PixAI-1008 fc1)
  EPI_SWIGLU = 3,    // s8: W rows are [gate 64 | up 64] pairs; fp16 out[m, n/2] = silu(gate) * up
  EPI_BIAS = 4,      // s8: fp16 out = y
  EPI_S32 = 5,       // s8: raw int32 accumulators (bit-exactness checks)
  EPI_STEM = 6,      // f16: fp16 x[image token row] = acc + pos_bias[patch, n]
  EPI_LOGITS = 7,    // f16: f32 out[m, n] = acc + bias[n] for n < n_valid
};

struct GemmArgs {
  int M, N, K;          // A [M, K], W [N, K]; K counts elements
  int num_kb;           // K bytes / 128
  int tiles_m;          // ceil(M / 128)
  const float* row_scale;  // [M]  per-token activation scale (s8)
  const float* col_scale;  // [N]  per-output-channel weight scale (s8)
  const float* bias;       // [N]
  void* out;
  int ldo;              // output row stride (elements)
  int n_valid;          // EPI_LOGITS: columns written
  const float* rope_cos;   // EPI_QKV_ROPE: angle-major [32, tokens]
  const float* rope_sin;
  int rope_cols;        // EPI_QKV_ROPE: columns [0, rope_cols) are rotated (q and k)
  // Separable RoPE (rope_grid > 0): the angle of pair i at position p depends on one grid coordinate of p,
  // so the tables shrink to [32, rope_grid] (a few KB, resident in L1). idx = p - rope_cls (negative: the
  // class token, identity); (r, c) = (idx / grid, idx % grid); pairs 0..15 take coordinate r and 16..31
  // coordinate c, or the other way round with rope_swap. The engine builds these from the full tables
  // only after checking that every full-table entry equals its compact one bit for bit.
  int rope_grid, rope_cls, rope_swap;
  const float* rope_cos_c;  // [32, rope_grid + 1]: column rope_grid is the identity (class token)
  const float* rope_sin_c;
  int tokens;           // tokens per image (RoPE position = m % tokens; stem row remap)
  const float* pos_bias;   // EPI_STEM: [patches, N] = patch bias + position embedding
  int patches;          // EPI_STEM: patches per image
  int* err;             // device error word
  int w_const;          // 1: no kernel writes W while a forward runs (the engine's weights), so the producer may
                        // load W tiles before the wait for the previous kernel (programmatic dependent launch)
};

}  // namespace ff
