// Orchestration of the Haruka tree attention pool head (kernels in pool.cu), shared by the engine and the
// ff_tree_pool entry point.
#pragma once
#include <cuda_fp16.h>

#include "foidfinder_b200.h"
#include "gemm.h"

namespace ff {

struct PoolBuffers {
  __half* xf = nullptr;  // [B*tokens, dim] final-normed tokens
  __half* xn = nullptr;  // [B*tokens, dim] pool-normed tokens
  __half* kv = nullptr;  // [B*tokens, 2*dim] keys | values
  float* z = nullptr;        // [B, leaves, dim] slot outputs (coarse pass uses the first coarse rows of each image)
  float* z_coarse = nullptr; // [B, coarse, dim]
  float* q_leaf = nullptr;   // [B, leaves, dim]
  float* z_child = nullptr;  // [B, leaves, dim]
  float* mass_c = nullptr;   // [B, pool_heads, coarse]
  float* mass_l = nullptr;   // [B, pool_heads, leaves]
};

// Bytes of the small f32 buffers (z .. mass_l) for B images.
size_t pool_small_bytes(const ff_model_config& c, int B);
// Carves the small f32 buffers out of `base` (pool_small_bytes bytes, 256-byte aligned).
void pool_carve_small(const ff_model_config& c, int B, void* base, PoolBuffers* pb);
int pool_validate(const ff_model_config& c, const ff_model_weights& w);
// Plans the key/value GEMM xn -> kv for B images of `tokens` tokens.
int pool_prepare(const ff_model_config& c, const ff_model_weights& w, int B, int tokens, const PoolBuffers& pb,
                 GemmPlan* kv_plan);
// x [B*tokens, dim] fp16 (backbone output before its final LayerNorm) -> leaf features
// leaf_out [B, leaves * leaf_dim] fp16. 7 launches.
int pool_run(const ff_model_config& c, const ff_model_weights& w, const __half* x, int B, int tokens,
             const PoolBuffers& pb, const GemmPlan& kv_plan, __half* leaf_out, cudaStream_t s);
constexpr int kPoolLaunches = 7;

}  // namespace ff
