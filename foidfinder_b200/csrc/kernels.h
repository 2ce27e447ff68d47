// Internal launchers shared between the per-op C ABI and the engine.
#pragma once
#include <cuda_runtime.h>
#include <cstdint>

namespace ff {

int rot_q8(const void* x, const float* g, const float* b, float eps, int rows, int cols, int valid, int block,
           int8_t* out, float* rs, cudaStream_t s);
int attention(const void* qkv, void* out, int num_seqs, int seq_len, int heads, const float* rope_cos,
              const float* rope_sin, float scale, cudaStream_t s);
int attention_tc(const void* qkv, void* out, int num_seqs, int seq_len, int heads, float scale, cudaStream_t s);
int topk(const float* logits, int B, int n, int k, int32_t* idx, float* val, cudaStream_t s);
int patchify(const uint8_t* img, int B, int S, int p, const float* mean, const float* stdv, void* out, int k_pad,
             cudaStream_t s);
int fill_cls(const void* cls, void* x, int B, int tokens, int dim, cudaStream_t s);
int layernorm(const void* x, int64_t stride, const float* g, const float* b, float eps, int rows, int cols, void* out,
              cudaStream_t s);

}  // namespace ff
