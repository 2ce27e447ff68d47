// Internal launchers shared between the per-op C ABI and the engine.
#pragma once
#include <cuda_runtime.h>
#include <cstdint>

namespace ff {

// err: device error word for bounded waits (nullptr: the library's per-device word).
int rot_q8(const void* x, const float* g, const float* b, float eps, int rows, int cols, int valid, int block,
           int8_t* out, float* rs, cudaStream_t s, int* err = nullptr);
int attention(const void* qkv, void* out, int num_seqs, int seq_len, int heads, const float* rope_cos,
              const float* rope_sin, float scale, cudaStream_t s);
int attention_tc(const void* qkv, void* out, int num_seqs, int seq_len, int heads, float scale, cudaStream_t s);
// Query rows (and keys) past the last full 128-row tile that attention_tc computes on the CUDA cores inside
// its one launch (1..4 of them, e.g. EVA02's 1025th token), or 0 when the last tiles are ragged instead.
int attention_tc_tail_rows(int seq_len);
int topk(const float* logits, int B, int n, int k, int32_t* idx, float* val, cudaStream_t s);
// img: uint8 pixels (normalised with mean/std) or, with f16_pixels, already normalised fp16 pixels.
int patchify(const void* img, int B, int S, int p, const float* mean, const float* stdv, void* out, int k_pad,
             cudaStream_t s, int win = 0, bool f16_pixels = false);
int fill_cls(const void* cls, void* x, int B, int tokens, int dim, cudaStream_t s);
int layernorm(const void* x, int64_t stride, const float* g, const float* b, float eps, int rows, int cols, void* out,
              cudaStream_t s, const void* pos = nullptr, int period = 0);
// H128 rotation + int8 of rows of any width that is a multiple of 128 (no LayerNorm): two passes per row.
int rot_q8_h128_wide(const void* x, int rows, int cols, int8_t* out, float* rs, cudaStream_t s);
// Attention of one learned query per head over all tokens: q [heads * 64] f32 (scale folded in),
// kv [B * tokens, 2 * dim] fp16 (keys | values) -> out [B, dim] fp16.
int pool_query_attention(const float* q, const void* kv, int B, int tokens, int heads, void* out, cudaStream_t s);
int slot_attend(const float* q, int64_t q_img_stride, const float* bias, int M, const void* kv, int B, int tokens,
                int dim, int heads, float* z, float* mass_part, cudaStream_t s);
int pool_trunk(const float* z, int B, int coarse, int leaves, int dim, const float* trunk_w, const float* trunk_b,
               const float* q_child, const float* child_w, const float* child_b, float eps, float* z_coarse,
               float* q_leaf, cudaStream_t s);
int pool_leaf(const float* z_coarse, const float* z_child, const float* mass_part, int B, int coarse, int leaves,
              int heads, int dim, int leaf_dim, const float* leaf_nw, const float* leaf_nb, float eps,
              const float* leaf_w, const float* leaf_b, void* out, int ld_out, cudaStream_t s);

}  // namespace ff
