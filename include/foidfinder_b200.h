/*
 * foidfinder_b200 — C ABI of the sm_100a int8 tagger forward.
 *
 * Every entry point takes plain device pointers, sizes and a cudaStream_t passed as void*, returns an
 * int status (FF_OK = 0) and never allocates caller-visible memory. On failure ff_last_error()
 * returns a message for the calling thread. Kernels launch asynchronously on the given stream; a
 * kernel whose bounded device-side wait ran out records a code in the per-device error word, which
 * ff_device_error() returns after synchronising.
 *
 * Pointers named fp16 are IEEE binary16 arrays (uint16_t storage). All matrices are row-major and
 * contiguous. Base pointers of TMA-fed operands (GEMM A and W) must be 16-byte aligned.
 */
#ifndef FOIDFINDER_B200_H
#define FOIDFINDER_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#pragma GCC visibility push(default)
#endif

/* ---------------------------------------------------------------- status codes */
#define FF_OK 0
#define FF_ERR_INVALID_ARGUMENT 1   /* shape, alignment or pointer check failed on the host */
#define FF_ERR_UNSUPPORTED_DEVICE 2 /* not an sm_100 device */
#define FF_ERR_LAUNCH 3             /* a kernel launch or CUDA runtime call failed */
#define FF_ERR_DEVICE_TIMEOUT 4     /* a bounded device wait ran out (see ff_device_error) */
#define FF_ERR_OUT_OF_MEMORY 5

/* Message describing the last failure on this thread ("" if none). */
const char* ff_last_error(void);

/* Library version, major * 10000 + minor * 100 + patch. */
int ff_version(void);

/* Reads (and, if clear != 0, resets) the error word of `device`; synchronises that device first.
 * *code = 0 when no kernel reported a failure. */
int ff_device_error(int device, int* code, int clear);

/* Measured dense int8 tensor-core peak of the current device (no reference counterpart): one CTA per SM
 * issues `iters` x 4 back-to-back tcgen05 kind::i8 MMAs (M128 N256 K32) on resident shared-memory operands,
 * timed with CUDA events on `stream` (synchronises it). ms: elapsed time; ops: 2 x multiply-adds done. */
int ff_int8_mma_peak(int iters, float* ms, double* ops, void* stream);

/* ---------------------------------------------------------------- GEMM epilogues */
#define FF_EPI_QKV_ROPE 0 /* fp16 out [M, N]; 2-D RoPE on columns [0, rope_cols) */
#define FF_EPI_RESIDUAL 1 /* fp16 out [M, N] = fp16(out + fp16(y)) (the residual stream) */
#define FF_EPI_SWIGLU 3   /* W rows interleaved [gate 64 | up 64]; fp16 out [M, N/2] = silu(gate) * up */
#define FF_EPI_GELU 2     /* fp16 out [M, N] = gelu_tanh(y) (PixAI fc1, csrc/common.cuh:50-56) */
#define FF_EPI_BIAS 4     /* fp16 out [M, N] = y */
#define FF_EPI_S32 5      /* int32 out [M, N] = raw accumulators */

/*
 * W8A8 GEMM on tcgen05: y[m, n] = int32(sum_k A[m, k] * W[n, k]) * row_scale[m] * col_scale[n] + bias[n],
 * then the epilogue `epi`.
 *   A [M, K] int8 (per-token codes), W [N, K] int8 (per-channel codes), K % 128 == 0, N % 128 == 0.
 *   rope_cos / rope_sin [32, tokens] f32 (angle-major) are read only by FF_EPI_QKV_ROPE: row m uses
 *   position m % tokens, and pair (2i, 2i+1) of every 64-wide head uses angle row (i % 32).
 *   tile_n: 0 = automatic, else 128 or 256 output columns per CTA tile (128 rows), or FF_TILE_PAIR256:
 *           256 x 256 tiles over a cluster of two CTAs on two SMs (tcgen05 cta_group::2; int8 operands,
 *           N % 256 == 0). Automatic picks the pair tiles for K >= 2048 when there are at least two
 *           256 x 256 tiles per SM.
 * Replaces torch.ops.foidfinder.gemm_s8 (foidfinder/backends/cuda/csrc/kernels.cu:187-217, schema
 * kernels.cu:267-271); the reference's `stages` knob becomes `tile_n`, and its q_scale is folded into
 * the q rows of W and bias at conversion time.
 */
#define FF_TILE_PAIR256 512
int ff_gemm_s8(const int8_t* A, const int8_t* W, const float* row_scale, const float* col_scale, const float* bias,
               void* out, int M, int N, int K, int epi, const float* rope_cos, const float* rope_sin, int rope_cols,
               int tokens, int tile_n, void* stream);

/*
 * fp16 GEMM on tcgen05 with f32 accumulation, for the stem and the tag head.
 *   FF_EPI_STEM:   A = patches [M = images * patches, K] fp16, W [N = dim, K] fp16;
 *                  x[(m / patches) * tokens + (tokens - patches) + m % patches, n] = fp16(acc + pos_bias[m % patches, n]);
 *                  tokens = patches + 1 leaves row 0 of each image to the class token, tokens = patches (PixAI)
 *                  does not.
 *   FF_EPI_LOGITS: A [M, K] fp16, W [N, K] fp16; out[m, n] = acc + bias[n] (f32) for n < n_valid,
 *                  out row stride ldo.
 *   FF_EPI_BIAS:   A [M, K] fp16, W [N, K] fp16; out[m, n] = fp16(acc + bias[n]), out row stride ldo
 *                  (the Haruka pool's key/value projection, foidfinder/backends/mlx/haruka.py:124).
 * Replaces the cuBLAS matmuls of engine.py:146 (patch embedding) and reference.py:140 (head linear).
 */
#define FF_EPI_STEM 6
#define FF_EPI_LOGITS 7
int ff_gemm_f16(const uint16_t* A, const uint16_t* W, const float* bias, void* out, int M, int N, int K, int epi,
                int ldo, int n_valid, const float* pos_bias, int patches, int tokens, int tile_n, void* stream);

/* ---------------------------------------------------------------- rotation + int8 quantisation */
/*
 * x [rows, cols] fp16 -> (LayerNorm over columns [0, valid_cols) with gamma/beta/eps when gamma != NULL;
 * columns >= valid_cols become 0) -> block-diagonal normalised Sylvester Hadamard of size `block`
 * -> per-row scale s = max(amax, 1e-12) / 127 -> codes clamp(rint(v / s), -127, 127).
 * Supported (cols, block): cols % 256 == 0 and block in {128, 256, 512, 1024} dividing cols, cols <= 4096.
 * Replaces rot_q8_1024 (kernels.cu:49-108, :220-235) and rot_q8_h128 (kernels.cu:112-160, :238-251).
 */
int ff_rot_q8(const uint16_t* x, const float* gamma, const float* beta, float eps, int rows, int cols,
              int valid_cols, int block, int8_t* out, float* row_scale, void* stream);

/* The reference's two entry points, same argument meaning (LayerNorm eps 1e-5 as in kernels.cu:91). */
int ff_rot_q8_1024(const uint16_t* x, const float* gamma, const float* beta, int rows, int8_t* out, float* row_scale,
                   void* stream);
int ff_rot_q8_h128(const uint16_t* x, int rows, int cols, int8_t* out, float* row_scale, void* stream);

/*
 * Activation quantisation + W8A8 GEMM in one call that allocates no device memory, for callers that may
 * not call cudaMalloc once running (a host that gives all GPU memory to its own pool at start-up, a
 * serving loop where allocation and the synchronisation of cudaFree are not allowed, a plugin that only
 * receives buffers). This entry point has no counterpart in the reference.
 *   Computes what ff_rot_q8(x, gamma, beta, eps, rows, cols, valid_cols, block, codes, scales) followed by
 *   ff_gemm_s8(codes, W, scales, col_scale, bias, out, rows, N, cols, epi, ...) computes, epi one of
 *   FF_EPI_BIAS, FF_EPI_RESIDUAL, FF_EPI_SWIGLU, but the codes and row scales live in a static device
 *   array built into the library (held by every GPU that loads it until the process exits).
 *   Limits: rows <= 8192 and rows * cols <= 8 MiB; larger calls fail with FF_ERR_INVALID_ARGUMENT.
 *   err: required device int (from the caller's pool) where a bounded-wait timeout is recorded as a
 *   non-zero code; the caller clears it. NULL fails with FF_ERR_INVALID_ARGUMENT.
 *   The array is part of the library's CUDA module, which the default lazy module loading brings onto a
 *   device only at the first call there (that call resolves the array's address). Make one call per
 *   device at start-up, before the host reserves the remaining GPU memory for its pool (or set
 *   CUDA_MODULE_LOADING=EAGER), and before any stream capture. All calls share the array and it keeps
 *   the last call's contents: calls that overlap on the GPU (e.g. on two streams) race.
 */
int ff_linear_w8a8_noalloc(const uint16_t* x, const float* gamma, const float* beta, float eps, int rows, int cols,
                           int valid_cols, int block, const int8_t* W, const float* col_scale, const float* bias,
                           void* out, int N, int epi, int* err, void* stream);

/* ---------------------------------------------------------------- attention */
/*
 * Non-causal multi-head attention, head dim 64, fp16 in/out, f32 softmax and accumulation.
 *   qkv [num_seqs * seq_len, 3 * heads * 64] fp16 (q | k | v column sections, head h at columns h*64),
 *   out [num_seqs * seq_len, heads * 64] fp16. Any seq_len >= 1 (ragged tail tiles are masked).
 *   rope_cos / rope_sin: must be NULL; q and k arrive rotated, as in the reference, whose QKV GEMM
 *   epilogue applies the RoPE (here FF_EPI_QKV_ROPE). scale multiplies q·k (1 when folded into q).
 *   Runs on the tcgen05 tensor cores (f16 MMAs, f32 accumulation in TMEM).
 * Replaces torch.ops.foidfinder.attention (foidfinder/backends/cuda/csrc/kernels.cu:255-265).
 */
int ff_attention(const uint16_t* qkv, uint16_t* out, int num_seqs, int seq_len, int heads, const float* rope_cos,
                 const float* rope_sin, float scale, void* stream);

/* ---------------------------------------------------------------- stem, norm, head */
/*
 * images [B, S, S, 3] uint8 -> patches [B * (S/p)^2, k_pad] fp16 with (kh, kw, c) column order
 * (reference.py:103-107), each value (pixel / 255 - mean[c]) / std[c]; columns >= p*p*3 are 0.
 */
int ff_patchify(const uint8_t* images, int B, int image_size, int patch, const float* mean3, const float* std3,
                uint16_t* patches, int k_pad, void* stream);

/* Writes the class-token row cls_row [dim] fp16 into token 0 of each of B images of x [B * tokens, dim]. */
int ff_fill_cls(const uint16_t* cls_row, uint16_t* x, int B, int tokens, int dim, void* stream);

/* out[r] = LayerNorm(x[r * row_stride : + cols]) in fp16, r < rows, f32 statistics. */
int ff_layernorm(const uint16_t* x, int64_t row_stride, const float* gamma, const float* beta, float eps, int rows,
                 int cols, uint16_t* out, void* stream);

/* Per row of logits [B, n]: the k (<= 64) largest values, descending, ties by lower index. */
int ff_topk(const float* logits, int B, int n, int k, int32_t* idx_out, float* val_out, void* stream);

/* ---------------------------------------------------------------- whole-model engine */
typedef struct ff_model_config {
  int image_size;       /* 448 */
  int patch;            /* 14 */
  int dim;              /* 1024 (EVA02-L) / 768 (EVA02-B) */
  int depth;            /* 24 / 12 */
  int heads;            /* dim / 64 */
  int mlp_hidden;       /* 2730 / 2048 real SwiGLU width */
  int mlp_hidden_pad;   /* 2816 / 2048 / 4864 (PixAI's 4736): multiple of 128, zero-padded weights */
  int num_tags;         /* 30877 */
  int num_tags_pad;     /* multiple of 256 */
  int rot_block_dim;    /* Hadamard block for dim-wide activations: 1024 / 256 */
  int rot_block_hidden; /* Hadamard block for hidden activations: 128 */
  int topk;             /* <= 64 */
  float ln_eps;         /* 1e-6 */
  float mean[3];
  float std[3];
  /* Head. FF_HEAD_CLS: final LayerNorm of the class token -> linear [num_tags, dim]. FF_HEAD_TREE: the
   * Haruka tree attention pool (foidfinder/backends/mlx/haruka.py:104-136) over all tokens ->
   * linear [num_tags, leaf_queries * leaf_dim]. */
  int head_kind;
  int pool_heads;     /* 16; dim / pool_heads in {48, 64} */
  int coarse_queries; /* 6 */
  int leaf_queries;   /* 18, a multiple of coarse_queries */
  int leaf_dim;       /* 64 */
  /* Architecture. FF_ARCH_EVA02: class token, SwiGLU with the hidden LayerNorm, every block global.
   * FF_ARCH_PIXAI: PixAI Tagger v1.0 (foidfinder/backends/cuda/reference.py:109-140): no class token, tokens
   * in window order, ln_pre after the stem, GELU MLP (mlp_hidden == mlp_hidden_pad, H128 on the hidden),
   * window x window attention except in the blocks whose bit is set in global_blocks, head_kind
   * FF_HEAD_POOL. */
  int arch;
  int window;                      /* window size in patches (PixAI: 24); the grid must be a multiple */
  unsigned long long global_blocks; /* bit i: block i attends over the whole image (PixAI: 7, 15, 23, 31) */
} ff_model_config;

#define FF_HEAD_CLS 0
#define FF_HEAD_TREE 1
#define FF_HEAD_POOL 2 /* PixAI: LN + pos -> kv -> one learned query per head -> proj (reference.py:133-140) */
#define FF_ARCH_EVA02 0
#define FF_ARCH_PIXAI 1

typedef struct ff_layer_weights {
  const float *norm1_w, *norm1_b;
  const int8_t* qkv_w; /* [3*dim, dim], q rows pre-scaled by 1/8 */
  const float *qkv_s, *qkv_b;
  const int8_t* proj_w; /* [dim, dim] */
  const float *proj_s, *proj_b;
  const float *norm2_w, *norm2_b;
  const int8_t* fc1_w; /* [2*hidden_pad, dim], rows interleaved [gate 64 | up 64] */
  const float *fc1_s, *fc1_b;
  const float *mlp_norm_w, *mlp_norm_b; /* [hidden_pad] */
  const int8_t* fc2_w; /* [dim, hidden_pad] */
  const float *fc2_s, *fc2_b;
} ff_layer_weights;

typedef struct ff_model_weights {
  const uint16_t* patch_w;  /* [dim, k_pad] fp16, k_pad = ceil(p*p*3 / 64) * 64 */
  const float* pos_bias;    /* [patches, dim] f32 = patch bias + pos_embed[1:] */
  const uint16_t* cls_row;  /* [dim] fp16 = cls_token + pos_embed[0] */
  const float *rope_cos, *rope_sin; /* [32, tokens], angle-major */
  const ff_layer_weights* layers;   /* [depth] */
  const float *norm_w, *norm_b;     /* final LayerNorm */
  const uint16_t* head_w;           /* [num_tags_pad, dim] (CLS) or [num_tags_pad, leaf_queries * leaf_dim] fp16 */
  const float* head_b;              /* [num_tags_pad] */
  /* FF_HEAD_TREE (and, for pool_norm_* and pool_kv_*, FF_HEAD_POOL, where the key rows are not pre-scaled)
   * only, NULL otherwise; layout of foidfinder/haruka.py:fold, f32 unless noted. */
  const float *pool_norm_w, *pool_norm_b;     /* [dim] */
  const uint16_t* pool_kv_w;                  /* [2*dim, dim] fp16, key rows pre-scaled by head_dim^-0.5 */
  const float* pool_kv_b;                     /* [2*dim] */
  const float *q_coarse, *q_coarse_bias;      /* [coarse, dim], [coarse] */
  const float *q_child, *q_child_bias;        /* [leaves, dim], [leaves] */
  const float *trunk_norm_w, *trunk_norm_b;   /* [dim] */
  const float *child_q_norm_w, *child_q_norm_b;
  const float *leaf_norm_w, *leaf_norm_b;
  const float *leaf_w, *leaf_b;               /* [leaves, dim, leaf_dim], [leaves, leaf_dim] */
  /* FF_ARCH_PIXAI only (NULL otherwise). cls_row, norm_w/b and the layers' mlp_norm_w/b are unused; fc1_w is
   * [hidden, dim] in the checkpoint's row order with the GELU in the epilogue; rope_cos/sin hold the
   * window table [32, window^2] and pos_bias the window-ordered position embedding [patches, dim]. */
  const float *ln_pre_w, *ln_pre_b;                /* [dim] */
  const float *rope_cos_global, *rope_sin_global;  /* [32, patches], angle-major, window order */
  const uint16_t* pool_pos;                        /* [patches, dim] fp16, window order */
  const float* pool_q;                             /* [dim], the 1/8 attention scale folded in */
  const uint16_t* pool_proj_w;                     /* [dim, dim] fp16 */
  const float* pool_proj_b;                        /* [dim] */
} ff_model_weights;

/*
 * The Haruka tree attention pool head on its own: x [B * tokens, dim] fp16 (the backbone's output before its
 * final LayerNorm; tokens = (image_size / patch)^2 + 1) -> leaf features leaf_out [B, leaf_queries * leaf_dim]
 * fp16, the input of the tag head. Runs: final LayerNorm (w->norm_*), pool LayerNorm, key/value GEMM
 * (tcgen05 fp16), coarse slot attention, trunk/child LayerNorms, leaf slot attention, leaf LayerNorm x
 * mass gate x per-leaf projection (foidfinder/backends/mlx/haruka.py:104-136). cfg->head_kind must be
 * FF_HEAD_TREE. workspace: caller-allocated device memory, 256-byte aligned, at least
 * ff_tree_pool_workspace_bytes(cfg, B) bytes.
 */
int ff_tree_pool(const ff_model_config* cfg, const struct ff_model_weights* w, const uint16_t* x, int B,
                 void* workspace, int64_t workspace_bytes, uint16_t* leaf_out, void* stream);
int64_t ff_tree_pool_workspace_bytes(const ff_model_config* cfg, int B);

/* Window-ordered patch rows (window > 0: the grid in window x window tiles, windows row-major, patches
 * row-major inside; foidfinder/backends/cuda/reference.py:21-24). window = 0 is ff_patchify. */
int ff_patchify_windowed(const uint8_t* images, int B, int image_size, int patch, const float* mean3, const float* std3,
                         uint16_t* patches, int k_pad, int window, void* stream);
/* LayerNorm (f32 statistics) to fp16, then + fp16 pos[row % period] in fp16 (the PixAI pool's
 * LN + position embedding, reference.py:135). */
int ff_layernorm_pos(const uint16_t* x, int64_t row_stride, const float* gamma, const float* beta, float eps, int rows,
                     int cols, const uint16_t* pos, int period, uint16_t* out, void* stream);
/* One learned query per head over all tokens of each image (the PixAI attention pool, reference.py:136-138):
 * q [heads * 64] f32 with the 1/8 scale folded in, kv [B * tokens, 2 * heads * 64] fp16 (keys | values)
 * -> out [B, heads * 64] fp16, f32 softmax. */
int ff_pool_query_attention(const float* q, const uint16_t* kv, int B, int tokens, int heads, uint16_t* out,
                            void* stream);

/* ---------------------------------------------------------------- preprocessing */
#define FF_RESAMPLE_BILINEAR 0
#define FF_RESAMPLE_BICUBIC 1 /* a = -0.5 */
/*
 * Letterbox on the GPU: src [h, w, 3] uint8 RGB -> dst [size, size, 3] uint8, the image resized to
 * (new_h, new_w) with Pillow's 8-bit separable resampling (filter FF_RESAMPLE_*, antialiased when
 * reducing) and centred at ((size - new_h) / 2, (size - new_w) / 2) on a canvas of value `fill`.
 * Bit-exact with PIL.Image.resize(filter) pasted on Image.new("RGB", (size, size), fill). The image step
 * before the engine: foidfinder/backends/cuda/preprocess.py:16-32 (PixAI, on black) and
 * foidfinder/backends/mlx/kernels.py:75-186 (Haruka, bicubic on white). workspace: device memory of at
 * least ff_resize_pad_workspace_bytes(...) bytes, 256-byte aligned (intermediate image + coefficients).
 */
int ff_resize_pad(const uint8_t* src, int h, int w, int new_h, int new_w, int size, int filter, int fill, uint8_t* dst,
                  void* workspace, int64_t workspace_bytes, void* stream);
int64_t ff_resize_pad_workspace_bytes(int h, int w, int new_h, int new_w, int filter);

/*
 * PixAI's letterbox in float on the GPU: src [h, w, 3] uint8 RGB -> dst [size, size, 3] fp16 normalised
 * pixels (the engine's float input): pixels / 255, resized to (new_h, new_w) by antialiased bilinear
 * interpolation in f32 (torch F.interpolate(mode="bilinear", align_corners=False, antialias=True)),
 * x * 2 - 1 rounded to fp16, centred at ((size - new_h) / 2, (size - new_w) / 2) on a canvas of -1.
 * Replaces foidfinder/backends/cuda/preprocess.py:16-32 (per image). No workspace.
 */
int ff_letterbox_aa_f16(const uint8_t* src, int h, int w, int new_h, int new_w, int size, uint16_t* dst,
                        void* stream);

typedef struct ff_engine ff_engine;

/* Validates the config, keeps the weight pointers (the caller keeps them alive) and binds to `device`. */
int ff_engine_create(const ff_model_config* cfg, const ff_model_weights* w, int device, ff_engine** out);

/*
 * images [B, S, S, 3] uint8 on the device -> logits [B, num_tags] f32 and, when topk_idx != NULL,
 * the top cfg.topk tag indices [B, topk] int32 (and values when topk_val != NULL).
 * The first call for a batch size allocates that size's activation buffers and captures the whole
 * forward in a CUDA graph; later calls replay it. Replaces PixAICuda.__call__ (engine.py:163-184).
 */
int ff_engine_forward(ff_engine* e, const uint8_t* images, int B, float* logits, int32_t* topk_idx, float* topk_val,
                      void* stream);

/* Same forward without a graph (each kernel launched directly); used for debugging and tests. */
int ff_engine_forward_eager(ff_engine* e, const uint8_t* images, int B, float* logits, int32_t* topk_idx,
                            float* topk_val, void* stream);

/*
 * The forward from normalised fp16 pixels [B, S, S, 3] on the device instead of uint8 images: the input
 * PixAICuda.__call__ takes (engine.py:163-165, "normalized pixels"; the reference casts any float dtype to
 * fp16 into its static input) and ff_letterbox_aa_f16 writes. The patch rows take the pixels as they are
 * (no mean/std). use_graph != 0: replay this batch size's graph for fp16 input (captured on first use);
 * 0: launch the kernels directly.
 */
int ff_engine_forward_pixels(ff_engine* e, const uint16_t* pixels, int B, float* logits, int32_t* topk_idx,
                             float* topk_val, int use_graph, void* stream);

/* Kernel classes of ff_engine_profile. */
#define FF_PROF_STEM_PREP 0 /* patchify + class-token rows */
#define FF_PROF_STEM_GEMM 1
#define FF_PROF_ROTATE 2    /* every LayerNorm/Hadamard/int8 quantisation launch */
#define FF_PROF_GEMM_QKV 3
#define FF_PROF_ATTENTION 4
#define FF_PROF_GEMM_PROJ 5
#define FF_PROF_GEMM_FC1 6  /* gate|up with the SwiGLU epilogue */
#define FF_PROF_GEMM_FC2 7
#define FF_PROF_HEAD 8      /* final LayerNorm, tag head GEMM, top-k */
#define FF_PROF_CLASSES 9

/*
 * Runs the forward `iters` times without a graph, with CUDA events around every launch, and writes the
 * mean milliseconds per forward spent in each kernel class to ms[FF_PROF_CLASSES] (and the number of
 * launches per forward of each class to launches[FF_PROF_CLASSES] when not NULL). Synchronises stream.
 */
int ff_engine_profile(ff_engine* e, const uint8_t* images, int B, int iters, float* ms, int* launches, void* stream);

/* Kernel launches in one forward of this configuration. */
int ff_engine_launches_per_forward(const ff_model_config* cfg);

/* Bytes of device memory the engine holds for activations of batch size B. */
int64_t ff_engine_workspace_bytes(const ff_model_config* cfg, int B);

int ff_engine_destroy(ff_engine* e);

#if defined(__GNUC__)
#pragma GCC visibility pop
#endif

#ifdef __cplusplus
}
#endif
#endif /* FOIDFINDER_B200_H */
