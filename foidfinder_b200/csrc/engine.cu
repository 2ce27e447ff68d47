// Whole-model int8 engine behind the C ABI: one object per device, activation buffers and a CUDA graph
// per batch size, weights owned by the caller.
//
// The layer loop follows PixAICuda._forward (foidfinder/backends/cuda/engine.py:142-161) with the EVA02
// block of foidfinder/backends/mlx/haruka.py:86-99:
//   per block: LN1+H(dim)+q8 -> QKV GEMM (+bias, 2-D RoPE) -> attention -> H(dim)+q8 -> proj GEMM
//              (+bias, residual) -> LN2+H(dim)+q8 -> gate|up GEMM (+bias, SwiGLU) -> mlp LN+H128+q8 ->
//              down GEMM (+bias, residual)
// followed by the head — the final LayerNorm of the class tokens (FF_HEAD_CLS) or the Haruka tree
// attention pool over all tokens (FF_HEAD_TREE, pool.cu) — the fp16 tag head and a device top-k.
// FF_ARCH_PIXAI runs PixAICuda._forward itself: window-ordered patches, ln_pre, window attention with the
// window RoPE table except in the global blocks, GELU fc1 epilogue, H128 of the 4736-wide hidden, and the
// one-query attention pool (reference.py:133-140) before the tag head.
// Graph capture per batch size replaces the torch.cuda.graph capture of engine.py:163-184.
#include <cuda_fp16.h>

#include <algorithm>
#include <cstring>
#include <map>
#include <mutex>
#include <vector>

#include "common.h"
#include "gemm.h"
#include "kernels.h"
#include "pool.h"

struct ff_engine {
  struct Batch {
    int B = 0;
    void* block = nullptr;  // one allocation for every activation buffer below
    uint8_t* images = nullptr;  // the input: uint8 pixels, or (fp16 input) normalised fp16 pixels
    __half* patches = nullptr;
    __half* x = nullptr;
    int8_t* a8 = nullptr;
    float* rs = nullptr;
    __half* qkv = nullptr;
    __half* o = nullptr;
    __half* h = nullptr;
    __half* cls = nullptr;  // head input: [B, dim] class rows or [B, leaves * leaf_dim] leaf features
    float* logits = nullptr;
    int32_t* top_idx = nullptr;
    float* top_val = nullptr;
    ff::GemmPlan stem, head, pool_kv, pool_proj;
    ff::PoolBuffers pool;
    std::vector<ff::GemmPlan> qkv_p, proj_p, fc1_p, fc2_p;
    cudaGraphExec_t exec[2] = {nullptr, nullptr};  // graph per input kind: [0] uint8, [1] fp16 pixels
    cudaStream_t capture_stream = nullptr;
  };
  ff_model_config cfg{};
  ff_model_weights w{};
  std::vector<ff_layer_weights> layers;
  int device = 0;
  int grid = 0, patches = 0, tokens = 0, k_pad = 0;
  // Separable form of the (window) RoPE tables, when every entry checks out (rope_separable): [cos | sin],
  // each [32, rope_grid + 1]; nullptr keeps the QKV epilogue on the full tables.
  float* rope_compact = nullptr;
  int rope_grid = 0, rope_cls = 0, rope_swap = 0;
  std::map<int, Batch*> batches;
  std::mutex mu;
};

namespace ff {
namespace {

struct DeviceScope {
  int prev = 0;
  explicit DeviceScope(int dev) {
    cudaGetDevice(&prev);
    cudaSetDevice(dev);
  }
  ~DeviceScope() { cudaSetDevice(prev); }
};

size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

// The full RoPE tables (angle-major [32, rows], rows = cls + G * G positions) as [32, G + 1] tables of one grid
// coordinate each: pairs 0..15 follow the row coordinate and 16..31 the column (or the reverse with swap),
// as the EVA02 and PixAI axial tables are built; column G holds the class token's identity rotation.
// Accepted only if every entry of the full tables equals its compact counterpart bit for bit (and the class
// token's column is the identity), so the QKV epilogue computes exactly what it computes from the full
// tables. Returns false (no compact form) otherwise.
bool rope_separable(const std::vector<float>& fc, const std::vector<float>& fs, int rows, int G, int cls, int swap,
                    std::vector<float>* compact) {
  if (G <= 0 || rows != cls + G * G) return false;
  const int W = G + 1;  // column G: the identity rotation of the class token
  std::vector<float> cc(32 * W), cs(32 * W);
  for (int j = 0; j < 32; ++j) {
    for (int a = 0; a < G; ++a) {
      const bool row_coord = (j < 16) != (swap != 0);  // this pair follows the row coordinate
      const int idx = row_coord ? a * G : a;
      cc[j * W + a] = fc[static_cast<size_t>(j) * rows + cls + idx];
      cs[j * W + a] = fs[static_cast<size_t>(j) * rows + cls + idx];
    }
    cc[j * W + G] = 1.f;
    cs[j * W + G] = 0.f;
  }
  auto same = [](float a, float b) { return std::memcmp(&a, &b, sizeof(float)) == 0; };
  for (int j = 0; j < 32; ++j) {
    if (cls && (!same(fc[static_cast<size_t>(j) * rows], 1.f) || !same(fs[static_cast<size_t>(j) * rows], 0.f)))
      return false;
    for (int idx = 0; idx < G * G; ++idx) {
      const int r = idx / G, c = idx % G;
      const int a = ((j < 16) != (swap != 0)) ? r : c;
      if (!same(fc[static_cast<size_t>(j) * rows + cls + idx], cc[j * W + a]) ||
          !same(fs[static_cast<size_t>(j) * rows + cls + idx], cs[j * W + a]))
        return false;
    }
  }
  compact->assign(cc.begin(), cc.end());
  compact->insert(compact->end(), cs.begin(), cs.end());
  return true;
}

struct Layout {
  size_t images, patches, x, a8, rs, qkv, o, h, cls, logits, top_idx, top_val, pool, total;
};

int head_in(const ff_model_config& c) { return c.head_kind == FF_HEAD_TREE ? c.leaf_queries * c.leaf_dim : c.dim; }

bool pixai(const ff_model_config& c) { return c.arch == FF_ARCH_PIXAI; }

int tokens_of(const ff_model_config& c) {
  const int G = c.image_size / c.patch;
  return G * G + (pixai(c) ? 0 : 1);
}

bool is_global(const ff_model_config& c, int block) {
  return !pixai(c) || (block < 64 && ((c.global_blocks >> block) & 1ull) != 0);
}

Layout layout_for(const ff_model_config& c, int B) {
  const size_t G = c.image_size / c.patch, P = G * G, T = tokens_of(c), M = static_cast<size_t>(B) * T;
  const size_t kpad = align_up(static_cast<size_t>(c.patch) * c.patch * 3, 64);
  const size_t wide = std::max<size_t>(c.dim, c.mlp_hidden_pad);
  Layout l{};
  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t at = off;
    off = align_up(off + bytes, 1024);
    return at;
  };
  l.images = take(static_cast<size_t>(B) * c.image_size * c.image_size * 3 * 2);  // room for fp16 pixels
  l.patches = take(static_cast<size_t>(B) * P * kpad * 2);
  l.x = take(M * c.dim * 2);
  l.a8 = take(M * wide);
  l.rs = take(M * 4);
  l.qkv = take(M * 3 * c.dim * 2);
  l.o = take(M * c.dim * 2);
  l.h = take(M * c.mlp_hidden_pad * 2);
  l.cls = take(static_cast<size_t>(B) * head_in(c) * 2);
  l.logits = take(static_cast<size_t>(B) * c.num_tags * 4);
  l.top_idx = take(static_cast<size_t>(B) * (c.topk > 0 ? c.topk : 1) * 4);
  l.top_val = take(static_cast<size_t>(B) * (c.topk > 0 ? c.topk : 1) * 4);
  l.pool = take(c.head_kind == FF_HEAD_TREE ? pool_small_bytes(c, B) : 0);
  l.total = off;
  return l;
}

int validate(const ff_model_config& c) {
  FF_REQUIRE(c.patch >= 1 && c.image_size % c.patch == 0, "engine: image_size %d not a multiple of patch %d", c.image_size, c.patch);
  FF_REQUIRE(c.dim == 768 || c.dim == 1024, "engine: dim %d (supported: 768, 1024)", c.dim);
  FF_REQUIRE(c.heads * 64 == c.dim, "engine: heads * 64 must equal dim");
  FF_REQUIRE(c.depth >= 1, "engine: depth %d", c.depth);
  FF_REQUIRE(c.mlp_hidden >= 1 && c.mlp_hidden <= c.mlp_hidden_pad && c.mlp_hidden_pad % 128 == 0,
             "engine: mlp_hidden %d / pad %d", c.mlp_hidden, c.mlp_hidden_pad);
  FF_REQUIRE(c.arch == FF_ARCH_EVA02 || c.arch == FF_ARCH_PIXAI, "engine: arch %d", c.arch);
  if (pixai(c)) {
    const int G = c.image_size / c.patch;
    FF_REQUIRE(c.head_kind == FF_HEAD_POOL, "engine: the PixAI architecture needs head_kind FF_HEAD_POOL");
    FF_REQUIRE(c.window >= 1 && G % c.window == 0, "engine: window %d does not tile the %d-patch grid", c.window, G);
    FF_REQUIRE(c.rot_block_hidden == 128, "engine: the PixAI GELU hidden takes an H128 rotation");
  } else {
    FF_REQUIRE(c.head_kind != FF_HEAD_POOL, "engine: FF_HEAD_POOL needs the PixAI architecture");
    FF_REQUIRE(c.mlp_hidden_pad == 2048 || c.mlp_hidden_pad == 2816 || c.mlp_hidden_pad == 4096,
               "engine: mlp_hidden_pad %d has no rotation kernel", c.mlp_hidden_pad);
  }
  FF_REQUIRE(c.num_tags >= 1 && c.num_tags <= c.num_tags_pad && c.num_tags_pad % 256 == 0,
             "engine: num_tags %d / pad %d", c.num_tags, c.num_tags_pad);
  FF_REQUIRE(c.dim % c.rot_block_dim == 0 && c.mlp_hidden_pad % c.rot_block_hidden == 0, "engine: rotation blocks");
  FF_REQUIRE(c.topk >= 0 && c.topk <= 64 && c.topk <= c.num_tags, "engine: topk %d", c.topk);
  FF_REQUIRE(c.head_kind == FF_HEAD_CLS || c.head_kind == FF_HEAD_TREE || c.head_kind == FF_HEAD_POOL,
             "engine: head_kind %d", c.head_kind);
  return FF_OK;
}

int build_batch(ff_engine* e, int B, ff_engine::Batch** out) {
  const ff_model_config& c = e->cfg;
  const Layout l = layout_for(c, B);
  auto* b = new ff_engine::Batch();
  b->B = B;
  if (cudaMalloc(&b->block, l.total) != cudaSuccess) {
    delete b;
    cudaGetLastError();
    set_error("engine: cudaMalloc of %zu bytes for batch %d failed", l.total, B);
    return FF_ERR_OUT_OF_MEMORY;
  }
  uint8_t* base = static_cast<uint8_t*>(b->block);
  b->images = base + l.images;
  b->patches = reinterpret_cast<__half*>(base + l.patches);
  b->x = reinterpret_cast<__half*>(base + l.x);
  b->a8 = reinterpret_cast<int8_t*>(base + l.a8);
  b->rs = reinterpret_cast<float*>(base + l.rs);
  b->qkv = reinterpret_cast<__half*>(base + l.qkv);
  b->o = reinterpret_cast<__half*>(base + l.o);
  b->h = reinterpret_cast<__half*>(base + l.h);
  b->cls = reinterpret_cast<__half*>(base + l.cls);
  b->logits = reinterpret_cast<float*>(base + l.logits);
  b->top_idx = reinterpret_cast<int32_t*>(base + l.top_idx);
  b->top_val = reinterpret_cast<float*>(base + l.top_val);
  if (c.head_kind == FF_HEAD_TREE) {
    // The pool reuses activation buffers that are free once the last block has run: the attention
    // output for the final-normed tokens, the residual stream for the pool-normed ones, qkv for keys/values.
    b->pool.xf = b->o;
    b->pool.xn = b->x;
    b->pool.kv = b->qkv;
    pool_carve_small(c, B, base + l.pool, &b->pool);
  }
  cudaMemset(b->block, 0, l.total);

  const int M = B * e->tokens, D = c.dim, H = c.mlp_hidden_pad;
  int rc = FF_OK;
  {
    GemmProblem p{};
    p.args.w_const = 1;  // the engine's weights stay constant while forwards run
    p.A = b->patches;
    p.W = e->w.patch_w;
    p.out = b->x;
    p.M = B * e->patches;
    p.N = D;
    p.K = e->k_pad;
    p.epi = EPI_STEM;
    p.f16 = true;
    p.args.ldo = D;
    p.args.pos_bias = e->w.pos_bias;
    p.args.patches = e->patches;
    p.args.tokens = e->tokens;
    rc = gemm_prepare(p, &b->stem);
  }
  if (rc == FF_OK) {
    GemmProblem p{};
    p.args.w_const = 1;  // the engine's weights stay constant while forwards run
    p.A = b->cls;
    p.W = e->w.head_w;
    p.out = b->logits;
    p.M = B;
    p.N = c.num_tags_pad;
    p.K = head_in(c);
    p.epi = EPI_LOGITS;
    p.f16 = true;
    p.args.bias = e->w.head_b;
    p.args.ldo = c.num_tags;
    p.args.n_valid = c.num_tags;
    rc = gemm_prepare(p, &b->head);
  }
  if (rc == FF_OK && c.head_kind == FF_HEAD_TREE) rc = pool_prepare(c, e->w, B, e->tokens, b->pool, &b->pool_kv);
  if (rc == FF_OK && c.head_kind == FF_HEAD_POOL) {
    // PixAI pool (reference.py:133-140): pool-normed tokens (+ pos) in o, keys|values in qkv, the attended
    // [B, dim] rows in h, the projected rows in cls (the tag head's input).
    GemmProblem p{};
    p.args.w_const = 1;  // the engine's weights stay constant while forwards run
    p.A = b->o;
    p.W = e->w.pool_kv_w;
    p.out = b->qkv;
    p.M = M;
    p.N = 2 * D;
    p.K = D;
    p.epi = EPI_BIAS;
    p.f16 = true;
    p.args.bias = e->w.pool_kv_b;
    p.args.ldo = 2 * D;
    rc = gemm_prepare(p, &b->pool_kv);
    if (rc == FF_OK) {
      GemmProblem q{};
      q.args.w_const = 1;
      q.A = b->h;
      q.W = e->w.pool_proj_w;
      q.out = b->cls;
      q.M = B;
      q.N = D;
      q.K = D;
      q.epi = EPI_BIAS;
      q.f16 = true;
      q.args.bias = e->w.pool_proj_b;
      q.args.ldo = D;
      rc = gemm_prepare(q, &b->pool_proj);
    }
  }
  b->qkv_p.resize(c.depth);
  b->proj_p.resize(c.depth);
  b->fc1_p.resize(c.depth);
  b->fc2_p.resize(c.depth);
  for (int i = 0; i < c.depth && rc == FF_OK; ++i) {
    const ff_layer_weights& lw = e->layers[i];
    const bool glob = is_global(c, i);
    const float* rcos = pixai(c) && glob ? e->w.rope_cos_global : e->w.rope_cos;
    const float* rsin = pixai(c) && glob ? e->w.rope_sin_global : e->w.rope_sin;
    const int rope_tokens = glob ? e->tokens : c.window * c.window;  // the RoPE table's rows
    auto prep = [&](GemmPlan* plan, const int8_t* W, const float* s, const float* bias, void* out, int N, int K, int epi) {
      GemmProblem p{};
      p.args.w_const = 1;  // the engine's weights stay constant while forwards run
      p.A = b->a8;
      p.W = W;
      p.out = out;
      p.M = M;
      p.N = N;
      p.K = K;
      p.epi = epi;
      p.f16 = false;
      p.args.row_scale = b->rs;
      p.args.col_scale = s;
      p.args.bias = bias;
      p.args.ldo = epi == EPI_SWIGLU ? N / 2 : N;
      p.args.rope_cos = rcos;
      p.args.rope_sin = rsin;
      p.args.rope_cols = epi == EPI_QKV_ROPE ? 2 * D : 0;
      p.args.tokens = rope_tokens;
      if (e->rope_compact && !(pixai(c) && glob)) {  // the table rope_separable checked
        p.args.rope_grid = e->rope_grid;
        p.args.rope_cls = e->rope_cls;
        p.args.rope_swap = e->rope_swap;
        p.args.rope_cos_c = e->rope_compact;
        p.args.rope_sin_c = e->rope_compact + 32 * (e->rope_grid + 1);
      }
      return gemm_prepare(p, plan);
    };
    rc = prep(&b->qkv_p[i], lw.qkv_w, lw.qkv_s, lw.qkv_b, b->qkv, 3 * D, D, EPI_QKV_ROPE);
    if (rc == FF_OK) rc = prep(&b->proj_p[i], lw.proj_w, lw.proj_s, lw.proj_b, b->x, D, D, EPI_RESIDUAL);
    if (rc == FF_OK && pixai(c)) rc = prep(&b->fc1_p[i], lw.fc1_w, lw.fc1_s, lw.fc1_b, b->h, H, D, EPI_GELU_F16);
    if (rc == FF_OK && !pixai(c)) rc = prep(&b->fc1_p[i], lw.fc1_w, lw.fc1_s, lw.fc1_b, b->h, 2 * H, D, EPI_SWIGLU);
    if (rc == FF_OK) rc = prep(&b->fc2_p[i], lw.fc2_w, lw.fc2_s, lw.fc2_b, b->x, D, H, EPI_RESIDUAL);
  }
  if (rc != FF_OK) {
    cudaFree(b->block);
    delete b;
    return rc;
  }
  *out = b;
  return FF_OK;
}

#define FF_TRY(expr)             \
  do {                           \
    const int rc_ = (expr);      \
    if (rc_ != FF_OK) return rc_; \
  } while (0)

// Optional per-launch timing: events recorded around every launch, accumulated per kernel class.
struct Profiler {
  std::vector<cudaEvent_t> ev;
  std::vector<int> cls;
  size_t next = 0;
  int begin(int klass, cudaStream_t s) {
    if (next + 1 >= ev.size()) return FF_OK;  // out of events: stop recording
    cls.push_back(klass);
    return cudaEventRecord(ev[next++], s) == cudaSuccess ? FF_OK : check_launch("profiler: event record");
  }
  int end(cudaStream_t s) {
    if (next >= ev.size() || cls.size() * 2 != next + 1) return FF_OK;
    return cudaEventRecord(ev[next++], s) == cudaSuccess ? FF_OK : check_launch("profiler: event record");
  }
};

#define FF_LAUNCH(klass, expr)                    \
  do {                                            \
    if (prof) FF_TRY(prof->begin((klass), s));    \
    FF_TRY(expr);                                 \
    if (prof) FF_TRY(prof->end(s));               \
  } while (0)

// Every launch of one forward of batch b on stream s.
int run_forward(ff_engine* e, ff_engine::Batch* b, cudaStream_t s, Profiler* prof = nullptr, bool f16_in = false) {
  const ff_model_config& c = e->cfg;
  const int B = b->B, M = B * e->tokens, D = c.dim, H = c.mlp_hidden_pad;
  FF_LAUNCH(FF_PROF_STEM_PREP, patchify(b->images, B, c.image_size, c.patch, c.mean, c.std, b->patches, e->k_pad, s,
                                        pixai(c) ? c.window : 0, f16_in));
  FF_LAUNCH(FF_PROF_STEM_GEMM, gemm_launch(b->stem, s));
  if (pixai(c))  // ln_pre, in place (engine.py:148)
    FF_LAUNCH(FF_PROF_STEM_PREP, layernorm(b->x, D, e->w.ln_pre_w, e->w.ln_pre_b, c.ln_eps, M, D, b->x, s));
  else
    FF_LAUNCH(FF_PROF_STEM_PREP, fill_cls(e->w.cls_row, b->x, B, e->tokens, D, s));
  for (int i = 0; i < c.depth; ++i) {
    const ff_layer_weights& lw = e->layers[i];
    const int seq = is_global(c, i) ? e->tokens : c.window * c.window;  // engine.py:152
    FF_LAUNCH(FF_PROF_ROTATE, rot_q8(b->x, lw.norm1_w, lw.norm1_b, c.ln_eps, M, D, D, c.rot_block_dim, b->a8, b->rs, s));
    FF_LAUNCH(FF_PROF_GEMM_QKV, gemm_launch(b->qkv_p[i], s));
    FF_LAUNCH(FF_PROF_ATTENTION, attention(b->qkv, b->o, M / seq, seq, c.heads, nullptr, nullptr, 1.f, s));
    FF_LAUNCH(FF_PROF_ROTATE, rot_q8(b->o, nullptr, nullptr, 0.f, M, D, D, c.rot_block_dim, b->a8, b->rs, s));
    FF_LAUNCH(FF_PROF_GEMM_PROJ, gemm_launch(b->proj_p[i], s));
    FF_LAUNCH(FF_PROF_ROTATE, rot_q8(b->x, lw.norm2_w, lw.norm2_b, c.ln_eps, M, D, D, c.rot_block_dim, b->a8, b->rs, s));
    FF_LAUNCH(FF_PROF_GEMM_FC1, gemm_launch(b->fc1_p[i], s));
    if (pixai(c))
      // zero padding columns (weights padded with zero rows) stay zero through the GELU and the H128 blocks
      FF_LAUNCH(FF_PROF_ROTATE, rot_q8(b->h, nullptr, nullptr, 0.f, M, H, H, c.rot_block_hidden, b->a8, b->rs, s));
    else
      FF_LAUNCH(FF_PROF_ROTATE, rot_q8(b->h, lw.mlp_norm_w, lw.mlp_norm_b, c.ln_eps, M, H, c.mlp_hidden,
                                       c.rot_block_hidden, b->a8, b->rs, s));
    FF_LAUNCH(FF_PROF_GEMM_FC2, gemm_launch(b->fc2_p[i], s));
  }
  if (c.head_kind == FF_HEAD_TREE) {
    FF_LAUNCH(FF_PROF_HEAD, pool_run(c, e->w, b->x, B, e->tokens, b->pool, b->pool_kv, b->cls, s));
  } else if (c.head_kind == FF_HEAD_POOL) {
    FF_LAUNCH(FF_PROF_HEAD, layernorm(b->x, D, e->w.pool_norm_w, e->w.pool_norm_b, c.ln_eps, M, D, b->o, s,
                                      e->w.pool_pos, e->tokens));
    FF_LAUNCH(FF_PROF_HEAD, gemm_launch(b->pool_kv, s));
    FF_LAUNCH(FF_PROF_HEAD, pool_query_attention(e->w.pool_q, b->qkv, B, e->tokens, c.heads, b->h, s));
    FF_LAUNCH(FF_PROF_HEAD, gemm_launch(b->pool_proj, s));
  } else
    FF_LAUNCH(FF_PROF_HEAD, layernorm(b->x, static_cast<int64_t>(e->tokens) * D, e->w.norm_w, e->w.norm_b, c.ln_eps, B,
                                      D, b->cls, s));
  FF_LAUNCH(FF_PROF_HEAD, gemm_launch(b->head, s));
  if (c.topk > 0) FF_LAUNCH(FF_PROF_HEAD, topk(b->logits, B, c.num_tags, c.topk, b->top_idx, b->top_val, s));
  return FF_OK;
}

// Kernel launches of one forward: 9 per block (2 rotations of the block's input and output of
// attention, 2 of the MLP, 4 GEMMs, 1 attention).
int launches_per_forward(const ff_model_config& c) {
  const int head = c.head_kind == FF_HEAD_TREE ? kPoolLaunches : c.head_kind == FF_HEAD_POOL ? 4 : 1;
  return 3 + 9 * c.depth + head + 1 + (c.topk > 0 ? 1 : 0);
}

int copy_out(ff_engine* e, ff_engine::Batch* b, float* logits, int32_t* top_idx, float* top_val, cudaStream_t s) {
  const ff_model_config& c = e->cfg;
  const int B = b->B;
  if (logits && cudaMemcpyAsync(logits, b->logits, static_cast<size_t>(B) * c.num_tags * 4, cudaMemcpyDeviceToDevice, s) != cudaSuccess)
    return check_launch("engine: logits copy");
  if (c.topk > 0 && top_idx &&
      cudaMemcpyAsync(top_idx, b->top_idx, static_cast<size_t>(B) * c.topk * 4, cudaMemcpyDeviceToDevice, s) != cudaSuccess)
    return check_launch("engine: top-k index copy");
  if (c.topk > 0 && top_val &&
      cudaMemcpyAsync(top_val, b->top_val, static_cast<size_t>(B) * c.topk * 4, cudaMemcpyDeviceToDevice, s) != cudaSuccess)
    return check_launch("engine: top-k value copy");
  return FF_OK;
}

int get_batch(ff_engine* e, int B, ff_engine::Batch** out) {
  auto it = e->batches.find(B);
  if (it != e->batches.end()) {
    *out = it->second;
    return FF_OK;
  }
  ff_engine::Batch* b = nullptr;
  FF_TRY(build_batch(e, B, &b));
  e->batches[B] = b;
  *out = b;
  return FF_OK;
}

int check_inputs(ff_engine* e, const uint8_t* images, int B, float* logits, int32_t* top_idx) {
  FF_REQUIRE(e != nullptr, "engine: NULL handle");
  FF_REQUIRE(images != nullptr && B >= 1, "engine: need images and B >= 1");
  FF_REQUIRE(logits != nullptr || top_idx != nullptr, "engine: no output requested");
  FF_REQUIRE(top_idx == nullptr || e->cfg.topk > 0, "engine: top-k requested but cfg.topk is 0");
  return FF_OK;
}

}  // namespace
}  // namespace ff

using namespace ff;

extern "C" int64_t ff_engine_workspace_bytes(const ff_model_config* cfg, int B) {
  if (cfg == nullptr || B < 1) return -1;
  return static_cast<int64_t>(layout_for(*cfg, B).total);
}

extern "C" int ff_engine_create(const ff_model_config* cfg, const ff_model_weights* w, int device, ff_engine** out) {
  FF_REQUIRE(cfg && w && out, "ff_engine_create: NULL argument");
  FF_TRY(validate(*cfg));
  const bool px = pixai(*cfg);
  FF_REQUIRE(w->patch_w && w->pos_bias && w->rope_cos && w->rope_sin && w->layers && w->head_w && w->head_b,
             "ff_engine_create: a model weight pointer is NULL");
  if (px)
    FF_REQUIRE(w->ln_pre_w && w->ln_pre_b && w->rope_cos_global && w->rope_sin_global && w->pool_norm_w &&
                   w->pool_norm_b && w->pool_pos && w->pool_q && w->pool_kv_w && w->pool_kv_b && w->pool_proj_w &&
                   w->pool_proj_b,
               "ff_engine_create: a PixAI weight pointer (ln_pre, global RoPE, attention pool) is NULL");
  else
    FF_REQUIRE(w->cls_row && w->norm_w && w->norm_b, "ff_engine_create: class row or final LayerNorm is NULL");
  if (cfg->head_kind == FF_HEAD_TREE) FF_TRY(pool_validate(*cfg, *w));
  for (int i = 0; i < cfg->depth; ++i) {
    const ff_layer_weights& l = w->layers[i];
    FF_REQUIRE(l.norm1_w && l.norm1_b && l.qkv_w && l.qkv_s && l.qkv_b && l.proj_w && l.proj_s && l.proj_b &&
                   l.norm2_w && l.norm2_b && l.fc1_w && l.fc1_s && l.fc1_b && (px || (l.mlp_norm_w && l.mlp_norm_b)) &&
                   l.fc2_w && l.fc2_s && l.fc2_b,
               "ff_engine_create: layer %d has a NULL weight pointer", i);
  }
  int ndev = 0;
  cudaGetDeviceCount(&ndev);
  FF_REQUIRE(device >= 0 && device < ndev, "ff_engine_create: device %d of %d", device, ndev);
  cudaDeviceProp prop;
  if (cudaGetDeviceProperties(&prop, device) != cudaSuccess || prop.major != 10) {
    set_error("ff_engine_create: device %d is not sm_100 (compute capability %d.%d)", device, prop.major, prop.minor);
    return FF_ERR_UNSUPPORTED_DEVICE;
  }
  auto* e = new ff_engine();
  e->cfg = *cfg;
  e->w = *w;
  e->layers.assign(w->layers, w->layers + cfg->depth);
  e->w.layers = e->layers.data();
  e->device = device;
  e->grid = cfg->image_size / cfg->patch;
  e->patches = e->grid * e->grid;
  e->tokens = tokens_of(*cfg);
  e->k_pad = static_cast<int>(align_up(static_cast<size_t>(cfg->patch) * cfg->patch * 3, 64));
  {
    // Separable RoPE tables for the QKV epilogue (EVA02's table; PixAI's window table), checked entry by entry.
    DeviceScope scope(device);
    const int G = pixai(*cfg) ? cfg->window : e->grid, cls = pixai(*cfg) ? 0 : 1;
    const int rows = cls + G * G;
    std::vector<float> fc(static_cast<size_t>(32) * rows), fs(fc.size()), compact;
    if (G > 0 && cudaMemcpy(fc.data(), w->rope_cos, fc.size() * 4, cudaMemcpyDeviceToHost) == cudaSuccess &&
        cudaMemcpy(fs.data(), w->rope_sin, fs.size() * 4, cudaMemcpyDeviceToHost) == cudaSuccess) {
      for (int swap = 0; swap < 2 && e->rope_compact == nullptr; ++swap)
        if (rope_separable(fc, fs, rows, G, cls, swap, &compact) &&
            cudaMalloc(&e->rope_compact, compact.size() * 4) == cudaSuccess) {
          if (cudaMemcpy(e->rope_compact, compact.data(), compact.size() * 4, cudaMemcpyHostToDevice) == cudaSuccess) {
            e->rope_grid = G;
            e->rope_cls = cls;
            e->rope_swap = swap;
          } else {
            cudaFree(e->rope_compact);
            e->rope_compact = nullptr;
          }
        }
    }
    cudaGetLastError();  // a table that is not separable (or a failed copy) only keeps the full tables
  }
  *out = e;
  return FF_OK;
}

namespace ff {
namespace {

size_t input_bytes(const ff_engine* e, int B, bool f16_in) {
  return static_cast<size_t>(B) * e->cfg.image_size * e->cfg.image_size * 3 * (f16_in ? 2 : 1);
}

// One forward of B images (uint8, or normalised fp16 pixels) already on the device: copy into the batch's
// input buffer, then the captured graph of this batch size and input kind (captured on first use) or the
// eager launch sequence, then the outputs to the caller's buffers, all on `stream`.
int forward_impl(ff_engine* e, const void* input, bool f16_in, int B, float* logits, int32_t* top_idx, float* top_val,
                 bool use_graph, void* stream) {
  std::lock_guard<std::mutex> lock(e->mu);
  DeviceScope scope(e->device);
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  ff_engine::Batch* b = nullptr;
  FF_TRY(get_batch(e, B, &b));
  cudaGraphExec_t& exec = b->exec[f16_in ? 1 : 0];
  if (use_graph && exec == nullptr) {
    // Warm up outside capture (kernel attributes, module loading), then capture on a private stream.
    if (b->capture_stream == nullptr &&
        cudaStreamCreateWithFlags(&b->capture_stream, cudaStreamNonBlocking) != cudaSuccess)
      return check_launch("engine: stream create");
    FF_TRY(run_forward(e, b, b->capture_stream, nullptr, f16_in));
    if (cudaStreamSynchronize(b->capture_stream) != cudaSuccess) return check_launch("engine: warm-up forward");
    cudaGraph_t graph = nullptr;
    if (cudaStreamBeginCapture(b->capture_stream, cudaStreamCaptureModeThreadLocal) != cudaSuccess)
      return check_launch("engine: begin capture");
    const int rc = run_forward(e, b, b->capture_stream, nullptr, f16_in);
    const cudaError_t ce = cudaStreamEndCapture(b->capture_stream, &graph);
    if (rc != FF_OK) {
      if (graph) cudaGraphDestroy(graph);
      return rc;
    }
    if (ce != cudaSuccess) return check_launch("engine: end capture");
    const cudaError_t ie = cudaGraphInstantiate(&exec, graph, 0);
    cudaGraphDestroy(graph);
    if (ie != cudaSuccess) {
      exec = nullptr;
      return check_launch("engine: graph instantiate");
    }
  }
  if (cudaMemcpyAsync(b->images, input, input_bytes(e, B, f16_in), cudaMemcpyDeviceToDevice, s) != cudaSuccess)
    return check_launch("engine: input copy");
  if (use_graph) {
    if (cudaGraphLaunch(exec, s) != cudaSuccess) return check_launch("engine: graph launch");
  } else {
    FF_TRY(run_forward(e, b, s, nullptr, f16_in));
  }
  return copy_out(e, b, logits, top_idx, top_val, s);
}

}  // namespace
}  // namespace ff

extern "C" int ff_engine_forward_eager(ff_engine* e, const uint8_t* images, int B, float* logits, int32_t* top_idx,
                                       float* top_val, void* stream) {
  FF_TRY(check_inputs(e, images, B, logits, top_idx));
  return forward_impl(e, images, false, B, logits, top_idx, top_val, false, stream);
}

extern "C" int ff_engine_forward(ff_engine* e, const uint8_t* images, int B, float* logits, int32_t* top_idx,
                                 float* top_val, void* stream) {
  FF_TRY(check_inputs(e, images, B, logits, top_idx));
  return forward_impl(e, images, false, B, logits, top_idx, top_val, true, stream);
}

extern "C" int ff_engine_forward_pixels(ff_engine* e, const uint16_t* pixels, int B, float* logits, int32_t* top_idx,
                                        float* top_val, int use_graph, void* stream) {
  FF_TRY(check_inputs(e, reinterpret_cast<const uint8_t*>(pixels), B, logits, top_idx));
  return forward_impl(e, pixels, true, B, logits, top_idx, top_val, use_graph != 0, stream);
}

extern "C" int ff_engine_profile(ff_engine* e, const uint8_t* images, int B, int iters, float* ms, int* launches,
                                 void* stream) {
  FF_REQUIRE(e && images && ms && B >= 1 && iters >= 1, "ff_engine_profile: bad arguments");
  std::lock_guard<std::mutex> lock(e->mu);
  DeviceScope scope(e->device);
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  ff_engine::Batch* b = nullptr;
  FF_TRY(get_batch(e, B, &b));
  const size_t in_bytes = static_cast<size_t>(B) * e->cfg.image_size * e->cfg.image_size * 3;
  if (cudaMemcpyAsync(b->images, images, in_bytes, cudaMemcpyDeviceToDevice, s) != cudaSuccess)
    return check_launch("engine: image copy");
  FF_TRY(run_forward(e, b, s));  // warm
  const int n = launches_per_forward(e->cfg);
  Profiler prof;
  prof.ev.resize(static_cast<size_t>(2 * n * iters));
  for (auto& ev : prof.ev)
    if (cudaEventCreate(&ev) != cudaSuccess) return check_launch("ff_engine_profile: event create");
  int rc = FF_OK;
  for (int it = 0; it < iters && rc == FF_OK; ++it) rc = run_forward(e, b, s, &prof);
  if (rc == FF_OK && cudaStreamSynchronize(s) != cudaSuccess) rc = check_launch("ff_engine_profile: sync");
  for (int k = 0; k < FF_PROF_CLASSES; ++k) {
    ms[k] = 0.f;
    if (launches) launches[k] = 0;
  }
  if (rc == FF_OK) {
    for (size_t i = 0; i < prof.cls.size() && 2 * i + 1 < prof.next; ++i) {
      float t = 0.f;
      cudaEventElapsedTime(&t, prof.ev[2 * i], prof.ev[2 * i + 1]);
      ms[prof.cls[i]] += t / static_cast<float>(iters);
      if (launches) launches[prof.cls[i]] += 1;
    }
    if (launches)
      for (int k = 0; k < FF_PROF_CLASSES; ++k) launches[k] /= iters;
  }
  for (auto& ev : prof.ev) cudaEventDestroy(ev);
  return rc;
}

extern "C" int ff_engine_launches_per_forward(const ff_model_config* cfg) {
  return cfg == nullptr ? -1 : launches_per_forward(*cfg);
}

extern "C" int ff_engine_destroy(ff_engine* e) {
  if (e == nullptr) return FF_OK;
  {
    DeviceScope scope(e->device);
    cudaDeviceSynchronize();
    for (auto& kv : e->batches) {
      ff_engine::Batch* b = kv.second;
      for (cudaGraphExec_t x : b->exec)
        if (x) cudaGraphExecDestroy(x);
      if (b->capture_stream) cudaStreamDestroy(b->capture_stream);
      cudaFree(b->block);
      delete b;
    }
    if (e->rope_compact) cudaFree(e->rope_compact);
  }
  delete e;
  return FF_OK;
}
