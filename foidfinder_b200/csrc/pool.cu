// Haruka tree attention pool (foidfinder/backends/mlx/haruka.py:104-136; the model card's MHAttnPool,
// tests/test_haruka.py:73-122): learned queries compete for every token and are gated per token,
//   logits[m, n] = q_m . k_n               (per pool head; 1/sqrt(head_dim) is folded into k)
//   attn[m, n]   = softmax_m(logits[:, n])[m] * sigmoid(logits[m, n] + bias[m])
//   z[m]         = sum_n attn[m, n] v_n
// first for the coarse queries, then for the leaf queries built from the coarse results. The softmax runs
// over the QUERY axis, so a token's weights never need a pass over other tokens: one sweep over the
// tokens suffices and nothing like flash attention's running max is needed.
//
// Kernels (all f32 arithmetic; key/value fp16 from the pool's projection GEMM):
//   slot_attend_kernel  one CTA per (pool head, image): tokens in chunks of 256, a thread per token for
//                       the logits/softmax/gate, then threads per (query, 4 dims) accumulate attn . V from
//                       shared memory; also the per-head attention mass of every query;
//   pool_trunk_kernel   one CTA per image: trunk LayerNorm of the coarse results, leaf queries
//                       LN(z_parent + q_child);
//   pool_leaf_kernel    one CTA per (leaf, image): LN(z_parent + z_child) scaled by mass / (mass + 4),
//                       then the leaf's [dim, leaf_dim] projection, written as the fp16 head input.
#include <cuda_fp16.h>

#include "common.h"
#include "kernels.h"
#include "pool.h"
#include "ptx.cuh"

namespace ff {
namespace {

constexpr int kChunk = 256;  // tokens per sweep step = threads per CTA
constexpr int kMaxQ = 32;

template <int HD, int M>
__global__ void __launch_bounds__(kChunk) slot_attend_kernel(const float* __restrict__ q, int64_t q_img_stride,
                                                             const float* __restrict__ bias,
                                                             const __half* __restrict__ kv, int tokens, int dim,
                                                             float* __restrict__ z, float* __restrict__ mass_part) {
  pdl_wait();
  pdl_trigger();
  static_assert(HD % 8 == 0 && M <= kMaxQ, "head dim must be a multiple of 8");
  constexpr int D4 = HD / 4;
  // v_s [kChunk][HD] | attn_s [M][kChunk] | q_s [M][HD] | red_s [kChunk / 32][M], all f32
  extern __shared__ float4 slot_smem[];
  auto v_s = reinterpret_cast<float(*)[HD]>(slot_smem);
  auto attn_s = reinterpret_cast<float(*)[kChunk]>(reinterpret_cast<float*>(slot_smem) + kChunk * HD);
  auto q_s = reinterpret_cast<float(*)[HD]>(reinterpret_cast<float*>(slot_smem) + kChunk * HD + M * kChunk);
  auto red_s = reinterpret_cast<float(*)[M]>(reinterpret_cast<float*>(slot_smem) + kChunk * HD + M * kChunk + M * HD);

  const int h = blockIdx.x, b = blockIdx.y, heads = gridDim.x;
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  const float* qb = q + static_cast<int64_t>(b) * q_img_stride;
  for (int i = t; i < M * HD; i += kChunk) q_s[i / HD][i % HD] = qb[(i / HD) * dim + h * HD + i % HD];
  float bias_r[M];
#pragma unroll
  for (int m = 0; m < M; ++m) bias_r[m] = bias[m];

  const int om = t / D4, od = (t % D4) * 4;  // this thread's output (query, 4 dims) in phase 2
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  float mass[M];
#pragma unroll
  for (int m = 0; m < M; ++m) mass[m] = 0.f;
  __syncthreads();

  const int64_t row_pitch = 2 * static_cast<int64_t>(dim);
  for (int c0 = 0; c0 < tokens; c0 += kChunk) {
    const int n = c0 + t;
    if (n < tokens) {
      const __half* kr = kv + (static_cast<int64_t>(b) * tokens + n) * row_pitch + h * HD;
      const __half* vr = kr + dim;
      float k[HD];
#pragma unroll
      for (int i = 0; i < HD; i += 8) {
        const uint4 raw = *reinterpret_cast<const uint4*>(kr + i);
        const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float2 f = unpack_half2(w[j]);
          k[i + 2 * j] = f.x;
          k[i + 2 * j + 1] = f.y;
        }
        const uint4 rv = *reinterpret_cast<const uint4*>(vr + i);
        const uint32_t wv[4] = {rv.x, rv.y, rv.z, rv.w};
        float4 lo, hi;
        float2 f0 = unpack_half2(wv[0]), f1 = unpack_half2(wv[1]), f2 = unpack_half2(wv[2]), f3 = unpack_half2(wv[3]);
        lo = make_float4(f0.x, f0.y, f1.x, f1.y);
        hi = make_float4(f2.x, f2.y, f3.x, f3.y);
        *reinterpret_cast<float4*>(&v_s[t][i]) = lo;
        *reinterpret_cast<float4*>(&v_s[t][i + 4]) = hi;
      }
      float l[M];
      float mx = -INFINITY;
#pragma unroll
      for (int m = 0; m < M; ++m) {
        float s = 0.f;
#pragma unroll
        for (int d = 0; d < HD; ++d) s = fmaf(q_s[m][d], k[d], s);
        l[m] = s;
        mx = fmaxf(mx, s);
      }
      float sum = 0.f;
      float e[M];
#pragma unroll
      for (int m = 0; m < M; ++m) {
        e[m] = __expf(l[m] - mx);
        sum += e[m];
      }
      const float inv = 1.f / sum;
#pragma unroll
      for (int m = 0; m < M; ++m) {
        const float gate = 1.f / (1.f + __expf(-(l[m] + bias_r[m])));
        const float a = e[m] * inv * gate;
        attn_s[m][t] = a;
        mass[m] += a;
      }
    } else {
#pragma unroll
      for (int m = 0; m < M; ++m) attn_s[m][t] = 0.f;
#pragma unroll
      for (int i = 0; i < HD; i += 4) *reinterpret_cast<float4*>(&v_s[t][i]) = make_float4(0.f, 0.f, 0.f, 0.f);
    }
    __syncthreads();
    if (om < M) {
      const int rows = min(kChunk, tokens - c0);
#pragma unroll 4
      for (int j = 0; j < rows; ++j) {
        const float a = attn_s[om][j];
        const float4 v = *reinterpret_cast<const float4*>(&v_s[j][od]);
        acc.x = fmaf(a, v.x, acc.x);
        acc.y = fmaf(a, v.y, acc.y);
        acc.z = fmaf(a, v.z, acc.z);
        acc.w = fmaf(a, v.w, acc.w);
      }
    }
    __syncthreads();
  }
  if (om < M) *reinterpret_cast<float4*>(z + (static_cast<int64_t>(b) * M + om) * dim + h * HD + od) = acc;
#pragma unroll
  for (int m = 0; m < M; ++m) {
    const float s = warp_sum(mass[m]);
    if (lane == 0) red_s[warp][m] = s;
  }
  __syncthreads();
  if (t < M) {
    float s = 0.f;
#pragma unroll
    for (int w = 0; w < kChunk / 32; ++w) s += red_s[w][t];
    mass_part[(static_cast<int64_t>(b) * heads + h) * M + t] = s;
  }
}

// Mean and reciprocal standard deviation of a row of `dim` f32 values held across the block (two-pass).
__device__ float2 block_ln_stats(const float* row_s, int dim, float eps, float* red) {
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5, nw = blockDim.x >> 5;
  float s = 0.f;
  for (int i = t; i < dim; i += blockDim.x) s += row_s[i];
  s = warp_sum(s);
  if (lane == 0) red[warp] = s;
  __syncthreads();
  float tot = 0.f;
  for (int w = 0; w < nw; ++w) tot += red[w];
  const float mean = tot / dim;
  __syncthreads();
  float q = 0.f;
  for (int i = t; i < dim; i += blockDim.x) {
    const float d = row_s[i] - mean;
    q += d * d;
  }
  q = warp_sum(q);
  if (lane == 0) red[warp] = q;
  __syncthreads();
  float var = 0.f;
  for (int w = 0; w < nw; ++w) var += red[w];
  __syncthreads();
  return make_float2(mean, rsqrtf(var / dim + eps));
}

// One CTA per image: z_coarse = LN_trunk(z[c]); q_leaf[c * branches + j] = LN_child(z_coarse[c] + q_child[...]).
__global__ void __launch_bounds__(256) pool_trunk_kernel(const float* __restrict__ z, int coarse, int leaves, int dim,
                                                         const float* __restrict__ trunk_w,
                                                         const float* __restrict__ trunk_b,
                                                         const float* __restrict__ q_child,
                                                         const float* __restrict__ child_w,
                                                         const float* __restrict__ child_b, float eps,
                                                         float* __restrict__ z_coarse, float* __restrict__ q_leaf) {
  pdl_wait();
  pdl_trigger();
  extern __shared__ float sm[];
  float* row = sm;         // [dim]
  float* zc = sm + dim;    // [dim]
  float* red = zc + dim;   // [32]
  const int b = blockIdx.x, t = threadIdx.x;
  const int branches = leaves / coarse;
  for (int c = 0; c < coarse; ++c) {
    const float* zr = z + (static_cast<int64_t>(b) * coarse + c) * dim;
    for (int i = t; i < dim; i += blockDim.x) row[i] = zr[i];
    __syncthreads();
    const float2 st = block_ln_stats(row, dim, eps, red);
    float* zco = z_coarse + (static_cast<int64_t>(b) * coarse + c) * dim;
    for (int i = t; i < dim; i += blockDim.x) {
      const float v = (row[i] - st.x) * st.y * trunk_w[i] + trunk_b[i];
      zc[i] = v;
      zco[i] = v;
    }
    __syncthreads();
    for (int j = 0; j < branches; ++j) {
      const int leaf = c * branches + j;
      for (int i = t; i < dim; i += blockDim.x) row[i] = zc[i] + q_child[static_cast<int64_t>(leaf) * dim + i];
      __syncthreads();
      const float2 s2 = block_ln_stats(row, dim, eps, red);
      float* ql = q_leaf + (static_cast<int64_t>(b) * leaves + leaf) * dim;
      for (int i = t; i < dim; i += blockDim.x) ql[i] = (row[i] - s2.x) * s2.y * child_w[i] + child_b[i];
      __syncthreads();
    }
  }
}

// One CTA per (leaf, image): z_tree = LN_leaf(z_coarse[parent] + z_child[leaf]) * mass / (mass + 4);
// out[b, leaf * L + f] = fp16(sum_d z_tree[d] * leaf_w[leaf, d, f] + leaf_b[leaf, f]).
__global__ void __launch_bounds__(256) pool_leaf_kernel(const float* __restrict__ z_coarse,
                                                        const float* __restrict__ z_child,
                                                        const float* __restrict__ mass_part, int coarse, int leaves,
                                                        int heads, int dim, int leaf_dim,
                                                        const float* __restrict__ leaf_nw,
                                                        const float* __restrict__ leaf_nb, float eps,
                                                        const float* __restrict__ leaf_w,
                                                        const float* __restrict__ leaf_b, __half* __restrict__ out,
                                                        int ld_out) {
  pdl_wait();
  pdl_trigger();
  extern __shared__ float sm[];
  float* row = sm;        // [dim]
  float* red = sm + dim;  // [32]
  float* part = red + 32; // [blockDim.x]
  const int leaf = blockIdx.x, b = blockIdx.y, t = threadIdx.x;
  const int parent = leaf / (leaves / coarse);
  const float* zc = z_coarse + (static_cast<int64_t>(b) * coarse + parent) * dim;
  const float* zl = z_child + (static_cast<int64_t>(b) * leaves + leaf) * dim;
  for (int i = t; i < dim; i += blockDim.x) row[i] = zc[i] + zl[i];
  float mass = 0.f;
  for (int h = 0; h < heads; ++h) mass += mass_part[(static_cast<int64_t>(b) * heads + h) * leaves + leaf];
  mass /= heads;
  const float gate = mass / (mass + 4.f);
  __syncthreads();
  const float2 st = block_ln_stats(row, dim, eps, red);
  for (int i = t; i < dim; i += blockDim.x) row[i] = ((row[i] - st.x) * st.y * leaf_nw[i] + leaf_nb[i]) * gate;
  __syncthreads();
  // leaf_dim outputs x (blockDim / leaf_dim) slices of the dim axis, then a shared-memory sum.
  const int f = t % leaf_dim, slices = blockDim.x / leaf_dim, sl = t / leaf_dim;
  const float* w = leaf_w + static_cast<int64_t>(leaf) * dim * leaf_dim;
  float s = 0.f;
  if (sl < slices)
    for (int d = sl; d < dim; d += slices) s = fmaf(row[d], w[static_cast<int64_t>(d) * leaf_dim + f], s);
  part[t] = s;
  __syncthreads();
  if (t < leaf_dim) {
    float tot = leaf_b[static_cast<int64_t>(leaf) * leaf_dim + t];
    for (int k = 0; k < slices; ++k) tot += part[k * leaf_dim + t];
    out[static_cast<int64_t>(b) * ld_out + leaf * leaf_dim + t] = __float2half_rn(tot);
  }
}

template <int HD, int M>
constexpr size_t slot_smem_bytes() {
  return sizeof(float) * (kChunk * HD + M * kChunk + M * HD + (kChunk / 32) * M);
}

template <int HD, int M>
int slot_launch(const float* q, int64_t q_stride, const float* bias, const __half* kv, int B, int tokens, int dim,
                int heads, float* z, float* mass, cudaStream_t s) {
  constexpr size_t smem = slot_smem_bytes<HD, M>();
  static bool configured[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64 || !configured[dev]) {
    if (cudaFuncSetAttribute(slot_attend_kernel<HD, M>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(smem)) != cudaSuccess)
      return check_launch("slot_attend_kernel: cudaFuncSetAttribute");
    if (dev >= 0 && dev < 64) configured[dev] = true;
  }
  launch(slot_attend_kernel<HD, M>, dim3(dim3(heads, B)), dim3(kChunk), smem, s, q, q_stride, bias, kv, tokens, dim, z, mass);
  return check_launch("slot_attend_kernel");
}

// PixAI attention-pool head (foidfinder/backends/cuda/reference.py:133-140): one learned query per head
// attends over all tokens of an image. One CTA per (head, image); each quarter-warp (8 lanes x 8 dims =
// one 128-byte key/value row) walks a share of the tokens with its own online softmax, four rows in
// flight, and the 40 partial (max, sum, output) triples are merged through shared memory.
constexpr int kPqThreads = 320;
__global__ void __launch_bounds__(kPqThreads) pool_query_kernel(const float* __restrict__ q, const __half* __restrict__ kv,
                                                               int tokens, int dim, __half* __restrict__ out) {
  pdl_wait();
  pdl_trigger();
  constexpr int HD = 64, NQ = kPqThreads / 8, UNR = 4;
  __shared__ float part_m[NQ], part_l[NQ];
  __shared__ float part_o[NQ][HD];
  const int h = blockIdx.x, b = blockIdx.y, t = threadIdx.x, qw = t >> 3, ql = t & 7;
  const unsigned qmask = 0xFFu << (t & 24);
  float qr[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) qr[e] = q[h * HD + 8 * ql + e] * 1.4426950408889634f;  // log2 units
  const size_t row0 = static_cast<size_t>(b) * tokens;
  float m = -INFINITY, l = 0.f, o[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) o[e] = 0.f;
  for (int k0 = qw; k0 < tokens; k0 += NQ * UNR) {
    uint4 kr[UNR], vr[UNR];
#pragma unroll
    for (int i = 0; i < UNR; ++i) {
      const int key = k0 + i * NQ;
      if (key < tokens) {
        const __half* base = kv + (row0 + key) * 2 * dim + h * HD;
        kr[i] = __ldg(reinterpret_cast<const uint4*>(base) + ql);
        vr[i] = __ldg(reinterpret_cast<const uint4*>(base + dim) + ql);
      }
    }
#pragma unroll
    for (int i = 0; i < UNR; ++i) {
      if (k0 + i * NQ >= tokens) break;  // uniform within the quarter-warp
      const uint32_t kw[4] = {kr[i].x, kr[i].y, kr[i].z, kr[i].w};
      float sc = 0.f;
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 f = unpack_half2(kw[e]);
        sc = fmaf(qr[2 * e], f.x, fmaf(qr[2 * e + 1], f.y, sc));
      }
      sc += __shfl_xor_sync(qmask, sc, 1, 8);
      sc += __shfl_xor_sync(qmask, sc, 2, 8);
      sc += __shfl_xor_sync(qmask, sc, 4, 8);
      const float m_new = fmaxf(m, sc);
      const float corr = ex2_approx(m - m_new);
      const float pk = ex2_approx(sc - m_new);
      m = m_new;
      l = l * corr + pk;
      const uint32_t vw[4] = {vr[i].x, vr[i].y, vr[i].z, vr[i].w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 f = unpack_half2(vw[e]);
        o[2 * e] = fmaf(pk, f.x, o[2 * e] * corr);
        o[2 * e + 1] = fmaf(pk, f.y, o[2 * e + 1] * corr);
      }
    }
  }
  if (ql == 0) {
    part_m[qw] = m;
    part_l[qw] = l;
  }
#pragma unroll
  for (int e = 0; e < 8; ++e) part_o[qw][8 * ql + e] = o[e];
  __syncthreads();
  if (t < HD) {
    float mm = -INFINITY;
    for (int i = 0; i < NQ; ++i) mm = fmaxf(mm, part_m[i]);
    float ll = 0.f, acc = 0.f;
    for (int i = 0; i < NQ; ++i) {
      const float w = part_m[i] == -INFINITY ? 0.f : ex2_approx(part_m[i] - mm);
      ll = fmaf(part_l[i], w, ll);
      acc = fmaf(part_o[i][t], w, acc);
    }
    out[static_cast<size_t>(b) * dim + h * HD + t] = __float2half_rn(acc / ll);
  }
}

template <int HD>
int slot_dispatch(int M, const float* q, int64_t q_stride, const float* bias, const __half* kv, int B, int tokens,
                  int dim, int heads, float* z, float* mass, cudaStream_t s) {
  switch (M) {
    case 6: return slot_launch<HD, 6>(q, q_stride, bias, kv, B, tokens, dim, heads, z, mass, s);
    case 18: return slot_launch<HD, 18>(q, q_stride, bias, kv, B, tokens, dim, heads, z, mass, s);
  }
  set_error("pool: %d queries (supported: 6, 18)", M);
  return FF_ERR_INVALID_ARGUMENT;
}

}  // namespace

int slot_attend(const float* q, int64_t q_img_stride, const float* bias, int M, const void* kv, int B, int tokens,
                int dim, int heads, float* z, float* mass_part, cudaStream_t s) {
  FF_REQUIRE(q && bias && kv && z && mass_part, "pool: NULL pointer");
  FF_REQUIRE(heads >= 1 && dim % heads == 0 && B >= 0 && tokens >= 1, "pool: bad shape");
  FF_REQUIRE(aligned16(kv) && aligned16(z) && dim % 8 == 0, "pool: key/value and z must be 16-byte aligned");
  if (B == 0) return FF_OK;
  const __half* kvh = static_cast<const __half*>(kv);
  switch (dim / heads) {
    case 48: return slot_dispatch<48>(M, q, q_img_stride, bias, kvh, B, tokens, dim, heads, z, mass_part, s);
    case 64: return slot_dispatch<64>(M, q, q_img_stride, bias, kvh, B, tokens, dim, heads, z, mass_part, s);
  }
  set_error("pool: head dim %d (supported: 48, 64)", dim / heads);
  return FF_ERR_INVALID_ARGUMENT;
}

int pool_query_attention(const float* q, const void* kv, int B, int tokens, int heads, void* out, cudaStream_t s) {
  FF_REQUIRE(q && kv && out && heads >= 1 && tokens >= 1, "pool query: bad arguments");
  FF_REQUIRE(aligned16(kv), "pool query: key/value must be 16-byte aligned");
  if (B == 0) return FF_OK;
  launch(pool_query_kernel, dim3(dim3(heads, B)), dim3(kPqThreads), 0, s, q, static_cast<const __half*>(kv), tokens, heads * 64,
                                                          static_cast<__half*>(out));
  return check_launch("pool_query_kernel");
}

int pool_trunk(const float* z, int B, int coarse, int leaves, int dim, const float* trunk_w, const float* trunk_b,
               const float* q_child, const float* child_w, const float* child_b, float eps, float* z_coarse,
               float* q_leaf, cudaStream_t s) {
  FF_REQUIRE(coarse >= 1 && leaves % coarse == 0 && dim >= 1, "pool: %d leaves over %d coarse queries", leaves, coarse);
  if (B == 0) return FF_OK;
  launch(pool_trunk_kernel, dim3(B), dim3(256), (2 * dim + 32) * sizeof(float), s, z, coarse, leaves, dim, trunk_w, trunk_b, q_child,
                                                                    child_w, child_b, eps, z_coarse, q_leaf);
  return check_launch("pool_trunk_kernel");
}

int pool_leaf(const float* z_coarse, const float* z_child, const float* mass_part, int B, int coarse, int leaves,
              int heads, int dim, int leaf_dim, const float* leaf_nw, const float* leaf_nb, float eps,
              const float* leaf_w, const float* leaf_b, void* out, int ld_out, cudaStream_t s) {
  FF_REQUIRE(leaf_dim >= 1 && leaf_dim <= 256 && 256 % leaf_dim == 0, "pool: leaf dim %d must divide 256", leaf_dim);
  FF_REQUIRE(ld_out >= leaves * leaf_dim, "pool: head input stride %d", ld_out);
  if (B == 0) return FF_OK;
  launch(pool_leaf_kernel, dim3(dim3(leaves, B)), dim3(256), (dim + 32 + 256) * sizeof(float), s, z_coarse, z_child, mass_part, coarse, leaves, heads, dim, leaf_dim, leaf_nw, leaf_nb, eps, leaf_w, leaf_b,
      static_cast<__half*>(out), ld_out);
  return check_launch("pool_leaf_kernel");
}

}  // namespace ff

// ---------------------------------------------------------------- orchestration

namespace ff {
namespace {
size_t up256(size_t v) { return (v + 255) / 256 * 256; }
}  // namespace

size_t pool_small_bytes(const ff_model_config& c, int B) {
  const size_t b = static_cast<size_t>(B), D = c.dim;
  return up256(b * c.leaf_queries * D * 4) + up256(b * c.coarse_queries * D * 4) + 2 * up256(b * c.leaf_queries * D * 4) +
         up256(b * c.pool_heads * c.coarse_queries * 4) + up256(b * c.pool_heads * c.leaf_queries * 4);
}

void pool_carve_small(const ff_model_config& c, int B, void* base, PoolBuffers* pb) {
  const size_t b = static_cast<size_t>(B), D = c.dim;
  auto* p = static_cast<uint8_t*>(base);
  auto take = [&](size_t bytes) {
    float* at = reinterpret_cast<float*>(p);
    p += up256(bytes);
    return at;
  };
  pb->z = take(b * c.leaf_queries * D * 4);
  pb->z_coarse = take(b * c.coarse_queries * D * 4);
  pb->q_leaf = take(b * c.leaf_queries * D * 4);
  pb->z_child = take(b * c.leaf_queries * D * 4);
  pb->mass_c = take(b * c.pool_heads * c.coarse_queries * 4);
  pb->mass_l = take(b * c.pool_heads * c.leaf_queries * 4);
}

int pool_validate(const ff_model_config& c, const ff_model_weights& w) {
  FF_REQUIRE(c.pool_heads >= 1 && c.dim % c.pool_heads == 0 &&
                 (c.dim / c.pool_heads == 48 || c.dim / c.pool_heads == 64),
             "tree pool: dim %d / pool_heads %d must be 48 or 64", c.dim, c.pool_heads);
  FF_REQUIRE(c.coarse_queries == 6 && c.leaf_queries == 18, "tree pool: %d coarse / %d leaf queries (supported: 6 / 18)",
             c.coarse_queries, c.leaf_queries);
  FF_REQUIRE(c.leaf_dim >= 1 && 256 % c.leaf_dim == 0 && (c.leaf_queries * c.leaf_dim) % 64 == 0,
             "tree pool: leaf_dim %d", c.leaf_dim);
  FF_REQUIRE(w.pool_norm_w && w.pool_norm_b && w.pool_kv_w && w.pool_kv_b && w.q_coarse && w.q_coarse_bias &&
                 w.q_child && w.q_child_bias && w.trunk_norm_w && w.trunk_norm_b && w.child_q_norm_w &&
                 w.child_q_norm_b && w.leaf_norm_w && w.leaf_norm_b && w.leaf_w && w.leaf_b && w.norm_w && w.norm_b,
             "tree pool: a pool weight pointer is NULL");
  return FF_OK;
}

int pool_prepare(const ff_model_config& c, const ff_model_weights& w, int B, int tokens, const PoolBuffers& pb,
                 GemmPlan* kv_plan) {
  GemmProblem p{};
  p.A = pb.xn;
  p.W = w.pool_kv_w;
  p.out = pb.kv;
  p.M = B * tokens;
  p.N = 2 * c.dim;
  p.K = c.dim;
  p.epi = EPI_BIAS;
  p.f16 = true;
  p.args.bias = w.pool_kv_b;
  p.args.ldo = 2 * c.dim;
  return gemm_prepare(p, kv_plan);
}

int pool_run(const ff_model_config& c, const ff_model_weights& w, const __half* x, int B, int tokens,
             const PoolBuffers& pb, const GemmPlan& kv_plan, __half* leaf_out, cudaStream_t s) {
  const int M = B * tokens, D = c.dim, C = c.coarse_queries, Qn = c.leaf_queries;
  int rc = layernorm(x, D, w.norm_w, w.norm_b, c.ln_eps, M, D, pb.xf, s);
  if (rc == FF_OK) rc = layernorm(pb.xf, D, w.pool_norm_w, w.pool_norm_b, c.ln_eps, M, D, pb.xn, s);
  if (rc == FF_OK) rc = gemm_launch(kv_plan, s);
  if (rc == FF_OK) rc = slot_attend(w.q_coarse, 0, w.q_coarse_bias, C, pb.kv, B, tokens, D, c.pool_heads, pb.z, pb.mass_c, s);
  if (rc == FF_OK)
    rc = pool_trunk(pb.z, B, C, Qn, D, w.trunk_norm_w, w.trunk_norm_b, w.q_child, w.child_q_norm_w, w.child_q_norm_b,
                    c.ln_eps, pb.z_coarse, pb.q_leaf, s);
  if (rc == FF_OK)
    rc = slot_attend(pb.q_leaf, static_cast<int64_t>(Qn) * D, w.q_child_bias, Qn, pb.kv, B, tokens, D, c.pool_heads,
                     pb.z_child, pb.mass_l, s);
  if (rc == FF_OK)
    rc = pool_leaf(pb.z_coarse, pb.z_child, pb.mass_l, B, C, Qn, c.pool_heads, D, c.leaf_dim, w.leaf_norm_w,
                   w.leaf_norm_b, c.ln_eps, w.leaf_w, w.leaf_b, leaf_out, Qn * c.leaf_dim, s);
  return rc;
}

}  // namespace ff

using namespace ff;

extern "C" int ff_pool_query_attention(const float* q, const uint16_t* kv, int B, int tokens, int heads,
                                       uint16_t* out, void* stream) {
  return pool_query_attention(q, kv, B, tokens, heads, out, static_cast<cudaStream_t>(stream));
}

extern "C" int64_t ff_tree_pool_workspace_bytes(const ff_model_config* cfg, int B) {
  if (cfg == nullptr || B < 1) return -1;
  const int64_t T = static_cast<int64_t>(cfg->image_size / cfg->patch) * (cfg->image_size / cfg->patch) + 1;
  const int64_t M = T * B, D = cfg->dim;
  return static_cast<int64_t>(up256(M * D * 2)) * 2 + static_cast<int64_t>(up256(M * 2 * D * 2)) +
         static_cast<int64_t>(pool_small_bytes(*cfg, B));
}

extern "C" int ff_tree_pool(const ff_model_config* cfg, const ff_model_weights* w, const uint16_t* x, int B,
                            void* workspace, int64_t workspace_bytes, uint16_t* leaf_out, void* stream) {
  FF_REQUIRE(cfg && w && x && workspace && leaf_out && B >= 1, "ff_tree_pool: NULL argument or B < 1");
  FF_REQUIRE(cfg->head_kind == FF_HEAD_TREE, "ff_tree_pool: config head_kind is not FF_HEAD_TREE");
  int rc = pool_validate(*cfg, *w);
  if (rc != FF_OK) return rc;
  const int64_t need = ff_tree_pool_workspace_bytes(cfg, B);
  FF_REQUIRE(workspace_bytes >= need, "ff_tree_pool: workspace of %lld bytes, %lld needed",
             static_cast<long long>(workspace_bytes), static_cast<long long>(need));
  FF_REQUIRE(aligned16(x) && (reinterpret_cast<uintptr_t>(workspace) & 255u) == 0 && aligned16(leaf_out),
             "ff_tree_pool: x and leaf_out must be 16-byte aligned, workspace 256-byte aligned");
  const int tokens = (cfg->image_size / cfg->patch) * (cfg->image_size / cfg->patch) + 1;
  const size_t M = static_cast<size_t>(tokens) * B, D = cfg->dim;
  auto* p = static_cast<uint8_t*>(workspace);
  PoolBuffers pb;
  pb.xf = reinterpret_cast<__half*>(p);
  p += up256(M * D * 2);
  pb.xn = reinterpret_cast<__half*>(p);
  p += up256(M * D * 2);
  pb.kv = reinterpret_cast<__half*>(p);
  p += up256(M * 2 * D * 2);
  pool_carve_small(*cfg, B, p, &pb);
  GemmPlan kv;
  rc = pool_prepare(*cfg, *w, B, tokens, pb, &kv);
  if (rc != FF_OK) return rc;
  return pool_run(*cfg, *w, reinterpret_cast<const __half*>(x), B, tokens, pb, kv, reinterpret_cast<__half*>(leaf_out),
                  static_cast<cudaStream_t>(stream));
}
