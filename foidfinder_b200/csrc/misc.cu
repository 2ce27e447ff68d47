// Stem input preparation, the final LayerNorm and the device top-k of the tag logits.
#include "common.h"
#include "kernels.h"
#include "ptx.cuh"

namespace ff {

// ---------------------------------------------------------------- patchify
// images [B, S, S, 3] -> patches [B * G * G, k_pad] fp16, column k = (kh * p + kw) * 3 + c (the (kh, kw, c)
// order of reference.py:103-107 and mlx/haruka.py:78). uint8 pixels become (px / 255 - mean) / std; fp16
// pixels are already normalised (PixAICuda's input, engine.py:163-165) and are copied as they are.
// Patch rows in row-major grid order, or (win > 0) window order: the grid cut into win x win windows,
// windows row-major, patches row-major inside each (foidfinder/backends/cuda/reference.py:21-24, 103-107).
__device__ __forceinline__ float pixel_value(uint8_t u, float mean, float istd) {
  return __fmul_rn(__fmaf_rn(static_cast<float>(u), 1.f / 255.f, -mean), istd);  // one rounding per step
}
__device__ __forceinline__ float pixel_value(__half h, float, float) { return __half2float(h); }

template <typename Px>
__global__ void patchify_kernel(const Px* __restrict__ img, int B, int S, int p, float m0, float m1, float m2,
                                float is0, float is1, float is2, __half* __restrict__ out, int k_pad, int win) {
  pdl_wait();
  pdl_trigger();
  const int G = S / p, P = G * G, kreal = p * p * 3;
  const int nw = win > 0 ? G / win : 1;
  const int64_t total = static_cast<int64_t>(B) * P * k_pad;
  for (int64_t t = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; t < total;
       t += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int k = static_cast<int>(t % k_pad);
    const int64_t row = t / k_pad;
    float v = 0.f;
    if (k < kreal) {
      const int b = static_cast<int>(row / P), pi = static_cast<int>(row % P);
      int py = pi / G, px = pi % G;
      if (win > 0) {
        const int w = pi / (win * win), r = (pi / win) % win, c = pi % win;
        py = (w / nw) * win + r;
        px = (w % nw) * win + c;
      }
      const int kh = k / (p * 3), rem = k % (p * 3);
      const int y = py * p + kh;
      const int c = rem % 3;
      const Px u = img[(static_cast<int64_t>(b) * S + y) * S * 3 + static_cast<int64_t>(px) * p * 3 + rem];
      const float mean = c == 0 ? m0 : (c == 1 ? m1 : m2);
      const float istd = c == 0 ? is0 : (c == 1 ? is1 : is2);
      v = pixel_value(u, mean, istd);
    }
    out[t] = __float2half_rn(v);
  }
}

__global__ void fill_cls_kernel(const __half* __restrict__ cls, __half* __restrict__ x, int B, int tokens, int dim) {
  pdl_wait();
  pdl_trigger();
  const int b = blockIdx.x;
  for (int c = threadIdx.x; c < dim; c += blockDim.x) x[static_cast<size_t>(b) * tokens * dim + c] = cls[c];
}

// ---------------------------------------------------------------- LayerNorm (one warp per row)
// LayerNorm of fp16 rows (f32 statistics) to fp16; with `pos`, the fp16 row pos[row % period] is added to
// the fp16 result (the PixAI attention pool's LN + position embedding, reference.py:135).
__global__ void layernorm_kernel(const __half* __restrict__ x, int64_t stride, const float* __restrict__ g,
                                 const float* __restrict__ b, float eps, int rows, int cols, __half* __restrict__ out,
                                 const __half* __restrict__ pos, int period) {
  pdl_wait();
  pdl_trigger();
  const int lane = threadIdx.x & 31;
  const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (row >= rows) return;
  const __half* xr = x + row * stride;
  float s = 0.f;
  for (int c = lane; c < cols; c += 32) s += __half2float(xr[c]);
  const float mean = warp_sum(s) / static_cast<float>(cols);
  float q = 0.f;
  for (int c = lane; c < cols; c += 32) {
    const float d = __half2float(xr[c]) - mean;
    q += d * d;
  }
  const float rstd = rsqrtf(warp_sum(q) / static_cast<float>(cols) + eps);
  __half* orow = out + static_cast<size_t>(row) * cols;
  const __half* prow = pos != nullptr ? pos + static_cast<size_t>(row % period) * cols : nullptr;
  for (int c = lane; c < cols; c += 32) {
    __half y = __float2half_rn((__half2float(xr[c]) - mean) * rstd * g[c] + b[c]);
    if (prow != nullptr) y = __float2half_rn(__half2float(y) + __half2float(prow[c]));
    orow[c] = y;
  }
}

// ---------------------------------------------------------------- top-k per row
// One CTA per row. The row's keys (order-preserving uint32 of the f32 logits) are staged in shared
// memory, a 4-pass 8-bit radix select finds the k-th largest key, then the winners are gathered
// (ties at the threshold taken in index order) and ranked by (value desc, index asc).
constexpr int kTopkThreads = 1024;
constexpr int kTopkMax = 64;

__device__ __forceinline__ uint32_t order_key(float f) {
  const uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// STAGED: the row's keys live in shared memory; otherwise (rows too long for it) every pass re-reads
// the logits, which stay in L2.
template <bool STAGED>
__global__ void __launch_bounds__(kTopkThreads) topk_kernel(const float* __restrict__ logits, int n, int k,
                                                            int32_t* __restrict__ idx_out, float* __restrict__ val_out) {
  pdl_wait();
  pdl_trigger();
  extern __shared__ uint32_t keys_smem[];  // [n] when STAGED
  __shared__ uint32_t hist[256];
  __shared__ uint32_t s_prefix, s_remaining;
  __shared__ uint32_t s_sel_key[kTopkMax];
  __shared__ int s_sel_idx[kTopkMax];
  __shared__ int s_count_gt, s_warp_ties[kTopkThreads / 32];
  const int row = blockIdx.x, tid = threadIdx.x;
  const float* lr = logits + static_cast<size_t>(row) * n;
  auto key_at = [&](int i) { return STAGED ? keys_smem[i] : order_key(lr[i]); };
  if constexpr (STAGED)
    for (int i = tid; i < n; i += kTopkThreads) keys_smem[i] = order_key(lr[i]);
  if (tid == 0) {
    s_prefix = 0;
    s_remaining = static_cast<uint32_t>(k);
    s_count_gt = 0;
  }
  __syncthreads();
  for (int shift = 24; shift >= 0; shift -= 8) {
    for (int i = tid; i < 256; i += kTopkThreads) hist[i] = 0;
    __syncthreads();
    const uint32_t prefix = s_prefix;
    const uint32_t hmask = shift == 24 ? 0u : (0xffffffffu << (shift + 8));
    for (int i = tid; i < n; i += kTopkThreads) {
      const uint32_t key = key_at(i);
      if ((key & hmask) == (prefix & hmask)) atomicAdd(&hist[(key >> shift) & 0xffu], 1u);
    }
    __syncthreads();
    if (tid == 0) {
      uint32_t rem = s_remaining, cum = 0;
      int d = 255;
      for (; d > 0; --d) {
        if (cum + hist[d] >= rem) break;
        cum += hist[d];
      }
      s_prefix = prefix | (static_cast<uint32_t>(d) << shift);
      s_remaining = rem - cum;
    }
    __syncthreads();
  }
  const uint32_t thr = s_prefix;
  const uint32_t ties_needed = s_remaining;  // how many keys equal to thr are taken
  // Gather: keys > thr (unordered), and the first `ties_needed` keys == thr in index order. Each thread
  // owns a contiguous index range so a block scan of tie counts preserves index order.
  const int per = (n + kTopkThreads - 1) / kTopkThreads;
  const int lo = tid * per, hi = min(n, lo + per);
  int my_ties = 0;
  for (int i = lo; i < hi; ++i) my_ties += key_at(i) == thr;
  // exclusive scan of my_ties over the block
  const int lane = tid & 31, warp = tid >> 5;
  int incl = my_ties;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int t = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += t;
  }
  if (lane == 31) s_warp_ties[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    int w = lane < kTopkThreads / 32 ? s_warp_ties[lane] : 0;
    int wi = w;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int t = __shfl_up_sync(0xffffffffu, wi, o);
      if (lane >= o) wi += t;
    }
    if (lane < kTopkThreads / 32) s_warp_ties[lane] = wi - w;  // exclusive warp offsets
  }
  __syncthreads();
  int tie_rank = s_warp_ties[warp] + incl - my_ties;
  const int n_gt = k - static_cast<int>(ties_needed);
  for (int i = lo; i < hi; ++i) {
    const uint32_t key = key_at(i);
    if (key > thr) {
      const int slot = atomicAdd(&s_count_gt, 1);
      s_sel_key[slot] = key;
      s_sel_idx[slot] = i;
    } else if (key == thr) {
      if (tie_rank < static_cast<int>(ties_needed)) {
        s_sel_key[n_gt + tie_rank] = key;
        s_sel_idx[n_gt + tie_rank] = i;
      }
      ++tie_rank;
    }
  }
  __syncthreads();
  if (tid < k) {
    const uint32_t mk = s_sel_key[tid];
    const int mi = s_sel_idx[tid];
    int rank = 0;
    for (int j = 0; j < k; ++j) {
      const uint32_t ok = s_sel_key[j];
      const int oi = s_sel_idx[j];
      rank += (ok > mk) || (ok == mk && oi < mi);
    }
    idx_out[static_cast<size_t>(row) * k + rank] = mi;
    if (val_out != nullptr) val_out[static_cast<size_t>(row) * k + rank] = lr[mi];
  }
}

int topk(const float* logits, int B, int n, int k, int32_t* idx, float* val, cudaStream_t s) {
  FF_REQUIRE(logits && idx, "ff_topk: NULL pointer");
  FF_REQUIRE(k >= 1 && k <= kTopkMax && n >= k, "ff_topk: need 1 <= k <= %d and k <= n (k=%d n=%d)", kTopkMax, k, n);
  const size_t smem = static_cast<size_t>(n) * sizeof(uint32_t);
  if (B == 0) return FF_OK;
  if (smem > 200 * 1024) {
    launch(topk_kernel<false>, dim3(B), dim3(kTopkThreads), 0, s, logits, n, k, idx, val);
    return check_launch("topk_kernel");
  }
  static bool configured[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64 || !configured[dev]) {
    if (cudaFuncSetAttribute(topk_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024) != cudaSuccess)
      return check_launch("ff_topk: cudaFuncSetAttribute");
    if (dev >= 0 && dev < 64) configured[dev] = true;
  }
  launch(topk_kernel<true>, dim3(B), dim3(kTopkThreads), smem, s, logits, n, k, idx, val);
  return check_launch("topk_kernel");
}

int patchify(const void* img, int B, int S, int p, const float* mean, const float* stdv, void* out, int k_pad,
             cudaStream_t s, int win, bool f16_pixels) {
  FF_REQUIRE(img && out && mean && stdv, "ff_patchify: NULL pointer");
  FF_REQUIRE(p >= 1 && S % p == 0 && k_pad >= p * p * 3, "ff_patchify: bad geometry S=%d p=%d k_pad=%d", S, p, k_pad);
  FF_REQUIRE(win >= 0 && (win == 0 || (S / p) % win == 0), "ff_patchify: window %d does not tile the %d-patch grid",
             win, S / p);
  if (B == 0) return FF_OK;
  const int64_t total = static_cast<int64_t>(B) * (S / p) * (S / p) * k_pad;
  const int grid = static_cast<int>(std::min<int64_t>((total + 255) / 256, 148 * 16));
  if (f16_pixels)
    launch(patchify_kernel<__half>, dim3(grid), dim3(256), 0, s, static_cast<const __half*>(img), B, S, p, 0.f, 0.f, 0.f, 1.f, 1.f,
                                                 1.f, static_cast<__half*>(out), k_pad, win);
  else
    launch(patchify_kernel<uint8_t>, dim3(grid), dim3(256), 0, s, static_cast<const uint8_t*>(img), B, S, p, mean[0], mean[1],
                                                  mean[2], 1.f / stdv[0], 1.f / stdv[1], 1.f / stdv[2],
                                                  static_cast<__half*>(out), k_pad, win);
  return check_launch("patchify_kernel");
}

int fill_cls(const void* cls, void* x, int B, int tokens, int dim, cudaStream_t s) {
  FF_REQUIRE(cls && x && tokens >= 1 && dim >= 1, "ff_fill_cls: bad arguments");
  if (B == 0) return FF_OK;
  launch(fill_cls_kernel, dim3(B), dim3(256), 0, s, static_cast<const __half*>(cls), static_cast<__half*>(x), B, tokens, dim);
  return check_launch("fill_cls_kernel");
}

int layernorm(const void* x, int64_t stride, const float* g, const float* b, float eps, int rows, int cols, void* out,
              cudaStream_t s, const void* pos, int period) {
  FF_REQUIRE(x && g && b && out && cols >= 1 && stride >= cols, "ff_layernorm: bad arguments");
  FF_REQUIRE(pos == nullptr || period >= 1, "ff_layernorm: position rows need a period");
  if (rows == 0) return FF_OK;
  launch(layernorm_kernel, dim3((rows + 7) / 8), dim3(256), 0, s, static_cast<const __half*>(x), stride, g, b, eps, rows, cols,
                                                  static_cast<__half*>(out), static_cast<const __half*>(pos), period);
  return check_launch("layernorm_kernel");
}

}  // namespace ff

extern "C" int ff_patchify(const uint8_t* images, int B, int image_size, int patch, const float* mean3,
                           const float* std3, uint16_t* patches, int k_pad, void* stream) {
  return ff::patchify(images, B, image_size, patch, mean3, std3, patches, k_pad, static_cast<cudaStream_t>(stream));
}

extern "C" int ff_fill_cls(const uint16_t* cls_row, uint16_t* x, int B, int tokens, int dim, void* stream) {
  return ff::fill_cls(cls_row, x, B, tokens, dim, static_cast<cudaStream_t>(stream));
}

extern "C" int ff_patchify_windowed(const uint8_t* images, int B, int image_size, int patch, const float* mean3,
                                    const float* std3, uint16_t* patches, int k_pad, int window, void* stream) {
  return ff::patchify(images, B, image_size, patch, mean3, std3, patches, k_pad, static_cast<cudaStream_t>(stream),
                      window);
}

extern "C" int ff_layernorm_pos(const uint16_t* x, int64_t row_stride, const float* gamma, const float* beta, float eps,
                                int rows, int cols, const uint16_t* pos, int period, uint16_t* out, void* stream) {
  return ff::layernorm(x, row_stride, gamma, beta, eps, rows, cols, out, static_cast<cudaStream_t>(stream), pos, period);
}

extern "C" int ff_layernorm(const uint16_t* x, int64_t row_stride, const float* gamma, const float* beta, float eps,
                            int rows, int cols, uint16_t* out, void* stream) {
  return ff::layernorm(x, row_stride, gamma, beta, eps, rows, cols, out, static_cast<cudaStream_t>(stream));
}

extern "C" int ff_topk(const float* logits, int B, int n, int k, int32_t* idx_out, float* val_out, void* stream) {
  return ff::topk(logits, B, n, k, idx_out, val_out, static_cast<cudaStream_t>(stream));
}
