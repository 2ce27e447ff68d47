// Non-causal flash attention, head dim 64, on the packed QKV activations [tokens, 3 * heads * 64] fp16.
// Follows the reference's attention (foidfinder/backends/cuda/csrc/attention.cuh:19-157) in what it
// computes, but accumulates S = Q K^T and O = P V in f32 (the reference uses f16 partials) and masks
// ragged tails, so any sequence length works (EVA02 at 448 px has 1025 tokens: 1024 patches + class).
//
// One CTA = 128 query rows of one head of one sequence (8 warps x 16 rows); K/V tiles of 64 keys are
// double-buffered through cp.async into 128-byte-swizzled shared memory. Softmax is online in base 2
// with f32 running max / normaliser. Optional 2-D RoPE (interleaved pairs, table [seq_len, 32]) is
// applied to the Q and K tiles in shared memory right after they land, for callers whose q/k are not
// rotated yet (the QKV GEMM epilogue already rotates them in the engine).
#include "common.h"
#include "kernels.h"
#include "ptx.cuh"

namespace ff {

namespace attn {
constexpr int D = 64, BQ = 128, BKV = 64, WARPS = 8, THREADS = WARPS * 32;
constexpr int SMEM = (BQ + 4 * BKV) * 128;  // Q + 2 x K + 2 x V, 128 bytes per row

__device__ __forceinline__ uint32_t swz(int row, int chunk) { return row * 128 + ((chunk ^ (row & 7)) << 4); }

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool pred) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(dst), "l"(src), "r"(pred ? 16 : 0));
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N>
__device__ __forceinline__ void cp_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N));
}
__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
// D (f32) += A (f16, 16x16 row) * B (f16, 16x8 col)
__device__ __forceinline__ void mma_f32(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Rotates `rows` rows (64 halves each, swizzled) of a tile in shared memory whose first row is
// sequence position pos0; rows at or beyond seq_len are left alone.
__device__ __forceinline__ void rope_tile(uint8_t* base, int rows, int pos0, int seq_len, const float* cos_t,
                                          const float* sin_t) {
  for (int i = threadIdx.x; i < rows * 32; i += THREADS) {
    const int r = i >> 5, pair = i & 31, pos = pos0 + r;
    if (pos >= seq_len) continue;
    const int col = pair * 2;
    __half2* p = reinterpret_cast<__half2*>(base + swz(r, col >> 3) + (col & 7) * 2);
    const float2 v = __half22float2(*p);
    const float c = cos_t[pos * 32 + pair], s = sin_t[pos * 32 + pair];
    *p = __floats2half2_rn(v.x * c - v.y * s, v.x * s + v.y * c);
  }
}
}  // namespace attn

template <bool ROPE>
__global__ void __launch_bounds__(attn::THREADS, 2)
    attention_kernel(const __half* __restrict__ qkv, __half* __restrict__ out, int seq_len, int heads, float scale_log2,
                     const float* __restrict__ rope_cos, const float* __restrict__ rope_sin) {
  using namespace attn;
  extern __shared__ __align__(128) uint8_t smem[];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int qt = blockIdx.x, h = blockIdx.y, seq = blockIdx.z;
  const int dim = heads * D, row_stride = 3 * dim;
  const size_t tok0 = static_cast<size_t>(seq) * seq_len;
  const __half* qbase = qkv + tok0 * row_stride + h * D;
  const __half* kbase = qbase + dim;
  const __half* vbase = qbase + 2 * dim;
  const int q0 = qt * BQ;
  const int nkv = (seq_len + BKV - 1) / BKV;
  const uint32_t s_q = smem_u32(smem);
  auto s_k = [&](int b) { return s_q + (BQ + b * BKV) * 128; };
  auto s_v = [&](int b) { return s_q + (BQ + (2 + b) * BKV) * 128; };

  auto load_rows = [&](uint32_t dst, const __half* src, int row0, int rows) {
    for (int i = tid; i < rows * 8; i += THREADS) {
      const int r = i >> 3, c = i & 7, tok = row0 + r;
      const bool ok = tok < seq_len;
      cp_async16(dst + swz(r, c), src + static_cast<size_t>(ok ? tok : 0) * row_stride + c * 8, ok);
    }
  };
  load_rows(s_q, qbase, q0, BQ);
  load_rows(s_k(0), kbase, 0, BKV);
  load_rows(s_v(0), vbase, 0, BKV);
  cp_commit();

  uint32_t qf[4][4];
  float o[8][4];
  float m_run[2] = {-INFINITY, -INFINITY}, l_run[2] = {0.f, 0.f};
#pragma unroll
  for (int i = 0; i < 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;

  for (int j = 0; j < nkv; ++j) {
    if (j + 1 < nkv) {
      load_rows(s_k((j + 1) & 1), kbase, (j + 1) * BKV, BKV);
      load_rows(s_v((j + 1) & 1), vbase, (j + 1) * BKV, BKV);
      cp_commit();
      cp_wait<1>();
    } else {
      cp_wait<0>();
    }
    __syncthreads();
    if constexpr (ROPE) {
      if (j == 0) rope_tile(smem, BQ, q0, seq_len, rope_cos, rope_sin);
      rope_tile(smem + (BQ + (j & 1) * BKV) * 128, BKV, j * BKV, seq_len, rope_cos, rope_sin);
      __syncthreads();
    }
    if (j == 0) {
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) ldsm_x4(qf[kk], s_q + swz(warp * 16 + (lane & 15), kk * 2 + (lane >> 4)));
    }
    const uint32_t kb = s_k(j & 1), vb = s_v(j & 1);

    float s[8][4];
#pragma unroll
    for (int i = 0; i < 8; ++i) s[i][0] = s[i][1] = s[i][2] = s[i][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < 4; ++kk)
#pragma unroll
      for (int np = 0; np < 4; ++np) {
        uint32_t t[4];
        ldsm_x4(t, kb + swz(np * 16 + ((lane >> 4) << 3) + (lane & 7), kk * 2 + ((lane >> 3) & 1)));
        mma_f32(s[2 * np], qf[kk], t[0], t[1]);
        mma_f32(s[2 * np + 1], qf[kk], t[2], t[3]);
      }
    // Scale into base 2 and mask keys past the end of the sequence.
    const int key0 = j * BKV;
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int key = key0 + i * 8 + (lane & 3) * 2 + (e & 1);
        s[i][e] = key < seq_len ? s[i][e] * scale_log2 : -INFINITY;
      }
    float corr[2];
    uint32_t pf[4][4];
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
      float mx = -INFINITY;
#pragma unroll
      for (int i = 0; i < 8; ++i) mx = fmaxf(mx, fmaxf(s[i][2 * hh], s[i][2 * hh + 1]));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
      const float m_new = fmaxf(m_run[hh], mx);  // finite: every tile holds at least one valid key
      corr[hh] = ex2(m_run[hh] - m_new);
      m_run[hh] = m_new;
      float sum = 0.f;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float p0 = ex2(s[i][2 * hh] - m_new), p1 = ex2(s[i][2 * hh + 1] - m_new);
        sum += p0 + p1;
        pf[i >> 1][(i & 1) * 2 + hh] = pack_half2(p0, p1);
      }
      l_run[hh] = l_run[hh] * corr[hh] + sum;
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      o[i][0] *= corr[0];
      o[i][1] *= corr[0];
      o[i][2] *= corr[1];
      o[i][3] *= corr[1];
    }
#pragma unroll
    for (int kk = 0; kk < 4; ++kk)
#pragma unroll
      for (int dp = 0; dp < 4; ++dp) {
        uint32_t t[4];
        ldsm_x4_t(t, vb + swz(kk * 16 + (lane & 15), dp * 2 + (lane >> 4)));
        mma_f32(o[2 * dp], pf[kk], t[0], t[1]);
        mma_f32(o[2 * dp + 1], pf[kk], t[2], t[3]);
      }
    __syncthreads();
  }

  // Normalise; each thread writes its own half2 pairs (rows past seq_len are dropped).
  const int dim_out = dim;
#pragma unroll
  for (int hh = 0; hh < 2; ++hh) {
    float l = l_run[hh];
    l += __shfl_xor_sync(0xffffffffu, l, 1);
    l += __shfl_xor_sync(0xffffffffu, l, 2);
    const float inv = 1.f / l;
    const int r = q0 + warp * 16 + (lane >> 2) + hh * 8;
    if (r < seq_len) {
      __half* orow = out + (tok0 + r) * dim_out + h * D;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int c = i * 8 + (lane & 3) * 2;
        *reinterpret_cast<__half2*>(orow + c) = __floats2half2_rn(o[i][2 * hh] * inv, o[i][2 * hh + 1] * inv);
      }
    }
  }
}

int attention(const void* qkv, void* out, int num_seqs, int seq_len, int heads, const float* rc, const float* rsn,
              float scale, cudaStream_t s) {
  using namespace attn;
  FF_REQUIRE(qkv && out, "ff_attention: NULL pointer");
  FF_REQUIRE(num_seqs >= 0 && seq_len >= 1 && heads >= 1 && heads <= 64, "ff_attention: bad shape");
  FF_REQUIRE((rc == nullptr) == (rsn == nullptr), "ff_attention: give both RoPE tables or neither");
  FF_REQUIRE(aligned16(qkv) && aligned16(out), "ff_attention: pointers must be 16-byte aligned");
  if (num_seqs == 0) return FF_OK;
  if (rc == nullptr) return attention_tc(qkv, out, num_seqs, seq_len, heads, scale, s);
  const float scale_log2 = scale * 1.4426950408889634f;
  const dim3 grid((seq_len + BQ - 1) / BQ, heads, num_seqs);
  static bool configured[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64 || !configured[dev]) {
    if (cudaFuncSetAttribute(attention_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM) != cudaSuccess ||
        cudaFuncSetAttribute(attention_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM) != cudaSuccess)
      return check_launch("ff_attention: cudaFuncSetAttribute");
    if (dev >= 0 && dev < 64) configured[dev] = true;
  }
  if (rc != nullptr)
    attention_kernel<true><<<grid, THREADS, SMEM, s>>>(static_cast<const __half*>(qkv), static_cast<__half*>(out),
                                                       seq_len, heads, scale_log2, rc, rsn);
  else
    attention_kernel<false><<<grid, THREADS, SMEM, s>>>(static_cast<const __half*>(qkv), static_cast<__half*>(out),
                                                        seq_len, heads, scale_log2, nullptr, nullptr);
  return check_launch("attention_kernel");
}

}  // namespace ff

extern "C" int ff_attention(const uint16_t* qkv, uint16_t* out, int num_seqs, int seq_len, int heads,
                            const float* rope_cos, const float* rope_sin, float scale, void* stream) {
  return ff::attention(qkv, out, num_seqs, seq_len, heads, rope_cos, rope_sin, scale,
                       static_cast<cudaStream_t>(stream));
}
