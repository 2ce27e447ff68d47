// Non-causal flash attention on the 5th-generation tensor cores (tcgen05), head dim 64.
//
// Computes what the reference's attention kernel computes (foidfinder/backends/cuda/csrc/attention.cuh:19-157:
// softmax(q k^T) v per head on the packed QKV activations, scale folded into q), with f32 accumulation and
// masked ragged tails (EVA02 at 448 px has 1025 tokens).
//
// One CTA = 128 queries of one (image, head); 192 threads, two CTAs per SM so one CTA's softmax overlaps
// the other's tensor-core work:
//   warp 0     TMA: Q once, then K/V tiles of 128 keys through a 2-stage ring (3-D tensor map
//              [images, tokens, 3*dim], so rows past an image's last token arrive as zeros)
//   warp 1     TMEM allocation (256 columns) and the MMA issuer:
//                S = Q K^T          (SS, M128 N128 K64)         -> TMEM columns [0, 128)
//                O += P V           (TS: P read from TMEM, V from smem as an MN-major operand) -> [128, 192)
//                l += P 1           (TS, N16 against a constant tile of ones)                   -> [192, 208)
//   warps 2-5  softmax, one query row per thread (TMEM lane = row, so no shuffles): mask, row max,
//              lazy rescale of O and l in TMEM when the max grows by more than 2^8, P = 2^(s - m) as fp16
//              pairs (ex2.approx.f16x2) written back over S; finally O / l -> fp16 -> global.
// The row sum runs on the tensor core against the ones tile, so it is rescaled together with O.
#include "common.h"
#include "ptx.cuh"

namespace ff {
namespace fa {

constexpr int BQ = 128, BKV = 128, HD = 64, STAGES = 2;
constexpr int TILE = 128 * 128;  // 128 rows x 128 bytes (64 fp16)
constexpr int OFF_Q = 0;
constexpr int OFF_K = OFF_Q + TILE;
constexpr int OFF_V = OFF_K + STAGES * TILE;
constexpr int OFF_ONES = OFF_V + STAGES * TILE;  // 2 K-atoms x 16 rows x 128 B of fp16 1.0
constexpr int OFF_BAR = OFF_ONES + 4096;
constexpr int SMEM = 1024 + OFF_BAR + 256;
constexpr uint32_t T_S = 0, T_O = 128, T_L = 192, T_COLS = 256;
constexpr float kRescaleThreshold = 8.f;  // log2 units: P may reach 2^8 before O and l are rescaled

// MN-major operand with 128-byte swizzle: K rows of 128 B (64 fp16 along N), 8-row groups 1024 B apart.
__device__ __forceinline__ uint64_t sdesc_mn_sw128(uint32_t saddr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>(TILE >> 4) << 16;      // leading byte offset: next 64-wide N atom (unused at N = 64)
  d |= static_cast<uint64_t>(1024u >> 4) << 32;     // stride byte offset: 8 K rows x 128 B
  d |= static_cast<uint64_t>(1u) << 46;
  d |= static_cast<uint64_t>(2u) << 61;
  return d;
}

__device__ __forceinline__ void mma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                           uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]),
      "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]),
      "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}
__device__ __forceinline__ void tmem_ld1(uint32_t taddr, uint32_t& r) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x1.b32 {%0}, [%1];" : "=r"(r) : "r"(taddr) : "memory");
}
__device__ __forceinline__ void tmem_st1(uint32_t taddr, uint32_t r) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x1.b32 [%0], {%1};" ::"r"(taddr), "r"(r) : "memory");
}
__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// (a - m, b - m) rounded to a half2, then 2^x on both halves in one MUFU operation.
__device__ __forceinline__ uint32_t exp2_pair(float a, float b, float m) {
  const uint32_t h = pack_half2(a - m, b - m);
  uint32_t p;
  asm("ex2.approx.f16x2 %0, %1;" : "=r"(p) : "r"(h));
  return p;
}

}  // namespace fa

__global__ void __launch_bounds__(192, 2)
    attention_tc_kernel(const __grid_constant__ CUtensorMap tm_qkv, __half* __restrict__ out, int T, int heads,
                        float scale_log2, int* err) {
  using namespace fa;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + OFF_BAR);
  uint64_t* q_full = bar + 0;
  uint64_t* kv_full = bar + 1;   // [STAGES]
  uint64_t* kv_empty = bar + 3;  // [STAGES]
  uint64_t* s_full = bar + 5;
  uint64_t* p_full = bar + 6;
  uint64_t* pv_done = bar + 7;
  uint64_t* o_full = bar + 8;
  uint64_t* drain = bar + 9;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar + 10);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(bar + 11);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int qt = blockIdx.x, h = blockIdx.y, img = blockIdx.z;
  const int dim = heads * HD;
  const int q0 = qt * BQ;
  const int nkv = (T + BKV - 1) / BKV;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    mbar_init(s_full, 1);
    mbar_init(p_full, 4);
    mbar_init(pv_done, 1);
    mbar_init(o_full, 1);
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) tma_prefetch_map(&tm_qkv);
  if (warp == 1) {
    tmem_alloc(tmem_slot, T_COLS);
    tmem_relinquish();
  }
  if (warp >= 2) {  // the constant ones operand of the row-sum MMA (4 KB of fp16 1.0)
    uint4* ones = reinterpret_cast<uint4*>(smem + OFF_ONES);
    for (int i = threadIdx.x - 64; i < 4096 / 16; i += 128) ones[i] = make_uint4(0x3C003C00u, 0x3C003C00u, 0x3C003C00u, 0x3C003C00u);
    fence_async_smem();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      mbar_arrive_expect_tx(q_full, TILE);
      tma_load_3d(smem + OFF_Q, &tm_qkv, q_full, h * HD, q0, img);
      int last_phase[STAGES] = {-1, -1};
      bool ok = true;
      for (int j = 0; j < nkv; ++j) {
        const int s = j % STAGES;
        const uint32_t ph = static_cast<uint32_t>(j / STAGES) & 1u;
        if (!mbar_wait(&kv_empty[s], ph ^ 1u, abort_flag, err, kDevTimeoutAttn)) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(&kv_full[s], 2 * TILE);
        tma_load_3d(smem + OFF_K + s * TILE, &tm_qkv, &kv_full[s], dim + h * HD, j * BKV, img);
        tma_load_3d(smem + OFF_V + s * TILE, &tm_qkv, &kv_full[s], 2 * dim + h * HD, j * BKV, img);
        last_phase[s] = static_cast<int>(ph);
      }
      // Let every issued copy land before the CTA can exit (bounded).
      const unsigned long long t0 = globaltimer();
      while (!mbar_try_wait(smem_u32(q_full), 0) && globaltimer() - t0 < kWaitLimitNs) {
      }
      if (!ok)
        for (int s = 0; s < STAGES; ++s)
          if (last_phase[s] >= 0)
            while (!mbar_try_wait(smem_u32(&kv_full[s]), static_cast<uint32_t>(last_phase[s])) &&
                   globaltimer() - t0 < kWaitLimitNs) {
            }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t id_s = idesc_f16(128, BKV);
      constexpr uint32_t id_o = idesc_f16(128, HD) | (1u << 16);  // B (V) is MN-major
      constexpr uint32_t id_l = idesc_f16(128, 16);
      const uint32_t sq = smem_u32(smem + OFF_Q), sones = smem_u32(smem + OFF_ONES);
      bool ok = mbar_wait(q_full, 0, abort_flag, err, kDevTimeoutAttn);
      for (int j = 0; j < nkv && ok; ++j) {
        const int s = j % STAGES;
        const uint32_t ph = static_cast<uint32_t>(j / STAGES) & 1u;
        if (!mbar_wait(&kv_full[s], ph, abort_flag, err, kDevTimeoutAttn)) break;
        // S_j overwrites the TMEM columns P_{j-1} was read from: wait for the previous P V to finish.
        if (j > 0 && !mbar_wait(pv_done, static_cast<uint32_t>(j - 1) & 1u, abort_flag, err, kDevTimeoutAttn)) break;
        tc_fence_after();
        const uint64_t qd = sdesc_k_sw128(sq);
        const uint64_t kd = sdesc_k_sw128(smem_u32(smem + OFF_K + s * TILE));
#pragma unroll
        for (int k = 0; k < 4; ++k) mma_f16(tmem + T_S, qd + 2 * k, kd + 2 * k, id_s, k > 0);
        tc_commit(s_full);
        if (!mbar_wait(p_full, static_cast<uint32_t>(j) & 1u, abort_flag, err, kDevTimeoutAttn)) break;
        tc_fence_after();
        const uint32_t sv = smem_u32(smem + OFF_V + s * TILE);
#pragma unroll
        for (int k = 0; k < 8; ++k) {  // 16 keys per step: P columns 8k.., V rows 16k..
          const uint32_t acc = (j > 0 || k > 0) ? 1u : 0u;
          mma_f16_ts(tmem + T_O, tmem + T_S + 8 * k, fa::sdesc_mn_sw128(sv + k * 2048), id_o, acc);
          mma_f16_ts(tmem + T_L, tmem + T_S + 8 * k,
                     sdesc_k_sw128(sones + (k >> 2) * 2048) + 2 * (k & 3), id_l, acc);
        }
        tc_commit(&kv_empty[s]);
        tc_commit(pv_done);
      }
      tc_commit(o_full);
      tc_commit(drain);
      const unsigned long long t0 = globaltimer();
      while (!mbar_try_wait(smem_u32(drain), 0)) {
        if (globaltimer() - t0 > kWaitLimitNs) {
          atomicCAS(err, 0, kDevTimeoutDrain);
          break;
        }
      }
    }
  } else {
    // ------------------------------------------------------------ softmax + epilogue (warps 2..5)
    const int q = warp & 3;
    const uint32_t lane_base = static_cast<uint32_t>(q * 32) << 16;
    const int row = q0 + q * 32 + lane;
    float m_ref = -INFINITY;
    bool ok = true;
    for (int j = 0; j < nkv && ok; ++j) {
      if (!mbar_wait(s_full, static_cast<uint32_t>(j) & 1u, abort_flag, err, kDevTimeoutAttn)) {
        ok = false;
        break;
      }
      tc_fence_after();
      // Pass 1: row max of the valid keys (keys at columns >= valid belong to no token of this image).
      const int valid = T - j * BKV;
      float mx = -INFINITY;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t raw[32];
        tmem_ld32(tmem + lane_base + T_S + 32 * c, raw);
        tmem_ld_wait();
#pragma unroll
        for (int e = 0; e < 32; ++e)
          if (32 * c + e < valid) mx = fmaxf(mx, __uint_as_float(raw[e]));
      }
      const float m_new = fmaxf(m_ref, mx * scale_log2);
      bool rescale = false;
      float corr = 1.f;
      if (j == 0) {
        m_ref = m_new;
      } else if (m_new > m_ref + kRescaleThreshold) {
        corr = ex2_approx(m_ref - m_new);
        m_ref = m_new;
        rescale = true;
      }
      if (__any_sync(0xffffffffu, rescale)) {
        uint32_t o[32];
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          tmem_ld32(tmem + lane_base + T_O + 32 * c, o);
          tmem_ld_wait();
#pragma unroll
          for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * corr);
          fa::tmem_st32(tmem + lane_base + T_O + 32 * c, o);
        }
        uint32_t l;
        fa::tmem_ld1(tmem + lane_base + T_L, l);
        tmem_ld_wait();
        fa::tmem_st1(tmem + lane_base + T_L, __float_as_uint(__uint_as_float(l) * corr));
      }
      // Pass 2: P = 2^(s * scale_log2 - m_ref) as fp16 pairs over TMEM columns [0, 64). Chunk c of S
      // (columns 32c..32c+31) is read before P chunk c (columns 16c..16c+15) is written, and P chunk c
      // only overlaps S columns of chunks <= c.
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t raw[32];
        tmem_ld32(tmem + lane_base + T_S + 32 * c, raw);
        tmem_ld_wait();
        uint32_t pk[16];
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          const float a = 32 * c + 2 * e < valid ? __uint_as_float(raw[2 * e]) * scale_log2 : -INFINITY;
          const float b = 32 * c + 2 * e + 1 < valid ? __uint_as_float(raw[2 * e + 1]) * scale_log2 : -INFINITY;
          pk[e] = fa::exp2_pair(a, b, m_ref);
        }
        fa::tmem_st16(tmem + lane_base + T_S + 16 * c, pk);
      }
      fa::tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(p_full);
    }
    if (ok && mbar_wait(o_full, 0, abort_flag, err, kDevTimeoutAttn)) {
      tc_fence_after();
      uint32_t o2[2][32], l;
      tmem_ld32(tmem + lane_base + T_O, o2[0]);
      tmem_ld32(tmem + lane_base + T_O + 32, o2[1]);
      const uint32_t* o = &o2[0][0];
      fa::tmem_ld1(tmem + lane_base + T_L, l);
      tmem_ld_wait();
      if (row < T) {
        const float inv = 1.f / __uint_as_float(l);
        uint4* dst = reinterpret_cast<uint4*>(out + (static_cast<size_t>(img) * T + row) * dim + h * HD);
#pragma unroll
        for (int v4 = 0; v4 < 8; ++v4)
          dst[v4] = make_uint4(pack_half2(__uint_as_float(o[8 * v4]) * inv, __uint_as_float(o[8 * v4 + 1]) * inv),
                               pack_half2(__uint_as_float(o[8 * v4 + 2]) * inv, __uint_as_float(o[8 * v4 + 3]) * inv),
                               pack_half2(__uint_as_float(o[8 * v4 + 4]) * inv, __uint_as_float(o[8 * v4 + 5]) * inv),
                               pack_half2(__uint_as_float(o[8 * v4 + 6]) * inv, __uint_as_float(o[8 * v4 + 7]) * inv));
      }
    }
  }

  __syncwarp();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, T_COLS);
}

int attention_tc(const void* qkv, void* out, int num_seqs, int seq_len, int heads, float scale, cudaStream_t s) {
  using namespace fa;
  CUtensorMap map;
  const int dim = heads * HD;
  int rc = make_tmap_3d(&map, qkv, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, static_cast<uint64_t>(3 * dim),
                        static_cast<uint64_t>(seq_len), static_cast<uint64_t>(num_seqs), 64, 128, 1);
  if (rc != FF_OK) return rc;
  int* err = device_error_word();
  FF_REQUIRE(err != nullptr, "attention: no device error word");
  static bool configured[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64 || !configured[dev]) {
    if (cudaFuncSetAttribute(attention_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM) != cudaSuccess)
      return check_launch("attention_tc: cudaFuncSetAttribute");
    if (dev >= 0 && dev < 64) configured[dev] = true;
  }
  const dim3 grid((seq_len + BQ - 1) / BQ, heads, num_seqs);
  attention_tc_kernel<<<grid, 192, SMEM, s>>>(map, static_cast<__half*>(out), seq_len, heads,
                                              scale * 1.4426950408889634f, err);
  return check_launch("attention_tc_kernel");
}

}  // namespace ff
