// Persistent tcgen05 GEMM for sm_100a: Y[m, n] = sum_k A[m, k] * W[n, k], both operands K-major.
//
// Replaces the reference's mma.sync int8 GEMM (foidfinder/backends/cuda/csrc/gemm.cuh:43-172) and the
// cuBLAS fp16 matmuls of the stem and head (foidfinder/backends/cuda/engine.py:146,
// foidfinder/backends/cuda/reference.py:133-140).
//
// Layout of one CTA (320 threads, one CTA per SM, grid = min(tiles, SMs)):
//   warp 0     TMA producer: A box 128 x 128 B and W box BN x 128 B per stage, 128-byte swizzle
//   warp 1     TMEM allocator and MMA issuer: 4 tcgen05.mma (K = 32 bytes each) per stage
//   warps 2-9  epilogue: tcgen05.ld of the accumulator (warp w reads TMEM lanes 32*(w%4)..+31, one
//              output row per thread; two warps per lane quarter split the columns), fused
//              dequantisation / bias / RoPE / SwiGLU / residual, then the warp's 32-row block goes out
//              through a swizzled shared-memory stage as whole 128-byte lines.
// The epilogue balances the issue slots against the narrow XU pipe: int->float uses the hardware
// conversion (acc_to_float), the SwiGLU sigmoid an ex2 and a reciprocal (silu_mul2), so the epilogue of one
// tile hides under the next tile's mainloop as far as possible.
// Accumulators are double-buffered in TMEM (2 x BN columns), so the epilogue of tile i overlaps the
// mainloop of tile i+1. Stages are a ring of STAGES smem buffers guarded by full/empty mbarriers.
//
// PAIR: clusters of two CTAs on two SMs share 256-row tiles through tcgen05.mma.cta_group::2 (M = 256):
// each CTA loads its own 128 rows of A and half of B's BN rows, the even CTA issues the MMAs, and each
// CTA's TMEM receives its 128 rows of the accumulator. Per SM this halves the B bytes moved through
// shared memory per multiply-add, which bounds the single-CTA mainloop (TMA writes + MMA operand reads
// of 48 KB per 128-byte K step against the shared-memory bandwidth). Both CTAs' copies of a stage signal
// the even CTA's full barrier (cta_group::2 loads, no multicast: each CTA loads its own rows); the MMA
// commits arrive on both CTAs' empty / accumulator-full barriers at once (commit with a CTA mask); the odd
// CTA's epilogue warps release the accumulator on the even CTA's tempty barrier (mapa address).
#pragma once
#include "ptx.cuh"
#include "gemm_args.h"

namespace ff {

template <int BN, int STAGES, bool PAIR = false>
struct GemmCfg {
  static constexpr int BM = 128;    // rows per CTA (a PAIR tile is 2 x BM)
  static constexpr int TILE_M = PAIR ? 2 * BM : BM;
  static constexpr int BKB = 128;  // K bytes per stage (one 128-byte swizzle row)
  static constexpr int A_BYTES = BM * BKB;
  static constexpr int B_ROWS = PAIR ? BN / 2 : BN;  // W rows this CTA loads per stage
  static constexpr int B_BYTES = B_ROWS * BKB;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int TMEM_COLS = 2 * BN;  // double-buffered accumulator
  static constexpr int EPI_WARPS = 8;       // two per TMEM sub-partition, each owning half the tile's columns
  static constexpr int THREADS = 64 + 32 * EPI_WARPS;
  static constexpr int STAGING = 4096;      // per epilogue warp: 32 rows x 128 B (one TMA store in flight;
                                            // a second buffer measured no faster and costs a stage)
  static constexpr int BAR_BYTES = 256;
  static constexpr int SMEM = 1024 /*alignment slack*/ + STAGES * STAGE_BYTES + EPI_WARPS * STAGING + BAR_BYTES;
  static_assert(BN == 128 || BN == 256, "BN");
  static_assert(TMEM_COLS == 256 || TMEM_COLS == 512, "TMEM columns must be a power of two");
  static_assert(SMEM <= 227 * 1024, "shared memory");
};

// tanh GELU as the reference's fc1 epilogue computes it (foidfinder/backends/cuda/csrc/common.cuh:50-56),
// with the hardware tanh.approx.
__device__ __forceinline__ float gelu_tanh(float x) {
  float t;
  asm("tanh.approx.f32 %0, %1;" : "=f"(t) : "f"(0.7978845608f * (x + 0.044715f * x * x * x)));
  return 0.5f * x * (1.f + t);
}

// silu(g) * u on two lanes: sigmoid(g) = 1 / (1 + 2^(-g log2 e)) by MUFU ex2 and MUFU rcp (rcp.approx, ~1 ulp),
// the products packed f32x2. A Newton reciprocal on the FMA pipe instead (magic-constant estimate + 3 steps)
// measured 2.4% slower for the gate/up GEMM at bs64: the epilogue is issue-bound, the XU pipe has room.
__device__ __forceinline__ float2 silu_mul2(float2 g, float2 u) {
  const float2 t = mul2(g, make_float2(-1.4426950408889634f, -1.4426950408889634f));
  const float2 e = make_float2(ex2_approx(fminf(t.x, 64.f)), ex2_approx(fminf(t.y, 64.f)));
  const float2 d = add2(make_float2(1.f, 1.f), e);
  float2 y;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y.x) : "f"(d.x));
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y.y) : "f"(d.y));
  return mul2(mul2(g, y), u);
}

// Coalesced store of a warp's 32-row x 128-byte block: each lane wrote its own row into `stg` (16-byte
// chunks XOR-swizzled by row % 8, so both phases are bank-conflict free); here every 8 lanes copy one
// full row, 4 rows (4 whole cache lines) per warp instruction.
__device__ __forceinline__ void stage_row128(uint8_t* stg, int lane, const uint32_t (&w)[32]) {
#pragma unroll
  for (int c = 0; c < 8; ++c)
    *reinterpret_cast<uint4*>(stg + lane * 128 + ((c ^ (lane & 7)) << 4)) =
        make_uint4(w[4 * c], w[4 * c + 1], w[4 * c + 2], w[4 * c + 3]);
}
// Half of a 128-byte row (16-byte chunks 4h .. 4h + 3), same swizzle as stage_row128.
__device__ __forceinline__ void stage_half_row128(uint8_t* stg, int lane, int h, const uint32_t (&w)[16]) {
#pragma unroll
  for (int c = 0; c < 4; ++c)
    *reinterpret_cast<uint4*>(stg + lane * 128 + (((4 * h + c) ^ (lane & 7)) << 4)) =
        make_uint4(w[4 * c], w[4 * c + 1], w[4 * c + 2], w[4 * c + 3]);
}
__device__ __forceinline__ uint4 staged_chunk128(const uint8_t* stg, int r, int c) {
  return *reinterpret_cast<const uint4*>(stg + r * 128 + ((c ^ (r & 7)) << 4));
}
// 64-byte rows (4 chunks, XOR-swizzled by (row / 2) % 4); 8 rows per warp instruction.
__device__ __forceinline__ void stage_row64(uint8_t* stg, int lane, const uint32_t (&w)[16]) {
#pragma unroll
  for (int c = 0; c < 4; ++c)
    *reinterpret_cast<uint4*>(stg + lane * 64 + ((c ^ ((lane >> 1) & 3)) << 4)) =
        make_uint4(w[4 * c], w[4 * c + 1], w[4 * c + 2], w[4 * c + 3]);
}
__device__ __forceinline__ uint4 staged_chunk64(const uint8_t* stg, int r, int c) {
  return *reinterpret_cast<const uint4*>(stg + r * 64 + ((c ^ ((r >> 1) & 3)) << 4));
}

// y[j] = acc[j] * rs * cs[n0 + j] + bias[n0 + j] for 32 consecutive columns.
// int32 accumulator -> f32, correctly rounded. The hardware conversion (I2F, on the XU pipe) costs one
// issue slot per 32 values; an exact integer/FMA-pipe form (two magic-number halves recombined by an FMA)
// costs six. With the current epilogues the XU pipe has room, and I2F measured faster on every GEMM
// shape (SwiGLU epilogue +12%).
__device__ __forceinline__ float acc_to_float(uint32_t raw) { return __int2float_rn(static_cast<int>(raw)); }

// dequant32 in packed f32x2 form: (acc * rs) * cs + b per lane, the same two roundings as the scalar form.
__device__ __forceinline__ void dequant32_x2(const uint32_t (&r)[32], float rs, const float* cs, const float* bias,
                                             float2 (&y)[16]) {
  const float2 rs2 = make_float2(rs, rs);
#pragma unroll
  for (int j = 0; j < 32; j += 4) {
    const float4 c4 = *reinterpret_cast<const float4*>(cs + j);
    const float4 b4 = *reinterpret_cast<const float4*>(bias + j);
    y[j / 2] = fma2(mul2(make_float2(acc_to_float(r[j]), acc_to_float(r[j + 1])), rs2), make_float2(c4.x, c4.y),
                    make_float2(b4.x, b4.y));
    y[j / 2 + 1] = fma2(mul2(make_float2(acc_to_float(r[j + 2]), acc_to_float(r[j + 3])), rs2),
                        make_float2(c4.z, c4.w), make_float2(b4.z, b4.w));
  }
}

__device__ __forceinline__ void dequant32(const uint32_t (&r)[32], float rs, const float* cs, const float* bias,
                                          float (&y)[32]) {
#pragma unroll
  for (int j = 0; j < 32; j += 4) {
    const float4 c4 = *reinterpret_cast<const float4*>(cs + j);
    const float4 b4 = *reinterpret_cast<const float4*>(bias + j);
    y[j] = acc_to_float(r[j]) * rs * c4.x + b4.x;
    y[j + 1] = acc_to_float(r[j + 1]) * rs * c4.y + b4.y;
    y[j + 2] = acc_to_float(r[j + 2]) * rs * c4.z + b4.z;
    y[j + 3] = acc_to_float(r[j + 3]) * rs * c4.w + b4.w;
  }
}

template <int BN, int STAGES, bool F16IN, int EPI, bool PAIR = false>
__global__ void __launch_bounds__(GemmCfg<BN, STAGES, PAIR>::THREADS, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const __grid_constant__ CUtensorMap tmC, const GemmArgs args) {
  // fp16 outputs of these epilogues leave through TMA stores of the swizzled staging buffer (tmC).
  constexpr bool kTmaStore =
      EPI == EPI_BIAS || EPI == EPI_QKV_ROPE || EPI == EPI_SWIGLU || EPI == EPI_RESIDUAL || EPI == EPI_GELU_F16;
  static_assert(!PAIR || !F16IN, "pair tiles are built for the int8 GEMMs");
  using C = GemmCfg<BN, STAGES, PAIR>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* staging = smem + STAGES * C::STAGE_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(staging + C::EPI_WARPS * C::STAGING);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tiles_n = args.N / BN;
  const int tiles = args.tiles_m * tiles_n;  // tiles_m counts TILE_M-row tiles
  const uint32_t rank = PAIR ? cluster_ctarank() : 0u;
  const bool leader = rank == 0;
  const int unit = PAIR ? static_cast<int>(blockIdx.x >> 1) : static_cast<int>(blockIdx.x);  // CTA or pair
  const int units = PAIR ? static_cast<int>(gridDim.x >> 1) : static_cast<int>(gridDim.x);
  // Waits on barriers the other CTA of a pair arrives on take cluster-scope acquire.
  // Waiting threads suspend rather than poll (mbar_wait<true>), leaving issue slots to the MMA thread and
  // the epilogue warps that share their schedulers.
  auto wait = [&](uint64_t* bar, uint32_t parity, int code) {
    if constexpr (PAIR)
      return mbar_wait_cluster<true>(bar, parity, abort_flag, args.err, code);
    else
      return mbar_wait<true>(bar, parity, abort_flag, args.err, code);
  };

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], (PAIR ? 2 : 1) * C::EPI_WARPS);  // one arrive per epilogue warp (of both CTAs)
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_map(&tmA);
    tma_prefetch_map(&tmB);
  }
  if (warp == 1) {
    if constexpr (PAIR) {
      tmem_alloc2(tmem_slot, C::TMEM_COLS);
      tmem_relinquish2();
    } else {
      tmem_alloc(tmem_slot, C::TMEM_COLS);
      tmem_relinquish();
    }
  }
  tc_fence_before();
  __syncthreads();
  if constexpr (PAIR) cluster_sync();  // both CTAs' barriers initialised and TMEM allocated
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // The prologue above overlapped the previous kernel (programmatic dependent launch). Each role waits for
  // that kernel's outputs (pdl_wait) only before its first access to them: with args.w_const the producer
  // first loads the weight tiles of its first stages, which no kernel of the forward writes.
  pdl_trigger();

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int last_phase[STAGES];
#pragma unroll
      for (int s = 0; s < STAGES; ++s) last_phase[s] = -1;
      constexpr int kElemsPerStage = F16IN ? C::BKB / 2 : C::BKB;
      // W tiles of the first tile's first stages, ahead of the wait for the previous kernel (the stages
      // are fresh, so no empty-wait; each full barrier expects the whole stage, A included).
      const int pre = (!PAIR && args.w_const && unit < tiles) ? (args.num_kb < STAGES ? args.num_kb : STAGES) : 0;
      if (!PAIR) {
        for (int kb = 0; kb < pre; ++kb) {
          mbar_arrive_expect_tx(&full[kb], C::STAGE_BYTES);
          tma_load_2d(smem + kb * C::STAGE_BYTES + C::A_BYTES, &tmB, &full[kb], kb * kElemsPerStage,
                      (unit % tiles_n) * BN);
        }
      }
      pdl_wait();
      bool ok = true;
      bool first = true;
      for (int t = unit; t < tiles && ok; t += units) {
        const int tm = t / tiles_n, tn = t % tiles_n;
        for (int kb = 0; kb < args.num_kb; ++kb) {
          uint8_t* sa = smem + stage * C::STAGE_BYTES;
          if (first && kb < pre) {  // W already on its way: only A
            tma_load_2d(sa, &tmA, &full[stage], kb * kElemsPerStage, tm * C::BM);
            last_phase[stage] = static_cast<int>(phase);
            if (++stage == STAGES) {
              stage = 0;
              phase ^= 1u;
            }
            continue;
          }
          if (!wait(&empty[stage], phase ^ 1u, kDevTimeoutSmemEmpty)) {
            ok = false;
            break;
          }
          if constexpr (PAIR) {
            // Both CTAs' copies of this stage complete on the even CTA's full barrier.
            if (leader) mbar_arrive_expect_tx(&full[stage], 2 * C::STAGE_BYTES);
            const uint32_t fb = mapa_shared(smem_u32(&full[stage]), 0u);
            tma_load_2d_pair(sa, &tmA, fb, kb * kElemsPerStage, tm * C::TILE_M + static_cast<int>(rank) * C::BM);
            tma_load_2d_pair(sa + C::A_BYTES, &tmB, fb, kb * kElemsPerStage,
                             tn * BN + static_cast<int>(rank) * C::B_ROWS);
          } else {
            mbar_arrive_expect_tx(&full[stage], C::STAGE_BYTES);
            tma_load_2d(sa, &tmA, &full[stage], kb * kElemsPerStage, tm * C::BM);
            tma_load_2d(sa + C::A_BYTES, &tmB, &full[stage], kb * kElemsPerStage, tn * BN);
          }
          last_phase[stage] = static_cast<int>(phase);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        first = false;
      }
      if (!ok && leader) {
        // Let every issued copy land before the CTA exits (bounded). In a pair the even CTA's full barrier
        // also counts the odd CTA's copies, and the odd CTA stays resident until the even one is done.
        for (int s = 0; s < STAGES; ++s)
          if (last_phase[s] >= 0) {
            const uint32_t addr = smem_u32(&full[s]);
            const unsigned long long t0 = globaltimer();
            while (!mbar_try_wait(addr, static_cast<uint32_t>(last_phase[s])) && globaltimer() - t0 < kWaitLimitNs) {
            }
          }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer (the even CTA of a pair)
    pdl_wait();
    if (lane == 0 && leader) {
      constexpr uint32_t idesc = F16IN ? idesc_f16(128, BN) : idesc_s8(C::TILE_M, BN);
      auto commit = [&](uint64_t* bar) {  // local barrier
        if constexpr (PAIR)
          tc_commit2(bar);
        else
          tc_commit(bar);
      };
      auto commit_both = [&](uint64_t* bar) {  // the barrier of both CTAs of a pair
        if constexpr (PAIR)
          tc_commit2_both(bar);
        else
          tc_commit(bar);
      };
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int t = unit; t < tiles && ok; t += units) {
        if (!wait(&tempty[acc], acc_phase ^ 1u, kDevTimeoutTmemEmpty)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem + static_cast<uint32_t>(acc * BN);
        for (int kb = 0; kb < args.num_kb; ++kb) {
          if (!wait(&full[stage], phase, kDevTimeoutTmaFull)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + stage * C::STAGE_BYTES);
          const uint64_t adesc = sdesc_k_sw128(sa);
          const uint64_t bdesc = sdesc_k_sw128(sa + C::A_BYTES);
#pragma unroll
          for (int k = 0; k < 4; ++k) {  // 4 x 32-byte K steps inside the 128-byte row
            const uint64_t step = static_cast<uint64_t>(k * 2);  // (32 bytes) >> 4
            if constexpr (F16IN)
              mma_f16(d, adesc + step, bdesc + step, idesc, (kb | k) != 0);
            else if constexpr (PAIR)
              mma_i8_pair(d, adesc + step, bdesc + step, idesc, (kb | k) != 0);
            else
              mma_i8(d, adesc + step, bdesc + step, idesc, (kb | k) != 0);
          }
          commit_both(&empty[stage]);  // frees the stage (in both CTAs) once these MMAs have read it
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        commit_both(&tfull[acc]);  // accumulator ready for the epilogue (of both CTAs)
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1u;
        }
      }
      // Drain: every MMA this thread issued must finish before TMEM is released.
      commit(drain);
      const uint32_t addr = smem_u32(drain);
      const unsigned long long t0 = globaltimer();
      while (!mbar_try_wait(addr, 0)) {
        if (globaltimer() - t0 > kWaitLimitNs) {
          atomicCAS(args.err, 0, kDevTimeoutDrain);
          break;
        }
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue (warps 2..9)
    pdl_wait();
    const int ew = warp - 2;
    const int q = warp & 3;         // TMEM sub-partition (lanes 32q..32q+31) this warp can read
    const int half = ew >> 2;       // which half of the tile's columns this warp owns
    const int row_in_tile = q * 32 + lane;
    uint8_t* const stg = staging + ew * C::STAGING;
    constexpr int HALF = BN / 2;
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int t = unit; t < tiles; t += units) {
      const int tm = t / tiles_n, tn = t % tiles_n;
      const int m_block = tm * C::TILE_M + static_cast<int>(rank) * C::BM + q * 32;  // this warp's 32-row block
      const int m = m_block + row_in_tile - q * 32;
      const bool row_ok = m < args.M;
      // RoPE: this row's 32 angles, loaded once per tile (every 64-column head of the tile rotates by the
      // same angles) and before the accumulator wait, so their L2 latency overlaps the mainloop. The
      // tables are angle-major [32, tokens]: the warp's 32 consecutive rows read 128 contiguous bytes per
      // angle (one wavefront); the table column of position 0 (class token) is the identity.
      float rope_c[EPI == EPI_QKV_ROPE ? 32 : 1], rope_s[EPI == EPI_QKV_ROPE ? 32 : 1];
      if constexpr (EPI == EPI_QKV_ROPE) {
        if (tn * BN < args.rope_cols) {
          const int pos = (row_ok ? m : 0) % args.tokens;
          // One load loop for both table forms: pointers and stride per form. Separable tables (L1-resident)
          // are [32, grid + 1], column `grid` the class token's identity rotation.
          const float *c0, *s0, *c1, *s1;
          int step;
          if (args.rope_grid > 0) {
            const int G = args.rope_grid, idx = pos - args.rope_cls;
            int r = G, c = G;
            if (idx >= 0) {
              r = idx / G;
              c = idx - r * G;
            }
            step = G + 1;
            const int a0 = args.rope_swap ? c : r, a1 = args.rope_swap ? r : c;
            c0 = args.rope_cos_c + a0;
            s0 = args.rope_sin_c + a0;
            c1 = args.rope_cos_c + 16 * step + a1;
            s1 = args.rope_sin_c + 16 * step + a1;
          } else {
            step = args.tokens;
            c0 = args.rope_cos + pos;
            s0 = args.rope_sin + pos;
            c1 = args.rope_cos + 16 * step + pos;
            s1 = args.rope_sin + 16 * step + pos;
          }
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            rope_c[j] = __ldg(c0 + j * step);
            rope_s[j] = __ldg(s0 + j * step);
            rope_c[16 + j] = __ldg(c1 + j * step);
            rope_s[16 + j] = __ldg(s1 + j * step);
          }
        }
      }
      if (!wait(&tfull[acc], acc_phase, kDevTimeoutTmemFull)) break;
      tc_fence_after();
      const uint32_t tbase = tmem + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(acc * BN);
      const int n_tile = tn * BN;
      float rs = 1.f;
      if constexpr (!F16IN) rs = row_ok ? args.row_scale[m] : 0.f;
      __half* out16 = static_cast<__half*>(args.out);

      if constexpr (EPI == EPI_SWIGLU) {
        // Tile columns hold [gate 64 | up 64] groups; the output h has N/2 columns.
        constexpr int OUTS = BN == 256 ? 64 : 32;  // output columns per warp
        const int cg0 = BN == 256 ? half * 128 : half * 32;
        const int col0 = (n_tile >> 1) + (BN == 256 ? half * 64 : half * 32);
        // The staging buffer is free once this warp's previous TMA store has read it; each 32-column
        // group of the output goes into it as soon as it is packed.
        if (lane == 0) bulk_wait_read_all();
        __syncwarp();
#pragma unroll
        for (int sub = 0; sub < OUTS / 32; ++sub) {
          uint32_t rg[32], ru[32];
          const int cg = cg0 + sub * 32, cu = cg + 64;
          __syncwarp();  // tcgen05.ld is .sync.aligned: the whole warp must arrive converged
          tmem_ld32(tbase + cg, rg);
          tmem_ld32(tbase + cu, ru);
          tmem_ld_wait();
          float2 g[16], u[16];
          dequant32_x2(rg, rs, args.col_scale + n_tile + cg, args.bias + n_tile + cg, g);
          dequant32_x2(ru, rs, args.col_scale + n_tile + cu, args.bias + n_tile + cu, u);
          uint32_t packed[16];
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const float2 h = silu_mul2(g[j], u[j]);
            packed[j] = pack_half2(h.x, h.y);
          }
          if constexpr (OUTS == 64) {
            stage_half_row128(stg, lane, sub, packed);
          } else {
            stage_row64(stg, lane, packed);
          }
        }
        fence_async_smem();
        __syncwarp();
        if (lane == 0) {
          tma_store_2d(&tmC, stg, col0, m_block);
          bulk_commit_group();
        }
      } else if constexpr (EPI == EPI_BIAS || EPI == EPI_QKV_ROPE || EPI == EPI_RESIDUAL || EPI == EPI_GELU_F16) {
        // 64 fp16 output columns per chunk; the warp owns HALF columns. The residual epilogue adds the
        // fp16-rounded y to the fp16 stream with a TMA add-reduction (x = fp16(x + fp16(y)), the reference's
        // __hadd2 of the staged fp16 result, foidfinder/backends/cuda/csrc/gemm.cuh:163-169).
#pragma unroll  // unrolled: QKV + RoPE 0.229 -> 0.216 ms at bs64 (rolled, the RoPE branch stayed inside)
        for (int ch = 0; ch < HALF / 64; ++ch) {
          const int c0 = half * HALF + ch * 64;  // tile column of this chunk
          const int n0 = n_tile + c0;
          // The staging buffer is free once this warp's previous TMA store has read it; each 32-column
          // half of the chunk goes into it as soon as it is packed.
          if (lane == 0) bulk_wait_read_all();
          __syncwarp();
#pragma unroll
          for (int sub = 0; sub < 2; ++sub) {
            uint32_t r[32];
            __syncwarp();
            tmem_ld32(tbase + c0 + sub * 32, r);
            tmem_ld_wait();
            float y[32];
            if constexpr (F16IN) {
              // fp16 operands: the accumulator is already f32; y = acc + bias.
              const float* bp = args.bias + n0 + sub * 32;
#pragma unroll
              for (int j = 0; j < 32; j += 4) {
                const float4 b4 = *reinterpret_cast<const float4*>(bp + j);
                y[j] = __uint_as_float(r[j]) + b4.x;
                y[j + 1] = __uint_as_float(r[j + 1]) + b4.y;
                y[j + 2] = __uint_as_float(r[j + 2]) + b4.z;
                y[j + 3] = __uint_as_float(r[j + 3]) + b4.w;
              }
            } else {
              dequant32(r, rs, args.col_scale + n0 + sub * 32, args.bias + n0 + sub * 32, y);
            }
            if constexpr (EPI == EPI_QKV_ROPE) {
              if (n0 < args.rope_cols) {
                // Interleaved pairs (2i, 2i+1) of each 64-wide head rotate by the angle of pair i at this
                // token's position.
#pragma unroll
                for (int j = 0; j < 16; ++j) {
                  const float cc = rope_c[sub * 16 + j], ss = rope_s[sub * 16 + j];
                  const float x0 = y[2 * j], x1 = y[2 * j + 1];
                  y[2 * j] = x0 * cc - x1 * ss;
                  y[2 * j + 1] = x0 * ss + x1 * cc;
                }
              }
            }
            if constexpr (EPI == EPI_GELU_F16) {
#pragma unroll
              for (int j = 0; j < 32; ++j) y[j] = gelu_tanh(y[j]);
            }
            uint32_t packed[16];
#pragma unroll
            for (int j = 0; j < 32; j += 2) packed[j / 2] = pack_half2(y[j], y[j + 1]);
            stage_half_row128(stg, lane, sub, packed);
          }
          fence_async_smem();
          __syncwarp();
          if (lane == 0) {
            if constexpr (EPI == EPI_RESIDUAL)
              tma_reduce_add_2d(&tmC, stg, n0, m_block);
            else
              tma_store_2d(&tmC, stg, n0, m_block);
            bulk_commit_group();
          }
        }
      } else {
        // S32 (debug), LOGITS (ragged tag count) and STEM (row remap): one row per thread, direct stores.
#pragma unroll 1
        for (int ch = 0; ch < HALF / 32; ++ch) {
          const int c0 = half * HALF + ch * 32;
          const int n0 = n_tile + c0;
          uint32_t r[32];
          __syncwarp();
          tmem_ld32(tbase + c0, r);
          tmem_ld_wait();
          if (!row_ok) {
            // rows past M: nothing to store
          } else if constexpr (EPI == EPI_S32) {
            int4* dst = reinterpret_cast<int4*>(static_cast<int*>(args.out) + static_cast<size_t>(m) * args.ldo + n0);
#pragma unroll
            for (int v = 0; v < 8; ++v)
              dst[v] = make_int4(static_cast<int>(r[4 * v]), static_cast<int>(r[4 * v + 1]),
                                 static_cast<int>(r[4 * v + 2]), static_cast<int>(r[4 * v + 3]));
          } else if constexpr (EPI == EPI_LOGITS) {
            float* dst = static_cast<float*>(args.out) + static_cast<size_t>(m) * args.ldo;
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              const int n = n0 + j;
              if (n < args.n_valid) dst[n] = __uint_as_float(r[j]) + args.bias[n];
            }
          } else if constexpr (EPI == EPI_STEM) {
            // Patch row m of image b = m / patches goes to token b * tokens + (tokens - patches) + (m % patches)
            // (with a class token, token 0 of each image). pos_bias = patch bias + position embedding.
            const int b = m / args.patches, p = m - b * args.patches;
            const float* pb = args.pos_bias + static_cast<size_t>(p) * args.N + n0;
            uint32_t packed[16];
#pragma unroll
            for (int j = 0; j < 32; j += 4) {
              const float4 pv = *reinterpret_cast<const float4*>(pb + j);
              packed[j / 2] = pack_half2(__uint_as_float(r[j]) + pv.x, __uint_as_float(r[j + 1]) + pv.y);
              packed[j / 2 + 1] = pack_half2(__uint_as_float(r[j + 2]) + pv.z, __uint_as_float(r[j + 3]) + pv.w);
            }
            uint4* d4 = reinterpret_cast<uint4*>(out16 + (static_cast<size_t>(b) * args.tokens + (args.tokens - args.patches) + p) * args.ldo + n0);
#pragma unroll
            for (int v = 0; v < 4; ++v)
              d4[v] = make_uint4(packed[4 * v], packed[4 * v + 1], packed[4 * v + 2], packed[4 * v + 3]);
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if (PAIR && !leader)
          mbar_arrive_cluster(mapa_shared(smem_u32(&tempty[acc]), 0u));  // the even CTA's MMA reuses it
        else
          mbar_arrive(&tempty[acc]);
      }
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1u;
      }
    }
  }

  if constexpr (kTmaStore)
    if (warp >= 2 && lane == 0) bulk_wait_all();  // this warp's output stores are complete
  __syncwarp();
  tc_fence_before();
  __syncthreads();
  if constexpr (PAIR) cluster_sync();  // the even CTA's MMAs into this CTA's TMEM have drained
  tc_fence_after();
  if (warp == 1) {
    if constexpr (PAIR)
      tmem_dealloc2(tmem, C::TMEM_COLS);
    else
      tmem_dealloc(tmem, C::TMEM_COLS);
  }
}

}  // namespace ff
