// Persistent tcgen05 GEMM for sm_100a: Y[m, n] = sum_k A[m, k] * W[n, k], both operands K-major.
//
// Replaces the reference's mma.sync int8 GEMM (foidfinder/backends/cuda/csrc/gemm.cuh:43-172) and the
// cuBLAS fp16 matmuls of the stem and head (foidfinder/backends/cuda/engine.py:146,
// foidfinder/backends/cuda/reference.py:133-140).
//
// Layout of one CTA (192 threads, one CTA per SM, grid = min(tiles, SMs)):
//   warp 0     TMA producer: A box 128 x 128 B and W box BN x 128 B per stage, 128-byte swizzle
//   warp 1     TMEM allocator and MMA issuer: 4 tcgen05.mma (K = 32 bytes each) per stage
//   warps 2-5  epilogue: tcgen05.ld of the accumulator (warp w reads TMEM lanes 32*(w%4)..+31, one
//              output row per thread), fused dequantisation / bias / RoPE / SwiGLU / residual, store.
// Accumulators are double-buffered in TMEM (2 x BN columns), so the epilogue of tile i overlaps the
// mainloop of tile i+1. Stages are a ring of STAGES smem buffers guarded by full/empty mbarriers.
#pragma once
#include "ptx.cuh"
#include "gemm_args.h"

namespace ff {

template <int BN, int STAGES>
struct GemmCfg {
  static constexpr int BM = 128;
  static constexpr int BKB = 128;  // K bytes per stage (one 128-byte swizzle row)
  static constexpr int A_BYTES = BM * BKB;
  static constexpr int B_BYTES = BN * BKB;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int TMEM_COLS = 2 * BN;  // double-buffered accumulator
  static constexpr int BAR_BYTES = 256;
  static constexpr int SMEM = 1024 /*alignment slack*/ + STAGES * STAGE_BYTES + BAR_BYTES;
  static_assert(BN % 32 == 0 && BN >= 64 && BN <= 256, "BN");
  static_assert(TMEM_COLS == 128 || TMEM_COLS == 256 || TMEM_COLS == 512, "TMEM columns must be a power of two");
  static_assert(SMEM <= 227 * 1024, "shared memory");
};

__device__ __forceinline__ float silu_mul(float g, float u) { return g / (1.f + __expf(-g)) * u; }

template <int BN, int STAGES, bool F16IN, int EPI>
__global__ void __launch_bounds__(192, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const GemmArgs args) {
  using C = GemmCfg<BN, STAGES>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * C::STAGE_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tiles_n = args.N / BN;
  const int tiles = args.tiles_m * tiles_n;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 4);  // one arrive per epilogue warp
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
    tmem_alloc(tmem_slot, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int last_phase[STAGES];
#pragma unroll
      for (int s = 0; s < STAGES; ++s) last_phase[s] = -1;
      constexpr int kElemsPerStage = F16IN ? C::BKB / 2 : C::BKB;
      bool ok = true;
      for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x) {
        const int tm = t / tiles_n, tn = t % tiles_n;
        for (int kb = 0; kb < args.num_kb; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag, args.err, kDevTimeoutSmemEmpty)) {
            ok = false;
            break;
          }
          uint8_t* sa = smem + stage * C::STAGE_BYTES;
          mbar_arrive_expect_tx(&full[stage], C::STAGE_BYTES);
          tma_load_2d(sa, &tmA, &full[stage], kb * kElemsPerStage, tm * C::BM);
          tma_load_2d(sa + C::A_BYTES, &tmB, &full[stage], kb * kElemsPerStage, tn * BN);
          last_phase[stage] = static_cast<int>(phase);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (!ok) {
        // Let every issued copy land before the CTA exits (bounded).
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
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = F16IN ? idesc_f16(128, BN) : idesc_s8(128, BN);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x) {
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1u, abort_flag, args.err, kDevTimeoutTmemEmpty)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem + static_cast<uint32_t>(acc * BN);
        for (int kb = 0; kb < args.num_kb; ++kb) {
          if (!mbar_wait(&full[stage], phase, abort_flag, args.err, kDevTimeoutTmaFull)) {
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
            else
              mma_i8(d, adesc + step, bdesc + step, idesc, (kb | k) != 0);
          }
          tc_commit(&empty[stage]);  // frees the stage once these MMAs have read it
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        tc_commit(&tfull[acc]);  // accumulator ready for the epilogue
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1u;
        }
      }
      // Drain: every MMA this thread issued must finish before TMEM is released.
      tc_commit(drain);
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
    // ------------------------------------------------------------ epilogue (warps 2..5)
    const int q = warp & 3;  // TMEM sub-partition this warp can read
    const int row_in_tile = q * 32 + lane;
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int t = blockIdx.x; t < tiles; t += gridDim.x) {
      if (!mbar_wait(&tfull[acc], acc_phase, abort_flag, args.err, kDevTimeoutTmemFull)) break;
      tc_fence_after();
      const int tm = t / tiles_n, tn = t % tiles_n;
      const int m = tm * C::BM + row_in_tile;
      const bool row_ok = m < args.M;
      const uint32_t tbase = tmem + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(acc * BN);
      const int n_tile = tn * BN;

      if constexpr (EPI == EPI_SWIGLU) {
        // Tile columns hold [gate 64 | up 64] pairs; output h has N/2 columns.
        const float rs = row_ok ? args.row_scale[m] : 0.f;
        for (int g = 0; g < BN / 128; ++g)
          for (int h = 0; h < 2; ++h) {
            uint32_t rg[32], ru[32];
            const int cg = g * 128 + h * 32, cu = cg + 64;
            __syncwarp();  // tcgen05.ld is .sync.aligned: the whole warp must arrive converged
            tmem_ld32(tbase + cg, rg);
            tmem_ld32(tbase + cu, ru);
            tmem_ld_wait();
            if (row_ok) {
              const int ng = n_tile + cg, nu = n_tile + cu;
              uint32_t packed[16];
#pragma unroll
              for (int j = 0; j < 32; j += 2) {
                const float2 csg = *reinterpret_cast<const float2*>(args.col_scale + ng + j);
                const float2 csu = *reinterpret_cast<const float2*>(args.col_scale + nu + j);
                const float2 bg = *reinterpret_cast<const float2*>(args.bias + ng + j);
                const float2 bu = *reinterpret_cast<const float2*>(args.bias + nu + j);
                const float g0 = static_cast<float>(static_cast<int>(rg[j])) * rs * csg.x + bg.x;
                const float g1 = static_cast<float>(static_cast<int>(rg[j + 1])) * rs * csg.y + bg.y;
                const float u0 = static_cast<float>(static_cast<int>(ru[j])) * rs * csu.x + bu.x;
                const float u1 = static_cast<float>(static_cast<int>(ru[j + 1])) * rs * csu.y + bu.y;
                packed[j / 2] = pack_half2(silu_mul(g0, u0), silu_mul(g1, u1));
              }
              const int no = (n_tile >> 1) + g * 64 + h * 32;
              uint4* dst = reinterpret_cast<uint4*>(static_cast<__half*>(args.out) + static_cast<size_t>(m) * args.ldo + no);
#pragma unroll
              for (int v = 0; v < 4; ++v)
                dst[v] = make_uint4(packed[4 * v], packed[4 * v + 1], packed[4 * v + 2], packed[4 * v + 3]);
            }
          }
      } else {
        float rs = 1.f;
        if constexpr (!F16IN) rs = row_ok ? args.row_scale[m] : 0.f;
        for (int c = 0; c < BN / 32; ++c) {
          uint32_t r[32];
          __syncwarp();  // tcgen05.ld is .sync.aligned: the whole warp must arrive converged
          tmem_ld32(tbase + c * 32, r);
          tmem_ld_wait();
          const int n0 = n_tile + c * 32;
          if (!row_ok) {
            // rows past M: nothing to store
          } else if constexpr (EPI == EPI_S32) {
            int4* dst = reinterpret_cast<int4*>(static_cast<int*>(args.out) + static_cast<size_t>(m) * args.ldo + n0);
#pragma unroll
            for (int v = 0; v < 8; ++v)
              dst[v] = make_int4(static_cast<int>(r[4 * v]), static_cast<int>(r[4 * v + 1]), static_cast<int>(r[4 * v + 2]),
                                 static_cast<int>(r[4 * v + 3]));
          } else if constexpr (EPI == EPI_LOGITS) {
            // f32 logits, columns >= n_valid (padding of the tag count) are dropped.
            float* dst = static_cast<float*>(args.out) + static_cast<size_t>(m) * args.ldo;
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              const int n = n0 + j;
              if (n < args.n_valid) dst[n] = __uint_as_float(r[j]) + args.bias[n];
            }
          } else if constexpr (EPI == EPI_STEM) {
            // Patch row m of image b = m / patches goes to token b * tokens + 1 + (m % patches)
            // (token 0 of each image is the class token). pos_bias = patch bias + position embedding.
            const int b = m / args.patches, p = m - b * args.patches;
            const float* pb = args.pos_bias + static_cast<size_t>(p) * args.N + n0;
            __half* dst = static_cast<__half*>(args.out) + (static_cast<size_t>(b) * args.tokens + 1 + p) * args.ldo + n0;
            uint32_t packed[16];
#pragma unroll
            for (int j = 0; j < 32; j += 4) {
              const float4 pv = *reinterpret_cast<const float4*>(pb + j);
              packed[j / 2] = pack_half2(__uint_as_float(r[j]) + pv.x, __uint_as_float(r[j + 1]) + pv.y);
              packed[j / 2 + 1] = pack_half2(__uint_as_float(r[j + 2]) + pv.z, __uint_as_float(r[j + 3]) + pv.w);
            }
            uint4* d4 = reinterpret_cast<uint4*>(dst);
#pragma unroll
            for (int v = 0; v < 4; ++v)
              d4[v] = make_uint4(packed[4 * v], packed[4 * v + 1], packed[4 * v + 2], packed[4 * v + 3]);
          } else {
            // int32 -> f32 dequantisation: y = acc * row_scale[m] * col_scale[n] + bias[n]
            float y[32];
#pragma unroll
            for (int j = 0; j < 32; j += 4) {
              const float4 cs = *reinterpret_cast<const float4*>(args.col_scale + n0 + j);
              const float4 bi = *reinterpret_cast<const float4*>(args.bias + n0 + j);
              y[j] = static_cast<float>(static_cast<int>(r[j])) * rs * cs.x + bi.x;
              y[j + 1] = static_cast<float>(static_cast<int>(r[j + 1])) * rs * cs.y + bi.y;
              y[j + 2] = static_cast<float>(static_cast<int>(r[j + 2])) * rs * cs.z + bi.z;
              y[j + 3] = static_cast<float>(static_cast<int>(r[j + 3])) * rs * cs.w + bi.w;
            }
            if constexpr (EPI == EPI_QKV_ROPE) {
              if (n0 < args.rope_cols) {
                // Interleaved pairs (2i, 2i+1) of each 64-wide head rotate by the angle of pair
                // (n % 64) / 2 at this token's position; the table row of position 0 (class token)
                // is the identity.
                const int pos = m % args.tokens;
                const float* cr = args.rope_cos + static_cast<size_t>(pos) * 32 + ((n0 & 63) >> 1);
                const float* sr = args.rope_sin + static_cast<size_t>(pos) * 32 + ((n0 & 63) >> 1);
#pragma unroll
                for (int j = 0; j < 16; j += 4) {
                  const float4 c4 = *reinterpret_cast<const float4*>(cr + j);
                  const float4 s4 = *reinterpret_cast<const float4*>(sr + j);
                  const float cc[4] = {c4.x, c4.y, c4.z, c4.w}, ss[4] = {s4.x, s4.y, s4.z, s4.w};
#pragma unroll
                  for (int e = 0; e < 4; ++e) {
                    const float x0 = y[2 * (j + e)], x1 = y[2 * (j + e) + 1];
                    y[2 * (j + e)] = x0 * cc[e] - x1 * ss[e];
                    y[2 * (j + e) + 1] = x0 * ss[e] + x1 * cc[e];
                  }
                }
              }
            }
            __half* dst = static_cast<__half*>(args.out) + static_cast<size_t>(m) * args.ldo + n0;
            uint4* d4 = reinterpret_cast<uint4*>(dst);
            if constexpr (EPI == EPI_RESIDUAL) {
              // fp16 residual stream: x = fp16(float(x) + y)
#pragma unroll
              for (int v = 0; v < 4; ++v) {
                const uint4 old = d4[v];
                const uint32_t ow[4] = {old.x, old.y, old.z, old.w};
                uint32_t nw[4];
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                  const float2 o2 = unpack_half2(ow[e]);
                  nw[e] = pack_half2(o2.x + y[8 * v + 2 * e], o2.y + y[8 * v + 2 * e + 1]);
                }
                d4[v] = make_uint4(nw[0], nw[1], nw[2], nw[3]);
              }
            } else {
#pragma unroll
              for (int v = 0; v < 4; ++v)
                d4[v] = make_uint4(pack_half2(y[8 * v], y[8 * v + 1]), pack_half2(y[8 * v + 2], y[8 * v + 3]),
                                   pack_half2(y[8 * v + 4], y[8 * v + 5]), pack_half2(y[8 * v + 6], y[8 * v + 7]));
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[acc]);
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1u;
      }
    }
  }

  __syncwarp();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, C::TMEM_COLS);
}

}  // namespace ff
