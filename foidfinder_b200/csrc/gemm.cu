// Host side of the tcgen05 GEMM: argument checks, TMA descriptors, tile-shape choice and launch.
#include "common.h"
#include "gemm.h"
#include "gemm_tc.cuh"

namespace ff {

namespace {

template <int BN, int STAGES, bool F16IN, int EPI>
int launch_one(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tc, const GemmArgs& a,
               cudaStream_t stream) {
  using C = GemmCfg<BN, STAGES>;
  auto kernel = gemm_tc_kernel<BN, STAGES, F16IN, EPI>;
  static bool configured[64] = {};  // per instantiation and device
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64 || !configured[dev]) {
    if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM) != cudaSuccess)
      return check_launch("gemm: cudaFuncSetAttribute");
    if (dev >= 0 && dev < 64) configured[dev] = true;
  }
  const int tiles = a.tiles_m * (a.N / BN);
  const int grid = tiles < sm_count() ? tiles : sm_count();
  launch(kernel, dim3(grid), dim3(C::THREADS), C::SMEM, stream, ta, tb, tc, a);
  return check_launch("gemm_tc_kernel");
}

// Pair tiles (256 x BN over a cluster of two CTAs): as many clusters as fit at once, each walking tiles.
constexpr int kPairStages = 6;

template <int EPI>
int launch_pair(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tc, const GemmArgs& a,
                cudaStream_t stream) {
  using C = GemmCfg<256, kPairStages, true>;
  auto kernel = gemm_tc_kernel<256, kPairStages, false, EPI, true>;
  static int max_clusters[64] = {};  // per instantiation and device, 0 = not configured yet
  int dev = 0;
  cudaGetDevice(&dev);
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;  // as ff::launch (common.h)
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.blockDim = dim3(C::THREADS);
  cfg.dynamicSmemBytes = C::SMEM;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int clusters = dev >= 0 && dev < 64 ? max_clusters[dev] : 0;
  if (clusters == 0) {
    if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM) != cudaSuccess)
      return check_launch("gemm (pair): cudaFuncSetAttribute");
    cfg.gridDim = dim3(2 * (sm_count() / 2));
    if (cudaOccupancyMaxActiveClusters(&clusters, kernel, &cfg) != cudaSuccess || clusters < 1)
      return check_launch("gemm (pair): cudaOccupancyMaxActiveClusters");
    if (dev >= 0 && dev < 64) max_clusters[dev] = clusters;
  }
  const int tiles = a.tiles_m * (a.N / 256);
  cfg.gridDim = dim3(2 * (tiles < clusters ? tiles : clusters));
  cfg.numAttrs = 2;
  if (cudaLaunchKernelEx(&cfg, kernel, ta, tb, tc, a) != cudaSuccess) return check_launch("gemm_tc_kernel (pair)");
  return check_launch("gemm_tc_kernel (pair)");
}

template <int BN, bool F16IN>
int dispatch_epi(int epi, const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tc, const GemmArgs& a,
                 cudaStream_t s) {
  constexpr int STAGES = BN == 256 ? 4 : 6;
  if constexpr (F16IN) {
    switch (epi) {
      case EPI_STEM: return launch_one<BN, STAGES, true, EPI_STEM>(ta, tb, tc, a, s);
      case EPI_LOGITS: return launch_one<BN, STAGES, true, EPI_LOGITS>(ta, tb, tc, a, s);
      case EPI_BIAS: return launch_one<BN, STAGES, true, EPI_BIAS>(ta, tb, tc, a, s);
    }
  } else {
    switch (epi) {
      case EPI_QKV_ROPE: return launch_one<BN, STAGES, false, EPI_QKV_ROPE>(ta, tb, tc, a, s);
      case EPI_RESIDUAL: return launch_one<BN, STAGES, false, EPI_RESIDUAL>(ta, tb, tc, a, s);
      case EPI_SWIGLU: return launch_one<BN, STAGES, false, EPI_SWIGLU>(ta, tb, tc, a, s);
      case EPI_BIAS: return launch_one<BN, STAGES, false, EPI_BIAS>(ta, tb, tc, a, s);
      case EPI_GELU_F16: return launch_one<BN, STAGES, false, EPI_GELU_F16>(ta, tb, tc, a, s);
      case EPI_S32: return launch_one<BN, STAGES, false, EPI_S32>(ta, tb, tc, a, s);
    }
  }
  set_error("gemm: epilogue %d is not available for %s inputs", epi, F16IN ? "fp16" : "int8");
  return FF_ERR_INVALID_ARGUMENT;
}

}  // namespace

bool pair_supported(int N, int bn, bool f16, int epi) {
  return !f16 && bn == 256 && N % 256 == 0 &&
         (epi == EPI_QKV_ROPE || epi == EPI_RESIDUAL || epi == EPI_SWIGLU || epi == EPI_BIAS || epi == EPI_GELU_F16 ||
          epi == EPI_S32);
}

// Pair tiles pay off on long K loops (measured at M = 65,600: K = 2816 +5-6%; K = 1024 within +-3%, the
// epilogue's output traffic being what bounds those) once there are enough 256-row tiles to keep every SM
// pair busy for a few waves.
bool choose_pair(int M, int N, int K, int bn, bool f16, int epi) {
  if (!pair_supported(N, bn, f16, epi) || epi == EPI_S32 || K < 2048) return false;
  const long long pair_tiles = static_cast<long long>((M + 255) / 256) * (N / 256);
  return pair_tiles >= 2LL * sm_count();
}

int choose_tile_n(int M, int N) {
  // Prefer 256-wide tiles; drop to 128 when 256 would leave most SMs idle (small M) or N needs it.
  if (N % 256 != 0) return 128;
  const int tiles256 = ((M + 127) / 128) * (N / 256);
  return tiles256 * 2 <= sm_count() ? 128 : 256;
}

int gemm_prepare(const GemmProblem& p, GemmPlan* plan) {
  const bool f16 = p.f16;
  const int elt = f16 ? 2 : 1;
  FF_REQUIRE(p.A != nullptr && p.W != nullptr && p.out != nullptr, "gemm: NULL operand");
  FF_REQUIRE(p.M >= 1 && p.N >= 1 && p.K >= 1, "gemm: bad shape M=%d N=%d K=%d", p.M, p.N, p.K);
  FF_REQUIRE((static_cast<int64_t>(p.K) * elt) % 128 == 0, "gemm: K*%d bytes must be a multiple of 128 (K=%d)", elt, p.K);
  FF_REQUIRE(aligned16(p.A) && aligned16(p.W), "gemm: A and W must be 16-byte aligned");
  int bn = p.tile_n == 0 ? choose_tile_n(p.M, p.N) : p.tile_n == FF_TILE_PAIR256 ? 256 : p.tile_n;
  FF_REQUIRE(bn == 128 || bn == 256, "gemm: tile_n must be 0, 128, 256 or FF_TILE_PAIR256 (got %d)", p.tile_n);
  const bool pair = p.tile_n == FF_TILE_PAIR256 || (p.tile_n == 0 && choose_pair(p.M, p.N, p.K, bn, f16, p.epi));
  FF_REQUIRE(!pair || pair_supported(p.N, bn, f16, p.epi),
             "gemm: pair tiles need int8 operands, N %% 256 == 0 and an s32/bias/QKV/SwiGLU/GELU/residual epilogue");
  FF_REQUIRE(p.N % bn == 0, "gemm: N=%d must be a multiple of the tile width %d", p.N, bn);
  const CUtensorMapDataType dt = f16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_UINT8;
  const uint32_t box_k = 128 / elt;
  int rc = make_tmap_2d(&plan->ta, p.A, dt, elt, static_cast<uint64_t>(p.K), static_cast<uint64_t>(p.M), box_k, 128);
  if (rc != FF_OK) return rc;
  rc = make_tmap_2d(&plan->tb, p.W, dt, elt, static_cast<uint64_t>(p.K), static_cast<uint64_t>(p.N), box_k,
                    static_cast<uint32_t>(pair ? bn / 2 : bn));  // a pair CTA loads half of the tile's W rows
  if (rc != FF_OK) return rc;
  // Output map for the TMA-store (and, for the residual, TMA add-reduce) epilogues: fp16 [M, out_cols] with
  // row pitch ldo, boxes of 32 rows x
  // 64 columns (128-byte swizzle) or, for the 128-wide SwiGLU tile, 32 columns (64-byte swizzle) — the
  // layouts the epilogue's staging buffer is written in.
  plan->tc = plan->ta;
  if (p.epi == EPI_BIAS || p.epi == EPI_QKV_ROPE || p.epi == EPI_SWIGLU || p.epi == EPI_RESIDUAL ||
      p.epi == EPI_GELU_F16) {
    const int out_cols = p.epi == EPI_SWIGLU ? p.N / 2 : p.N;
    const int ldo = p.args.ldo;
    FF_REQUIRE(ldo >= out_cols && ldo % 8 == 0, "gemm: output row stride %d for %d columns", ldo, out_cols);
    FF_REQUIRE(aligned16(p.out), "gemm: out must be 16-byte aligned");
    const bool narrow = p.epi == EPI_SWIGLU && bn == 128;
    rc = make_tmap_2d_pitched(&plan->tc, p.out, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, static_cast<uint64_t>(out_cols),
                              static_cast<uint64_t>(p.M), static_cast<uint64_t>(ldo) * 2, narrow ? 32 : 64, 32,
                              narrow ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc != FF_OK) return rc;
  }
  plan->args = p.args;
  plan->args.M = p.M;
  plan->args.N = p.N;
  plan->args.K = p.K;
  plan->args.num_kb = static_cast<int>((static_cast<int64_t>(p.K) * elt) / 128);
  plan->args.tiles_m = pair ? (p.M + 255) / 256 : (p.M + 127) / 128;
  plan->args.out = p.out;
  plan->args.err = p.err_word != nullptr ? p.err_word : device_error_word();
  FF_REQUIRE(plan->args.err != nullptr, "gemm: no device error word");
  plan->bn = bn;
  plan->pair = pair;
  plan->f16 = f16;
  plan->epi = p.epi;
  return FF_OK;
}

int gemm_launch(const GemmPlan& plan, cudaStream_t stream) {
  if (plan.pair) {
    switch (plan.epi) {
      case EPI_QKV_ROPE: return launch_pair<EPI_QKV_ROPE>(plan.ta, plan.tb, plan.tc, plan.args, stream);
      case EPI_RESIDUAL: return launch_pair<EPI_RESIDUAL>(plan.ta, plan.tb, plan.tc, plan.args, stream);
      case EPI_SWIGLU: return launch_pair<EPI_SWIGLU>(plan.ta, plan.tb, plan.tc, plan.args, stream);
      case EPI_BIAS: return launch_pair<EPI_BIAS>(plan.ta, plan.tb, plan.tc, plan.args, stream);
      case EPI_GELU_F16: return launch_pair<EPI_GELU_F16>(plan.ta, plan.tb, plan.tc, plan.args, stream);
      case EPI_S32: return launch_pair<EPI_S32>(plan.ta, plan.tb, plan.tc, plan.args, stream);
    }
    set_error("gemm: epilogue %d has no pair-tile kernel", plan.epi);
    return FF_ERR_INVALID_ARGUMENT;
  }
  if (plan.f16)
    return plan.bn == 256 ? dispatch_epi<256, true>(plan.epi, plan.ta, plan.tb, plan.tc, plan.args, stream)
                          : dispatch_epi<128, true>(plan.epi, plan.ta, plan.tb, plan.tc, plan.args, stream);
  return plan.bn == 256 ? dispatch_epi<256, false>(plan.epi, plan.ta, plan.tb, plan.tc, plan.args, stream)
                        : dispatch_epi<128, false>(plan.epi, plan.ta, plan.tb, plan.tc, plan.args, stream);
}

}  // namespace ff

using namespace ff;

extern "C" int ff_gemm_s8(const int8_t* A, const int8_t* W, const float* row_scale, const float* col_scale,
                          const float* bias, void* out, int M, int N, int K, int epi, const float* rope_cos,
                          const float* rope_sin, int rope_cols, int tokens, int tile_n, void* stream) {
  FF_REQUIRE(epi == EPI_QKV_ROPE || epi == EPI_RESIDUAL || epi == EPI_SWIGLU || epi == EPI_BIAS || epi == EPI_S32 ||
                 epi == EPI_GELU_F16,
             "ff_gemm_s8: unknown epilogue %d", epi);
  if (epi != EPI_S32) FF_REQUIRE(row_scale && col_scale && bias, "ff_gemm_s8: scales and bias are required");
  FF_REQUIRE(N % 128 == 0, "ff_gemm_s8: N=%d must be a multiple of 128", N);
  if (epi == EPI_QKV_ROPE) {
    FF_REQUIRE(rope_cos && rope_sin && tokens >= 1, "ff_gemm_s8: QKV epilogue needs RoPE tables and tokens");
    FF_REQUIRE(rope_cols % 64 == 0 && rope_cols >= 0 && rope_cols <= N, "ff_gemm_s8: bad rope_cols %d", rope_cols);
  }
  GemmProblem p{};
  p.A = A;
  p.W = W;
  p.out = out;
  p.M = M;
  p.N = N;
  p.K = K;
  p.epi = epi;
  p.tile_n = tile_n;
  p.f16 = false;
  p.args.row_scale = row_scale;
  p.args.col_scale = col_scale;
  p.args.bias = bias;
  p.args.ldo = epi == EPI_SWIGLU ? N / 2 : N;
  p.args.rope_cos = rope_cos;
  p.args.rope_sin = rope_sin;
  p.args.rope_cols = epi == EPI_QKV_ROPE ? rope_cols : 0;
  p.args.tokens = tokens > 0 ? tokens : 1;
  GemmPlan plan;
  int rc = gemm_prepare(p, &plan);
  if (rc != FF_OK) return rc;
  return gemm_launch(plan, static_cast<cudaStream_t>(stream));
}

extern "C" int ff_gemm_f16(const uint16_t* A, const uint16_t* W, const float* bias, void* out, int M, int N, int K,
                           int epi, int ldo, int n_valid, const float* pos_bias, int patches, int tokens, int tile_n,
                           void* stream) {
  FF_REQUIRE(epi == EPI_STEM || epi == EPI_LOGITS || epi == EPI_BIAS, "ff_gemm_f16: unknown epilogue %d", epi);
  if (epi == EPI_BIAS) {
    FF_REQUIRE(bias != nullptr && ldo >= N && ldo % 8 == 0, "ff_gemm_f16: bias epilogue needs bias and ldo >= N, ldo %% 8 == 0");
  } else if (epi == EPI_STEM) {
    FF_REQUIRE(pos_bias != nullptr && patches >= 1 && (tokens == patches || tokens == patches + 1),
               "ff_gemm_f16: stem needs pos_bias, patches and tokens = patches (+ 1 with a class token)");
    FF_REQUIRE(ldo >= N && ldo % 8 == 0, "ff_gemm_f16: stem ldo %d", ldo);
  } else {
    FF_REQUIRE(bias != nullptr && n_valid >= 1 && n_valid <= N && ldo >= n_valid, "ff_gemm_f16: logits need bias, n_valid <= N, ldo >= n_valid");
  }
  GemmProblem p{};
  p.A = A;
  p.W = W;
  p.out = out;
  p.M = M;
  p.N = N;
  p.K = K;
  p.epi = epi;
  p.tile_n = tile_n;
  p.f16 = true;
  p.args.bias = bias;
  p.args.ldo = ldo;
  p.args.n_valid = n_valid;
  p.args.pos_bias = pos_bias;
  p.args.patches = patches;
  p.args.tokens = tokens;
  GemmPlan plan;
  int rc = gemm_prepare(p, &plan);
  if (rc != FF_OK) return rc;
  return gemm_launch(plan, static_cast<cudaStream_t>(stream));
}
