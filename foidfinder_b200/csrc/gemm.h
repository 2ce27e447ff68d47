// Internal GEMM planning API: the engine encodes TMA descriptors once per buffer (gemm_prepare) and
// replays the launch (gemm_launch) inside its CUDA graph.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>

#include "gemm_args.h"

namespace ff {

struct GemmProblem {
  const void* A;
  const void* W;
  void* out;
  int M, N, K;
  int epi;
  int tile_n;  // 0 = automatic
  bool f16;
  GemmArgs args;  // epilogue fields; M/N/K/num_kb/tiles_m/out/err are filled in by gemm_prepare
  int* err_word = nullptr;  // device error word to use instead of the library's allocated one
};

struct GemmPlan {
  CUtensorMap ta, tb, tc;  // tc: fp16 output, for the epilogues that store through TMA
  GemmArgs args;
  int bn;
  bool pair;  // 256-row tiles over a cluster of two CTAs
  bool f16;
  int epi;
};

int choose_tile_n(int M, int N);
bool choose_pair(int M, int N, int K, int bn, bool f16, int epi);
int gemm_prepare(const GemmProblem& p, GemmPlan* plan);
int gemm_launch(const GemmPlan& plan, cudaStream_t stream);

}  // namespace ff
