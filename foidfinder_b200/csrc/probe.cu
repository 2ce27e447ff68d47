// Measured int8 tensor-core peak of this GPU (the roofline denominator for the W8A8 GEMMs, which the
// measured-peaks file only gives for bf16): one CTA per SM issues back-to-back
// tcgen05.mma.cta_group::1.kind::i8 (M128 N256 K32, the GEMM's instruction shape) on shared-memory operands
// that stay resident, accumulating into TMEM, with no global-memory traffic and no epilogue. The operands
// hold pseudo-random bytes so the datapath toggles as in a real GEMM.
#include "common.h"
#include "ptx.cuh"

namespace ff {
namespace {

constexpr int kProbeThreads = 128;
constexpr int kA = 128 * 128, kB = 256 * 128;  // one 128-byte K row of A (128 rows) and B (256 rows)
constexpr int kProbeSmem = 1024 + kA + kB + 64;

__global__ void __launch_bounds__(kProbeThreads, 1) int8_mma_peak_kernel(int iters, int* err) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* done = reinterpret_cast<uint64_t*>(smem + kA + kB);
  uint32_t* slot = reinterpret_cast<uint32_t*>(done + 1);
  const int warp = threadIdx.x >> 5;
  uint32_t seed = 0x9E3779B9u * (blockIdx.x * kProbeThreads + threadIdx.x + 1);
  for (int i = threadIdx.x; i < (kA + kB) / 4; i += kProbeThreads) {
    seed = seed * 1664525u + 1013904223u;
    reinterpret_cast<uint32_t*>(smem)[i] = seed;
  }
  fence_async_smem();
  if (threadIdx.x == 0) {
    mbar_init(done, 1);
    fence_mbar_init();
  }
  if (warp == 0) {
    tmem_alloc(slot, 256);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *slot;
  if (threadIdx.x == 0) {
    constexpr uint32_t idesc = idesc_s8(128, 256);
    const uint64_t ad = sdesc_k_sw128(smem_u32(smem)), bd = sdesc_k_sw128(smem_u32(smem + kA));
    for (int it = 0; it < iters; ++it)
#pragma unroll
      for (int k = 0; k < 4; ++k) mma_i8(tmem, ad + 2 * k, bd + 2 * k, idesc, (it | k) != 0);
    tc_commit(done);
    const unsigned long long t0 = globaltimer();
    while (!mbar_try_wait(smem_u32(done), 0)) {
      if (globaltimer() - t0 > kWaitLimitNs) {
        atomicCAS(err, 0, kDevTimeoutDrain);
        break;
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0) tmem_dealloc(tmem, 256);
}

}  // namespace
}  // namespace ff

using namespace ff;

extern "C" int ff_int8_mma_peak(int iters, float* ms, double* ops, void* stream) {
  FF_REQUIRE(ms && ops && iters >= 1 && iters <= (1 << 22), "ff_int8_mma_peak: bad arguments (iters %d)", iters);
  int* err = device_error_word();
  FF_REQUIRE(err != nullptr, "ff_int8_mma_peak: no device error word");
  if (cudaFuncSetAttribute(int8_mma_peak_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kProbeSmem) != cudaSuccess)
    return check_launch("ff_int8_mma_peak: cudaFuncSetAttribute");
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaEvent_t e0, e1;
  if (cudaEventCreate(&e0) != cudaSuccess || cudaEventCreate(&e1) != cudaSuccess)
    return check_launch("ff_int8_mma_peak: event create");
  const int grid = sm_count();
  int8_mma_peak_kernel<<<grid, kProbeThreads, kProbeSmem, s>>>(iters / 10 + 1, err);  // warm-up
  cudaEventRecord(e0, s);
  int8_mma_peak_kernel<<<grid, kProbeThreads, kProbeSmem, s>>>(iters, err);
  cudaEventRecord(e1, s);
  int rc = check_launch("int8_mma_peak_kernel");
  if (rc == FF_OK && cudaEventSynchronize(e1) != cudaSuccess) rc = check_launch("ff_int8_mma_peak: sync");
  if (rc == FF_OK) {
    cudaEventElapsedTime(ms, e0, e1);
    *ops = 2.0 * 128 * 256 * 128 * static_cast<double>(iters) * grid;  // 4 MMAs x K 32 = 128 per iteration
  }
  cudaEventDestroy(e0);
  cudaEventDestroy(e1);
  return rc;
}
