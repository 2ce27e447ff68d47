// ff_linear_w8a8_noalloc: the activation-quantise -> W8A8 GEMM pair without any device allocation.
//
// Some callers cannot allocate device memory once they are running: a host application that hands all
// GPU memory to its own pool at start-up and forbids later cudaMalloc calls, a latency-bound serving
// loop where an allocation (and the implicit synchronisation cudaFree brings) is not allowed on the hot
// path, or a plugin that only receives buffers from its host. The ordinary entry points need the caller
// to provide the int8 activation codes and row scales (ff_rot_q8 then ff_gemm_s8), and the library
// allocates its error word on first use. This entry point keeps the codes and scales in one file-scope
// static device array instead, and reports bounded-wait timeouts in an error word the caller passes (a
// device int from the caller's own pool; NULL is rejected, so a timeout can never go unreported). It
// calls neither cudaMalloc nor cudaFree nor any allocating library routine.
//
// The array belongs to this library's CUDA module. Under the CUDA runtime's default lazy module loading
// the module, and with it the array, is loaded on a device at the first call there (its
// cudaGetSymbolAddress), not when the library is opened; a host that reserves all free GPU memory for its
// own pool must therefore make one call per device at start-up, before that reservation (or run with
// CUDA_MODULE_LOADING=EAGER), and before any stream capture. From then on every GPU that loaded it holds
// kNoallocCodeBytes of int8 codes and kNoallocRows row scales until the process exits. All calls on a
// device share the array and it keeps the last call's contents; codes and scales are fully rewritten by
// every call before they are read. Calls that overlap on the GPU (two streams, or a second call queued
// before the first one's GEMM has read the codes on another stream) race on it.
#include <mutex>

#include "common.h"
#include "gemm.h"
#include "kernels.h"

namespace ff {
namespace {

constexpr size_t kNoallocCodeBytes = size_t(8) << 20;  // rows x cols int8 codes
constexpr int kNoallocRows = 8192;                      // row scales
constexpr size_t kScaleOffset = kNoallocCodeBytes;
constexpr size_t kNoallocBytes = kScaleOffset + sizeof(float) * kNoallocRows;

static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoallocBytes];

std::mutex g_noalloc_mu;
uint8_t* g_noalloc_ptr[64] = {};  // device address of g_noalloc_scratch, per device

// Once per device, with that device current: resolve the array's device address (the host-side name is
// only a stand-in; passing it to a kernel would fault or silently use the wrong memory).
int noalloc_setup(uint8_t** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
    set_error("ff_linear_w8a8_noalloc: no current device");
    return FF_ERR_UNSUPPORTED_DEVICE;
  }
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (g_noalloc_ptr[dev] == nullptr) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr) {
      set_error("ff_linear_w8a8_noalloc: cudaGetSymbolAddress failed: %s", cudaGetErrorString(e));
      return FF_ERR_LAUNCH;
    }
    g_noalloc_ptr[dev] = static_cast<uint8_t*>(p);
  }
  *out = g_noalloc_ptr[dev];
  return FF_OK;
}

}  // namespace
}  // namespace ff

using namespace ff;

extern "C" int ff_linear_w8a8_noalloc(const uint16_t* x, const float* gamma, const float* beta, float eps, int rows,
                                      int cols, int valid_cols, int block, const int8_t* W, const float* col_scale,
                                      const float* bias, void* out, int N, int epi, int* err, void* stream) {
  FF_REQUIRE(x && W && col_scale && bias && out, "ff_linear_w8a8_noalloc: NULL pointer");
  FF_REQUIRE(err != nullptr,
             "ff_linear_w8a8_noalloc: err is NULL (pass a device int; bounded-wait timeouts are reported there)");
  FF_REQUIRE(epi == EPI_BIAS || epi == EPI_RESIDUAL || epi == EPI_SWIGLU,
             "ff_linear_w8a8_noalloc: epilogue %d (supported: FF_EPI_BIAS, FF_EPI_RESIDUAL, FF_EPI_SWIGLU)", epi);
  FF_REQUIRE(rows >= 1 && cols >= 1, "ff_linear_w8a8_noalloc: bad shape rows=%d cols=%d", rows, cols);
  FF_REQUIRE(rows <= kNoallocRows, "ff_linear_w8a8_noalloc: %d rows exceed the static scratch limit of %d rows", rows,
             kNoallocRows);
  FF_REQUIRE(static_cast<size_t>(rows) * static_cast<size_t>(cols) <= kNoallocCodeBytes,
             "ff_linear_w8a8_noalloc: rows x cols = %zu codes exceed the static scratch limit of %zu bytes",
             static_cast<size_t>(rows) * static_cast<size_t>(cols), kNoallocCodeBytes);
  FF_REQUIRE(N % 128 == 0, "ff_linear_w8a8_noalloc: N=%d must be a multiple of 128", N);
  uint8_t* scratch = nullptr;
  int rc = noalloc_setup(&scratch);
  if (rc != FF_OK) return rc;
  int8_t* codes = reinterpret_cast<int8_t*>(scratch);
  float* row_scale = reinterpret_cast<float*>(scratch + kScaleOffset);
  int* err_word = err;
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  rc = rot_q8(x, gamma, beta, eps, rows, cols, valid_cols, block, codes, row_scale, s, err_word);
  if (rc != FF_OK) return rc;
  GemmProblem p{};
  p.A = codes;
  p.W = W;
  p.out = out;
  p.M = rows;
  p.N = N;
  p.K = cols;
  p.epi = epi;
  p.tile_n = 0;
  p.f16 = false;
  p.err_word = err_word;
  p.args.row_scale = row_scale;
  p.args.col_scale = col_scale;
  p.args.bias = bias;
  p.args.ldo = epi == EPI_SWIGLU ? N / 2 : N;
  p.args.tokens = 1;
  GemmPlan plan;
  rc = gemm_prepare(p, &plan);
  if (rc != FF_OK) return rc;
  return gemm_launch(plan, s);
}
