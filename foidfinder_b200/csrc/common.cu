// Host helpers: error reporting, device queries, the per-device error word and TMA descriptor encoding.
#include <cudaTypedefs.h>

#include <cstdarg>
#include <mutex>

#include "common.h"

namespace ff {

namespace {
thread_local char g_last_error[512] = "";
std::mutex g_mu;
int* g_err_word[64] = {};  // per-device error word, allocated on first use and held until exit
int g_sm_count[64] = {};
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
}  // namespace

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
}

int check_launch(const char* what) {
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_error("%s: %s", what, cudaGetErrorString(e));
    return FF_ERR_LAUNCH;
  }
  return FF_OK;
}

int sm_count() {
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return 148;
  if (g_sm_count[dev] == 0) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    g_sm_count[dev] = n > 0 ? n : 148;
  }
  return g_sm_count[dev];
}

int* device_error_word() {
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return nullptr;
  if (g_err_word[dev] == nullptr) {
    std::lock_guard<std::mutex> lock(g_mu);
    if (g_err_word[dev] == nullptr) {
      int* p = nullptr;
      if (cudaMalloc(&p, sizeof(int)) != cudaSuccess) return nullptr;
      cudaMemset(p, 0, sizeof(int));
      cudaDeviceSynchronize();
      g_err_word[dev] = p;
    }
  }
  return g_err_word[dev];
}

static int load_encode() {
  if (g_encode == nullptr) {
    std::lock_guard<std::mutex> lock(g_mu);
    if (g_encode == nullptr) {
      void* fn = nullptr;
      cudaDriverEntryPointQueryResult q;
      if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) != cudaSuccess ||
          q != cudaDriverEntryPointSuccess || fn == nullptr) {
        set_error("cuTensorMapEncodeTiled is not available from the driver");
        return FF_ERR_UNSUPPORTED_DEVICE;
      }
      g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    }
  }
  return FF_OK;
}

int make_tmap_2d(CUtensorMap* map, const void* base, CUtensorMapDataType dtype, int elt_bytes, uint64_t inner,
                 uint64_t outer, uint32_t box_inner, uint32_t box_outer) {
  return make_tmap_2d_pitched(map, base, dtype, elt_bytes, inner, outer, inner * static_cast<uint64_t>(elt_bytes),
                              box_inner, box_outer, CU_TENSOR_MAP_SWIZZLE_128B);
}

int make_tmap_2d_pitched(CUtensorMap* map, const void* base, CUtensorMapDataType dtype, int elt_bytes, uint64_t inner,
                         uint64_t outer, uint64_t pitch_bytes, uint32_t box_inner, uint32_t box_outer,
                         CUtensorMapSwizzle swizzle) {
  const int lrc = load_encode();
  if (lrc != FF_OK) return lrc;
  if (!aligned16(base) || pitch_bytes % 16 != 0 || pitch_bytes < inner * elt_bytes) {
    set_error("TMA operand must be 16-byte aligned with a 16-byte multiple row pitch");
    return FF_ERR_INVALID_ARGUMENT;
  }
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {pitch_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  const CUresult r = g_encode(map, dtype, 2, const_cast<void*>(base), dims, strides, box, estr,
                              CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("cuTensorMapEncodeTiled failed (%d) for [%llu, %llu] box [%u, %u]", static_cast<int>(r),
              static_cast<unsigned long long>(outer), static_cast<unsigned long long>(inner), box_outer, box_inner);
    return FF_ERR_INVALID_ARGUMENT;
  }
  return FF_OK;
}

int make_tmap_3d(CUtensorMap* map, const void* base, CUtensorMapDataType dtype, int elt_bytes, uint64_t d0, uint64_t d1,
                 uint64_t d2, uint32_t box0, uint32_t box1, uint32_t box2) {
  const int lrc = load_encode();
  if (lrc != FF_OK) return lrc;
  if (!aligned16(base) || (d0 * elt_bytes) % 16 != 0) {
    set_error("TMA operand must be 16-byte aligned with a 16-byte multiple row pitch");
    return FF_ERR_INVALID_ARGUMENT;
  }
  cuuint64_t dims[3] = {d0, d1, d2};
  cuuint64_t strides[2] = {d0 * static_cast<uint64_t>(elt_bytes), d0 * d1 * static_cast<uint64_t>(elt_bytes)};
  cuuint32_t box[3] = {box0, box1, box2};
  cuuint32_t estr[3] = {1, 1, 1};
  const CUresult r = g_encode(map, dtype, 3, const_cast<void*>(base), dims, strides, box, estr,
                              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("cuTensorMapEncodeTiled (3-D) failed (%d)", static_cast<int>(r));
    return FF_ERR_INVALID_ARGUMENT;
  }
  return FF_OK;
}

}  // namespace ff

extern "C" {

const char* ff_last_error(void) { return ff::g_last_error; }

int ff_version(void) { return 100; }

int ff_device_error(int device, int* code, int clear) {
  FF_REQUIRE(code != nullptr, "ff_device_error: code is NULL");
  int prev = 0;
  cudaGetDevice(&prev);
  if (cudaSetDevice(device) != cudaSuccess) {
    ff::set_error("ff_device_error: bad device %d", device);
    return FF_ERR_INVALID_ARGUMENT;
  }
  int* w = ff::device_error_word();
  int rc = FF_OK;
  *code = 0;
  if (w == nullptr) {
    ff::set_error("ff_device_error: could not allocate the error word");
    rc = FF_ERR_OUT_OF_MEMORY;
  } else if (cudaDeviceSynchronize() != cudaSuccess || cudaMemcpy(code, w, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess) {
    ff::set_error("ff_device_error: %s", cudaGetErrorString(cudaGetLastError()));
    rc = FF_ERR_LAUNCH;
  } else if (clear && *code != 0) {
    cudaMemset(w, 0, sizeof(int));
    cudaDeviceSynchronize();
  }
  cudaSetDevice(prev);
  return rc;
}

}  // extern "C"
