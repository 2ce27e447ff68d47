// Host-side helpers shared by the C-ABI translation units: status codes, the thread-local error
// string, device properties and TMA descriptor encoding through the driver entry point.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <cstdint>
#include <cstdio>
#include <string>

#include "../../include/foidfinder_b200.h"

namespace ff {

void set_error(const char* fmt, ...);

// Returns FF_ERR_LAUNCH (and records the CUDA error) when the last launch failed.
int check_launch(const char* what);

int sm_count();  // of the current device

// Per-device error word that kernels with bounded waits write (allocated on first use, held until exit).
int* device_error_word();

// 2-D tensor map over a row-major [outer, inner] matrix, 128-byte swizzle, box {box_inner, box_outer}.
int make_tmap_2d(CUtensorMap* map, const void* base, CUtensorMapDataType dtype, int elt_bytes, uint64_t inner,
                 uint64_t outer, uint32_t box_inner, uint32_t box_outer);
// Same with an explicit row pitch (bytes) and swizzle mode.
int make_tmap_2d_pitched(CUtensorMap* map, const void* base, CUtensorMapDataType dtype, int elt_bytes, uint64_t inner,
                         uint64_t outer, uint64_t pitch_bytes, uint32_t box_inner, uint32_t box_outer,
                         CUtensorMapSwizzle swizzle);

// 3-D tensor map over a row-major [d2, d1, d0] array (d0 innermost), 128-byte swizzle.
int make_tmap_3d(CUtensorMap* map, const void* base, CUtensorMapDataType dtype, int elt_bytes, uint64_t d0, uint64_t d1,
                 uint64_t d2, uint32_t box0, uint32_t box1, uint32_t box2);

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Launches `kernel` on stream `s` with programmatic stream serialization: the launch may start while the
// previous kernel in the stream finishes; the kernel's pdl_wait() (ptx.cuh) orders its memory accesses after
// that kernel's completion.
template <typename... KArgs, typename... Args>
cudaError_t launch(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

}  // namespace ff

#define FF_REQUIRE(cond, ...)         \
  do {                                \
    if (!(cond)) {                    \
      ::ff::set_error(__VA_ARGS__);   \
      return FF_ERR_INVALID_ARGUMENT; \
    }                                 \
  } while (0)
