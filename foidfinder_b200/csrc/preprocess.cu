// Letterbox preprocessing on the GPU: an RGB uint8 image resized with Pillow's 8-bit separable resampling
// (bilinear or bicubic, antialiased when reducing) and centred on a square canvas of a fill colour, written
// directly as the engine's uint8 input. Bit-exact with PIL.Image.resize + paste.
//
// The reference does this step on the host (foidfinder/backends/cuda/preprocess.py:16-32) or, for the
// Haruka model, on the GPU with the same fixed-point arithmetic (foidfinder/backends/mlx/kernels.py:75-186,
// tested against Pillow in tests/test_haruka.py:36-55). The coefficients follow Pillow's Resample.c:
// precompute_coeffs (float64, taps normalised by their sequential sum) then 22-bit fixed point
// (normalize_coeffs_8bpc); each output is (2^21 + sum in * k) >> 22 clamped to [0, 255]. Two passes with
// an 8-bit intermediate, so their order changes the result: Pillow (12.x, the version these tests run
// against) resamples horizontally first unless the source is more than 100 times taller than wide — a
// rule established by comparing both orders against PIL.Image.resize over a few hundred random shapes.
// Horizontal-first reads only the source rows the vertical pass needs.
#include <cuda_fp16.h>

#include <cmath>
#include <vector>

#include "common.h"
#include "ptx.cuh"

namespace ff {
namespace {

constexpr int kPrecisionBits = 22;

double bilinear_filter(double x) {
  if (x < 0.0) x = -x;
  return x < 1.0 ? 1.0 - x : 0.0;
}

double bicubic_filter(double x) {  // a = -0.5
  const double a = -0.5;
  if (x < 0.0) x = -x;
  if (x < 1.0) return ((a + 2.0) * x - (a + 3.0)) * x * x + 1.0;
  if (x < 2.0) return (((x - 5.0) * x + 8.0) * x - 4.0) * a;
  return 0.0;
}

struct Coeffs {
  int ksize = 0;
  std::vector<int32_t> kk;      // [out, ksize] fixed-point taps
  std::vector<int32_t> bounds;  // [out, 2]: first source index, tap count
};

Coeffs pillow_coeffs(int in_size, int out_size, int filter) {
  const double support_1 = filter == FF_RESAMPLE_BICUBIC ? 2.0 : 1.0;
  const double scale = static_cast<double>(in_size) / out_size;
  const double filterscale = scale > 1.0 ? scale : 1.0;
  const double support = support_1 * filterscale;
  Coeffs c;
  c.ksize = static_cast<int>(std::ceil(support)) * 2 + 1;
  c.kk.assign(static_cast<size_t>(out_size) * c.ksize, 0);
  c.bounds.assign(static_cast<size_t>(out_size) * 2, 0);
  std::vector<double> k(c.ksize);
  const double ss = 1.0 / filterscale;
  for (int xx = 0; xx < out_size; ++xx) {
    const double center = (xx + 0.5) * scale;
    int xmin = static_cast<int>(center - support + 0.5);
    if (xmin < 0) xmin = 0;
    int xmax = static_cast<int>(center + support + 0.5);
    if (xmax > in_size) xmax = in_size;
    xmax -= xmin;
    double ww = 0.0;
    for (int x = 0; x < xmax; ++x) {
      const double arg = (x + xmin - center + 0.5) * ss;
      const double w = filter == FF_RESAMPLE_BICUBIC ? bicubic_filter(arg) : bilinear_filter(arg);
      k[x] = w;
      ww += w;
    }
    for (int x = 0; x < xmax; ++x)
      if (ww != 0.0) k[x] /= ww;
    for (int x = 0; x < c.ksize; ++x) {
      const double w = x < xmax ? k[x] : 0.0;
      c.kk[static_cast<size_t>(xx) * c.ksize + x] =
          static_cast<int32_t>(w < 0 ? -0.5 + w * (1 << kPrecisionBits) : 0.5 + w * (1 << kPrecisionBits));
    }
    c.bounds[2 * xx] = xmin;
    c.bounds[2 * xx + 1] = xmax;
  }
  return c;
}

// One pass along AXIS (0: width, 1: height). Output canvas [out_h, out_w, 3]; pixels inside the region
// (top, left, h, w) are resampled, the rest take the fill value. Source rows are offset by row0.
template <int AXIS>
__global__ void resample_kernel(const uint8_t* __restrict__ src, int src_w, int row0, const int32_t* __restrict__ kk,
                                const int32_t* __restrict__ bounds, int ksize, int out_w, int out_h, int top, int left,
                                int h, int w, int fill, uint8_t* __restrict__ out) {
  pdl_wait();
  pdl_trigger();
  const int x = blockIdx.x * blockDim.x + threadIdx.x, y = blockIdx.y;
  if (x >= out_w || y >= out_h) return;
  const int yy = y - top, xx = x - left;
  uint8_t v[3] = {static_cast<uint8_t>(fill), static_cast<uint8_t>(fill), static_cast<uint8_t>(fill)};
  if (yy >= 0 && yy < h && xx >= 0 && xx < w) {
    const int i_out = AXIS == 0 ? xx : yy;
    const int first = bounds[2 * i_out], taps = bounds[2 * i_out + 1];
    const int32_t* k = kk + static_cast<size_t>(i_out) * ksize;
    const uint8_t* in = AXIS == 0 ? src + (static_cast<size_t>(row0 + yy) * src_w + first) * 3
                                  : src + (static_cast<size_t>(row0 + first) * src_w + xx) * 3;
    const size_t stride = AXIS == 0 ? 3 : static_cast<size_t>(src_w) * 3;
    int s0 = 1 << (kPrecisionBits - 1), s1 = s0, s2 = s0;
    for (int i = 0; i < taps; ++i) {
      const uint8_t* p = in + i * stride;
      s0 += static_cast<int>(p[0]) * k[i];
      s1 += static_cast<int>(p[1]) * k[i];
      s2 += static_cast<int>(p[2]) * k[i];
    }
    v[0] = static_cast<uint8_t>(min(max(s0 >> kPrecisionBits, 0), 255));
    v[1] = static_cast<uint8_t>(min(max(s1 >> kPrecisionBits, 0), 255));
    v[2] = static_cast<uint8_t>(min(max(s2 >> kPrecisionBits, 0), 255));
  }
  uint8_t* o = out + (static_cast<size_t>(y) * out_w + x) * 3;
  o[0] = v[0];
  o[1] = v[1];
  o[2] = v[2];
}

size_t up256(size_t v) { return (v + 255) / 256 * 256; }

struct Plan {
  Coeffs ch, cv;
  bool vertical_first;
  int row0, rows;    // horizontal-first: the source rows the vertical pass reads
  size_t tmp_bytes;  // intermediate image
  size_t total;
};

Plan make_plan(int h, int w, int new_h, int new_w, int filter) {
  Plan p;
  p.ch = pillow_coeffs(w, new_w, filter);
  p.cv = pillow_coeffs(h, new_h, filter);
  p.vertical_first = h > 100 * static_cast<int64_t>(w);
  p.row0 = p.cv.bounds[0];
  p.rows = p.cv.bounds[2 * (new_h - 1)] + p.cv.bounds[2 * (new_h - 1) + 1] - p.row0;
  if (!p.vertical_first)
    for (int i = 0; i < new_h; ++i) p.cv.bounds[2 * i] -= p.row0;
  p.tmp_bytes = p.vertical_first ? static_cast<size_t>(new_h) * w * 3 : static_cast<size_t>(p.rows) * new_w * 3;
  p.total = up256(p.tmp_bytes) + up256(p.ch.kk.size() * 4) + up256(p.ch.bounds.size() * 4) + up256(p.cv.kk.size() * 4) +
            up256(p.cv.bounds.size() * 4);
  return p;
}

int check_geometry(int h, int w, int new_h, int new_w, int size, int filter) {
  FF_REQUIRE(h >= 1 && w >= 1 && new_h >= 1 && new_w >= 1 && new_h <= size && new_w <= size,
             "ff_resize_pad: bad geometry %dx%d -> %dx%d on %d", h, w, new_h, new_w, size);
  FF_REQUIRE(filter == FF_RESAMPLE_BILINEAR || filter == FF_RESAMPLE_BICUBIC, "ff_resize_pad: filter %d", filter);
  return FF_OK;
}

}  // namespace
}  // namespace ff

using namespace ff;

extern "C" int64_t ff_resize_pad_workspace_bytes(int h, int w, int new_h, int new_w, int filter) {
  if (h < 1 || w < 1 || new_h < 1 || new_w < 1 || (filter != FF_RESAMPLE_BILINEAR && filter != FF_RESAMPLE_BICUBIC))
    return -1;
  return static_cast<int64_t>(make_plan(h, w, new_h, new_w, filter).total);
}

extern "C" int ff_resize_pad(const uint8_t* src, int h, int w, int new_h, int new_w, int size, int filter, int fill,
                             uint8_t* dst, void* workspace, int64_t workspace_bytes, void* stream) {
  FF_REQUIRE(src && dst && workspace, "ff_resize_pad: NULL pointer");
  const int rc = check_geometry(h, w, new_h, new_w, size, filter);
  if (rc != FF_OK) return rc;
  FF_REQUIRE(fill >= 0 && fill <= 255, "ff_resize_pad: fill %d", fill);
  const Plan p = make_plan(h, w, new_h, new_w, filter);
  FF_REQUIRE(workspace_bytes >= static_cast<int64_t>(p.total), "ff_resize_pad: workspace of %lld bytes, %zu needed",
             static_cast<long long>(workspace_bytes), p.total);
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  uint8_t* base = static_cast<uint8_t*>(workspace);
  uint8_t* tmp = base;
  size_t off = up256(p.tmp_bytes);
  auto put = [&](const std::vector<int32_t>& v) -> int32_t* {
    int32_t* d = reinterpret_cast<int32_t*>(base + off);
    off += up256(v.size() * 4);
    // Pageable source: the copy is staged before this call returns, so the vector may be freed.
    if (cudaMemcpyAsync(d, v.data(), v.size() * 4, cudaMemcpyHostToDevice, s) != cudaSuccess) return nullptr;
    return d;
  };
  int32_t* kh = put(p.ch.kk);
  int32_t* bh = put(p.ch.bounds);
  int32_t* kv = put(p.cv.kk);
  int32_t* bv = put(p.cv.bounds);
  if (!kh || !bh || !kv || !bv) return check_launch("ff_resize_pad: coefficient copy");
  const int top = (size - new_h) / 2, left = (size - new_w) / 2;
  constexpr int TX = 128;
  if (p.vertical_first) {
    launch(resample_kernel<1>, dim3(dim3((w + TX - 1) / TX, new_h)), dim3(TX), 0, s, src, w, 0, kv, bv, p.cv.ksize, w, new_h, 0, 0,
                                                                    new_h, w, fill, tmp);
    launch(resample_kernel<0>, dim3(dim3((size + TX - 1) / TX, size)), dim3(TX), 0, s, tmp, w, 0, kh, bh, p.ch.ksize, size, size, top,
                                                                      left, new_h, new_w, fill, dst);
  } else {
    launch(resample_kernel<0>, dim3(dim3((new_w + TX - 1) / TX, p.rows)), dim3(TX), 0, s, src, w, p.row0, kh, bh, p.ch.ksize, new_w,
                                                                         p.rows, 0, 0, p.rows, new_w, fill, tmp);
    launch(resample_kernel<1>, dim3(dim3((size + TX - 1) / TX, size)), dim3(TX), 0, s, tmp, new_w, 0, kv, bv, p.cv.ksize, size, size,
                                                                      top, left, new_h, new_w, fill, dst);
  }
  return check_launch("resample_kernel");
}

// ---------------------------------------------------------------- PixAI's float letterbox
// The reference's PixAI preprocessing (foidfinder/backends/cuda/preprocess.py:16-32): pixels / 255 in f32,
// F.interpolate(mode="bilinear", align_corners=False, antialias=True) to (new_h, new_w), then x * 2 - 1
// rounded to fp16, centred on a canvas of -1 (black after the normalisation). No 8-bit rounding anywhere.
//
// The antialiased bilinear resize is separable: each output index i along an axis of scale
// s = in / out takes the source indices [xmin, xmin + n) around center = s * (i + 0.5) with the triangle
// filter stretched by max(s, 1) (support = max(s, 1)), weights normalised by their sum (torch's
// _compute_weights_aa, the same rule as Pillow's precompute_coeffs but in float, not fixed point). One
// thread per output pixel sums over the rows of its vertical taps the horizontal sums of each row (the
// horizontal pass first, as torch's separable CPU kernel runs its width pass first), in f32.
namespace ff {
namespace {

struct AaAxis {
  float scale, support, invscale;
};

__host__ __device__ inline AaAxis aa_axis(int in_size, int out_size) {
  AaAxis a;
  a.scale = static_cast<float>(in_size) / static_cast<float>(out_size);
  a.support = a.scale >= 1.f ? a.scale : 1.f;  // interp size 2 for bilinear: support = 2/2 * max(scale, 1)
  a.invscale = a.scale >= 1.f ? 1.f / a.scale : 1.f;
  return a;
}

__device__ inline float tri(float x) {
  x = fabsf(x);
  return x < 1.f ? 1.f - x : 0.f;
}

// Taps of output index i: first source index, count, and the sum of the unnormalised weights.
__device__ inline void aa_taps(const AaAxis& a, int i, int in_size, int* first, int* count, float* total) {
  const float center = a.scale * (static_cast<float>(i) + 0.5f);
  int lo = static_cast<int>(center - a.support + 0.5f);
  if (lo < 0) lo = 0;
  int hi = static_cast<int>(center + a.support + 0.5f);
  if (hi > in_size) hi = in_size;
  float t = 0.f;
  for (int j = 0; j < hi - lo; ++j) t += tri((static_cast<float>(j + lo) - center + 0.5f) * a.invscale);
  *first = lo;
  *count = hi - lo;
  *total = t;
}

__device__ inline float aa_weight(const AaAxis& a, int i, int j, int first, float total) {
  const float center = a.scale * (static_cast<float>(i) + 0.5f);
  const float w = tri((static_cast<float>(j + first) - center + 0.5f) * a.invscale);
  return total != 0.f ? w / total : 0.f;
}

__global__ void letterbox_aa_f16_kernel(const uint8_t* __restrict__ src, int h, int w, int new_h, int new_w, int size,
                                        int top, int left, __half* __restrict__ dst) {
  pdl_wait();
  pdl_trigger();
  const int x = blockIdx.x * blockDim.x + threadIdx.x, y = blockIdx.y;
  if (x >= size || y >= size) return;
  const int yy = y - top, xx = x - left;
  float v[3] = {-1.f, -1.f, -1.f};
  if (yy >= 0 && yy < new_h && xx >= 0 && xx < new_w) {
    const AaAxis ax = aa_axis(w, new_w), ay = aa_axis(h, new_h);
    int x0, nx, y0, ny;
    float tx, ty;
    aa_taps(ax, xx, w, &x0, &nx, &tx);
    aa_taps(ay, yy, h, &y0, &ny, &ty);
    float acc[3] = {0.f, 0.f, 0.f};
    for (int jy = 0; jy < ny; ++jy) {
      const uint8_t* row = src + (static_cast<size_t>(y0 + jy) * w + x0) * 3;
      float hs[3] = {0.f, 0.f, 0.f};
      for (int jx = 0; jx < nx; ++jx) {
        const float wx = aa_weight(ax, xx, jx, x0, tx);
        for (int c = 0; c < 3; ++c) hs[c] += __fdiv_rn(static_cast<float>(row[jx * 3 + c]), 255.f) * wx;
      }
      const float wy = aa_weight(ay, yy, jy, y0, ty);
      for (int c = 0; c < 3; ++c) acc[c] += hs[c] * wy;
    }
    for (int c = 0; c < 3; ++c) v[c] = __fsub_rn(acc[c] * 2.f, 1.f);
  }
  __half* o = dst + (static_cast<size_t>(y) * size + x) * 3;
  o[0] = __float2half_rn(v[0]);
  o[1] = __float2half_rn(v[1]);
  o[2] = __float2half_rn(v[2]);
}

}  // namespace
}  // namespace ff

extern "C" int ff_letterbox_aa_f16(const uint8_t* src, int h, int w, int new_h, int new_w, int size, uint16_t* dst,
                                   void* stream) {
  FF_REQUIRE(src && dst, "ff_letterbox_aa_f16: NULL pointer");
  FF_REQUIRE(h >= 1 && w >= 1 && new_h >= 1 && new_w >= 1 && new_h <= size && new_w <= size,
             "ff_letterbox_aa_f16: bad geometry %dx%d -> %dx%d on %d", h, w, new_h, new_w, size);
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int top = (size - new_h) / 2, left = (size - new_w) / 2;
  constexpr int TX = 128;
  launch(letterbox_aa_f16_kernel, dim3(dim3((size + TX - 1) / TX, size)), dim3(TX), 0, s, src, h, w, new_h, new_w, size, top, left,
                                                                         reinterpret_cast<__half*>(dst));
  return check_launch("letterbox_aa_f16_kernel");
}
