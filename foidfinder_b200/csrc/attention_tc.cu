// Non-causal flash attention on the 5th-generation tensor cores (tcgen05), head dim 64.
//
// Computes what the reference's attention kernel computes (foidfinder/backends/cuda/csrc/attention.cuh:19-157:
// softmax(q k^T) v per head on the packed QKV activations, scale folded into q), with f32 accumulation and
// masked ragged tails (EVA02 at 448 px has 1025 tokens).
//
// Persistent CTAs (one per SM, 320 threads, or 384 with tail rows; all 512 TMEM columns) walk work items of
// up to 256 queries (two 128-row tiles, Q0 and Q1) of one (image, head); consecutive items overlap in the
// pipeline:
//   warp 0     TMA: each item's Q0/Q1 into one of two Q buffers, K/V tiles of 128 keys through a 3-stage
//              ring. The tensor map is 3-D [images, tokens, 3*dim], so rows past an image's last token
//              arrive as zeros.
//   warp 1     TMEM allocation and the MMA issuer, ping-ponging the two query tiles:
//                S_i = Q_i K^T        (SS, M128 N128 K64)                           -> TMEM [128 i, +128)
//                [O_i | l_i] += P_i [V | 1]  (TS: P_i read from TMEM; B = the V tile plus a constant
//                                 64-wide atom of ones, MN-major, N = 80)     -> [256 + 80 i, +80)
//              issue order per key tile j: PV_0(j), S_0(j+1), PV_1(j), S_1(j+1). An S MMA overwrites the
//              columns its tile's P was read from; tcgen05.mma operations of one thread execute in issue
//              order, so the preceding P V has consumed P by then. Each P V starts in two halves: keys
//              0..63 as soon as the softmax has written their P (p_half), keys 64..127 after the rest
//              (p_full), so the first half of the product overlaps the second half of the softmax.
//   warps 2-5  softmax of Q0, warps 6-9 softmax of Q1: one query row per thread (TMEM lane = row),
//              row max, lazy rescale of O and l in TMEM when the max grows by more than 2^8, then
//              P = 2^(s log2e scale - m + 7) as fp16 pairs written back over S. The two warpgroups run
//              their exponential phases independently (making them alternate through barriers measured
//              1.5-2.5% slower once the kernel went persistent). Exponentials go through MUFU ex2, or
//              (build-time option) a degree-3 polynomial whose fp16 bits are assembled with integer ops.
//              The 2^7 factor keeps every P in fp16 range (<= 2^15) while polynomial results below 2^-14
//              (saturated there) are at most 2^-21 of the row maximum; it cancels in O / l.
//   warps 10-11  (sequences with 1..kTailRows rows past the last full query tile, e.g. EVA02's 1025th)
//              those rows on the CUDA cores; their keys stay in the ragged last key tile of the others.
// The row sum l is column 64 of the widened P V product: it costs no extra MMA instruction (every
// tcgen05.mma of M128 K16 costs ~50-54 cycles of issue at N <= 80, measured) and is rescaled together with O.
#include <algorithm>

#include "common.h"
#include "kernels.h"
#include "ptx.cuh"

namespace ff {
namespace fa {

constexpr int BQ = 128, BKV = 128, HD = 64, STAGES = 3;
constexpr int TILE = 128 * 128;  // 128 rows x 128 bytes (64 fp16)
constexpr int OFF_Q = 0;         // two buffers of (Q0, Q1): buffer b tile i at OFF_Q + (2 b + i) TILE
constexpr int OFF_K = OFF_Q + 4 * TILE;
constexpr int OFF_V = OFF_K + STAGES * TILE;
constexpr int ONES_LBO = STAGES * TILE;          // V stage s + ONES_LBO: its atom of fp16 1.0
constexpr int OFF_ONES = OFF_V + ONES_LBO;       // STAGES atoms of 128 rows x 128 B
constexpr int OFF_BAR = OFF_ONES + STAGES * TILE;
constexpr int SMEM = 1024 + OFF_BAR + 256;
constexpr int THREADS = 320;          // load, MMA, 2 x 4 softmax warps
constexpr int THREADS_TAIL = 384;     // + 2 tail-row warps (sequences with kTailRows or fewer extra rows)
constexpr uint32_t T_COLS = 512;
__host__ __device__ constexpr uint32_t t_s(int i) { return 128u * i; }
__host__ __device__ constexpr uint32_t t_o(int i) { return 256u + 80u * i; }  // O in [0, 64), l at 64
__host__ __device__ constexpr uint32_t t_l(int i) { return t_o(i) + 64u; }
constexpr float kRescaleThreshold = 8.f;  // log2 units: P may grow by 2^8 before O and l are rescaled
constexpr float kPScaleLog2 = 7.f;        // P is computed as 2^(x + 7): max 2^15, inside fp16

// Degree-3 minimax polynomial for 2^f on [-0.5, 0.5]: a Remez exchange on the relative error (5 reference
// points, float64), coefficients rounded to f32. Max relative error 7.48e-5, measured against exp2 in
// float64 at 2^20 evenly spaced points of the interval: below half an fp16 ulp (2^-11). Only the
// build-time option FF_ATTN_POLY_CHUNKS != 0 uses it; the default build runs MUFU ex2 everywhere.
constexpr float kP0 = 0.99992806f, kP1 = 0.69326103f, kP2 = 0.24261114f, kP3 = 0.055171605f;

// MN-major operand with 128-byte swizzle: K rows of 128 B (64 fp16 along N), 8-row groups 1024 B apart,
// the next 64-wide N atom (the ones) ONES_LBO bytes further.
__device__ __forceinline__ uint64_t sdesc_mn_sw128(uint32_t saddr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>(ONES_LBO >> 4) << 16;  // leading byte offset: next 64-wide N atom
  d |= static_cast<uint64_t>(1024u >> 4) << 32;  // stride byte offset: 8 K rows x 128 B
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

// (2^x.x, 2^x.y) as fp16x2 through MUFU ex2 and the f32->f16x2 conversion; exact zeros for x = -inf.
// (Assembling the fp16 bits with integer ops instead of the conversion measured 20% slower on B200.)
__device__ __forceinline__ uint32_t exp2_mufu(float2 x) { return pack_half2(ex2_approx(x.x), ex2_approx(x.y)); }

// (2^x.x, 2^x.y) as fp16x2 for x <= 15 on the FMA/ALU pipes: x = n + f (n = rint(x), |f| <= 1/2), 2^f
// by the polynomial, then the fp16 exponent n + 15 is added to the rounded 10-bit mantissa of 2^f.
// x is clamped to >= -14 (results below 2^-14 saturate there).
__device__ __forceinline__ uint32_t exp2_poly(float2 x) {
  const float2 magic = make_float2(12582912.f, 12582912.f);  // 1.5 * 2^23: rint(x) lands in the low bits
  x = make_float2(fmaxf(x.x, -14.f), fmaxf(x.y, -14.f));
  const float2 t = add2(x, magic);
  const float2 f = sub2(x, sub2(t, magic));
  float2 q = fma2(make_float2(kP3, kP3), f, make_float2(kP2, kP2));
  q = fma2(q, f, make_float2(kP1, kP1));
  q = fma2(q, f, make_float2(kP0, kP0));
  // (q rounded to 10 mantissa bits with its exponent rebased from f32 to fp16) + (n << 10);
  // 0xC8001000 = 0x1000 - (112 << 23) (mod 2^32): rounding bias and exponent rebase in one add.
  const uint32_t h0 = ((__float_as_uint(q.x) + 0xC8001000u) >> 13) + __float_as_uint(t.x) * 1024u;
  const uint32_t h1 = ((__float_as_uint(q.y) + 0xC8001000u) >> 13) + __float_as_uint(t.y) * 1024u;
  return __byte_perm(h0, h1, 0x5410);
}

// Which 32-key chunks of a tile take the polynomial path (bit c set: chunk c; the others use MUFU).
// Tunable at build time. Measured on B200 (EVA02-L, 1025 tokens, batch 64): all-MUFU is fastest (0.531 ms
// per launch vs 0.549 with one polynomial chunk of four, 0.552 with the last chunk), because the
// polynomial's ~15 instructions per pair cost more issue slots than the MUFU time they save.
#ifndef FF_ATTN_POLY_CHUNKS
#define FF_ATTN_POLY_CHUNKS 0x0u
#endif
constexpr unsigned kPolyChunks = FF_ATTN_POLY_CHUNKS;


}  // namespace fa

// Query rows past the last full 128-row tile, when there are at most kTailRows of them (EVA02: 1025 =
// 8 x 128 + 1), are computed on the CUDA cores in f32 by kTailWarps extra warps of the persistent kernel,
// during one of the items of their (image, head), so their keys and values are read while the TMA loads
// of that (image, head)'s items bring the same rows into L2 (a tensor-core tile for them
// would run a whole 128-row query tile for one row; a separate launch re-read all keys and values from
// HBM). Each quarter-warp (8 lanes x 8 dims = one 128-byte key/value row, coalesced) walks its share of
// the keys (quarter-warp w: keys w, w + 4 kTailWarps, ...) with its own online softmax (running max m, sum
// l, o over its 8 dims per lane), UNR keys in flight; the partial results are then merged through shared
// memory in a fixed order. UNR does not change the arithmetic, only how many rows are requested at once:
//  - UNR = 2 when the tail warps run beside an item's softmax warps (4 measured 0.6% slower there);
//  - UNR = 8 when they run in CTAs of their own (small batches, fewer items than SMs: there, on an item's
//    CTA at UNR = 2, they kept EVA02-L's bs1 launch at 36 us against 19 us for 1024 tokens).
// Called by every thread of the tail warps (t = 0 .. 32 kTailWarps - 1), which synchronise among
// themselves on named barrier 1.
namespace fa {
constexpr int kTailRows = 4;
constexpr int kTailWarps = (THREADS_TAIL - THREADS) / 32;

// Named barrier 1 over the tail warps. The quarter-warps leave their key loops at different points, so the
// warps reconverge first (bar.sync is the warp-aligned form).
__device__ __forceinline__ void tail_bar() {
  __syncwarp();
  asm volatile("bar.sync 1, %0;" ::"n"(kTailWarps * 32) : "memory");
}

template <int UNR>
__device__ __forceinline__ void attention_tail_rows(const __half* __restrict__ qkv, __half* __restrict__ out, int T,
                                                 int T_main, int heads, float scale_log2, int img, int h, int t) {
  constexpr int NQ = kTailWarps * 4;  // quarter-warps (8 lanes each)
  __shared__ float part_m[NQ], part_l[NQ];
  __shared__ float part_o[NQ][HD];
  const int dim = heads * HD, qw = t >> 3, ql = t & 7;
  const size_t img_row0 = static_cast<size_t>(img) * T;
  const unsigned qmask = 0xFFu << (t & 24);  // this quarter-warp's lanes
  for (int r = T_main; r < T; ++r) {
    // q: this lane's 8 dims, in log2 units.
    float q[8];
    {
      const uint4 u = __ldg(reinterpret_cast<const uint4*>(qkv + (img_row0 + r) * 3 * dim + h * HD) + ql);
      const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 f = unpack_half2(w[e]);
        q[2 * e] = f.x * scale_log2;
        q[2 * e + 1] = f.y * scale_log2;
      }
    }
    float m = -INFINITY, l = 0.f, o[8];
#pragma unroll
    for (int d = 0; d < 8; ++d) o[d] = 0.f;
    // One key of this quarter-warp's chain: its score, then the online-softmax update of m, l and o.
    auto add_key = [&](const uint4& kr, const uint4& vr) {
      const uint32_t kw[4] = {kr.x, kr.y, kr.z, kr.w};
      float sc = 0.f;
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 f = unpack_half2(kw[e]);
        sc = fmaf(q[2 * e], f.x, fmaf(q[2 * e + 1], f.y, sc));
      }
      sc += __shfl_xor_sync(qmask, sc, 1, 8);
      sc += __shfl_xor_sync(qmask, sc, 2, 8);
      sc += __shfl_xor_sync(qmask, sc, 4, 8);
      const float m_new = fmaxf(m, sc);
      const float corr = ex2_approx(m - m_new);  // 0 while m is still -inf
      const float p = ex2_approx(sc - m_new);
      m = m_new;
      l = fmaf(l, corr, p);
      const uint32_t vw[4] = {vr.x, vr.y, vr.z, vr.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 f = unpack_half2(vw[e]);
        o[2 * e] = fmaf(p, f.x, o[2 * e] * corr);
        o[2 * e + 1] = fmaf(p, f.y, o[2 * e + 1] * corr);
      }
    };
    for (int k0 = qw; k0 < T; k0 += NQ * UNR) {
      uint4 kr[UNR], vr[UNR];
#pragma unroll
      for (int i = 0; i < UNR; ++i) {
        const int key = k0 + i * NQ;
        if (key < T) {
          const __half* base = qkv + (img_row0 + key) * 3 * dim + h * HD;
          kr[i] = __ldg(reinterpret_cast<const uint4*>(base + dim) + ql);
          vr[i] = __ldg(reinterpret_cast<const uint4*>(base + 2 * dim) + ql);
        }
      }
      if (UNR > 2 && k0 + (UNR - 1) * NQ < T) {
        // every key of the step is valid: no branch between them, so their dot products and shuffles overlap
        // (with the branches, the dedicated tail CTAs took ~23 us for one row of 1025 keys)
#pragma unroll
        for (int i = 0; i < UNR; ++i) add_key(kr[i], vr[i]);
      } else {
#pragma unroll
        for (int i = 0; i < UNR; ++i) {
          if (k0 + i * NQ >= T) break;  // uniform within the quarter-warp
          add_key(kr[i], vr[i]);
        }
      }
    }
    tail_bar();  // the previous row's merge has read the partials
    if (ql == 0) {
      part_m[qw] = m;
      part_l[qw] = l;
    }
#pragma unroll
    for (int d = 0; d < 8; ++d) part_o[qw][8 * ql + d] = o[d];
    tail_bar();
    if (t < HD) {
      float mm = -INFINITY;
#pragma unroll 8
      for (int i = 0; i < NQ; ++i) mm = fmaxf(mm, part_m[i]);
      float ll = 0.f, acc = 0.f;
#pragma unroll 8
      for (int i = 0; i < NQ; ++i) {
        const float w = part_m[i] == -INFINITY ? 0.f : ex2_approx(part_m[i] - mm);
        ll = fmaf(part_l[i], w, ll);
        acc = fmaf(part_o[i][t], w, acc);
      }
      out[(img_row0 + r) * dim + h * HD + t] = __float2half_rn(acc / ll);
    }
  }
}
}  // namespace fa

namespace fa {
// Cold paths of the softmax warps, kept out of line so the full-tile loop stays compact in the
// instruction cache. Row maximum over the first `valid` (< BKV) keys of a ragged tile (raw S values).
__device__ __noinline__ float ragged_max(uint32_t ts, int valid) {
  float mx = -INFINITY;
  for (int c = 0; c < 4; ++c) {
    uint32_t raw[32];
    tmem_ld32(ts + 32 * c, raw);
    tmem_ld_wait();
#pragma unroll
    for (int e = 0; e < 32; ++e)
      if (32 * c + e < valid) mx = fmaxf(mx, __uint_as_float(raw[e]));
  }
  return mx;
}
// P of a ragged tile: exact zeros for keys >= valid; chunks of 32 keys past `valid` are not written.
__device__ __noinline__ void ragged_p(uint32_t ts, int valid, float sc, float nm) {
  const float2 sc2 = make_float2(sc, sc), nm2 = make_float2(nm, nm);
  for (int c = 0; c < 4; ++c) {
    if (32 * c >= valid) break;
    uint32_t raw[32], pk[16];
    tmem_ld32(ts + 32 * c, raw);
    tmem_ld_wait();
#pragma unroll
    for (int e = 0; e < 16; ++e) {
      float2 x = fma2(make_float2(__uint_as_float(raw[2 * e]), __uint_as_float(raw[2 * e + 1])), sc2, nm2);
      if (32 * c + 2 * e >= valid) x.x = -INFINITY;
      if (32 * c + 2 * e + 1 >= valid) x.y = -INFINITY;
      pk[e] = exp2_mufu(x);
    }
    tmem_st16(ts + 16 * c, pk);
  }
}
// O and l (80 TMEM columns from to) scaled by corr.
__device__ __noinline__ void rescale_o(uint32_t to, float corr) {
  for (int c = 0; c < 2; ++c) {
    uint32_t o[32];
    tmem_ld32(to + 32 * c, o);
    tmem_ld_wait();
#pragma unroll
    for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * corr);
    tmem_st32(to + 32 * c, o);
  }
  uint32_t l;
  tmem_ld1(to + 64, l);
  tmem_ld_wait();
  tmem_st1(to + 64, __float_as_uint(__uint_as_float(l) * corr));
}
}  // namespace fa

// Persistent: min(items, SMs) CTAs, each walking work items (image, head, pair of query tiles) with a grid
// stride, pair index fastest so the items running at once share their keys/values in L2. The pipeline
// runs across item boundaries: the producer loads the next item's Q into the other Q buffer and its
// keys/values into the same ring while this item computes; the MMA warp issues the next item's first S
// right after this item's last P V; the softmax warps drain O (tcgen05.ld) and release it (o_empty) before
// storing, so the next item's first P V, which overwrites O, waits only for that read. Every barrier
// phase is counted per CTA (items, tiles), not per item. An item whose second query tile is empty runs
// that warpgroup's protocol without work (its S and P V are skipped, its barriers still advance).
// TAIL: 0 no tail rows; 1 tail rows on warps 10-11 of the item CTAs; 2 tail rows in CTAs of their own, the
// launch's CTAs past the first `items` (one item per CTA: only when there are fewer items than SMs).
template <int TAIL>
__global__ void __launch_bounds__(TAIL ? fa::THREADS_TAIL : fa::THREADS, 1)
    attention_tc_kernel(const __grid_constant__ CUtensorMap tm_qkv, const __half* __restrict__ qkv,
                        __half* __restrict__ out, int T, int T_main, int heads, int num_seqs, float scale_log2,
                        int pair_items, int* err) {
  using namespace fa;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + OFF_BAR);
  uint64_t* q_full = bar + 0;              // [2] Q buffers
  uint64_t* q_empty = bar + 2;             // [2]
  uint64_t* kv_full = bar + 4;             // [STAGES]
  uint64_t* kv_empty = kv_full + STAGES;   // [STAGES]
  uint64_t* s_full = kv_empty + STAGES;    // [2] per query tile
  uint64_t* p_full = s_full + 2;           // [2]
  uint64_t* p_half = p_full + 2;           // [2] P of keys 0..63 written
  uint64_t* o_full = p_half + 2;           // [2]
  uint64_t* o_empty = o_full + 2;          // [2]
  uint64_t* drain = o_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int dim = heads * HD;
  const int n_pairs = (T_main + 2 * BQ - 1) / (2 * BQ);
  // Items [0, pair_items) are pairs of query tiles; the pairs after them run as one item per query tile
  // (TAIL == 2 only: a single round of items; the other instantiations take pairs only).
  const int items =
      TAIL == 2 ? pair_items + 2 * (num_seqs * heads * n_pairs - pair_items) : num_seqs * heads * n_pairs;
  const int nkv = (T + BKV - 1) / BKV;
  // The last key tile may be ragged: its S and P V products only cover the first kv_tail_n keys
  // (a multiple of 16; keys past T inside them are masked in the softmax).
  const int kv_tail = T - (nkv - 1) * BKV;
  const int kv_tail_n = (kv_tail + 15) & ~15;
  // Item -> (image, head, first query row, whether a second query tile follows). `tail`: the item that
  // carries its (image, head)'s tail rows on the steady schedule (one per (image, head), spread so that a
  // CTA's items mostly share the pair index when the grid is a multiple of n_pairs).
  auto item_of = [&](int it, int& img, int& h, int& q0, bool& two, bool& tail) {
    int pi = it, tile = 0;
    if constexpr (TAIL == 2) {
      if (it >= pair_items) {
        pi = pair_items + ((it - pair_items) >> 1);
        tile = (it - pair_items) & 1;
      }
    }
    const int pair = pi % n_pairs, r = pi / n_pairs;
    h = r % heads;
    img = r / heads;
    q0 = pair * 2 * BQ + tile * BQ;
    two = (TAIL != 2 || it < pair_items) && q0 + BQ < T_main;
    tail = pair == r % n_pairs && tile == 0;
  };

  if constexpr (TAIL == 2) {
    if (static_cast<int>(blockIdx.x) >= items) {  // a tail-row CTA: no TMEM, none of the item pipeline's barriers
      pdl_wait();
      pdl_trigger();
      if (warp < kTailWarps) {
        const int tails = num_seqs * heads, stride = static_cast<int>(gridDim.x) - items;
        for (int s = static_cast<int>(blockIdx.x) - items; s < tails; s += stride)
          attention_tail_rows<8>(qkv, out, T, T_main, heads, scale_log2, s / heads, s % heads, threadIdx.x);
      }
      return;
    }
  }

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&q_full[i], 1);
      mbar_init(&q_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], 4);
      mbar_init(&p_half[i], 4);
      mbar_init(&o_full[i], 1);
      mbar_init(&o_empty[i], 4);
    }
    for (int st = 0; st < STAGES; ++st) {
      mbar_init(&kv_full[st], 1);
      mbar_init(&kv_empty[st], 1);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) tma_prefetch_map(&tm_qkv);
  if (warp == 1) {
    tmem_alloc(tmem_slot, T_COLS);
    tmem_relinquish();
  }
  if (warp >= 2) {  // the constant ones atoms that widen V (fp16 1.0; the TMA never writes them)
    uint4* ones = reinterpret_cast<uint4*>(smem + OFF_ONES);
    for (int i = threadIdx.x - 64; i < STAGES * TILE / 16; i += static_cast<int>(blockDim.x) - 64)
      ones[i] = make_uint4(0x3C003C00u, 0x3C003C00u, 0x3C003C00u, 0x3C003C00u);
    fence_async_smem();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  pdl_wait();
  pdl_trigger();

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      int q_phase[2] = {-1, -1}, kv_phase[STAGES];
#pragma unroll
      for (int st = 0; st < STAGES; ++st) kv_phase[st] = -1;
      bool ok = true;
      int kv_count = 0, n = 0;
      for (int it = blockIdx.x; it < items && ok; it += gridDim.x, ++n) {
        int img, h, q0;
        bool has1, tail;
        item_of(it, img, h, q0, has1, tail);
        const int qb = n & 1;
        if (n >= 2 && !mbar_wait(&q_empty[qb], static_cast<uint32_t>((n >> 1) - 1) & 1u, abort_flag, err,
                                 kDevTimeoutAttn)) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(&q_full[qb], has1 ? 2 * TILE : TILE);
        tma_load_3d(smem + OFF_Q + 2 * qb * TILE, &tm_qkv, &q_full[qb], h * HD, q0, img);
        if (has1) tma_load_3d(smem + OFF_Q + (2 * qb + 1) * TILE, &tm_qkv, &q_full[qb], h * HD, q0 + BQ, img);
        q_phase[qb] = (n >> 1) & 1;
        for (int j = 0; j < nkv; ++j, ++kv_count) {
          const int st = kv_count % STAGES;
          const uint32_t ph = static_cast<uint32_t>(kv_count / STAGES) & 1u;
          if (!mbar_wait(&kv_empty[st], ph ^ 1u, abort_flag, err, kDevTimeoutAttn)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&kv_full[st], 2 * TILE);
          tma_load_3d(smem + OFF_K + st * TILE, &tm_qkv, &kv_full[st], dim + h * HD, j * BKV, img);
          tma_load_3d(smem + OFF_V + st * TILE, &tm_qkv, &kv_full[st], 2 * dim + h * HD, j * BKV, img);
          kv_phase[st] = static_cast<int>(ph);
        }
      }
      // Normally the MMA warp has consumed every copy. After an abort, let the issued ones land (bounded)
      // before the CTA can exit: the last phase of each barrier completes with its last copy.
      if (!ok) {
        const unsigned long long t0 = globaltimer();
        for (int b = 0; b < 2; ++b)
          if (q_phase[b] >= 0)
            while (!mbar_try_wait(smem_u32(&q_full[b]), static_cast<uint32_t>(q_phase[b])) &&
                   globaltimer() - t0 < kWaitLimitNs) {
            }
        for (int st = 0; st < STAGES; ++st)
          if (kv_phase[st] >= 0)
            while (!mbar_try_wait(smem_u32(&kv_full[st]), static_cast<uint32_t>(kv_phase[st])) &&
                   globaltimer() - t0 < kWaitLimitNs) {
            }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t id_s = idesc_f16(128, BKV);
      const uint32_t id_s_tail = idesc_f16(128, kv_tail_n);
      constexpr uint32_t id_o = idesc_f16(128, HD + 16) | (1u << 16);  // B = [V | ones] is MN-major, N = 80
      auto issue_s = [&](int i, int qb, int c, bool tail) {  // S_i = Q_i K^T for key tile count c
        const uint64_t qd = sdesc_k_sw128(smem_u32(smem + OFF_Q + (2 * qb + i) * TILE));
        const uint64_t kd = sdesc_k_sw128(smem_u32(smem + OFF_K + (c % STAGES) * TILE));
        const uint32_t id = tail ? id_s_tail : id_s;
#pragma unroll
        for (int k = 0; k < 4; ++k) mma_f16(tmem + t_s(i), qd + 2 * k, kd + 2 * k, id, k > 0);
        tc_commit(&s_full[i]);
      };
      auto issue_pv = [&](int i, int j, int c, bool tail, int k0) {  // K steps k0 .. k0 + 3
        const uint32_t sv = smem_u32(smem + OFF_V + (c % STAGES) * TILE);
        const uint64_t vd = fa::sdesc_mn_sw128(sv + k0 * 2048);
        const uint32_t d = tmem + t_o(i), a = tmem + t_s(i) + 8 * k0;
        if (!tail) {  // straight-line issue: no branch between the MMAs
          mma_f16_ts(d, a, vd, id_o, (j > 0 || k0 > 0) ? 1u : 0u);
#pragma unroll
          for (int k = 1; k < 4; ++k) mma_f16_ts(d, a + 8 * k, vd + static_cast<uint64_t>(k * 128), id_o, 1u);
        } else {
          const int steps = kv_tail_n / 16;
#pragma unroll
          for (int k = k0; k < k0 + 4; ++k) {  // 16 keys per step: P columns 8k.., V rows 16k..
            if (k < steps) {
              const uint32_t acc = (j > 0 || k > 0) ? 1u : 0u;
              mma_f16_ts(tmem + t_o(i), tmem + t_s(i) + 8 * k, fa::sdesc_mn_sw128(sv + k * 2048), id_o, acc);
            }
          }
        }
      };
      auto kv_wait = [&](int c) {
        return mbar_wait(&kv_full[c % STAGES], static_cast<uint32_t>(c / STAGES) & 1u, abort_flag, err,
                         kDevTimeoutAttn);
      };
      // One flat sequence of key tiles over this CTA's items: per tile, P V of query tile 0, then S of query
      // tile 0 for the next key tile (the next item's first when this tile is an item's last, so the next
      // item starts while this one drains), then the same for query tile 1.
      bool ok = true;
      int kv_count = 0, tiles = 0, n = 0, it = blockIdx.x;
      int img, h, q0;
      bool has1 = false, tail;
      if (it < items) {
        item_of(it, img, h, q0, has1, tail);
        ok = mbar_wait(&q_full[0], 0u, abort_flag, err, kDevTimeoutAttn) && kv_wait(0);
        if (ok) {
          tc_fence_after();
          issue_s(0, 0, 0, nkv == 1);
          if (has1)
            issue_s(1, 0, 0, nkv == 1);
          else
            tc_commit(&s_full[1]);  // warpgroup 1 idles on this item; its barriers still advance
        }
      }
      for (; it < items && ok; it += gridDim.x, ++n) {
        const int qb = n & 1;
        const int it_next = it + gridDim.x;
        const bool more = it_next < items;
        bool has1_next = false;
        if (more) {
          int img2, h2, q02;
          item_of(it_next, img2, h2, q02, has1_next, tail);
        }
        for (int j = 0; j < nkv; ++j, ++kv_count, ++tiles) {
          const bool last = j == nkv - 1;
          // The key tile after this one: (this item, j + 1), or (next item, 0) with the other Q buffer.
          const bool next = !last || more;
          const int nqb = last ? qb ^ 1 : qb;
          const bool ntail = last ? nkv == 1 : j + 1 == nkv - 1;
          const bool nhas1 = last ? has1_next : has1;
          const uint32_t par = static_cast<uint32_t>(tiles) & 1u;
          const uint32_t opar = static_cast<uint32_t>(n - 1) & 1u;
          if (last) tc_commit(&q_empty[qb]);  // every S of this item is issued: Q frees when they complete
          if (!mbar_wait(&p_half[0], par, abort_flag, err, kDevTimeoutAttn) ||
              (j == 0 && n > 0 && !mbar_wait(&o_empty[0], opar, abort_flag, err, kDevTimeoutAttn))) {
            ok = false;
            break;
          }
          tc_fence_after();
          issue_pv(0, j, kv_count, last, 0);
          if (!mbar_wait(&p_full[0], par, abort_flag, err, kDevTimeoutAttn)) {
            ok = false;
            break;
          }
          tc_fence_after();
          issue_pv(0, j, kv_count, last, 4);
          if (last) tc_commit(&o_full[0]);
          if (next) {
            if (!kv_wait(kv_count + 1) ||
                (last && !mbar_wait(&q_full[nqb], static_cast<uint32_t>((n + 1) >> 1) & 1u, abort_flag, err,
                                    kDevTimeoutAttn))) {
              ok = false;
              break;
            }
            tc_fence_after();
            issue_s(0, nqb, kv_count + 1, ntail);
          }
          if (!mbar_wait(&p_half[1], par, abort_flag, err, kDevTimeoutAttn) ||
              (has1 && j == 0 && n > 0 && !mbar_wait(&o_empty[1], opar, abort_flag, err, kDevTimeoutAttn))) {
            ok = false;
            break;
          }
          tc_fence_after();
          if (has1) issue_pv(1, j, kv_count, last, 0);
          if (!mbar_wait(&p_full[1], par, abort_flag, err, kDevTimeoutAttn)) {
            ok = false;
            break;
          }
          tc_fence_after();
          if (has1) issue_pv(1, j, kv_count, last, 4);
          if (last) tc_commit(&o_full[1]);
          tc_commit(&kv_empty[kv_count % STAGES]);
          if (next) {
            if (nhas1)
              issue_s(1, nqb, kv_count + 1, ntail);
            else
              tc_commit(&s_full[1]);
          }
        }
        has1 = has1_next;
      }
      tc_commit(drain);
      const unsigned long long t0 = globaltimer();
      while (!mbar_try_wait(smem_u32(drain), 0)) {
        if (globaltimer() - t0 > kWaitLimitNs) {
          atomicCAS(err, 0, kDevTimeoutDrain);
          break;
        }
      }
    }
  } else if (warp >= 10) {
    // ------------------------------------------------------------ tail query rows (warps 10, 11)
    if constexpr (TAIL == 1) {
      for (int it = blockIdx.x; it < items; it += gridDim.x) {
        int img, h, q0;
        bool two, tail;
        item_of(it, img, h, q0, two, tail);
        if (!tail) continue;
        attention_tail_rows<2>(qkv, out, T, T_main, heads, scale_log2, img, h, threadIdx.x - THREADS);
      }
    }
  } else {
    // ------------------------------------------------------------ softmax + epilogue (warps 2..9)
    const int g = (warp - 2) >> 2;  // query tile of this warpgroup
    const int q = warp & 3;
    const uint32_t lane_base = static_cast<uint32_t>(q * 32) << 16;
    const uint32_t ts = tmem + lane_base + t_s(g);
    bool ok = true;
    int tiles = 0, n = 0;
    for (int it = blockIdx.x; it < items && ok; it += gridDim.x, ++n) {
      int img, h, q0;
      bool two, tail;
      item_of(it, img, h, q0, two, tail);
      const bool active = g == 0 || two;  // warp-uniform
      const int row = q0 + g * BQ + q * 32 + lane;
      float m_ref = -INFINITY;
      for (int j = 0; j < nkv; ++j, ++tiles) {
        if (!mbar_wait(&s_full[g], static_cast<uint32_t>(tiles) & 1u, abort_flag, err, kDevTimeoutAttn)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const int valid = T - j * BKV;  // keys at columns >= valid belong to no token of this image
        const bool full_tile = valid >= BKV;
        if (active) {
          // Pass 1: row maximum, 64 keys (two loads, one wait) at a time: holding all 128 in registers
          // pushed the kernel to the 168-register cap with spills (measured 5-10% slower).
          float mx = -INFINITY;
          if (full_tile) {
            // Four independent running maxima (max is exact, so the order does not change the result): a
            // single chain of 64 dependent max instructions per tile left the two softmax warps of each
            // scheduler waiting on its latency.
            float mq[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
            for (int hf = 0; hf < 2; ++hf) {
              uint32_t raw[2][32];
#pragma unroll
              for (int c = 0; c < 2; ++c) tmem_ld32(ts + 64 * hf + 32 * c, raw[c]);
              tmem_ld_wait();
#pragma unroll
              for (int c = 0; c < 2; ++c)
#pragma unroll
                for (int e = 0; e < 32; e += 2)
                  mq[(e >> 1) & 3] = max3(mq[(e >> 1) & 3], __uint_as_float(raw[c][e]), __uint_as_float(raw[c][e + 1]));
            }
            mx = max3(mq[0], mq[1], fmaxf(mq[2], mq[3]));
          } else {
            mx = fa::ragged_max(ts, valid);
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
          if (__any_sync(0xffffffffu, rescale)) fa::rescale_o(tmem + lane_base + t_o(g), corr);
        }
        // P of keys 0..63 is in TMEM: the first half of this tile's P V may start.
        auto signal_half = [&]() {
          __syncwarp();
          tmem_st_wait();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&p_half[g]);
        };
        bool half_sent = false;
        if (active) {
          // Pass 2: P = 2^(s * scale_log2 - m_ref + 7) as fp16 pairs over S columns [0, 64), in two halves
          // of 64 keys (two loads, one wait each). P of half hf (columns 32hf..32hf+31) only overlaps S
          // columns already read (those of half 0).
          const float2 sc2 = make_float2(scale_log2, scale_log2);
          const float2 nm2 = make_float2(kPScaleLog2 - m_ref, kPScaleLog2 - m_ref);
          if (full_tile) {
#pragma unroll
            for (int hf = 0; hf < 2; ++hf) {
              uint32_t raw[2][32];
              tmem_ld32(ts + 64 * hf, raw[0]);
              tmem_ld32(ts + 64 * hf + 32, raw[1]);
              tmem_ld_wait();
#pragma unroll
              for (int cc = 0; cc < 2; ++cc) {
                const int c = 2 * hf + cc;
                uint32_t pk[16];
#pragma unroll
                for (int e = 0; e < 16; ++e) {
                  const float2 x = fma2(
                      make_float2(__uint_as_float(raw[cc][2 * e]), __uint_as_float(raw[cc][2 * e + 1])), sc2, nm2);
                  pk[e] = ((kPolyChunks >> c) & 1u) ? fa::exp2_poly(x) : fa::exp2_mufu(x);
                }
                tmem_st16(ts + 16 * c, pk);
              }
              if (hf == 0) {
                signal_half();
                half_sent = true;
              }
            }
          } else {
            fa::ragged_p(ts, valid, scale_log2, kPScaleLog2 - m_ref);
          }
        }
        if (!half_sent) signal_half();
        __syncwarp();
        tmem_st_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&p_full[g]);
      }
      if (!ok) break;
      // Epilogue: read O and l, release them to the next item's P V, then normalise and store.
      if (!mbar_wait(&o_full[g], static_cast<uint32_t>(n) & 1u, abort_flag, err, kDevTimeoutAttn)) {
        ok = false;
        break;
      }
      tc_fence_after();
      uint32_t packed[32];  // O / l as fp16 pairs, 32 columns at a time through registers
      if (active) {
        uint32_t o[32], l;
        fa::tmem_ld1(tmem + lane_base + t_l(g), l);
        tmem_ld32(tmem + lane_base + t_o(g), o);
        tmem_ld_wait();
        const float inv = 1.f / __uint_as_float(l);
#pragma unroll
        for (int e = 0; e < 16; ++e) packed[e] = pack_half2(__uint_as_float(o[2 * e]) * inv, __uint_as_float(o[2 * e + 1]) * inv);
        tmem_ld32(tmem + lane_base + t_o(g) + 32, o);
        tmem_ld_wait();
#pragma unroll
        for (int e = 0; e < 16; ++e)
          packed[16 + e] = pack_half2(__uint_as_float(o[2 * e]) * inv, __uint_as_float(o[2 * e + 1]) * inv);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&o_empty[g]);
      if (active && row < T_main) {
        uint4* dst = reinterpret_cast<uint4*>(out + (static_cast<size_t>(img) * T + row) * dim + h * HD);
#pragma unroll
        for (int v4 = 0; v4 < 8; ++v4)
          dst[v4] = make_uint4(packed[4 * v4], packed[4 * v4 + 1], packed[4 * v4 + 2], packed[4 * v4 + 3]);
      }
    }
  }

  __syncwarp();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, T_COLS);
}

// Query rows past the last full 128-row tile that attention_tc computes on the CUDA cores inside its one
// launch (1..kTailRows of them, e.g. EVA02's 1025th token), or 0 when the last query tile is ragged instead.
int attention_tc_tail_rows(int seq_len) {
  const int rem = seq_len % fa::BQ;
  return rem != 0 && rem <= fa::kTailRows && seq_len > fa::BQ ? rem : 0;
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
    if (cudaFuncSetAttribute(attention_tc_kernel<0>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM) != cudaSuccess ||
        cudaFuncSetAttribute(attention_tc_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM) != cudaSuccess ||
        cudaFuncSetAttribute(attention_tc_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM) != cudaSuccess)
      return check_launch("attention_tc: cudaFuncSetAttribute");
    if (dev >= 0 && dev < 64) configured[dev] = true;
  }
  const float scale_log2 = scale * 1.4426950408889634f;
  const int t_main = seq_len - attention_tc_tail_rows(seq_len);
  const long long pairs = static_cast<long long>(num_seqs) * heads * ((t_main + 2 * BQ - 1) / (2 * BQ));
  FF_REQUIRE(pairs <= 0x3fffffff, "attention: %lld work items", pairs);
  const long long sms = sm_count();
  // Items are pairs of query tiles. With tail rows, when even single query tiles fill less than one round
  // over the SMs (EVA02-L bs1: 64 pairs, 128 tiles), each tile is an item of its own: 18.9 vs 21.9 us per
  // bs1 launch. (Single tiles for the pairs left over after full rounds, e.g. bs8's last 68 of 512,
  // measured slower: 79.2 vs 73.3 us.) Only when every pair holds two tiles; a query tile gives the same
  // bits either way.
  const bool singles = t_main < seq_len && t_main % (2 * BQ) == 0 && 2 * pairs < sms;
  const long long pair_items = singles ? 0 : pairs;
  const long long items = pair_items + 2 * (pairs - pair_items);
  const int grid = static_cast<int>(std::min<long long>(items, sm_count()));
  // Tail rows (EVA02's 1025th) run on two extra warps of the same launch; without them the kernel keeps
  // 320 threads (the extra warps, idle, measured 2.6% slower on 1024-token sequences). With fewer items
  // than SMs the tail rows run in CTAs of their own on the idle SMs instead (same arithmetic, more rows in
  // flight; see attention_tail_rows), one (image, head) after another.
  const long long tails = static_cast<long long>(num_seqs) * heads;
  if (t_main < seq_len && items < sm_count()) {
    const int tail_ctas = static_cast<int>(std::min<long long>(tails, sm_count() - items));
    launch(attention_tc_kernel<2>, dim3(static_cast<int>(items) + tail_ctas), dim3(THREADS_TAIL), SMEM, s, map,
           static_cast<const __half*>(qkv), static_cast<__half*>(out), seq_len, t_main, heads, num_seqs, scale_log2,
           static_cast<int>(pair_items), err);
  } else if (t_main < seq_len)
    launch(attention_tc_kernel<1>, dim3(grid), dim3(THREADS_TAIL), SMEM, s, map, static_cast<const __half*>(qkv),
                                                               static_cast<__half*>(out), seq_len, t_main, heads,
                                                               num_seqs, scale_log2, static_cast<int>(pair_items), err);
  else
    launch(attention_tc_kernel<0>, dim3(grid), dim3(THREADS), SMEM, s, map, static_cast<const __half*>(qkv),
                                                           static_cast<__half*>(out), seq_len, t_main, heads,
                                                           num_seqs, scale_log2, static_cast<int>(pair_items), err);
  return check_launch("attention_tc_kernel");
}

}  // namespace ff

namespace ff {

// ff_attention: the reference's attention operator (torch.ops.foidfinder.attention, kernels.cu:255-265) on
// the tensor-core kernel above. As in the reference, q and k arrive rotated (the QKV GEMM epilogue applies
// the 2-D RoPE, FF_EPI_QKV_ROPE), so the RoPE table arguments must be NULL.
int attention(const void* qkv, void* out, int num_seqs, int seq_len, int heads, const float* rc, const float* rsn,
              float scale, cudaStream_t s) {
  FF_REQUIRE(qkv && out, "ff_attention: NULL pointer");
  FF_REQUIRE(num_seqs >= 0 && seq_len >= 1 && heads >= 1 && heads <= 64, "ff_attention: bad shape");
  FF_REQUIRE(rc == nullptr && rsn == nullptr,
             "ff_attention: RoPE tables must be NULL (rotate q and k in the QKV GEMM epilogue, FF_EPI_QKV_ROPE)");
  FF_REQUIRE(aligned16(qkv) && aligned16(out), "ff_attention: pointers must be 16-byte aligned");
  if (num_seqs == 0) return FF_OK;
  return attention_tc(qkv, out, num_seqs, seq_len, heads, scale, s);
}

}  // namespace ff

extern "C" int ff_attention(const uint16_t* qkv, uint16_t* out, int num_seqs, int seq_len, int heads,
                            const float* rope_cos, const float* rope_sin, float scale, void* stream) {
  return ff::attention(qkv, out, num_seqs, seq_len, heads, rope_cos, rope_sin, scale,
                       static_cast<cudaStream_t>(stream));
}
