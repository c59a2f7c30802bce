// cp_backward.cuh — the backward pass of the folded CP sum layer (K = N = 64), and the gradient
// of the state table read by the second layer of a circuit.
//
// The forward (cp_layer.cuh, lse_gemm.cuh) is
//   Y[f,m,o] = log( sum_k exp(X[f,m,k] - s) w[f,o,k] ) + s,   s = max_k (or min_k) X[f,m,:],
// with X = A, A + A2 (the folded Hadamard product fused, translate.py:706-718) or the sum of two
// state-table rows picked by pixel values, and w (F, O, K) the layer's linear weights (the softmax
// of its logits; the contraction's B operand is w[f]^T).  The reference differentiates its torch
// executor's calls, in which the shift is a stop_gradient (backend_translation/translate.py:727-740).
// With G = dL/dY:
//   A'[m,k] = exp(X[m,k] - s),   V[m,o] = G[m,o] exp(s - Y[m,o])      (V = G / P)
//   dX[m,k] = A'[m,k] sum_o V[m,o] w[o,k],   dw[o,k] = sum_m V[m,o] A'[m,k],
// dX being the gradient of A and of A2 alike.  cpb_kernel computes both from one read of X, Y, G:
//
//  * a tile is 64 rows of one fold; each CTA takes a contiguous range of tiles and two pairs own
//    alternate tiles: pair p is the 64 TMEM lanes 64p.. (quarters 2p, 2p+1) and the four warps
//    that reach them, two threads per row (warp w: quarter w & 3, columns 32 (w >> 2) ..+31);
//  * tiles rotate through three 64 KB stages, so the loads of the next two tiles are in flight
//    while one is computed; a stage receives the tile's rows of X (two tensors for a pair source),
//    Y and G by TMA (table rows by cp.async of 16 bytes, a warp instruction per two rows);
//  * each thread reads its half row, takes the row extreme with the other half (through a TMEM
//    column of its own dX' half, free until the pair's next product, and a bounded mbarrier
//    phase on which all the pair's threads arrive), forms A' and V, writes V as
//    TF32 hi / lo into its TMEM lane, and writes the operands of the weight product in place of
//    its half row of the inputs: S (A'^T hi over A'^T lo, M = 128) and V^T hi / lo (N = 64),
//    MN-major with the tile's rows as K, so that a thread's k-rows are the 128-byte rows its
//    inputs came in and no other thread touches them;
//  * one thread issues dX' = V w with A = V from TMEM (M = 128 lanes, of which the pair's 64 are
//    its rows; split TF32 over w^T hi / lo, three products per k-step) and the weight product
//    D_B[(h,k), o] = sum over the tile's rows of S[(h,k), m] (V^T hi + V^T lo)[o, m];
//  * the pair's epilogue stores dX = dX' * A' from registers; a drain group (warps 4-7, one TMEM
//    lane quarter each) adds every tile's D_B into fp32 registers, rounding to nearest (the tensor
//    core's accumulator truncates, so it restarts with every tile), and writes the two halves
//    h = 0, 1 of its sums to a workspace slot of the fold when its range leaves the fold;
//  * the load warp splits w^T into TF32 hi / lo at each fold's start;
//  * cpb_reduce_kernel adds the slots of each fold in a fixed order, so dw is deterministic.
//
// table_grad_pair_kernel: the second layer's X is T[f, x_m] + T[f + pair, x'_m] for a state
// table T (2F, states, 64) and pixel values x_m, x'_m of the variables of folds f and f + pair;
// dT[t, s, :] is the sum of dX[f, m, :] over the rows m whose pixel selects state s of table fold
// t (the backward of the gather).  A CTA takes whole folds f of dX; warp w owns the states s
// with s % 31 == w, sums their rows in registers in increasing m: the sums are deterministic.
#pragma once

#include "cp_layer.cuh"

namespace xe {
namespace cpb {

using namespace gemm;
using cp::bulk_commit;
using cp::bulk_wait_all;
using cp::bulk_wait_read;
using cp::tma_store_3d;

// Event times of CTA 0 (trace builds only).  cpb_kernel, per tile: pair warps 0-4, MMA 6-9, loads
// 10, drain 11-12; table_grad_pair_kernel, per chunk: issue 0, warp 0's wait 1-2, warps 0-7 done 3-10.
#define XE_CPB_TRACE(n, ev) XE_TILE_TRACE(n, ev)

constexpr int kRows = 64;  // rows per tile
constexpr int kComputeWarps = 8;
constexpr int kDrainWarp0 = 8;  // 8-11: TMEM lane quarters 0-3
constexpr int kMmaWarp = 12;
constexpr int kProducerWarp = 13;
constexpr int kThreads = (kProducerWarp + 1) * 32;
constexpr int kBlock = 32 * 32 * 4;       // 32 rows x 32 fp32 (4 KB)
constexpr int kRegion = 8 * kBlock;       // one warp's 32 rows of X1, X2, Y, G (two column halves each)
constexpr int kStage = 2 * kRegion;       // one tile
constexpr int kStages = 3;
constexpr int kWPlane = 2 * 64 * 32 * 4;  // w^T hi or lo: two o-blocks of [64 k][32 o], K-major
constexpr int kOffStage = 0;
constexpr int kOffWHi = kOffStage + kStages * kStage;
constexpr int kOffWLo = kOffWHi + kWPlane;
constexpr int kOffBar = kOffWLo + kWPlane;
constexpr int kSmemBytes = 1024 + kOffBar + 256;
static_assert(kSmemBytes <= 232448, "shared memory");
// Blocks of a warp's region: the inputs, tensor t (0 X1, 1 X2, 2 Y, 3 G) and column half c at
// (2t + c) kBlock (128-byte swizzle, K-major: row m at m * 128); once read, the MN-major operands
// of the weight product in their place (32-element MN blocks of 4 KB, k-row m at m * 128):
// S (four MN blocks) over X1 / X2, V^T hi (two) over Y, V^T lo over G.
constexpr int kOffS = 0, kOffVtHi = 4 * kBlock, kOffVtLo = 6 * kBlock;
// TMEM columns of pair p (base 256 p): V hi, V lo (the A operand of dX'), dX', D_B
constexpr uint32_t kTmVHi = 0, kTmVLo = 64, kTmDX = 128, kTmDB = 192;

enum Source : int { kDense = 0, kDense2 = 1, kGather2 = 2 };

struct Params {
  const float* w;  // (folds, 64 o, 64 k)
  float* dx;       // (folds, M, 64)
  int folds, M, tiles_m, num_tiles;
  int g_folds;  // G[f] = g[f % g_folds]: the next layer's dX is the gradient of both halves of its input
  int shift_min;
  int pieces;       // workspace slots per fold
  float* partials;  // [folds][pieces][2][64 o][64 k]
  // kGather2: X[f,m,:] = T[f, x_m, :] + T[f + pair, x'_m, :], x_m the pixel of sample m and
  // variable var[f]: pixels[m * px_sm + var[f] * px_sv]
  const float* table;  // (table folds, states, 64)
  const uint8_t* pixels;
  const int32_t* var;  // nullptr: variable = table fold
  int64_t px_sm, px_sv, variables;
  int states, pair;
};

// The CTA whose range holds tile t when num_tiles tiles are split into `grid` contiguous ranges
// [floor(num_tiles c / grid), floor(num_tiles (c + 1) / grid)): the largest c with
// num_tiles c < (t + 1) grid.
__host__ __device__ __forceinline__ int cta_of_tile(int64_t t, int64_t num_tiles, int64_t grid) {
  return (int)(((t + 1) * grid - 1) / num_tiles);
}

__device__ __forceinline__ float2 lds_v2(uint32_t addr) {
  float2 v;
  asm volatile("ld.shared.v2.f32 {%0,%1}, [%2];" : "=f"(v.x), "=f"(v.y) : "r"(addr));
  return v;
}

// One fp32 column of the calling warp's 32 TMEM lanes.
__device__ __forceinline__ void tmem_st1(uint32_t taddr, float v) {
  __syncwarp();
  asm volatile("tcgen05.st.sync.aligned.32x32b.x1.b32 [%0], {%1};" ::"r"(taddr), "f"(v) : "memory");
}

__device__ __forceinline__ float tmem_ld1(uint32_t taddr) {
  __syncwarp();
  uint32_t r;
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x1.b32 {%0}, [%1];" : "=r"(r) : "r"(taddr) : "memory");
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
  return __uint_as_float(r);
}

// 16 bytes global -> shared memory through L2 (not L1), asynchronous.
__device__ __forceinline__ void cp_async_16(uint32_t dst, const float* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}

// One arrival on `bar` once every cp.async this thread issued before has landed; the arrival is
// one of the barrier's expected count.
__device__ __forceinline__ void cp_async_arrive_noinc(uint64_t* bar) {
  asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(bar)) : "memory");
}


template <int SRC>
__global__ void __launch_bounds__(kThreads, 1)
    cpb_kernel(const __grid_constant__ Params p, const __grid_constant__ CUtensorMap tmap_x1,
               const __grid_constant__ CUtensorMap tmap_x2, const __grid_constant__ CUtensorMap tmap_y,
               const __grid_constant__ CUtensorMap tmap_g) {
  constexpr bool PAIR = SRC != kDense;
  // bytes the TMA brings into a stage per tile: 64 rows x 64 fp32 of X1 (and X2; the table rows of
  // kGather2 come by cp.async, which arrives on the barrier once per load lane), Y and G
  constexpr uint32_t kStageTx = (SRC == kGather2 ? 2 : PAIR ? 4 : 3) * kRows * 64 * 4;
  constexpr uint32_t kStageArrivals = SRC == kGather2 ? 33 : 1;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  const uint32_t smem_base = smem_u32(smem);
  uint64_t* bars = (uint64_t*)(smem + kOffBar);
  uint64_t* stage_full = bars;               // [kStages] the tile's inputs have landed
  uint64_t* stage_free = bars + kStages;     // [kStages] the weight product has read the stage
  uint64_t* ready = bars + 2 * kStages;      // [2] the pair's V (TMEM) and S, V^T (stage) written
  uint64_t* dx_full = ready + 2;             // [2] dX' complete
  uint64_t* db_full = dx_full + 2;           // [2] D_B complete
  uint64_t* db_free = db_full + 2;           // [2] D_B drained
  uint64_t* w_ready = db_free + 2;           // the fold's w^T hi / lo split
  uint64_t* w_free = w_ready + 1;            // the fold's last dX' product done with them
  uint64_t* drain = w_free + 1;
  uint64_t* x_ready = drain + 1;             // [2] both halves' row extremes of the pair's tile written
  uint32_t* tmem_slot = (uint32_t*)(x_ready + 2);
  volatile int* abort_flag = (volatile int*)(tmem_slot + 1);
  ArmedCopies* stage_copies = (ArmedCopies*)(tmem_slot + 2);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int i = 0; i < kStages; ++i) {
      mbar_init(&stage_full[i], kStageArrivals);
      mbar_init(&stage_free[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&ready[i], 4);
      mbar_init(&dx_full[i], 1);
      mbar_init(&db_full[i], 1);
      mbar_init(&db_free[i], 4);
      mbar_init(&x_ready[i], 4 * 32);
    }
    mbar_init(w_ready, 1);
    mbar_init(w_free, 1);
    mbar_init(drain, 1);
    *abort_flag = 0;
    *stage_copies = ArmedCopies{0u, 0u};
    fence_mbarrier_init();
  }
  if (warp == kMmaWarp) tmem_alloc<512>(tmem_slot);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int first = (int)(((int64_t)p.num_tiles * blockIdx.x) / gridDim.x);
  const int last = (int)(((int64_t)p.num_tiles * (blockIdx.x + 1)) / gridDim.x);

  if (warp < kComputeWarps) {
    // ------------------------------------------------------------ pairs (two threads per row)
    const int quarter = warp & 3;
    const int half = warp >> 2;  // columns 32 half .. 32 half + 31 of the row
    const int pair = quarter >> 1;
    const int wq = quarter & 1;
    const uint32_t tp = tmem + pair * 256 + ((uint32_t)(quarter * 32) << 16);
    const bool is_min = p.shift_min != 0;
    const uint32_t roff = lane * 128;
    bool ok = true;
    for (int i = first + pair; i < last && ok; i += 2) {
      const int n = i - first;
      const int j = n >> 1;
      const int st = n % kStages;
      const int f = i / p.tiles_m;
      const int mt = i - f * p.tiles_m;
      const int row = mt * kRows + wq * 32 + lane;
      const bool valid = row < p.M;
      const uint32_t region = smem_base + kOffStage + st * kStage + wq * kRegion;
      const bool tr = half == 0 && wq == 0 && lane == 0;
      if (tr) XE_CPB_TRACE(n, 0);
      if (!mbar_wait_warp(&stage_full[st], (n / kStages) & 1, kSiteAStaged, abort_flag)) {
        ok = false;
        break;
      }
      if (tr) XE_CPB_TRACE(n, 1);
      float a[32];
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const uint32_t off = roff + ((q ^ (lane & 7)) << 4);
        float4 v = lds_v4(region + half * kBlock + off);
        if (PAIR) {
          const float4 u = lds_v4(region + (2 + half) * kBlock + off);
          v.x += u.x;
          v.y += u.y;
          v.z += u.z;
          v.w += u.w;
        }
        a[4 * q] = v.x;
        a[4 * q + 1] = v.y;
        a[4 * q + 2] = v.z;
        a[4 * q + 3] = v.w;
      }
      float e0 = is_min ? INFINITY : -INFINITY, e1 = e0, e2 = e0, e3 = e0;
#pragma unroll
      for (int k = 0; k < 32; k += 4) {
        e0 = extreme(e0, a[k], is_min);
        e1 = extreme(e1, a[k + 1], is_min);
        e2 = extreme(e2, a[k + 2], is_min);
        e3 = extreme(e3, a[k + 3], is_min);
      }
      const float e_half = extreme(extreme(e0, e1, is_min), extreme(e2, e3, is_min), is_min);
      // the row extreme: each half leaves its own in the first column of its dX' half (its own
      // epilogue has read the previous dX' there; the pair's next product is issued after every
      // thread of the pair has read the other half's); the pair's phase j of x_ready completes
      // once all 128 threads have written
      tmem_st1(tp + kTmDX + 32 * half, e_half);
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(&x_ready[pair]);
      if (!mbar_wait_warp(&x_ready[pair], j & 1, kSiteAStaged, abort_flag)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const float e_other = tmem_ld1(tp + kTmDX + 32 * (1 - half));
      const float s = valid ? extreme(e_half, e_other, is_min) : 0.0f;
      // A' and its S columns (M = k for hi, 64 + k for lo), in this thread's k-rows of blocks
      // half and 2 + half (its X rows, read above)
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        float4 hi, lo;
#pragma unroll
        for (int t = 0; t < 4; ++t) a[4 * q + t] = valid ? exp_shifted(a[4 * q + t], s) : 0.0f;
        split_rn(a[4 * q], hi.x, lo.x);
        split_rn(a[4 * q + 1], hi.y, lo.y);
        split_rn(a[4 * q + 2], hi.z, lo.z);
        split_rn(a[4 * q + 3], hi.w, lo.w);
        sts_v4(region + kOffS + mnmajor_off(lane, 8 * half + q), hi);
        sts_v4(region + kOffS + mnmajor_off(lane, 16 + 8 * half + q), lo);
      }
      // V = G exp(s - Y) for this half: its Y and G rows are read whole before its V^T chunks
      // (MN block `half` of V^T hi / lo, this thread's k-row) replace them
      float v[32];
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const uint32_t off = roff + ((q ^ (lane & 7)) << 4);
        const float4 yv = lds_v4(region + (4 + half) * kBlock + off);
        const float4 gv = lds_v4(region + (6 + half) * kBlock + off);
        v[4 * q] = valid ? gv.x * exp_shifted(s, yv.x) : 0.0f;
        v[4 * q + 1] = valid ? gv.y * exp_shifted(s, yv.y) : 0.0f;
        v[4 * q + 2] = valid ? gv.z * exp_shifted(s, yv.z) : 0.0f;
        v[4 * q + 3] = valid ? gv.w * exp_shifted(s, yv.w) : 0.0f;
      }
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        float hi[16], lo[16];
#pragma unroll
        for (int t = 0; t < 16; ++t) split_rn(v[16 * hh + t], hi[t], lo[t]);
        tmem_st16(tp + kTmVHi + 32 * half + 16 * hh, hi);
        tmem_st16(tp + kTmVLo + 32 * half + 16 * hh, lo);
#pragma unroll
        for (int qq = 0; qq < 4; ++qq) {
          const int oq = 8 * half + 4 * hh + qq;
          sts_v4(region + kOffVtHi + mnmajor_off(lane, oq), make_float4(hi[4 * qq], hi[4 * qq + 1], hi[4 * qq + 2], hi[4 * qq + 3]));
          sts_v4(region + kOffVtLo + mnmajor_off(lane, oq), make_float4(lo[4 * qq], lo[4 * qq + 1], lo[4 * qq + 2], lo[4 * qq + 3]));
        }
      }
      tmem_wait_st();
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&ready[pair]);
      if (tr) XE_CPB_TRACE(n, 2);
      // -------- epilogue: dX = dX' * A', this thread's half row
      if (!mbar_wait_warp(&dx_full[pair], j & 1, kSiteDrainChunk, abort_flag)) {
        ok = false;
        break;
      }
      if (tr) XE_CPB_TRACE(n, 3);
      tc_fence_after();
      float d[32];
      tmem_ld16(tp + kTmDX + 32 * half, d);
      tmem_ld16(tp + kTmDX + 32 * half + 16, d + 16);
      tmem_wait_ld();
      if (valid) {
        float* dst = p.dx + ((int64_t)f * p.M + row) * 64 + 32 * half;
#pragma unroll
        for (int c = 0; c < 8; ++c)
          stg_v4(dst + 4 * c, make_float4(d[4 * c] * a[4 * c], d[4 * c + 1] * a[4 * c + 1], d[4 * c + 2] * a[4 * c + 2],
                                          d[4 * c + 3] * a[4 * c + 3]));
      }
      // dX' has been read: the pair's next V (and its product) may replace it
      tc_fence_before();
      if (tr) XE_CPB_TRACE(n, 4);
    }
  } else if (warp < kMmaWarp) {
    // ------------------------------------------------------------ D_B drain (lane = row (h, k))
    const int q = warp - kDrainWarp0;
    const int h = q >> 1;
    const int k = 32 * (q & 1) + lane;
    const uint32_t lane_bits = (uint32_t)(q * 32) << 16;
    float run[64];
#pragma unroll
    for (int o = 0; o < 64; ++o) run[o] = 0.0f;
    int cur = first < last ? first / p.tiles_m : 0;
    // this CTA's partial sums of fold f into its slot (slot 0 for the fold's first CTA)
    auto flush = [&](int f) {
      const int piece = (int)blockIdx.x - cta_of_tile((int64_t)f * p.tiles_m, p.num_tiles, gridDim.x);
      float* dst = p.partials + (((int64_t)f * p.pieces + piece) * 2 + h) * 4096 + k;
#pragma unroll
      for (int o = 0; o < 64; ++o) {
        dst[o * 64] = run[o];
        run[o] = 0.0f;
      }
    };
    bool ok = true;
    for (int i = first, n = 0; i < last; ++i, ++n) {
      const int pair = n & 1;
      const int j = n >> 1;
      const int f = i / p.tiles_m;
      if (f != cur) {
        flush(cur);
        cur = f;
      }
      if (!mbar_wait_warp(&db_full[pair], j & 1, kSiteDrainChunk, abort_flag)) {
        ok = false;
        break;
      }
      if (q == 0 && lane == 0) XE_CPB_TRACE(n, 11);
      tc_fence_after();
      const uint32_t t = tmem + pair * 256 + kTmDB + lane_bits;
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        float d[32];
        tmem_ld16(t + 32 * c, d);
        tmem_ld16(t + 32 * c + 16, d + 16);
        tmem_wait_ld();
#pragma unroll
        for (int o = 0; o < 32; ++o) run[32 * c + o] += d[o];
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&db_free[pair]);
      if (q == 0 && lane == 0) XE_CPB_TRACE(n, 12);
    }
    if (ok && first < last) flush(cur);
  } else if (warp == kMmaWarp) {
    // ------------------------------------------------------------ MMA issue
    if (lane == 0) {
      constexpr uint32_t idesc_x = idesc_tf32(kBM, 64, false, false);  // V (TMEM) x w^T (K-major)
      constexpr uint32_t idesc_w = idesc_tf32(kBM, 64, true, true);    // S x V^T, both MN-major
      int fold_count = 0;
      for (int i = first, n = 0; i < last; ++i, ++n) {
        const int pair = n & 1;
        const int j = n >> 1;
        const int st = n % kStages;
        const int f = i / p.tiles_m;
        if (i == first || f != (i - 1) / p.tiles_m) {
          if (!mbar_wait(w_ready, fold_count & 1, kSiteMmaChunk, abort_flag)) break;
          ++fold_count;
        }
        if (!mbar_wait(&ready[pair], j & 1, kSiteMmaFull, abort_flag)) break;
        XE_CPB_TRACE(n, 6);
        tc_fence_after();
        const uint32_t tb = tmem + pair * 256;
        // dX'[m, k] = sum_o V[m, o] w[o, k]: 8 k-steps over o, hi*hi + hi*lo + lo*hi
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint32_t boff = (kk >> 2) * (64 * 128) + (kk & 3) * 32;
          const uint64_t dh = smem_desc(smem_base + kOffWHi + boff, 16, 1024, kLayoutSW128);
          const uint64_t dl = smem_desc(smem_base + kOffWLo + boff, 16, 1024, kLayoutSW128);
          umma_tf32_ts(tb + kTmDX, tb + kTmVHi + 8 * kk, dh, idesc_x, kk != 0);
          umma_tf32_ts(tb + kTmDX, tb + kTmVHi + 8 * kk, dl, idesc_x, 1);
          umma_tf32_ts(tb + kTmDX, tb + kTmVLo + 8 * kk, dh, idesc_x, 1);
        }
        umma_commit(&dx_full[pair]);
        XE_CPB_TRACE(n, 7);
        // the fold's last tile: its w^T split may be replaced once these products are done
        if (i + 1 < last && (i + 1) / p.tiles_m != f) umma_commit(w_free);
        // the weight product, once the previous D_B of the pair is drained: per warp of the pair
        // (32 rows, MN-major k-rows) four 8-row k-steps of 1 KB
        if (j > 0 && !mbar_wait(&db_free[pair], (j - 1) & 1, kSiteMmaCorr, abort_flag)) break;
        XE_CPB_TRACE(n, 8);
        tc_fence_after();
        const uint32_t stage = smem_base + kOffStage + st * kStage;
#pragma unroll
        for (int w = 0; w < 2; ++w)
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            const uint32_t reg = stage + w * kRegion + kk * 1024;
            const uint64_t da = smem_desc(reg + kOffS, 4096, 512, kLayoutSW128Base32B);
            const uint64_t dvh = smem_desc(reg + kOffVtHi, 4096, 512, kLayoutSW128Base32B);
            const uint64_t dvl = smem_desc(reg + kOffVtLo, 4096, 512, kLayoutSW128Base32B);
            umma_tf32(tb + kTmDB, da, dvh, idesc_w, (w | kk) != 0);
            umma_tf32(tb + kTmDB, da, dvl, idesc_w, 1);
          }
        umma_commit(&stage_free[st]);
        umma_commit(&db_full[pair]);
        XE_CPB_TRACE(n, 9);
      }
      // All issued MMAs must finish before TMEM is released.
      umma_commit(drain);
      mbar_wait(drain, 0, kSiteGemmDrain, abort_flag, /*honor_abort=*/false);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ loads and the weight split
    bool ok = true;
    int fold_count = 0;
    // kGather2: the pixel values of a tile's row copies, looked up a tile ahead (the variables of
    // a fold once per fold)
    int pxv[4] = {0, 0, 0, 0};
    int var_fold = -1;
    int64_t var0 = 0, var1 = 0;
    auto lookup = [&](int i2) {
      const int f2 = i2 / p.tiles_m;
      const int mt2 = i2 - f2 * p.tiles_m;
      if (f2 != var_fold) {
        var_fold = f2;
        var0 = p.var ? (int64_t)__ldg(p.var + f2) : f2;
        var1 = p.var ? (int64_t)__ldg(p.var + f2 + p.pair) : (int64_t)f2 + p.pair;
        if (var0 < 0 || var0 >= p.variables || var1 < 0 || var1 >= p.variables) {
          record_bad_index(kSiteGemmGatherState);
          var0 = var1 = 0;
        }
      }
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        const int inst = 32 * t + lane;
        const int m = mt2 * kRows + (inst & 63);
        pxv[t] = m < p.M ? (int)__ldg(p.pixels + (int64_t)m * p.px_sm + ((inst >> 6) ? var1 : var0) * p.px_sv) : 0;
      }
    };
    if (SRC == kGather2 && first < last) lookup(first);
    for (int i = first, n = 0; i < last && ok; ++i, ++n) {
      const int f = i / p.tiles_m;
      const int st = n % kStages;
      const int mt = i - f * p.tiles_m;
      bool armed = true;
      if (lane == 0) {
        armed = mbar_wait(&stage_free[st], ((n / kStages) & 1) ^ 1, kSiteProducer, abort_flag);
        if (armed) {
          XE_CPB_TRACE(n, 10);
          mbar_expect_tx(&stage_full[st], kStageTx);
          stage_copies->note(st, n / kStages);
        }
      }
      if (__shfl_sync(0xffffffffu, armed ? 1 : 0, 0) == 0) {  // the warp leaves together
        ok = false;
        break;
      }
      const uint32_t stage = smem_base + kOffStage + st * kStage;
      if (SRC == kGather2) {
        // 128 row copies, rows 0..63 of the tile from table folds f and f + pair (instance i: fold
        // f + (i >> 6) pair, row i & 63), two per warp instruction: lanes 0-15 and 16-31 each copy one
        // 256-byte row as sixteen 16-byte cp.async into its swizzled K-major place.  Lane l holds the
        // pixel values of instances l, 32 + l, 64 + l and 96 + l, loaded a tile ahead; a row past M
        // copies its fold's first row (the pair threads mask it).
        int rowoff[4];
#pragma unroll
        for (int t = 0; t < 4; ++t) {
          const int inst = 32 * t + lane;
          int sv = pxv[t];
          if (sv >= p.states) {
            record_bad_index(kSiteGemmGatherState);
            sv = p.states - 1;
          }
          rowoff[t] = (int)((((int64_t)f + (int64_t)(inst >> 6) * p.pair) * p.states + sv) * 64);
        }
        if (i + 1 < last) lookup(i + 1);
        const int q = lane & 15;
#pragma unroll
        for (int it = 0; it < 64; ++it) {
          const int inst = 2 * it + (lane >> 4);
          const int off = __shfl_sync(0xffffffffu, rowoff[it >> 4], inst & 31);
          const int h = inst >> 6, r = inst & 63;
          const uint32_t dst = stage + (r >> 5) * kRegion + (2 * h + (q >> 3)) * kBlock + (r & 31) * 128 +
                               (((q & 7) ^ (r & 7)) << 4);
          cp_async_16(dst, p.table + off + 4 * q);
        }
        cp_async_arrive_noinc(&stage_full[st]);
      }
      if (lane == 0) {
        const int gz = f % p.g_folds;
#pragma unroll
        for (int w = 0; w < 2; ++w) {
          const uint32_t reg = stage + w * kRegion;
          const int r0 = mt * kRows + w * 32;
          if (SRC != kGather2) {
            tma_load_3d(reg, &tmap_x1, 0, r0, f, &stage_full[st]);
            tma_load_3d(reg + kBlock, &tmap_x1, 32, r0, f, &stage_full[st]);
            if (PAIR) {
              tma_load_3d(reg + 2 * kBlock, &tmap_x2, 0, r0, f, &stage_full[st]);
              tma_load_3d(reg + 3 * kBlock, &tmap_x2, 32, r0, f, &stage_full[st]);
            }
          }
          tma_load_3d(reg + 4 * kBlock, &tmap_y, 0, r0, f, &stage_full[st]);
          tma_load_3d(reg + 5 * kBlock, &tmap_y, 32, r0, f, &stage_full[st]);
          tma_load_3d(reg + 6 * kBlock, &tmap_g, 0, r0, gz, &stage_full[st]);
          tma_load_3d(reg + 7 * kBlock, &tmap_g, 32, r0, gz, &stage_full[st]);
        }
      }
      __syncwarp();
      if (i == first || f != (i - 1) / p.tiles_m) {
        // the fold's first tile: split its w into w^T hi / lo once the previous fold's dX'
        // products are done with them.  Lane l holds chunks c = l + 32 i: (k = c & 63, o = 4 (c >> 6)
        // .. + 3), read from w (o, k) in four batches of eight (coalesced over k); the first batch
        // is in flight during the wait.
        const float* wf = p.w + (int64_t)f * 4096;
        bool wfree = true;
#pragma unroll 1
        for (int b = 0; b < 4; ++b) {
          float4 wr[8];
#pragma unroll
          for (int t = 0; t < 8; ++t) {
            const int idx = 8 * b + t;
            const int kr = lane + 32 * (idx & 1), o = 4 * (idx >> 1);
            wr[t] = make_float4(__ldg(wf + o * 64 + kr), __ldg(wf + (o + 1) * 64 + kr), __ldg(wf + (o + 2) * 64 + kr),
                                __ldg(wf + (o + 3) * 64 + kr));
          }
          if (b == 0) {
            if (lane == 0 && fold_count > 0)
              wfree = mbar_wait(w_free, (fold_count - 1) & 1, kSiteProducer, abort_flag);
            wfree = __shfl_sync(0xffffffffu, wfree ? 1 : 0, 0) != 0;
            if (!wfree) break;
          }
#pragma unroll
          for (int t = 0; t < 8; ++t) {
            const int idx = 8 * b + t;
            const int kr = lane + 32 * (idx & 1), oc = idx >> 1;
            float4 hi, lo;
            split_rn(wr[t].x, hi.x, lo.x);
            split_rn(wr[t].y, hi.y, lo.y);
            split_rn(wr[t].z, hi.z, lo.z);
            split_rn(wr[t].w, hi.w, lo.w);
            const uint32_t dst = (oc >> 3) * (64 * 128) + kmajor_off(kr, oc & 7);
            sts_v4(smem_base + kOffWHi + dst, hi);
            sts_v4(smem_base + kOffWLo + dst, lo);
          }
        }
        if (!wfree) {
          ok = false;
          break;
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(w_ready);
        ++fold_count;
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (*abort_flag) {  // uniform: every thread has passed its last wait
    stage_copies->drain(stage_full, abort_flag);
    __syncthreads();
  }
  tc_fence_after();
  if (warp == kMmaWarp) tmem_dealloc<512>(tmem);
}

// dw[f] = the sum of fold f's workspace slots (its CTAs in order, each slot's halves h = 0, 1);
// one thread per 4 consecutive elements.
__global__ void __launch_bounds__(256) cpb_reduce_kernel(const float* __restrict__ partials, int folds, int pieces,
                                                         int tiles_m, int num_tiles, int grid, float* __restrict__ dw) {
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (int64_t)folds * 1024) return;
  const int f = (int)(idx >> 10);
  const int e4 = (int)(idx & 1023);
  const int c0 = cta_of_tile((int64_t)f * tiles_m, num_tiles, grid);
  const int c1 = cta_of_tile((int64_t)f * tiles_m + tiles_m - 1, num_tiles, grid);
  float4 s = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
  for (int pc = 0; pc <= c1 - c0; ++pc)
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const float4 v = __ldg(reinterpret_cast<const float4*>(partials + (((int64_t)f * pieces + pc) * 2 + h) * 4096) + e4);
      s.x += v.x;
      s.y += v.y;
      s.z += v.z;
      s.w += v.w;
    }
  reinterpret_cast<float4*>(dw)[idx] = s;
}

// ---------------------------------------------------------------------------- state-table gradient
constexpr int kTgWarps = 31;  // consumer warps; warp w owns the states s with s % 31 == w
constexpr int kTgStatesPerWarp = (256 + kTgWarps - 1) / kTgWarps;  // 9
constexpr int kTgThreads = (kTgWarps + 1) * 32;
constexpr int kTgChunk = 64;  // rows of dX per bulk copy (16 KB)
constexpr int kTgStages = 4;
constexpr int kTgRing = kTgStages * kTgChunk * 256;
constexpr int kTgSmemBytes = kTgRing + 128;

// A warp's sums live in registers: lane l holds units 2l, 2l+1 of its (at most 9) states of both
// table folds; a row is added to its state's pair through a switch on the state index (uniform over the
// warp), in increasing row order.  The pixel values are loaded a chunk ahead.  Rows reach shared memory in 64-row chunks through a 4-slot
// ring filled by the last warp.  A CTA takes folds blockIdx.x, blockIdx.x + gridDim.x, ...
__global__ void __launch_bounds__(kTgThreads, 1)
    table_grad_pair_kernel(const float* __restrict__ dx, int folds, int M, const uint8_t* __restrict__ pixels,
                           int64_t px_sm, int64_t px_sv, int64_t variables, const int32_t* __restrict__ var, int pair,
                           int states, float* __restrict__ dt) {
  extern __shared__ __align__(16) uint8_t tg_smem[];
  const uint32_t ring = smem_u32(tg_smem);
  uint64_t* full = reinterpret_cast<uint64_t*>(tg_smem + kTgRing);
  uint64_t* empty = full + kTgStages;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(empty + kTgStages);
  ArmedCopies* copies = reinterpret_cast<ArmedCopies*>(const_cast<int*>(abort_flag) + 1);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int i = 0; i < kTgStages; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], kTgWarps);
    }
    *abort_flag = 0;
    *copies = ArmedCopies{0u, 0u};
    fence_mbarrier_init();
  }
  __syncthreads();
  const int chunks = (M + kTgChunk - 1) / kTgChunk;
  if (warp == kTgWarps) {
    if (lane == 0) {
      int c_all = 0;  // chunks over every fold of this CTA, in order
      for (int f = blockIdx.x; f < folds; f += gridDim.x) {
        const float* src = dx + (int64_t)f * M * 64;
        bool fine = true;
        for (int c = 0; c < chunks; ++c, ++c_all) {
          const int slot = c_all % kTgStages;
          const uint32_t u = c_all / kTgStages;
          if (!mbar_wait(&empty[slot], (u & 1) ^ 1, kSiteProducer, abort_flag)) {
            fine = false;
            break;
          }
          const int rows = min(kTgChunk, M - c * kTgChunk);
          XE_CPB_TRACE(c_all, 0);
          mbar_expect_tx(&full[slot], rows * 256);
          copies->note(slot, u);
          bulk_load(ring + slot * (kTgChunk * 256), src + (int64_t)c * kTgChunk * 64, rows * 256, &full[slot]);
        }
        if (!fine) break;
      }
    }
  } else {
    int c_all = 0;
    bool fine = true;
    for (int f = blockIdx.x; f < folds && fine; f += gridDim.x) {
      int64_t v1 = var ? (int64_t)__ldg(var + f) : f;
      int64_t v2 = var ? (int64_t)__ldg(var + f + pair) : (int64_t)f + pair;
      if (v1 < 0 || v1 >= variables || v2 < 0 || v2 >= variables) {
        record_bad_index(kSiteGatherState);
        v1 = v2 = 0;
      }
      float2 acc[2][kTgStatesPerWarp];
#pragma unroll
      for (int t = 0; t < 2; ++t)
#pragma unroll
        for (int k = 0; k < kTgStatesPerWarp; ++k) acc[t][k] = make_float2(0.0f, 0.0f);
      // the pixel values of rows lane and 32 + lane of chunk c (-1 past M), loaded a chunk ahead
      // and checked where they are used
      const uint8_t* px1 = pixels + v1 * px_sv;
      const uint8_t* px2 = pixels + v2 * px_sv;
      auto pixels_of = [&](int c, int (&s1)[2], int (&s2)[2]) {
#pragma unroll
        for (int hf = 0; hf < 2; ++hf) {
          const int m = c * kTgChunk + 32 * hf + lane;
          const bool in = c < chunks && m < M;
          s1[hf] = in ? (int)__ldg(px1 + (int64_t)m * px_sm) : -1;
          s2[hf] = in ? (int)__ldg(px2 + (int64_t)m * px_sm) : -1;
        }
      };
      int n1[2], n2[2];
      pixels_of(0, n1, n2);
      for (int c = 0; c < chunks; ++c, ++c_all) {
        const int slot = c_all % kTgStages;
        const uint32_t u = c_all / kTgStages;
        int s1[2] = {n1[0], n1[1]}, s2[2] = {n2[0], n2[1]};
        pixels_of(c + 1, n1, n2);
        if (warp == 0 && lane == 0) XE_CPB_TRACE(c_all, 1);
        if (!mbar_wait_warp(&full[slot], u & 1, kSiteAStaged, abort_flag)) {
          fine = false;
          break;
        }
        if (warp == 0 && lane == 0) XE_CPB_TRACE(c_all, 2);
#pragma unroll
        for (int hf = 0; hf < 2; ++hf) {
          if (s1[hf] >= states || s2[hf] >= states) {
            record_bad_index(kSiteGatherState);
            s1[hf] = min(s1[hf], states - 1);
            s2[hf] = min(s2[hf], states - 1);
          }
        }
#pragma unroll
        for (int hf = 0; hf < 2; ++hf) {
          const uint32_t rows = ring + slot * (kTgChunk * 256) + hf * (32 * 256) + lane * 8;
#pragma unroll
          for (int t = 0; t < 2; ++t) {
            const int sv = t == 0 ? s1[hf] : s2[hf];
            uint32_t own = __ballot_sync(0xffffffffu, sv >= 0 && sv % kTgWarps == warp);
            while (own) {
              const int b = __ffs(own) - 1;
              own &= own - 1;
              const int k = __shfl_sync(0xffffffffu, sv, b) / kTgWarps;  // this warp's state index (uniform)
              const float2 x = lds_v2(rows + b * 256);
              switch (k) {
#define XE_TG_ADD(kk)          \
  case kk:                     \
    acc[t][kk].x += x.x;       \
    acc[t][kk].y += x.y;       \
    break;
                XE_TG_ADD(0) XE_TG_ADD(1) XE_TG_ADD(2) XE_TG_ADD(3) XE_TG_ADD(4) XE_TG_ADD(5) XE_TG_ADD(6)
                XE_TG_ADD(7) XE_TG_ADD(8)
#undef XE_TG_ADD
                default: break;
              }
            }
          }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[slot]);
        if (lane == 0) XE_CPB_TRACE(c_all, 3 + (warp & 7));
      }
      if (!fine) break;
      // both table folds' rows of this warp's states (zero where no row selected them)
#pragma unroll
      for (int t = 0; t < 2; ++t) {
        float* base = dt + ((int64_t)f + (int64_t)t * pair) * states * 64;
#pragma unroll
        for (int kk = 0; kk < kTgStatesPerWarp; ++kk) {
          const int st = warp + kTgWarps * kk;
          if (st < states) reinterpret_cast<float2*>(base + (int64_t)st * 64)[lane] = acc[t][kk];
        }
      }
    }
  }
  __syncthreads();
  if (*abort_flag) copies->drain(full, abort_flag);
}

}  // namespace cpb
}  // namespace xe
