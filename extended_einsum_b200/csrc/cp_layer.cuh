// cp_layer.cuh — the folded CP sum layer of a circuit with K = N = 64.
//
// C[f,m,n] = log( sum_k exp(X[f,m,k] - s) W'[f,k,n] ) + s,  X = A (+ A2),
// s = max_k (or min_k) X[f,m,:], W' linear (the softmax of the layer's
// logits): the folded CP layer 'dac,dbc->dab' (preprocess.py:1310-1337) with
// the folded Hadamard product of the previous level fused into X
// (translate.py:706-718), lowered by _append_logspace_einsum
// (translate.py:686-750).  It computes what lse_gemm_kernel computes for these
// shapes, with the same arithmetic in the same order (split-TF32, the same
// exp / split / log helpers, the same MMA sequence), so the results are
// identical; its schedule is built for tiles whose tensor work is small:
//
//  * each CTA takes a contiguous range of 128-row tiles (tiles of one fold are
//    consecutive), so the fold's weights are split into TF32 hi / lo once per
//    fold, not once per tile;
//  * two warp groups own alternate tiles, each doing the row scan, the exp /
//    split into its own TMEM columns and the epilogue of its tiles, so that one
//    group's transform overlaps the other's epilogue and the tensor work; a
//    row (64 values) is held in registers, and its staging slot is released
//    as soon as the row extreme is known;
//  * outputs leave through TMA stores of 32 x 32 blocks.
//
// Sources of X: kDense (A), kDense2 (A + A2, both TMA-staged per tile), and
// kSlab2, the second sum layer over a state table T (folds0, states, 64):
// X[f,m,:] = T[f, x_m, :] + T[f + pair, x'_m, :] with x_m = pixels[m, var[f]]
// and x'_m = pixels[m, var[f + pair]] (xe_logspace_gemm_gather_pair).  For
// kSlab2 the two folds' table slabs (states x 64 each) are loaded into shared
// memory once per fold and every row is read from them by its pixel value.
//
// Warps 0-3 and 4-7: the warp groups (thread = tile row); warp 8: TMEM
// allocation and MMA issue; warp 9: TMA loads and the weight split.
#pragma once

#include "lse_gemm.cuh"

namespace xe {
namespace cp {

#define XE_CP_TRACE(n, ev) XE_TILE_TRACE(n, ev)

using namespace gemm;
constexpr int kK = 64;
constexpr int kN = 64;
constexpr int kThreads = 320;
constexpr int kMmaWarp = 8;
constexpr int kProducerWarp = 9;
constexpr int kAKBlock = kBM * 32 * 4;  // 16 KB: 128 rows x 32 k, 128-byte swizzle
constexpr int kATile = 2 * kAKBlock;    // one operand tile (both k-blocks)
constexpr int kBKBlock = kN * 32 * 4;   // 8 KB: 64 n x 32 k
constexpr int kBBytes = 2 * kBKBlock;   // one of raw / hi / lo
constexpr int kOutBytes = 32 * 32 * 4;  // per warp: 32 rows x 32 columns
// TMEM columns of a warp group: A hi/lo for k-block 0 [0, 64), k-block 1 [64, 128);
// main accumulator [128, 192); correction accumulator [192, 256)
constexpr uint32_t kTmemMain = 128, kTmemCorr = 192, kTmemPerGroup = 256;

enum Source : int { kDense = 0, kDense2 = 1, kSlab2 = 2 };
constexpr int kSlabKBlock = 256 * 128;  // one k-block of a slab: up to 256 states x 32 k

template <int SRC>
struct Cfg {
  static constexpr bool kPair = SRC != kDense;
  static constexpr int kStageBytes = (kPair ? 2 : 1) * kATile;
  static constexpr int kStages = SRC == kDense ? 2 : 1;  // per warp group
  static constexpr int kOffA = 0;  // A stages, or the two slabs [2][2 k-blocks]
  static constexpr int kABytes = SRC == kSlab2 ? 4 * kSlabKBlock : 2 * kStages * kStageBytes;
  static constexpr int kOffBRaw = kOffA + kABytes;
  static constexpr int kOffBHi = kOffBRaw + kBBytes;
  static constexpr int kOffBLo = kOffBHi + kBBytes;
  static constexpr int kOffOut = kOffBLo + kBBytes;
  static constexpr int kOffBar = kOffOut + 8 * kOutBytes;
  static constexpr int kSmemBytes = 1024 + kOffBar + 512;
  static_assert(kSmemBytes <= 232448, "shared memory");
};

struct Params {
  int folds, M, tiles_m, num_tiles;
  int shift_min;
  // kSlab2
  const uint8_t* pixels;
  const int32_t* var;  // nullptr: variable = fold
  int64_t pixel_stride;
  int states, pair;
};

__device__ __forceinline__ void tma_store_3d(const CUtensorMap* map, uint32_t src, int x, int y, int z) {
  asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.tile.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(map),
               "r"(src), "r"(x), "r"(y), "r"(z)
               : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_read() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

// Tiles [first, last) of this CTA: contiguous, fold-major.
__device__ __forceinline__ void tile_range(const Params& p, int& first, int& last) {
  first = (int)(((int64_t)p.num_tiles * blockIdx.x) / gridDim.x);
  last = (int)(((int64_t)p.num_tiles * (blockIdx.x + 1)) / gridDim.x);
}

template <int SRC>
__global__ void __launch_bounds__(kThreads, 1)
    cp_layer_kernel(const Params p, const __grid_constant__ CUtensorMap tmap_a,
                    const __grid_constant__ CUtensorMap tmap_a2, const __grid_constant__ CUtensorMap tmap_w,
                    const __grid_constant__ CUtensorMap tmap_c) {
  using C = Cfg<SRC>;
  constexpr bool PAIR = C::kPair;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  const uint32_t smem_base = smem_u32(smem);
  uint64_t* bars = (uint64_t*)(smem + C::kOffBar);
  uint64_t* a_full = bars;                       // [2][kStages]
  uint64_t* a_empty = a_full + 2 * C::kStages;   // [2][kStages]
  uint64_t* a_ready = a_empty + 2 * C::kStages;  // [2]
  uint64_t* acc_full = a_ready + 2;              // [2]
  uint64_t* b_ready = acc_full + 2;
  uint64_t* b_free = b_ready + 1;
  uint64_t* raw_full = b_free + 1;
  uint64_t* drain = raw_full + 1;
  uint64_t* slab_full = drain + 1;
  uint64_t* slab_empty = slab_full + 1;
  uint32_t* tmem_slot = (uint32_t*)(slab_empty + 1);
  volatile int* abort_flag = (volatile int*)(tmem_slot + 1);
  // the barriers the producer armed, drained at wind-down after an abort
  ArmedCopies* a_copies = (ArmedCopies*)(tmem_slot + 2);
  ArmedCopies* raw_copies = a_copies + 1;
  ArmedCopies* slab_copies = a_copies + 2;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int i = 0; i < 2 * C::kStages; ++i) {
      mbar_init(&a_full[i], 1);
      mbar_init(&a_empty[i], 128);
    }
    for (int g = 0; g < 2; ++g) {
      mbar_init(&a_ready[g], 4);
      mbar_init(&acc_full[g], 1);
    }
    mbar_init(b_ready, 1);
    mbar_init(b_free, 1);
    mbar_init(raw_full, 1);
    mbar_init(drain, 1);
    mbar_init(slab_full, 1);
    mbar_init(slab_empty, 256);
    *abort_flag = 0;
    *a_copies = *raw_copies = *slab_copies = ArmedCopies{0u, 0u};
    fence_mbarrier_init();
  }
  if (warp == kMmaWarp) tmem_alloc<512>(tmem_slot);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const bool is_min = p.shift_min != 0;

  int first, last;
  tile_range(p, first, last);
  auto fold_of = [&](int tile) { return tile / p.tiles_m; };

  if (warp < 8) {
    // ------------------------------------------------------------ warp groups
    const int group = warp >> 2;
    const int q = warp & 3;
    const int r = q * 32 + lane;
    const uint32_t lane_bits = (uint32_t)(q * 32) << 16;
    const uint32_t tg = tmem + group * kTmemPerGroup + lane_bits;
    const uint32_t out_buf = smem_base + C::kOffOut + warp * kOutBytes;
    const float fill = -INFINITY;
    bool ok = true;
    // kSlab2: pixel values of this thread's row in the group's next tile (loaded a tile ahead).
    // Every group acquires the slabs of every fold of the CTA in order (a wait on slab_full
    // phase g), whether or not it has a tile there, and releases fold g (an arrival on
    // slab_empty) only after acquiring it: neither barrier then runs more than one phase
    // ahead of a waiter, and each release lands in its own fold's phase.
    int px1 = 0, px2 = 0, released = 0, acquired = 0;
    const int fold0 = first < last ? fold_of(first) : 0;
    auto load_pixels = [&](int tile, int& s1, int& s2) {
      const int f = fold_of(tile);
      const int m = (tile - f * p.tiles_m) * kBM + r;
      int64_t v1 = p.var ? (int64_t)__ldg(p.var + f) : f;
      int64_t v2 = p.var ? (int64_t)__ldg(p.var + f + p.pair) : (int64_t)f + p.pair;
      if (v1 < 0 || v1 >= p.pixel_stride || v2 < 0 || v2 >= p.pixel_stride) {
        record_bad_index(kSiteGemmGatherState);
        v1 = v2 = 0;
      }
      s1 = m < p.M ? (int)__ldg(p.pixels + (int64_t)m * p.pixel_stride + v1) : 0;
      s2 = m < p.M ? (int)__ldg(p.pixels + (int64_t)m * p.pixel_stride + v2) : 0;
    };
    // The row of local tile j (tile i of the CTA) in registers, and its extreme (the shift);
    // false if a wait gave up.  Releases the staging slot (dense sources) once every value has
    // been used.
    auto load_row = [&](int i, int j, float (&x)[64], float& shift) -> bool {
      const int bb = fold_of(i);
      const int mt = i - bb * p.tiles_m;
      const bool valid = mt * kBM + r < p.M;
      const int sidx = j % C::kStages;
      if (SRC == kSlab2) {
        const int g = bb - fold0;
        bool fine = true;
        while (fine && acquired <= g) {
          while (released < acquired) {  // folds before `acquired` are done with
            mbar_arrive(slab_empty);
            ++released;
          }
          fine = mbar_wait_warp(slab_full, acquired & 1, kSiteAStaged, abort_flag);
          ++acquired;
        }
        if (!fine) return false;
        int s1 = px1, s2 = px2;
        if (i + 2 < last) load_pixels(i + 2, px1, px2);
        if (s1 >= p.states || s2 >= p.states) {
          record_bad_index(kSiteGemmGatherState);
          s1 = min(s1, p.states - 1);
          s2 = min(s2, p.states - 1);
        }
#pragma unroll
        for (int kb = 0; kb < 2; ++kb) {
          const uint32_t row1 = smem_base + C::kOffA + kb * kSlabKBlock + s1 * 128;
          const uint32_t row2 = smem_base + C::kOffA + (2 + kb) * kSlabKBlock + s2 * 128;
#pragma unroll
          for (int c = 0; c < 8; ++c) {
            float4 v = lds_v4(row1 + ((c ^ (s1 & 7)) << 4));
            const float4 w = lds_v4(row2 + ((c ^ (s2 & 7)) << 4));
            v.x += w.x;
            v.y += w.y;
            v.z += w.z;
            v.w += w.w;
            x[32 * kb + 4 * c] = valid ? v.x : fill;
            x[32 * kb + 4 * c + 1] = valid ? v.y : fill;
            x[32 * kb + 4 * c + 2] = valid ? v.z : fill;
            x[32 * kb + 4 * c + 3] = valid ? v.w : fill;
          }
        }
      } else {
        const uint32_t u = j / C::kStages;
        if (!mbar_wait_warp(&a_full[group * C::kStages + sidx], u & 1, kSiteAStaged, abort_flag)) return false;
        const uint32_t stage = smem_base + C::kOffA + (group * C::kStages + sidx) * C::kStageBytes;
#pragma unroll
        for (int kb = 0; kb < 2; ++kb) {
          const uint32_t row = stage + kb * kAKBlock + r * 128;
#pragma unroll
          for (int c = 0; c < 8; ++c) {
            float4 v = lds_v4(row + ((c ^ (r & 7)) << 4));
            if (PAIR) {
              const float4 w = lds_v4(row + kATile + ((c ^ (r & 7)) << 4));
              v.x += w.x;
              v.y += w.y;
              v.z += w.z;
              v.w += w.w;
            }
            x[32 * kb + 4 * c] = valid ? v.x : fill;
            x[32 * kb + 4 * c + 1] = valid ? v.y : fill;
            x[32 * kb + 4 * c + 2] = valid ? v.z : fill;
            x[32 * kb + 4 * c + 3] = valid ? v.w : fill;
          }
        }
      }
      // four independent chains (max / min are exact: the order does not change the result)
      float e0 = is_min ? INFINITY : -INFINITY, e1 = e0, e2 = e0, e3 = e0;
#pragma unroll
      for (int k = 0; k < 64; k += 4) {
        e0 = extreme(e0, x[k], is_min);
        e1 = extreme(e1, x[k + 1], is_min);
        e2 = extreme(e2, x[k + 2], is_min);
        e3 = extreme(e3, x[k + 3], is_min);
      }
      const float e = extreme(extreme(e0, e1, is_min), extreme(e2, e3, is_min), is_min);
      shift = valid ? e : 0.0f;
      // every value of the row has been used: the slot may be refilled
      if (SRC != kSlab2) mbar_arrive(&a_empty[group * C::kStages + sidx]);
      return true;
    };
    if (SRC == kSlab2 && first + group < last) load_pixels(first + group, px1, px2);
    float x[64], shift = 0.0f;
    if (first + group < last) ok = load_row(first + group, 0, x, shift);
    // Pipelined (kPipelined): the transform of tile j, then the row of tile j+1 while tile j's
    // products run, then tile j's epilogue; otherwise the row of tile j+1 follows the epilogue
    // (one staging slot per group: its next tile is still in flight).  Either way the transform
    // of tile j+1 (into the A columns tile j's products read) follows the epilogue of tile j,
    // which waited for those products.
    constexpr bool kPipelined = C::kStages > 1 || SRC == kSlab2;
    for (int i = first + group, j = 0; i < last && ok; i += 2, ++j) {
      const int bb = fold_of(i);
      const int mt = i - bb * p.tiles_m;
      const float tile_shift = shift;
      if (r == 0) XE_CP_TRACE(i - first, 0);
      // -------- exp / split into this group's A columns
#pragma unroll
      for (int kb = 0; kb < 2; ++kb) {
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          float hi[16], lo[16];
#pragma unroll
          for (int t = 0; t < 16; ++t) split_rn(exp_shifted(x[32 * kb + 16 * h + t], tile_shift), hi[t], lo[t]);
          tmem_st16(tg + 64 * kb + 16 * h, hi);
          tmem_st16(tg + 64 * kb + 32 + 16 * h, lo);
        }
      }
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&a_ready[group]);
      if (r == 0) XE_CP_TRACE(i - first, 1);
      // -------- the group's next row while this tile's products run
      if (kPipelined && i + 2 < last && !load_row(i + 2, j + 1, x, shift)) ok = false;
      if (r == 0) XE_CP_TRACE(i - first, 2);
      // -------- epilogue
      if (!mbar_wait_warp(&acc_full[group], j & 1, kSiteDrainChunk, abort_flag)) {
        ok = false;
        break;
      }
      tc_fence_after();
      if (r == 0) XE_CP_TRACE(i - first, 3);
#pragma unroll 1
      for (int sl = 0; sl < 2; ++sl) {
        float out[32], w[32];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          tmem_ld16(tg + kTmemMain + 32 * sl + 16 * h, out + 16 * h);
          tmem_ld16(tg + kTmemCorr + 32 * sl + 16 * h, w + 16 * h);
        }
        tmem_wait_ld();
#pragma unroll
        for (int t = 0; t < 32; ++t) {
          // an overflowed main term carries the result; its correction is NaN
          const float s = isinf(out[t]) ? out[t] : out[t] + w[t];
          out[t] = fast_log(s) + tile_shift;
        }
        // the previous block's store has read this warp's staging buffer
        if (lane == 0) bulk_wait_read();
        __syncwarp();
#pragma unroll
        for (int c = 0; c < 8; ++c)
          sts_v4(out_buf + lane * 128 + ((c ^ (lane & 7)) << 4),
                 make_float4(out[4 * c], out[4 * c + 1], out[4 * c + 2], out[4 * c + 3]));
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          tma_store_3d(&tmap_c, out_buf, 32 * sl, mt * kBM + q * 32, bb);
          bulk_commit();
        }
      }
      // this tile's accumulator has been read: the MMAs of the group's next tile may
      // overwrite it once its A columns are written (a_ready orders both)
      tc_fence_before();
      if (r == 0) XE_CP_TRACE(i - first, 4);
      if (!kPipelined && i + 2 < last && !load_row(i + 2, j + 1, x, shift)) ok = false;
    }
    // kSlab2: release the remaining folds' slabs (this group may have no tile in the last ones)
    if (SRC == kSlab2 && first < last && ok) {
      const int folds_here = fold_of(last - 1) - fold0 + 1;
      while (ok && acquired < folds_here) {
        while (released < acquired) {
          mbar_arrive(slab_empty);
          ++released;
        }
        ok = mbar_wait_warp(slab_full, acquired & 1, kSiteAStaged, abort_flag);
        ++acquired;
      }
      while (released < acquired) {
        mbar_arrive(slab_empty);
        ++released;
      }
    }
    if (lane == 0) bulk_wait_all();
    __syncwarp();
  } else if (warp == kMmaWarp) {
    // ------------------------------------------------------------ MMA issue
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_tf32(kBM, kN, false, false);
      int fold_count = 0;
      for (int i = first, n = 0; i < last; ++i, ++n) {
        const int group = n & 1;
        const int j = n >> 1;
        if (i == first || fold_of(i) != fold_of(i - 1)) {
          if (!mbar_wait(b_ready, fold_count & 1, kSiteMmaChunk, abort_flag)) break;
          ++fold_count;
        }
        XE_CP_TRACE(n, 5);
        if (!mbar_wait(&a_ready[group], j & 1, kSiteMmaFull, abort_flag)) break;
        tc_fence_after();
        XE_CP_TRACE(n, 6);
        const uint32_t tg = tmem + group * kTmemPerGroup;
        const uint32_t d_main = tg + kTmemMain, d_corr = tg + kTmemCorr;
#pragma unroll
        for (int kb = 0; kb < 2; ++kb) {
          const uint32_t a_hi = tg + 64 * kb, a_lo = a_hi + 32;
          const uint32_t b_hi = smem_base + C::kOffBHi + kb * kBKBlock, b_lo = smem_base + C::kOffBLo + kb * kBKBlock;
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            const uint64_t dbh = smem_desc(b_hi + kk * 32, 16, 1024, kLayoutSW128);
            const uint64_t dbl = smem_desc(b_lo + kk * 32, 16, 1024, kLayoutSW128);
            umma_tf32_ts(d_main, a_hi + kk * 8, dbh, idesc, (kb | kk) != 0);
            umma_tf32_ts(d_corr, a_hi + kk * 8, dbl, idesc, (kb | kk) != 0);
            umma_tf32_ts(d_corr, a_lo + kk * 8, dbh, idesc, 1);
          }
        }
        umma_commit(&acc_full[group]);
        // the fold's last tile: the weights may be replaced once these products are done
        if (i + 1 < last && fold_of(i + 1) != fold_of(i)) umma_commit(b_free);
      }
      // All issued MMAs must finish before TMEM is released.
      umma_commit(drain);
      mbar_wait(drain, 0, kSiteGemmDrain, abort_flag, /*honor_abort=*/false);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ TMA loads, weight split
    bool ok = true;
    int fold_count = 0;
    uint32_t raw_arms = 0;
    // the first fold's raw weights
    if (lane == 0 && first < last) {
      mbar_expect_tx(raw_full, kBBytes);
      raw_copies->note(0, raw_arms++);
      const int f = fold_of(first);
      tma_load_3d(smem_base + C::kOffBRaw, &tmap_w, 0, 0, f, raw_full);
      tma_load_3d(smem_base + C::kOffBRaw + kBKBlock, &tmap_w, 32, 0, f, raw_full);
    }
    for (int i = first, n = 0; i < last && ok; ++i, ++n) {
      const int bb = fold_of(i);
      if (i == first || bb != fold_of(i - 1)) {
        // kSlab2: both warp groups are done with the previous fold's slabs; load this fold's
        bool ready = true;
        if (SRC == kSlab2 && lane == 0) {
          if (fold_count > 0) ready = mbar_wait(slab_empty, (fold_count - 1) & 1, kSiteProducer, abort_flag);
          if (ready) {
            mbar_expect_tx(slab_full, 4 * p.states * 128);
            slab_copies->note(0, fold_count);
#pragma unroll
            for (int h = 0; h < 2; ++h)
#pragma unroll
              for (int kb = 0; kb < 2; ++kb)
                tma_load_3d(smem_base + C::kOffA + (2 * h + kb) * kSlabKBlock, &tmap_a, 32 * kb, 0, bb + h * p.pair,
                            slab_full);
          }
        }
        // the previous fold's products are done with hi / lo; the raw weights have landed
        if (lane == 0) {
          if (ready && fold_count > 0) ready = mbar_wait(b_free, (fold_count - 1) & 1, kSiteProducer, abort_flag);
          if (ready) ready = mbar_wait(raw_full, fold_count & 1, kSiteProducer, abort_flag);
        }
        if (__shfl_sync(0xffffffffu, ready ? 1 : 0, 0) == 0) break;
        // split: raw [n][32 k] per k-block (unswizzled) -> hi / lo, K-major 128-byte swizzle
#pragma unroll 4
        for (int c = lane; c < 2 * kN * 8; c += 32) {
          const int kb = c >> 9, nn = (c >> 3) & (kN - 1), qq = c & 7;
          const float4 v = lds_v4(smem_base + C::kOffBRaw + kb * kBKBlock + (nn * 32 + 4 * qq) * 4);
          float4 h, l;
          split_rn(v.x, h.x, l.x);
          split_rn(v.y, h.y, l.y);
          split_rn(v.z, h.z, l.z);
          split_rn(v.w, h.w, l.w);
          const uint32_t off = kb * kBKBlock + kmajor_off(nn, qq);
          sts_v4(smem_base + C::kOffBHi + off, h);
          sts_v4(smem_base + C::kOffBLo + off, l);
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(b_ready);
          // the next fold's raw weights (the raw buffer has been read)
          int next = i + 1;
          while (next < last && fold_of(next) == bb) ++next;
          if (next < last) {
            mbar_expect_tx(raw_full, kBBytes);
            raw_copies->note(0, raw_arms++);
            tma_load_3d(smem_base + C::kOffBRaw, &tmap_w, 0, 0, fold_of(next), raw_full);
            tma_load_3d(smem_base + C::kOffBRaw + kBKBlock, &tmap_w, 32, 0, fold_of(next), raw_full);
          }
        }
        ++fold_count;
      }
      if (SRC != kSlab2 && lane == 0) {
        const int group = n & 1;
        const int j = n >> 1;
        const int sidx = j % C::kStages;
        const uint32_t u = j / C::kStages;
        const int slot = group * C::kStages + sidx;
        if (!mbar_wait(&a_empty[slot], (u & 1) ^ 1, kSiteProducer, abort_flag)) {
          ok = false;
        } else {
          const int mt = i - bb * p.tiles_m;
          const uint32_t dst = smem_base + C::kOffA + slot * C::kStageBytes;
          mbar_expect_tx(&a_full[slot], C::kStageBytes);
          a_copies->note(slot, u);
          tma_load_3d(dst, &tmap_a, 0, mt * kBM, bb, &a_full[slot]);
          tma_load_3d(dst + kAKBlock, &tmap_a, 32, mt * kBM, bb, &a_full[slot]);
          if (PAIR) {
            tma_load_3d(dst + kATile, &tmap_a2, 0, mt * kBM, bb, &a_full[slot]);
            tma_load_3d(dst + kATile + kAKBlock, &tmap_a2, 32, mt * kBM, bb, &a_full[slot]);
          }
        }
      }
      ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (*abort_flag) {  // uniform: every thread has passed its last wait
    a_copies->drain(a_full, abort_flag);
    raw_copies->drain(raw_full, abort_flag);
    slab_copies->drain(slab_full, abort_flag);
    __syncthreads();
  }
  tc_fence_after();
  if (warp == kMmaWarp) tmem_dealloc<512>(tmem);
}

}  // namespace cp
}  // namespace xe
