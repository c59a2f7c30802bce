// tucker_layer.cuh — the log-space Tucker layer 'bfi,bfj,foij->bfo' with I = J = O = 32.
//
// y[b,f,o] = log( sum_ij exp(l[b,f,i]-sl) exp(r[b,f,j]-sr) w[f,o,i,j] ) + sl + sr,
// the ternary einsum that OptimizeContractionPaths fuses for Tucker circuits
// (preprocess.py:1095-1106), lowered by _append_logspace_einsum
// (translate.py:686-750), with sl / sr the max (or min) of l / r over i / j and
// w linear (a softmax of the layer's logits).  The contraction runs in two
// stages, j first (the path torch.einsum takes for the three operands):
//
//   T[b,(o,i)] = sum_j er[b,j] w[f,o,i,j]     tensor cores: M = 128 rows b, N = 128
//                                             (four o) per chunk, K = 32 j, split-TF32
//                                             (hi*hi + hi*lo + lo*hi: 96 products per
//                                             output, accumulated in fp32)
//   y[b,o]     = sum_i el[b,i] T[b,(o,i)]     fp32 FMAs in the epilogue
//
// with el = exp(l - sl), er = exp(r - sr).  That is half the tensor work of the
// fused (i,j) product, and the A operand (er) is 32 values per row instead of
// 1024.  Per 128-row tile of fold f the weights w[f] stream through shared memory
// in 8 chunks of 128 (o,i) rows x 32 j, split into TF32 hi / lo as they arrive.
//
// Warps 0-3 and 4-7: two row groups owning alternate tiles of the CTA's
// contiguous range (scan, exp, A operand in TMEM, epilogue), each with one
// accumulator: while a group drains a chunk, the other group's products run;
// warps 8-11: TF32 split of the weight chunks;
// warp 12: TMEM allocation and MMA issue (the two tiles' chunks interleaved);
// warp 13: TMA loads.
#pragma once

#include "cp_layer.cuh"

namespace xe {
namespace tk {

using namespace gemm;
constexpr int kDim = 32;                        // I = J = O
constexpr int kChunkN = 128;                    // (o,i) rows per chunk: four o
constexpr int kChunks = kDim * kDim / kChunkN;  // 8 per tile
constexpr int kThreads = 448;
constexpr int kLoWarp0 = 8, kMmaWarp = 12, kProducerWarp = 13;
constexpr int kRowBytes = kBM * kDim * 4;    // 16 KB: 128 rows x 32, 128-byte swizzle
constexpr int kWBytes = kChunkN * kDim * 4;  // 16 KB: 128 (o,i) rows x 32 j
constexpr int kWStages = 4;
constexpr int kOutBytes = 32 * kDim * 4;  // per row warp: 32 rows x 32 o
// TMEM of a row group (256 columns each): er hi [0,32), er lo [32,64), the accumulator
// [64,192)
constexpr uint32_t kTmemGroup = 256, kTmemAcc = 64;

struct Cfg {
  static constexpr int kOffLR = 0;                          // [group][l, r] rows
  static constexpr int kOffW = kOffLR + 2 * 2 * kRowBytes;  // [stage][hi, lo]
  static constexpr int kOffOut = kOffW + kWStages * 2 * kWBytes;
  static constexpr int kOffBar = kOffOut + 8 * kOutBytes;
  static constexpr int kSmemBytes = 1024 + kOffBar + 512;
  static_assert(kSmemBytes <= 232448, "shared memory");
};

struct Params {
  int rows, folds, tiles_m, num_tiles;
  int shift_min;
};

__global__ void __launch_bounds__(kThreads, 1)
    tucker_layer_kernel(const Params p, const __grid_constant__ CUtensorMap tmap_l,
                        const __grid_constant__ CUtensorMap tmap_r, const __grid_constant__ CUtensorMap tmap_w,
                        const __grid_constant__ CUtensorMap tmap_y) {
  using C = Cfg;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  const uint32_t smem_base = smem_u32(smem);
  uint64_t* bars = (uint64_t*)(smem + C::kOffBar);
  uint64_t* lr_full = bars;                // [group]
  uint64_t* lr_empty = lr_full + 2;        // [group]
  uint64_t* w_full = lr_empty + 2;         // [kWStages]
  uint64_t* w_ready = w_full + kWStages;   // [kWStages]
  uint64_t* w_empty = w_ready + kWStages;  // [kWStages]
  uint64_t* a_ready = w_empty + kWStages;  // [group]
  uint64_t* acc_full = a_ready + 2;        // [group]
  uint64_t* acc_empty = acc_full + 2;      // [group]
  uint64_t* drain = acc_empty + 2;
  uint32_t* tmem_slot = (uint32_t*)(drain + 1);
  volatile int* abort_flag = (volatile int*)(tmem_slot + 1);
  // the barriers the producer armed, drained at wind-down after an abort
  ArmedCopies* lr_copies = (ArmedCopies*)(tmem_slot + 2);
  ArmedCopies* w_copies = lr_copies + 1;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int g = 0; g < 2; ++g) {
      mbar_init(&lr_full[g], 1);
      mbar_init(&lr_empty[g], 128);
      mbar_init(&a_ready[g], 4);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], 4);
    }
    for (int s = 0; s < kWStages; ++s) {
      mbar_init(&w_full[s], 1);
      mbar_init(&w_ready[s], 4);
      mbar_init(&w_empty[s], 1);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    *lr_copies = *w_copies = ArmedCopies{0u, 0u};
    fence_mbarrier_init();
  }
  if (warp == kMmaWarp) tmem_alloc<512>(tmem_slot);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const bool is_min = p.shift_min != 0;
  // tiles [first, last) of this CTA, contiguous; local tile n belongs to group n & 1
  const int first = (int)(((int64_t)p.num_tiles * blockIdx.x) / gridDim.x);
  const int last = (int)(((int64_t)p.num_tiles * (blockIdx.x + 1)) / gridDim.x);
  const int count = last - first;

  if (warp < 8) {
    // ------------------------------------------------------------ rows: scan, A operand, epilogue
    const int group = warp >> 2;
    const int q = warp & 3;
    const int r = q * 32 + lane;
    const uint32_t lane_bits = (uint32_t)(q * 32) << 16;
    const uint32_t tg = tmem + group * kTmemGroup;
    const uint32_t out_buf = smem_base + C::kOffOut + warp * kOutBytes;
    const uint32_t yrow = out_buf + lane * 128;
    uint32_t gc = 0;  // this group's chunk count
    bool ok = true;
    for (int n = group, j = 0; n < count && ok; n += 2, ++j) {
      const int tile = first + n;
      const int f = tile / p.tiles_m;
      const int mt = tile - f * p.tiles_m;
      const bool valid = mt * kBM + r < p.rows;
      if (!mbar_wait_warp(&lr_full[group], j & 1, kSiteAStaged, abort_flag)) break;
      XE_CP_TRACE(r == 0 ? n : 1 << 20, 0);
      float lv[kDim], rv[kDim];
      const uint32_t lrow = smem_base + C::kOffLR + group * 2 * kRowBytes + r * 128;
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        const float4 a = lds_v4(lrow + ((c ^ (r & 7)) << 4));
        const float4 b = lds_v4(lrow + kRowBytes + ((c ^ (r & 7)) << 4));
        lv[4 * c] = a.x, lv[4 * c + 1] = a.y, lv[4 * c + 2] = a.z, lv[4 * c + 3] = a.w;
        rv[4 * c] = b.x, rv[4 * c + 1] = b.y, rv[4 * c + 2] = b.z, rv[4 * c + 3] = b.w;
      }
      float sl = is_min ? INFINITY : -INFINITY, sr = sl;
#pragma unroll
      for (int k = 0; k < kDim; ++k) {
        sl = extreme(sl, lv[k], is_min);
        sr = extreme(sr, rv[k], is_min);
      }
      mbar_arrive(&lr_empty[group]);  // every value has been used
      sl = valid ? sl : 0.0f;
      sr = valid ? sr : 0.0f;
      float el[kDim];
#pragma unroll
      for (int k = 0; k < kDim; ++k) el[k] = valid ? exp_shifted(lv[k], sl) : 0.0f;
      // A operand: er hi / lo (the group's previous tile's products are done: its chunks
      // were drained)
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        float hi[16], lo[16];
#pragma unroll
        for (int k = 0; k < 16; ++k) split_rn(valid ? exp_shifted(rv[16 * h + k], sr) : 0.0f, hi[k], lo[k]);
        tmem_st16(tg + lane_bits + 16 * h, hi);
        tmem_st16(tg + lane_bits + 32 + 16 * h, lo);
      }
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&a_ready[group]);
      // -------- chunks: y[o] = sum_i el[i] T[(o,i)] for the chunk's two o, written to this
      // thread's row of the warp's staging buffer (its previous store has read it)
      if (lane == 0) cp::bulk_wait_read();
      __syncwarp();
#pragma unroll 1
      for (int c = 0; c < kChunks; ++c, ++gc) {
        if (!mbar_wait_warp(&acc_full[group], gc & 1, kSiteDrainChunk, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        float y[4];
#pragma unroll
        for (int h = 0; h < 2; ++h) {  // two o at a time
          float t0[kDim], t1[kDim];
          tmem_ld32(tg + lane_bits + kTmemAcc + 64 * h, t0);
          tmem_ld32(tg + lane_bits + kTmemAcc + 64 * h + kDim, t1);
          tmem_wait_ld();
          if (h == 1) {  // the accumulator has been read
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&acc_empty[group]);
          }
          float a0 = 0.0f, a1 = 0.0f, a2 = 0.0f, a3 = 0.0f, b0 = 0.0f, b1 = 0.0f, b2 = 0.0f, b3 = 0.0f;
#pragma unroll
          for (int i = 0; i < kDim; i += 4) {
            a0 = fmaf(el[i], t0[i], a0);
            a1 = fmaf(el[i + 1], t0[i + 1], a1);
            a2 = fmaf(el[i + 2], t0[i + 2], a2);
            a3 = fmaf(el[i + 3], t0[i + 3], a3);
            b0 = fmaf(el[i], t1[i], b0);
            b1 = fmaf(el[i + 1], t1[i + 1], b1);
            b2 = fmaf(el[i + 2], t1[i + 2], b2);
            b3 = fmaf(el[i + 3], t1[i + 3], b3);
          }
          y[2 * h] = (a0 + a1) + (a2 + a3);
          y[2 * h + 1] = (b0 + b1) + (b2 + b3);
        }
        // columns 4c .. 4c+3: the 16-byte chunk c (swizzled by the row)
        sts_v4(yrow + ((c ^ (lane & 7)) << 4), make_float4(y[0], y[1], y[2], y[3]));
      }
      if (!ok) break;
      XE_CP_TRACE(r == 0 ? n : 1 << 20, 1);
      // -------- log + shifts in place, then the TMA store of the warp's 32 rows
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        const uint32_t a = yrow + ((c ^ (lane & 7)) << 4);
        const float4 v = lds_v4(a);
        sts_v4(a, make_float4(fast_log(v.x) + sl + sr, fast_log(v.y) + sl + sr, fast_log(v.z) + sl + sr,
                              fast_log(v.w) + sl + sr));
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        cp::tma_store_3d(&tmap_y, out_buf, 0, f, mt * kBM + q * 32);
        cp::bulk_commit();
      }
    }
    if (lane == 0) cp::bulk_wait_all();
    __syncwarp();
  } else if (warp < kMmaWarp) {
    // ------------------------------------------------------------ weight chunks: TF32 hi / lo
    const int tt = threadIdx.x - kLoWarp0 * 32;  // 0..127
    const int total = count * kChunks;           // every tile's chunks, in ring order
    for (int gw = 0; gw < total; ++gw) {
      const uint32_t s = gw % kWStages;
      if (!mbar_wait_warp(&w_full[s], (gw / kWStages) & 1, kSiteAStage, abort_flag)) break;
      if (tt == 0 && (gw % (2 * kChunks) == 0 || gw % (2 * kChunks) == 16)) XE_CP_TRACE(2 * (gw / (2 * kChunks)), gw % (2 * kChunks) == 0 ? 6 : 7);
      const uint32_t hi = smem_base + C::kOffW + s * 2 * kWBytes, lo = hi + kWBytes;
#pragma unroll
      for (int k = 0; k < kWBytes / 16 / 128; ++k) {  // 8 chunks of 16 bytes per thread
        const uint32_t off = (uint32_t)(tt + 128 * k) * 16;
        const float4 v = lds_v4(hi + off);
        float4 h, l;
        split_rn(v.x, h.x, l.x);
        split_rn(v.y, h.y, l.y);
        split_rn(v.z, h.z, l.z);
        split_rn(v.w, h.w, l.w);
        sts_v4(hi + off, h);
        sts_v4(lo + off, l);
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&w_ready[s]);
    }
  } else if (warp == kMmaWarp) {
    // ------------------------------------------------------------ MMA issue
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_tf32(kBM, kChunkN, false, false);
      uint32_t gw = 0;           // weight chunks, in ring order
      uint32_t gcg[2] = {0, 0};  // chunks per group
      bool ok = true;
      for (int n0 = 0, j = 0; n0 < count && ok; n0 += 2, ++j) {
        const int groups = n0 + 1 < count ? 2 : 1;
        for (int g = 0; g < groups && ok; ++g)
          if (!mbar_wait(&a_ready[g], j & 1, kSiteMmaFull, abort_flag)) ok = false;
        tc_fence_after();
        for (int c = 0; c < kChunks && ok; ++c) {
          for (int g = 0; g < groups; ++g, ++gw) {
            const uint32_t s = gw % kWStages;
            if (!mbar_wait(&w_ready[s], (gw / kWStages) & 1, kSiteMmaFull, abort_flag) ||
                !mbar_wait(&acc_empty[g], (gcg[g] & 1) ^ 1, kSiteMmaChunk, abort_flag)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t tg = tmem + g * kTmemGroup;
            const uint32_t d = tg + kTmemAcc;
            const uint32_t b_hi = smem_base + C::kOffW + s * 2 * kWBytes, b_lo = b_hi + kWBytes;
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
              const uint64_t dbh = smem_desc(b_hi + kk * 32, 16, 1024, kLayoutSW128);
              const uint64_t dbl = smem_desc(b_lo + kk * 32, 16, 1024, kLayoutSW128);
              umma_tf32_ts(d, tg + kk * 8, dbh, idesc, kk != 0);
              umma_tf32_ts(d, tg + kk * 8, dbl, idesc, 1);
              umma_tf32_ts(d, tg + 32 + kk * 8, dbh, idesc, 1);
            }
            umma_commit(&acc_full[g]);
            umma_commit(&w_empty[s]);
            if (c == 0 || c == 8) XE_CP_TRACE(n0 + g, c == 0 ? 2 : 3);
            ++gcg[g];
          }
        }
      }
      umma_commit(drain);
      mbar_wait(drain, 0, kSiteGemmDrain, abort_flag, /*honor_abort=*/false);
    }
    __syncwarp();
  } else if (lane == 0) {
    // ------------------------------------------------------------ TMA loads
    // The weight chunks in a ring, in the MMA warp's order; the l and r rows of a group's
    // next tile (one slot per group, freed once the group has read its current rows) after
    // the weight chunks of the current pair.
    auto load_lr = [&](int n, int j) -> bool {
      const int tile = first + n;
      const int f = tile / p.tiles_m;
      const int mt = tile - f * p.tiles_m;
      const int g = n & 1;
      if (!mbar_wait(&lr_empty[g], (j & 1) ^ 1, kSiteProducer, abort_flag)) return false;
      const uint32_t dst = smem_base + C::kOffLR + g * 2 * kRowBytes;
      mbar_expect_tx(&lr_full[g], 2 * kRowBytes);
      lr_copies->note(g, j);
      tma_load_3d(dst, &tmap_l, 0, f, mt * kBM, &lr_full[g]);
      tma_load_3d(dst + kRowBytes, &tmap_r, 0, f, mt * kBM, &lr_full[g]);
      return true;
    };
    bool ok = true;
    for (int n = 0; n < 2 && n < count && ok; ++n) ok = load_lr(n, 0);
    uint32_t gw = 0;
    for (int n0 = 0, j = 0; n0 < count && ok; n0 += 2, ++j) {
      const int groups = n0 + 1 < count ? 2 : 1;
      for (int c = 0; c < kChunks && ok; ++c) {
        for (int g = 0; g < groups; ++g, ++gw) {
          const uint32_t s = gw % kWStages;
          if (!mbar_wait(&w_empty[s], ((gw / kWStages) & 1) ^ 1, kSiteProducer, abort_flag)) {
            ok = false;
            break;
          }
          const int f = (first + n0 + g) / p.tiles_m;
          if (c == 0 || c == 8) XE_CP_TRACE(n0 + g, c == 0 ? 4 : 5);
          mbar_expect_tx(&w_full[s], kWBytes);
          w_copies->note(s, gw / kWStages);
          tma_load_3d(smem_base + C::kOffW + s * 2 * kWBytes, &tmap_w, 0, c * kChunkN, f, &w_full[s]);
        }
      }
      for (int n = n0 + 2; n < n0 + 4 && n < count && ok; ++n) ok = load_lr(n, j + 1);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (*abort_flag) {  // uniform: every thread has passed its last wait
    lr_copies->drain(lr_full, abort_flag);
    w_copies->drain(w_full, abort_flag);
    __syncthreads();
  }
  tc_fence_after();
  if (warp == kMmaWarp) tmem_dealloc<512>(tmem);
}

}  // namespace tk
}  // namespace xe
