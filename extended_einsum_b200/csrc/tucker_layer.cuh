// tucker_layer.cuh — the log-space Tucker layer 'bfi,bfj,foij->bfo' with I = J = O = 32.
//
// y[b,f,o] = log( sum_ij exp(l[b,f,i]-sl) exp(r[b,f,j]-sr) w[f,o,i,j] ) + sl + sr,
// the ternary einsum that OptimizeContractionPaths fuses for Tucker circuits
// (preprocess.py:1095-1106), lowered by _append_logspace_einsum
// (translate.py:686-750), with sl / sr the max (or min) of l / r over i / j and
// w linear (a softmax of the layer's logits).  The contraction runs in two
// stages, j first (the path torch.einsum takes for the three operands):
//
//   T[b,(o,i)] = sum_j er[b,j] w[f,o,i,j]     tensor cores: M = 128 rows b, N = 64
//                                             (two o) per chunk, K = 32 j, split-TF32
//                                             (hi*hi main, hi*lo + lo*hi correction)
//   y[b,o]     = sum_i el[b,i] T[b,(o,i)]     fp32 FMAs in the epilogue
//
// with el = exp(l - sl), er = exp(r - sr).  That is half the tensor work of the
// fused (i,j) product, and the A operand (er) is 32 values per row instead of
// 1024.  Per 128-row tile of fold f the weights w[f] stream through shared memory
// in 16 chunks of 64 (o,i) rows x 32 j.
//
// Warps 0-3: rows (scan, exp, A operand, epilogue); warps 4-7: TF32 split of
// the weight chunks; warp 8: TMEM allocation and MMA issue; warp 9: TMA loads.
#pragma once

#include "lse_gemm.cuh"

namespace xe {
namespace tk {

using namespace gemm;
constexpr int kDim = 32;          // I = J = O
constexpr int kChunkN = 64;       // (o,i) rows per chunk: two o
constexpr int kChunks = kDim * kDim / kChunkN;  // 16 per tile
constexpr int kThreads = 320;
constexpr int kLoWarp0 = 4, kMmaWarp = 8, kProducerWarp = 9;
constexpr int kRowBytes = kBM * kDim * 4;      // 16 KB: 128 rows x 32, 128-byte swizzle
constexpr int kWBytes = kChunkN * kDim * 4;    // 8 KB: 64 (o,i) rows x 32 j
constexpr int kWStages = 4;
constexpr int kOutBytes = 32 * kDim * 4;       // per row warp: 32 rows x 32 o
// TMEM: er hi [0,32), er lo [32,64); accumulators per buffer: main 64 + correction 64
constexpr uint32_t kTmemAcc = 64, kTmemAccStride = 128;

struct Cfg {
  static constexpr int kOffLR = 0;                           // [2 slots][l, r] rows
  static constexpr int kOffW = kOffLR + 2 * 2 * kRowBytes;   // [stage][hi, lo]
  static constexpr int kOffOut = kOffW + kWStages * 2 * kWBytes;
  static constexpr int kOffBar = kOffOut + 4 * kOutBytes;
  static constexpr int kSmemBytes = 1024 + kOffBar + 512;
  static_assert(kSmemBytes <= 232448, "shared memory");
};

struct Params {
  int rows, folds, tiles_m, num_tiles;
  int shift_min;
};

__device__ __forceinline__ void tma_store_3d(const CUtensorMap* map, uint32_t src, int x, int y, int z) {
  asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.tile.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(map),
               "r"(src), "r"(x), "r"(y), "r"(z)
               : "memory");
}

__global__ void __launch_bounds__(kThreads, 1)
    tucker_layer_kernel(const Params p, const __grid_constant__ CUtensorMap tmap_l,
                        const __grid_constant__ CUtensorMap tmap_r, const __grid_constant__ CUtensorMap tmap_w,
                        const __grid_constant__ CUtensorMap tmap_y) {
  using C = Cfg;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  const uint32_t smem_base = smem_u32(smem);
  uint64_t* bars = (uint64_t*)(smem + C::kOffBar);
  uint64_t* lr_full = bars;              // [2]
  uint64_t* lr_empty = lr_full + 2;      // [2]
  uint64_t* w_full = lr_empty + 2;       // [kWStages]
  uint64_t* w_ready = w_full + kWStages;   // [kWStages]
  uint64_t* w_empty = w_ready + kWStages;  // [kWStages]
  uint64_t* a_ready = w_empty + kWStages;
  uint64_t* acc_full = a_ready + 1;      // [2]
  uint64_t* acc_empty = acc_full + 2;    // [2]
  uint64_t* drain = acc_empty + 2;
  uint32_t* tmem_slot = (uint32_t*)(drain + 1);
  volatile int* abort_flag = (volatile int*)(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&lr_full[i], 1);
      mbar_init(&lr_empty[i], 128);
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], 4);
    }
    for (int s = 0; s < kWStages; ++s) {
      mbar_init(&w_full[s], 1);
      mbar_init(&w_ready[s], 4);
      mbar_init(&w_empty[s], 1);
    }
    mbar_init(a_ready, 4);
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbarrier_init();
  }
  if (warp == kMmaWarp) tmem_alloc<512>(tmem_slot);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const bool is_min = p.shift_min != 0;

  if (warp < kLoWarp0) {
    // ------------------------------------------------------------ rows: scan, A operand, epilogue
    const int q = warp;
    const int r = q * 32 + lane;
    const uint32_t lane_bits = (uint32_t)(q * 32) << 16;
    const uint32_t out_buf = smem_base + C::kOffOut + q * kOutBytes;
    uint32_t t = 0, gc = 0;
    bool ok = true;
    for (int tile = blockIdx.x; tile < p.num_tiles && ok; tile += gridDim.x, ++t) {
      const int f = tile / p.tiles_m;
      const int mt = tile - f * p.tiles_m;
      const bool valid = mt * kBM + r < p.rows;
      const int slot = t & 1;
      if (!mbar_wait(&lr_full[slot], (t >> 1) & 1, kSiteAStaged, abort_flag)) break;
      float lv[kDim], rv[kDim];
      const uint32_t lrow = smem_base + C::kOffLR + slot * 2 * kRowBytes + r * 128;
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
      mbar_arrive(&lr_empty[slot]);  // every value has been used
      sl = valid ? sl : 0.0f;
      sr = valid ? sr : 0.0f;
      float el[kDim];
#pragma unroll
      for (int k = 0; k < kDim; ++k) el[k] = valid ? exp_shifted(lv[k], sl) : 0.0f;
      // A operand: er hi / lo (the previous tile's products are done: its chunks were drained)
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        float hi[16], lo[16];
#pragma unroll
        for (int k = 0; k < 16; ++k) split_rn(valid ? exp_shifted(rv[16 * h + k], sr) : 0.0f, hi[k], lo[k]);
        tmem_st16(tmem + lane_bits + 16 * h, hi);
        tmem_st16(tmem + lane_bits + 32 + 16 * h, lo);
      }
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(a_ready);
      // -------- chunks: y[o] = sum_i el[i] T[(o,i)] for the chunk's two o
      float y[kDim];
#pragma unroll
      for (int c = 0; c < kChunks; ++c, ++gc) {
        const uint32_t buf = gc & 1;
        if (!mbar_wait_warp(&acc_full[buf], (gc >> 1) & 1, kSiteDrainChunk, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t acc = tmem + lane_bits + kTmemAcc + buf * kTmemAccStride;
#pragma unroll
        for (int oo = 0; oo < 2; ++oo) {
          float v[kDim], w[kDim];
          tmem_ld16(acc + kDim * oo, v);
          tmem_ld16(acc + kDim * oo + 16, v + 16);
          tmem_ld16(acc + 64 + kDim * oo, w);
          tmem_ld16(acc + 64 + kDim * oo + 16, w + 16);
          tmem_wait_ld();
          if (oo == 1) {  // the buffer has been read
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&acc_empty[buf]);
          }
          float s = 0.0f;
#pragma unroll
          for (int i = 0; i < kDim; ++i) {
            // an overflowed main term carries the result; its correction is NaN
            const float tv = isinf(v[i]) ? v[i] : v[i] + w[i];
            s = fmaf(el[i], tv, s);
          }
          y[2 * c + oo] = s;
        }
      }
      if (!ok) break;
      // -------- log + shifts, staged per warp and stored by TMA
#pragma unroll
      for (int o = 0; o < kDim; ++o) y[o] = fast_log(y[o]) + sl + sr;
      if (lane == 0) asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
      __syncwarp();
#pragma unroll
      for (int c = 0; c < 8; ++c)
        sts_v4(out_buf + lane * 128 + ((c ^ (lane & 7)) << 4), make_float4(y[4 * c], y[4 * c + 1], y[4 * c + 2], y[4 * c + 3]));
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        tma_store_3d(&tmap_y, out_buf, 0, f, mt * kBM + q * 32);
        asm volatile("cp.async.bulk.commit_group;" ::: "memory");
      }
    }
    if (lane == 0) asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
    __syncwarp();
  } else if (warp < kMmaWarp) {
    // ------------------------------------------------------------ weight chunks: TF32 hi / lo
    const int tt = threadIdx.x - kLoWarp0 * 32;  // 0..127
    uint32_t gc = 0;
    for (int tile = blockIdx.x; tile < p.num_tiles; tile += gridDim.x) {
      bool ok = true;
      for (int c = 0; c < kChunks; ++c, ++gc) {
        const uint32_t s = gc % kWStages;
        if (!mbar_wait(&w_full[s], (gc / kWStages) & 1, kSiteAStage, abort_flag)) {
          ok = false;
          break;
        }
        const uint32_t hi = smem_base + C::kOffW + s * 2 * kWBytes, lo = hi + kWBytes;
#pragma unroll
        for (int k = 0; k < kWBytes / 16 / 128; ++k) {  // 4 chunks of 16 bytes per thread
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
      if (!ok) break;
    }
  } else if (warp == kMmaWarp) {
    // ------------------------------------------------------------ MMA issue
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_tf32(kBM, kChunkN, false, false);
      uint32_t t = 0, gc = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < p.num_tiles && ok; tile += gridDim.x, ++t) {
        if (!mbar_wait(a_ready, t & 1, kSiteMmaFull, abort_flag)) break;
        tc_fence_after();
        for (int c = 0; c < kChunks; ++c, ++gc) {
          const uint32_t s = gc % kWStages, buf = gc & 1;
          if (!mbar_wait(&w_ready[s], (gc / kWStages) & 1, kSiteMmaFull, abort_flag) ||
              !mbar_wait(&acc_empty[buf], ((gc >> 1) & 1) ^ 1, kSiteMmaChunk, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t d_main = tmem + kTmemAcc + buf * kTmemAccStride, d_corr = d_main + 64;
          const uint32_t b_hi = smem_base + C::kOffW + s * 2 * kWBytes, b_lo = b_hi + kWBytes;
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            const uint64_t dbh = smem_desc(b_hi + kk * 32, 16, 1024, kLayoutSW128);
            const uint64_t dbl = smem_desc(b_lo + kk * 32, 16, 1024, kLayoutSW128);
            umma_tf32_ts(d_main, tmem + kk * 8, dbh, idesc, kk != 0);
            umma_tf32_ts(d_corr, tmem + kk * 8, dbl, idesc, kk != 0);
            umma_tf32_ts(d_corr, tmem + 32 + kk * 8, dbh, idesc, 1);
          }
          umma_commit(&acc_full[buf]);
          umma_commit(&w_empty[s]);
        }
      }
      umma_commit(drain);
      mbar_wait(drain, 0, kSiteGemmDrain, abort_flag, /*honor_abort=*/false);
    }
    __syncwarp();
  } else if (lane == 0) {
    // ------------------------------------------------------------ TMA loads
    // l and r rows of a tile one tile ahead (two slots), the weight chunks in a ring
    auto load_lr = [&](int tile, uint32_t t) -> bool {
      const int f = tile / p.tiles_m;
      const int mt = tile - f * p.tiles_m;
      const int slot = t & 1;
      if (!mbar_wait(&lr_empty[slot], ((t >> 1) & 1) ^ 1, kSiteProducer, abort_flag)) return false;
      const uint32_t dst = smem_base + C::kOffLR + slot * 2 * kRowBytes;
      mbar_expect_tx(&lr_full[slot], 2 * kRowBytes);
      tma_load_3d(dst, &tmap_l, 0, f, mt * kBM, &lr_full[slot]);
      tma_load_3d(dst + kRowBytes, &tmap_r, 0, f, mt * kBM, &lr_full[slot]);
      return true;
    };
    uint32_t t = 0, gc = 0;
    bool ok = (int)blockIdx.x >= p.num_tiles || load_lr(blockIdx.x, 0);
    for (int tile = blockIdx.x; tile < p.num_tiles && ok; tile += gridDim.x, ++t) {
      if (tile + (int)gridDim.x < p.num_tiles && !load_lr(tile + gridDim.x, t + 1)) break;
      const int f = tile / p.tiles_m;
      for (int c = 0; c < kChunks; ++c, ++gc) {
        const uint32_t s = gc % kWStages;
        if (!mbar_wait(&w_empty[s], ((gc / kWStages) & 1) ^ 1, kSiteProducer, abort_flag)) {
          ok = false;
          break;
        }
        mbar_expect_tx(&w_full[s], kWBytes);
        tma_load_3d(smem_base + C::kOffW + s * 2 * kWBytes, &tmap_w, 0, c * kChunkN, f, &w_full[s]);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == kMmaWarp) tmem_dealloc<512>(tmem);
}

}  // namespace tk
}  // namespace xe
