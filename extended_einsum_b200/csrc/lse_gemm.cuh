// Log-space batched contraction on the sm_100a tensor cores.
//
//   C[b,m,n] = log( sum_k exp(A[b,m,k]-sA[b,m]) * exp(B[b,k,n]-sB[b,n]) ) + sA[b,m] + sB[b,n]
//
// This is the arithmetic that _append_logspace_einsum
// (backend_translation/translate.py:686-750) spreads over ~16 backend calls
// for a binary contraction, fused into one persistent kernel.  Roles (warps):
//
//   A rows (0-3)       one thread per tile row: raw fp32 (from a TMA-filled
//                      staging ring, or global loads) -> exp(x - shift) (or
//                      the linear value, or the Tucker outer product) -> TF32
//                      hi/lo split -> tcgen05.st into a TMEM stage
//   B tiles (4-7)      global fp32 -> exp / split -> 128B-swizzled smem stage
//   MMA (8, 1 thread)  per 8-wide k-step: main += A_hi*B_hi,
//                      corr += A_hi*B_lo + A_lo*B_hi  (tcgen05.mma, A in TMEM)
//   drain (9-12)       one thread per row: adds each finished main-accumulator
//                      chunk into an fp32 running sum in smem (round to
//                      nearest), then log(running + corr) + shifts -> global
//   producer (13)      one thread: TMA loads of the raw A tiles (and of the
//                      fused addend) into the staging ring of this CTA alone
//
// The tensor core accumulates in fp32 with truncation, a bias that grows
// linearly with the number of accumulating instructions; the main
// accumulator is therefore restarted every kChunkKB k-blocks (two chunk
// buffers, so the MMA continues while the previous chunk is drained).  The
// correction products are ~2^-10 of the main ones and accumulate over the
// whole tile.  Row shifts reach the drain warps through shared memory.
// Stages, chunks and shift slots are handed over with mbarriers; every wait
// is bounded (xe_common.cuh).
#pragma once

#include <cuda.h>

#include "xe_common.cuh"

namespace xe {
namespace gemm {

constexpr int kBM = 128;  // UMMA M (cta_group::1) = TMEM lanes
constexpr int kBK = 32;   // k per stage
constexpr int kAWarps = 4;
constexpr int kBWarps = 4;
constexpr int kMmaWarp = kAWarps + kBWarps;  // 8
// With prepared B the B warps idle, and one of them issues the correction products
// (hi*lo + lo*hi, their own accumulator) beside the MMA warp's main products, so that the
// tensor pipe is fed from two instruction streams.
constexpr int kCorrMmaWarp = kAWarps + 1;  // 5
constexpr int kDrainWarp0 = kMmaWarp + 1;    // 9..12
constexpr int kDrainWarps = 4;
constexpr int kProducerWarp = kDrainWarp0 + kDrainWarps;  // 13
constexpr int kThreads = (kProducerWarp + 1) * 32;        // 448
constexpr int kStages = 2;
constexpr int kChunkKB = 8;  // 256 k per main-accumulator chunk
constexpr int kATileBytes = kBM * kBK * 4;  // one raw A tile (16 KB)

enum AMode : int { kALog = 0, kALinear = 1, kATucker = 2 };
// What one MMA-issuing thread issues (see mma_issue in lse_gemm_kernel).
enum MmaRole : int { kMmaAll = 0, kMmaMain = 1, kMmaCorr = 2 };
// Where the A rows come from: a TMA-filled staging ring (K-major A with
// 16-byte aligned strides), the same plus a second ring for the fused addend,
// or per-thread global loads (any layout).
// kAGather: the A rows are gathered rows of a table (Params::g_pixels), staged in
// the same swizzled ring by TMA tile::gather4 loads (four table rows each).
// kAGather2: two gathered rows per A row (folds bb and bb + Params::g_pair of the
// table), staged like the kATma2 pair and added by the A warps.
enum ASource : int { kATma = 0, kATma2 = 1, kALdg = 2, kAGather = 3, kAGather2 = 4 };

__host__ __device__ constexpr bool a_pair(int asrc) { return asrc == kATma2 || asrc == kAGather2; }
__host__ __device__ constexpr bool a_gathered(int asrc) { return asrc == kAGather || asrc == kAGather2; }
// Where the raw B tiles come from: a TMA-filled staging ring (16-byte aligned
// strides), or global loads with or without 16-byte vectors.  kBPlanes: B was
// prepared by b_planes_kernel (exp'd, split into TF32 hi / lo, laid out as the
// MMA's K-major stages), and each stage arrives by one bulk copy; the B warps idle.
enum BSource : int { kBTma = 0, kBLdgVec = 1, kBLdg = 2, kBPlanes = 3 };

struct Params {
  const float* a;
  const float* a2;
  int64_t a_sb, a_sm, a_sk;
  const float* b;
  int64_t b_sb, b_sk, b_sn;
  float* c;
  int64_t c_sb, c_sm, c_sn;
  const float* shift_a;  // [batch*M] (log A with K > kInlineShiftK); else nullptr
  const float* shift_b;  // [batch*N] for a log-domain B; nullptr when B is linear
  const float* b_planes;  // kBPlanes: the prepared B, one kPlaneBlockBytes block per (bb, nt, kb)
  // element strides of the shift vectors: shift_a[bb * sa_sb + m * sa_sm], shift_b[bb * sb_sb + n * sb_sn]
  // ((M, 1) and (N, 1) for one shift per row / column; a stride 0 repeats one value)
  int64_t sa_sb, sa_sm, sb_sb, sb_sn;
  int batch, M, N, K;
  int tiles_m, tiles_n, num_tiles, num_kb;
  int c_vec;      // output rows may be written with 16-byte stores
  int a_vec;      // LDG source: rows are k-contiguous and 16-byte aligned
  int shift_min;  // row extremes computed in-kernel use min instead of max
  int raw_out;    // write the plain sums (linear operands, scaled modes) instead of log + shifts
  // A rows gathered from a (folds, states, K) table by uint8 pixels (categorical input units
  // feeding a sum layer): row (bb, m) = a + bb * a_sb + pixels[m * g_stride + var[bb]] * a_sm
  const uint8_t* g_pixels;
  const int32_t* g_var;  // nullptr: variable bb
  int64_t g_stride;
  int g_states;
  // > 0: the row gathered from fold bb + g_pair (its variable var[bb + g_pair]) is added
  // (the Hadamard product of two input units feeding the sum layer)
  int64_t g_pair;
  // Tucker layer: l (rows, folds, I), r (rows, folds, J) contiguous; batch = fold
  const float* tl;
  const float* tr;
  int t_folds, t_i;
  int64_t t_l_sb, t_l_sf, t_r_sb, t_r_sf;  // element strides of l and r over (batch row, fold); units contiguous
};

__host__ __device__ constexpr int pow2_at_least(int x) {
  int p = 32;
  while (p < x) p <<= 1;
  return p;
}

template <int BN, int ASRC, int BSRC>
struct Cfg {
  static_assert(BN == 32 || BN == 64 || BN == 128, "BN");
  static constexpr int kSmemLimit = 232448;
  static constexpr int kBTile = BN * kBK * 4;  // bytes, one of hi/lo (also one raw B tile)
  static constexpr int kStageBytes = 2 * kBTile;
  // B stages in shared memory: with prepared B they are filled by bulk copies and run deeper
  // than the two TMEM A stages (the copies' latency is hidden by the ring alone)
  static constexpr int kBStages = BSRC == kBPlanes ? (a_pair(ASRC) ? 2 : 3) : kStages;
  // the running sum of the accumulation chunks before the last; gathered sources have
  // K <= 128 (one chunk) and need none
  static constexpr int kRunningBytes = a_gathered(ASRC) ? 0 : BN * kBM * 4;
  static constexpr int kShiftBytes = 2 * 2 * kBM * 4;  // [slot][s1,s2][row]
  // Tiles of at most 64 columns have little tensor work per tile and are
  // bound by the epilogue: two drain warp groups take alternate tiles
  // (warps 14..17 join 9..12; each group owns one staging buffer).
  static constexpr int kDrainGroups = BN <= 64 ? 2 : 1;
  static constexpr int kThreads = (kProducerWarp + 1 + 4 * (kDrainGroups - 1)) * 32;
  static constexpr int kColShiftBytes = 4 * kDrainGroups * BN * 4;  // [drain warp][BN]
  static constexpr int kOutBytes = kBM * 32 * 4;       // one [128 rows][32 cols] output staging buffer
  static constexpr int kAStageBytes = a_pair(ASRC) ? 2 * kATileBytes : kATileBytes;
  // everything except the two TMA rings and the output staging
  static constexpr int kFixed = 1024 + kBStages * kStageBytes + kRunningBytes + kShiftBytes + kColShiftBytes + 512;
  static constexpr int kBRawBytes = BSRC == kBTma ? kBTile : 0;
  static constexpr int kMinRings = (ASRC == kALdg ? 0 : 2 * kAStageBytes) + 2 * kBRawBytes;
  // With a running-sum buffer and one drain group, each warp stages its output rows in place, in
  // its own rows' part of the running sums of the slice it copies out (no separate buffer).
  static constexpr bool kStageInPlace = kRunningBytes > 0 && kDrainGroups == 1;
  static constexpr int kOutBufs =
      kStageInPlace ? 0 : (kDrainGroups == 2 || kFixed + kMinRings + 2 * kOutBytes <= kSmemLimit) ? 2 : 1;
  static constexpr int kRingBudget = kSmemLimit - kFixed - kOutBufs * kOutBytes - 1024;
  // up to four stages per ring, A first
  static constexpr int kAStages =
      ASRC == kALdg ? 0
                    : ((kRingBudget - 2 * kBRawBytes) / kAStageBytes >= 4 ? 4 : (kRingBudget - 2 * kBRawBytes) / kAStageBytes);
  static constexpr int kBRawStages =
      BSRC != kBTma ? 0 : ((kRingBudget - kAStages * kAStageBytes) / kBRawBytes >= 4 ? 4 : (kRingBudget - kAStages * kAStageBytes) / kBRawBytes);
  // TMEM columns: A stages (hi 32 + lo 32 each), two main chunks, correction
  static constexpr int kTmemA = 0;
  static constexpr int kTmemMain = 64 * kStages;
  static constexpr int kTmemCorr = kTmemMain + 2 * BN;
  // two correction accumulators (the next tile's MMAs need not wait for this
  // tile's epilogue) where TMEM has room: BN <= 64
  static constexpr int kCorrBufs = kTmemCorr + 2 * BN <= 512 ? 2 : 1;
  static constexpr int kTmemCols = pow2_at_least(kTmemCorr + kCorrBufs * BN);
  static constexpr int kOffB = 0;
  static constexpr int kOffA = kOffB + kBStages * kStageBytes;
  static constexpr int kOffBRaw = kOffA + kAStages * kAStageBytes;
  static constexpr int kOffRun = kOffBRaw + kBRawStages * kBRawBytes;
  static constexpr int kOffShift = kOffRun + kRunningBytes;
  static constexpr int kOffColShift = kOffShift + kShiftBytes;
  static constexpr int kOffOutAligned = (kOffColShift + kColShiftBytes + 1023) / 1024 * 1024;
  static constexpr int kOffBar = kOffOutAligned + kOutBufs * kOutBytes;
  static constexpr int kSmemBytes = 1024 + kOffBar + 512;
  static_assert(kTmemCorr + kCorrBufs * BN <= 512, "TMEM");
  // whether this combination fits (both rings at least double-buffered)
  static constexpr bool kFits = (ASRC == kALdg || kAStages >= 2) && (BSRC != kBTma || kBRawStages >= 2) &&
                                kSmemBytes <= kSmemLimit;
};

// Byte offset of the 16-byte chunk holding elements (row, 4q..4q+3) of a
// K-major tile (rows x 32 fp32, 128-byte rows, 8-row swizzle atoms).
__device__ __forceinline__ uint32_t kmajor_off(int row, int q) {
  return (uint32_t)((row >> 3) * 1024 + (row & 7) * 128 + ((q ^ (row & 7)) << 4));
}
// Byte offset of the 16-byte chunk holding elements (k, 4q..4q+3) of an
// MN-major tile (32 k-rows x MN): 32-element MN blocks every 4096 B, inside a
// block 4-row k-groups of 512 B, 32-byte chunks swizzled with (k & 3).
__device__ __forceinline__ uint32_t mnmajor_off(int k, int q) {
  return (uint32_t)((q >> 3) * 4096 + (k >> 2) * 512 + (k & 3) * 128 + ((((q >> 1) & 3) ^ (k & 3)) << 5) +
                    ((q & 1) << 4));
}

// exp(x - s) as 2^((x - s) * log2 e): x - s is exact for the terms that
// dominate a row (Sterbenz), the product adds one rounding, ex2.approx ~2 ulp.
__device__ __forceinline__ float exp_shifted(float x, float s) {
  const float y = (x - s) * 1.4426950408889634f;
  float e;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e) : "f"(y));
  return e;
}

// hi = e rounded to the nearest TF32 (10 explicit mantissa bits, ties away),
// lo = e - hi exactly; the tensor core reads lo's top 10 mantissa bits.
__device__ __forceinline__ void split_rn(float e, float& hi, float& lo) {
  hi = __uint_as_float((__float_as_uint(e) + 0x1000u) & 0xFFFFE000u);
  lo = e - hi;
}

__device__ __forceinline__ float4 ldg_v4(const float* p) {
  float4 v;
  asm volatile("ld.global.nc.v4.f32 {%0,%1,%2,%3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "l"(p));
  return v;
}

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const float (&v)[32]) {
  __syncwarp();  // .sync.aligned: the whole warp, converged
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "f"(v[0]), "f"(v[1]), "f"(v[2]), "f"(v[3]), "f"(v[4]), "f"(v[5]), "f"(v[6]), "f"(v[7]), "f"(v[8]), "f"(v[9]),
      "f"(v[10]), "f"(v[11]), "f"(v[12]), "f"(v[13]), "f"(v[14]), "f"(v[15]), "f"(v[16]), "f"(v[17]), "f"(v[18]),
      "f"(v[19]), "f"(v[20]), "f"(v[21]), "f"(v[22]), "f"(v[23]), "f"(v[24]), "f"(v[25]), "f"(v[26]), "f"(v[27]),
      "f"(v[28]), "f"(v[29]), "f"(v[30]), "f"(v[31])
      : "memory");
}

// 16 consecutive fp32 columns of the calling warp's 32 TMEM lanes.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float* v) {
  __syncwarp();  // .sync.aligned: the whole warp, converged
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void tmem_st16(uint32_t taddr, const float (&v)[16]) {
  __syncwarp();  // .sync.aligned: the whole warp, converged
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(
          taddr),
      "f"(v[0]), "f"(v[1]), "f"(v[2]), "f"(v[3]), "f"(v[4]), "f"(v[5]), "f"(v[6]), "f"(v[7]), "f"(v[8]), "f"(v[9]),
      "f"(v[10]), "f"(v[11]), "f"(v[12]), "f"(v[13]), "f"(v[14]), "f"(v[15])
      : "memory");
}

__device__ __forceinline__ void tmem_wait_st() {
  __syncwarp();
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// D[tmem] (+)= A[tmem] * B[smem], kind::tf32, one CTA.
__device__ __forceinline__ void umma_tf32_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                             uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// 3-D tiled TMA load into this CTA's shared memory, completing on an mbarrier.
__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap* map, int x, int y, int z, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(dst),
      "l"(map), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
      : "memory");
}

// Four rows (r0..r3, each one box of the 2-D tensor map: columns x .. x+31) gathered into
// four consecutive 128-byte rows of shared memory at dst, swizzled as the map says.
__device__ __forceinline__ void tma_gather4(uint32_t dst, const CUtensorMap* map, int x, int r0, int r1, int r2, int r3,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile::gather4.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4, %5, %6}], [%7];" ::"r"(dst),
      "l"(map), "r"(x), "r"(r0), "r"(r1), "r"(r2), "r"(r3), "r"(smem_u32(bar))
      : "memory");
}

// Contiguous bulk copy global -> shared memory (16-byte aligned addresses and size), completing
// on an mbarrier; this CTA's shared memory only.
__device__ __forceinline__ void bulk_load(uint32_t dst, const float* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
               "l"(src), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}

__device__ __forceinline__ float4 lds_v4(uint32_t addr) {
  float4 v;
  asm volatile("ld.shared.v4.f32 {%0,%1,%2,%3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "r"(addr));
  return v;
}

// log(x) = log2(x) * ln 2 (lg2.approx: absolute error ~2^-22 in log2).
__device__ __forceinline__ float fast_log(float x) {
  float y;
  asm("lg2.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y * 0.6931471805599453f;
}


__device__ __forceinline__ float extreme(float a, float b, bool is_min) {
  float r;
  if (is_min)
    asm("min.NaN.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
  else
    asm("max.NaN.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
  return r;
}

// Tile order within a batch entry: groups of kGroupM row tiles, the row tile fastest inside a
// group, so that the ~148 tiles in flight at once (one per CTA) share their A row blocks and B
// column tiles in L2 (about kGroupM CTAs read each B tile at the same time, instead of the one or
// two of a row-major order, which left a 32768-column B streaming from HBM once per CTA).
constexpr int kGroupM = 16;
__device__ __forceinline__ void decode_tile(const Params& p, int tile, int& bb, int& mt, int& nt) {
  const int per_batch = p.tiles_m * p.tiles_n;
  bb = tile / per_batch;
  const int t = tile - bb * per_batch;
  const int group = t / (kGroupM * p.tiles_n);
  const int m0 = group * kGroupM;
  const int gm = min(kGroupM, p.tiles_m - m0);  // the last group may hold fewer row tiles
  const int idx = t - group * kGroupM * p.tiles_n;
  mt = m0 + idx % gm;
  nt = idx / gm;
}

// ---------------------------------------------------------------------------
// A operand, one thread per tile row.

template <int AMODE, int TJ>
struct ARow {
  static constexpr int kTJ = TJ > 0 ? TJ : 1;
  const float* row = nullptr;   // element (m, 0) of this row (global-load source)
  const float* row2 = nullptr;  // fused addend
  int64_t step = 1;             // element stride along k
  bool valid = false;
  float shift = 0.0f;  // exp(x - shift): the row shift (sr for Tucker)
  // Tucker
  const float* lrow = nullptr;
  float sl = 0.0f;
  float er[kTJ];

  // Element offset of the table row that pixel (m, var[fold]) selects in fold `fold`.
  __device__ static int64_t gathered_row(const Params& p, int64_t fold, int m, bool valid) {
    int64_t v = p.g_var ? (int64_t)__ldg(p.g_var + fold) : fold;
    if (v < 0 || v >= p.g_stride) {
      record_bad_index(kSiteGemmGatherState);
      v = 0;
    }
    int64_t state = valid ? (int64_t)__ldg(p.g_pixels + (int64_t)m * p.g_stride + v) : 0;
    if (state >= p.g_states) {
      record_bad_index(kSiteGemmGatherState);
      state = p.g_states - 1;
    }
    return fold * p.a_sb + state * p.a_sm;
  }

  __device__ void set_row(const Params& p, int bb, int m) {
    valid = m < p.M;
    const int64_t base = (int64_t)bb * p.a_sb + (int64_t)(valid ? m : 0) * p.a_sm;
    if (p.g_pixels) {
      row = p.a + gathered_row(p, bb, m, valid);
      row2 = p.g_pair > 0 ? p.a + gathered_row(p, bb + p.g_pair, m, valid) : nullptr;
    } else {
      row = p.a + base;
      row2 = p.a2 ? p.a2 + base : nullptr;
    }
    step = p.a_sk;
  }

  // Row extreme over all k by global loads (small K, global-load source).
  __device__ float scan_extreme(const Params& p, bool is_min) const {
    float e = is_min ? INFINITY : -INFINITY;
    if (p.a_vec) {
#pragma unroll 4
      for (int k = 0; k < p.K; k += 4) {
        float4 v = ldg_v4(row + k);
        if (row2) {
          const float4 w = ldg_v4(row2 + k);
          v.x += w.x;
          v.y += w.y;
          v.z += w.z;
          v.w += w.w;
        }
        e = extreme(extreme(e, v.x, is_min), extreme(v.y, extreme(v.z, v.w, is_min), is_min), is_min);
      }
      return e;
    }
#pragma unroll 8
    for (int k = 0; k < p.K; ++k) {
      float v = __ldg(row + k * step);
      if (row2) v += __ldg(row2 + k * step);
      e = extreme(e, v, is_min);
    }
    return e;
  }

  // Tucker: row extremes of l and r; exp(r - sr) kept for the whole tile.
  __device__ void tucker_row(const Params& p, int bb, int m, bool want_er) {
    valid = m < p.M;
    const bool is_min = p.shift_min != 0;
    const int64_t row = valid ? m : 0;
    lrow = p.tl + row * p.t_l_sb + bb * p.t_l_sf;
    const float* rrow = p.tr + row * p.t_r_sb + bb * p.t_r_sf;
    float e1 = is_min ? INFINITY : -INFINITY, e2 = e1;
#pragma unroll 4
    for (int i = 0; i < p.t_i; i += 4) {
      const float4 v = ldg_v4(lrow + i);
      e1 = extreme(extreme(e1, v.x, is_min), extreme(v.y, extreme(v.z, v.w, is_min), is_min), is_min);
    }
    float4 rv[kTJ / 4 > 0 ? kTJ / 4 : 1];
#pragma unroll
    for (int j = 0; j < kTJ / 4; ++j) {
      rv[j] = ldg_v4(rrow + 4 * j);
      e2 = extreme(extreme(e2, rv[j].x, is_min), extreme(rv[j].y, extreme(rv[j].z, rv[j].w, is_min), is_min), is_min);
    }
    sl = e1;
    shift = e2;
    if (want_er) {
#pragma unroll
      for (int j = 0; j < kTJ / 4; ++j) {
        er[4 * j] = valid ? exp_shifted(rv[j].x, e2) : 0.0f;
        er[4 * j + 1] = valid ? exp_shifted(rv[j].y, e2) : 0.0f;
        er[4 * j + 2] = valid ? exp_shifted(rv[j].z, e2) : 0.0f;
        er[4 * j + 3] = valid ? exp_shifted(rv[j].w, e2) : 0.0f;
      }
    }
  }

  // Raw values of k0 .. k0+31 (with the fused addend) by global loads.
  __device__ void load_global(const Params& p, int k0, float (&v)[32]) const {
    if (AMODE == kATucker) {
      v[0] = valid ? __ldg(lrow + k0 / kTJ) : -INFINITY;  // one l value per k-block
      return;
    }
    const float fill = (AMODE == kALinear) ? 0.0f : -INFINITY;
    if (p.a_vec && valid && k0 + 32 <= p.K) {
      const float* r = row + k0;
#pragma unroll
      for (int j = 0; j < 32; j += 4) {
        float4 x = ldg_v4(r + j);
        if (row2) {
          const float4 y = ldg_v4(row2 + k0 + j);
          x.x += y.x;
          x.y += y.y;
          x.z += y.z;
          x.w += y.w;
        }
        v[j] = x.x;
        v[j + 1] = x.y;
        v[j + 2] = x.z;
        v[j + 3] = x.w;
      }
      return;
    }
    const float* r = row + (int64_t)k0 * step;
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      const bool ok = valid && k0 + j < p.K;
      float x = ok ? __ldg(r + j * step) : fill;
      if (row2 && ok) x += __ldg(row2 + (int64_t)(k0 + j) * step);
      v[j] = x;
    }
  }

  // exp / split of loaded values 16*H .. 16*H+15 -> hi, lo
  template <int H>
  __device__ void transform_half(const float (&v)[32], int k0, float (&hi)[16], float (&lo)[16]) const {
    if (AMODE == kATucker) {
      const float el = exp_shifted(v[0], sl);
      // J = 64 spans two k-blocks per i: the odd ones use er[32..63]
      const bool second = kTJ == 64 && ((k0 >> 5) & 1);
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        float r = er[(16 * H + j) % kTJ];
        if (kTJ == 64) r = second ? er[(32 + 16 * H + j) % kTJ] : r;
        split_rn(el * r, hi[j], lo[j]);
      }
      return;
    }
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const float x = v[16 * H + j];
      const float e = (AMODE == kALinear) ? x : exp_shifted(x, shift);
      split_rn(e, hi[j], lo[j]);
    }
  }
};

// Raw values of row r of a TMA-staged A tile (128 rows x 32 fp32, 128-byte
// swizzle: 16-byte chunk j of row r at chunk j ^ (r & 7)), plus the staged
// addend, masked to the tile's valid rows and k.
template <int ASRC>
__device__ __forceinline__ void load_staged_row(uint32_t stage, int r, bool valid, int kvalid, float fill,
                                                float (&v)[32]) {
  const uint32_t row = stage + r * 128;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    float4 x = lds_v4(row + ((j ^ (r & 7)) << 4));
    if (a_pair(ASRC)) {
      const float4 y = lds_v4(row + kATileBytes + ((j ^ (r & 7)) << 4));
      x.x += y.x;
      x.y += y.y;
      x.z += y.z;
      x.w += y.w;
    }
    v[4 * j] = x.x;
    v[4 * j + 1] = x.y;
    v[4 * j + 2] = x.z;
    v[4 * j + 3] = x.w;
  }
  if (!valid || kvalid < 32) {
#pragma unroll
    for (int j = 0; j < 32; ++j)
      if (!valid || j >= kvalid) v[j] = fill;
  }
}

// ---------------------------------------------------------------------------
// B operand: 128 threads, 16-byte chunks.  MN-major: thread t covers n-quad
// t % (BN/4) of k-rows t / (BN/4) + (512/BN)*i; K-major: k-quad t % 8 of
// n-rows t / 8 + 16*i.
template <int BN, bool B_KMAJ, int BSRC>
struct BTile {
  static constexpr bool VEC = BSRC != kBLdg;
  static constexpr int kQ = BN / 16;  // float4 per thread
  static constexpr int kQPR = BN / 4;
  static constexpr int kRPP = 128 / kQPR;
  static constexpr int kS = B_KMAJ ? kQ : 4;
  float shift[kS];

  __device__ static void coords(int t, int i, int& n_local, int& k_local) {
    if (B_KMAJ) {
      n_local = (t >> 3) + 16 * i;
      k_local = 4 * (t & 7);
    } else {
      k_local = t / kQPR + kRPP * i;
      n_local = 4 * (t % kQPR);
    }
  }

  __device__ void begin_tile(const Params& p, int bb, int n0, int t) {
#pragma unroll
    for (int i = 0; i < kS; ++i) {
      const int n = B_KMAJ ? n0 + (t >> 3) + 16 * i : n0 + 4 * (t % kQPR) + i;
      shift[i] = (p.shift_b && n < p.N) ? __ldg(p.shift_b + (int64_t)bb * p.sb_sb + (int64_t)n * p.sb_sn) : 0.0f;
    }
  }

  __device__ void load(const Params& p, int bb, int n0, int k0, int t, float4 (&v)[kQ]) const {
    const bool lin = p.shift_b == nullptr;
    const float fill = lin ? 0.0f : -INFINITY;
    const float* base = p.b + (int64_t)bb * p.b_sb;
#pragma unroll
    for (int i = 0; i < kQ; ++i) {
      int nl, kl;
      coords(t, i, nl, kl);
      const int n = n0 + nl, k = k0 + kl;
      const float* q = base + (int64_t)n * p.b_sn + (int64_t)k * p.b_sk;
      if (B_KMAJ) {
        const bool nv = n < p.N;
        if (VEC) {
          v[i] = (nv && k + 4 <= p.K) ? ldg_v4(q) : make_float4(fill, fill, fill, fill);
        } else {
          v[i].x = (nv && k < p.K) ? __ldg(q) : fill;
          v[i].y = (nv && k + 1 < p.K) ? __ldg(q + p.b_sk) : fill;
          v[i].z = (nv && k + 2 < p.K) ? __ldg(q + 2 * p.b_sk) : fill;
          v[i].w = (nv && k + 3 < p.K) ? __ldg(q + 3 * p.b_sk) : fill;
        }
      } else {
        const bool kv = k < p.K;
        if (VEC) {
          v[i] = (kv && n + 4 <= p.N) ? ldg_v4(q) : make_float4(fill, fill, fill, fill);
        } else {
          v[i].x = (kv && n < p.N) ? __ldg(q) : fill;
          v[i].y = (kv && n + 1 < p.N) ? __ldg(q + p.b_sn) : fill;
          v[i].z = (kv && n + 2 < p.N) ? __ldg(q + 2 * p.b_sn) : fill;
          v[i].w = (kv && n + 3 < p.N) ? __ldg(q + 3 * p.b_sn) : fill;
        }
      }
    }
  }

  // Raw values from a TMA-staged tile (unswizzled: MN-major [32 k][BN n],
  // K-major [BN n][32 k]), masked to the operand's extents.
  __device__ void load_staged(const Params& p, uint32_t stage, int n0, int k0, int t, float4 (&v)[kQ]) const {
    if (n0 + BN <= p.N && k0 + kBK <= p.K) {  // interior tile: nothing to mask
#pragma unroll
      for (int i = 0; i < kQ; ++i) {
        int nl, kl;
        coords(t, i, nl, kl);
        v[i] = lds_v4(stage + (B_KMAJ ? (uint32_t)(nl * 32 + kl) * 4 : (uint32_t)(kl * BN + nl) * 4));
      }
      return;
    }
    const float fill = p.shift_b == nullptr ? 0.0f : -INFINITY;
#pragma unroll
    for (int i = 0; i < kQ; ++i) {
      int nl, kl;
      coords(t, i, nl, kl);
      const uint32_t off = B_KMAJ ? (uint32_t)(nl * 32 + kl) * 4 : (uint32_t)(kl * BN + nl) * 4;
      float4 x = lds_v4(stage + off);
      const int n = n0 + nl, k = k0 + kl;
      if (B_KMAJ) {
        if (n >= p.N) x = make_float4(fill, fill, fill, fill);
        if (k + 4 > p.K) {
          if (k >= p.K) x.x = fill;
          if (k + 1 >= p.K) x.y = fill;
          if (k + 2 >= p.K) x.z = fill;
          if (k + 3 >= p.K) x.w = fill;
        }
      } else {
        if (k >= p.K) x = make_float4(fill, fill, fill, fill);
        if (n + 4 > p.N) {
          if (n >= p.N) x.x = fill;
          if (n + 1 >= p.N) x.y = fill;
          if (n + 2 >= p.N) x.z = fill;
          if (n + 3 >= p.N) x.w = fill;
        }
      }
      v[i] = x;
    }
  }

  __device__ void store(const Params& p, uint32_t hi, uint32_t lo, int t, const float4 (&v)[kQ]) const {
    if (p.shift_b == nullptr) {  // linear B: the split alone
#pragma unroll
      for (int i = 0; i < kQ; ++i) {
        int nl, kl;
        coords(t, i, nl, kl);
        float4 h, l;
        split_rn(v[i].x, h.x, l.x);
        split_rn(v[i].y, h.y, l.y);
        split_rn(v[i].z, h.z, l.z);
        split_rn(v[i].w, h.w, l.w);
        const uint32_t off = B_KMAJ ? kmajor_off(nl, kl >> 2) : mnmajor_off(kl, nl >> 2);
        sts_v4(hi + off, h);
        sts_v4(lo + off, l);
      }
      return;
    }
#pragma unroll
    for (int i = 0; i < kQ; ++i) {
      int nl, kl;
      coords(t, i, nl, kl);
      float4 e;
      if (B_KMAJ) {
        const float s = shift[i];
        e = make_float4(exp_shifted(v[i].x, s), exp_shifted(v[i].y, s), exp_shifted(v[i].z, s), exp_shifted(v[i].w, s));
      } else {
        e = make_float4(exp_shifted(v[i].x, shift[0]), exp_shifted(v[i].y, shift[1]), exp_shifted(v[i].z, shift[2]),
                        exp_shifted(v[i].w, shift[3]));
      }
      float4 h, l;
      split_rn(e.x, h.x, l.x);
      split_rn(e.y, h.y, l.y);
      split_rn(e.z, h.z, l.z);
      split_rn(e.w, h.w, l.w);
      const uint32_t off = B_KMAJ ? kmajor_off(nl, kl >> 2) : mnmajor_off(kl, nl >> 2);
      sts_v4(hi + off, h);
      sts_v4(lo + off, l);
    }
  }
};

// ---------------------------------------------------------------------------

// ---------------------------------------------------------------------------
// Prepared B operand.  A B operand is transformed (exp(B - sB), split into TF32 hi / lo) once
// per (batch, 128-column tile, 32-k block) and written as the 32 KB shared-memory stage that the
// contraction kernel's MMAs read: the hi tile, then the lo tile, each 128 n-rows x 32 k, K-major
// with the 128-byte swizzle (kmajor_off).  The kernel then fills a stage with one bulk copy
// (kBPlanes), which takes the B transform (raw tile in, raw values out, hi / lo in) off the
// tensor core's shared-memory path and does it once instead of once per 128-row tile of A.
// Values are bit-identical to the in-kernel transform: same shift, same exp_shifted and
// split_rn; rows past N and k past K are zeros (exp(-inf), or a linear zero).
constexpr int kPlaneN = 128;
constexpr int kPlaneBlockBytes = 2 * kPlaneN * kBK * 4;  // 32 KB

// The general preparation (any K; n or k contiguous) runs as two launches, each spread over
// k: b_col_extreme_kernel reduces a kPrepKRows-row slice of a 128-column tile to per-column
// partial extremes (max.NaN / min.NaN, as the shift pre-pass), and b_planes_kernel combines the
// partials of its tile into sB (written by the CTAs of the first k group) and writes the stages of
// kPrepGroupKB k-blocks.  B_KMAJ: element (k, n) at n * b_sn + k (k contiguous); else at
// k * b_sk + n (n contiguous).  Both need 16-byte aligned rows (the host checks the strides, N or
// K % 4, and the base).
constexpr int kPrepKRows = 1024;  // k rows per partial-extreme CTA
constexpr int kPrepGroupKB = 8;   // k-blocks per stage-writing CTA
__host__ __device__ constexpr int prep_ksplit(int k) { return (k + kPrepKRows - 1) / kPrepKRows; }

// partials: [ksplit][batch][tiles_n * 128]
template <bool B_KMAJ>
__global__ void __launch_bounds__(256) b_col_extreme_kernel(const float* __restrict__ b, int64_t b_sb, int64_t b_sk,
                                                            int64_t b_sn, int N, int K, int tiles_n, int batch,
                                                            int shift_min, float* __restrict__ partials) {
  __shared__ float red[8][kPlaneN];
  const int t = threadIdx.x;
  const int ks = blockIdx.x % prep_ksplit(K);
  const int rest = blockIdx.x / prep_ksplit(K);
  const int nt = rest % tiles_n;
  const int64_t bb = rest / tiles_n;
  const int n0 = nt * kPlaneN;
  const int k_lo = ks * kPrepKRows, k_hi = min(K, k_lo + kPrepKRows);
  const float* base = b + bb * b_sb;
  const bool is_min = shift_min != 0;
  float* out = partials + ((int64_t)ks * batch + bb) * (tiles_n * kPlaneN) + n0;
  if (!B_KMAJ) {
    const int cq = t & 31, kr = t >> 5;  // columns n0 + 4cq .. +3, k = k_lo + kr, + 8, ...
    const int n = n0 + 4 * cq;
    float e[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) e[i] = is_min ? INFINITY : -INFINITY;
    if (n < N) {  // N % 4 == 0: the quad is whole
      const float* q = base + n;
#pragma unroll 8
      for (int k = k_lo + kr; k < k_hi; k += 8) {
        const float4 v = ldg_v4(q + (int64_t)k * b_sk);
        e[0] = extreme(e[0], v.x, is_min);
        e[1] = extreme(e[1], v.y, is_min);
        e[2] = extreme(e[2], v.z, is_min);
        e[3] = extreme(e[3], v.w, is_min);
      }
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) red[kr][4 * cq + i] = e[i];
    __syncthreads();
    if (t < kPlaneN) {
      float x = red[0][t];
#pragma unroll
      for (int r = 1; r < 8; ++r) x = extreme(x, red[r][t], is_min);
      out[t] = x;
    }
  } else {
    const int nl = t >> 1, half = t & 1;  // row n0 + nl, k quads half, half + 2, ...
    const int n = n0 + nl;
    float e = is_min ? INFINITY : -INFINITY;
    if (n < N) {
      const float* q = base + (int64_t)n * b_sn;
#pragma unroll 8
      for (int k = k_lo + 4 * half; k < k_hi; k += 8) {  // K % 4 == 0
        const float4 v = ldg_v4(q + k);
        e = extreme(extreme(e, v.x, is_min), extreme(v.y, extreme(v.z, v.w, is_min), is_min), is_min);
      }
    }
    e = extreme(e, __shfl_xor_sync(0xffffffffu, e, 1), is_min);
    if (half == 0) out[nl] = e;
  }
}

// One CTA (256 threads) per (batch, 128-column tile, group of kPrepGroupKB k-blocks).
template <bool B_KMAJ, bool LOG>
__global__ void __launch_bounds__(256) b_planes_kernel(const float* __restrict__ b, int64_t b_sb, int64_t b_sk,
                                                       int64_t b_sn, int N, int K, int tiles_n, int batch,
                                                       int shift_min, const float* __restrict__ partials,
                                                       float* __restrict__ planes, float* __restrict__ shift_out) {
  __shared__ __align__(1024) uint8_t stage[kPlaneBlockBytes];
  __shared__ float colshift[kPlaneN];
  const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
  const int num_kb = (K + kBK - 1) / kBK;
  const int groups = (num_kb + kPrepGroupKB - 1) / kPrepGroupKB;
  const int kg = blockIdx.x % groups;
  const int rest = blockIdx.x / groups;
  const int nt = rest % tiles_n;
  const int64_t bb = rest / tiles_n;
  const int n0 = nt * kPlaneN;
  const float* base = b + bb * b_sb;
  const bool is_min = shift_min != 0;
  const float fill = LOG ? -INFINITY : 0.0f;

  // -------- column shifts: the partial extremes of the tile's columns over all k slices
  if (LOG) {
    if (t < kPlaneN) {
      const int ksplit = prep_ksplit(K);
      const float* part = partials + bb * (tiles_n * kPlaneN) + n0 + t;
      float x = part[0];
      for (int ks = 1; ks < ksplit; ++ks) x = extreme(x, part[(int64_t)ks * batch * (tiles_n * kPlaneN)], is_min);
      colshift[t] = x;
      if (kg == 0 && n0 + t < N) shift_out[bb * N + n0 + t] = x;
    }
    __syncthreads();
  }

  // -------- the group's stages, one 32-k block at a time, assembled in shared memory
  float* dst_base = planes + ((bb * tiles_n + nt) * (int64_t)num_kb) * (kPlaneBlockBytes / 4);
  const int kb_end = min(num_kb, (kg + 1) * kPrepGroupKB);
  for (int kb = kg * kPrepGroupKB; kb < kb_end; ++kb) {
    const int k0 = kb * kBK;
    const uint32_t hi = smem_u32(stage), lo = hi + kPlaneBlockBytes / 2;
    if (!B_KMAJ) {
      // warp: columns 32 * (warp & 3) .. +31, k 16 * (warp >> 2) .. +15; lane: column quad
      // lane >> 2, k quad lane & 3.  A 4 x 4 block per thread, transposed into four chunks
      // (one per column: 4 consecutive k); every store instruction fills the 32 banks 4 times.
      const int nl0 = 32 * (warp & 3) + 4 * (lane >> 2);
      const int q = 4 * (warp >> 2) + (lane & 3);  // k quad within the block
      const int n = n0 + nl0;
      float v[4][4];  // [k][column]
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int k = k0 + 4 * q + j;
        if (k < K && n < N) {
          const float4 x = ldg_v4(base + (int64_t)k * b_sk + n);
          v[j][0] = x.x;
          v[j][1] = x.y;
          v[j][2] = x.z;
          v[j][3] = x.w;
        } else {
          v[j][0] = v[j][1] = v[j][2] = v[j][3] = fill;
        }
      }
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float s = LOG ? colshift[nl0 + i] : 0.0f;
        float4 h, l;
        float e0 = LOG ? exp_shifted(v[0][i], s) : v[0][i];
        float e1 = LOG ? exp_shifted(v[1][i], s) : v[1][i];
        float e2 = LOG ? exp_shifted(v[2][i], s) : v[2][i];
        float e3 = LOG ? exp_shifted(v[3][i], s) : v[3][i];
        if (LOG && n >= N) e0 = e1 = e2 = e3 = 0.0f;  // a column past N (its shift is a fill value)
        split_rn(e0, h.x, l.x);
        split_rn(e1, h.y, l.y);
        split_rn(e2, h.z, l.z);
        split_rn(e3, h.w, l.w);
        const uint32_t off = kmajor_off(nl0 + i, q);
        sts_v4(hi + off, h);
        sts_v4(lo + off, l);
      }
    } else {
      // warp: rows 16 * warp .. +15, four at a time; lane: row + (lane >> 3), k quad lane & 7
      const int q = lane & 7;
#pragma unroll
      for (int r = 0; r < 4; ++r) {
        const int nl = 16 * warp + 4 * r + (lane >> 3);
        const int n = n0 + nl, k = k0 + 4 * q;
        float4 x = make_float4(fill, fill, fill, fill);
        if (n < N && k < K) x = ldg_v4(base + (int64_t)n * b_sn + k);
        float4 e = x;
        if (LOG) {
          const float s = colshift[nl];
          e = make_float4(exp_shifted(x.x, s), exp_shifted(x.y, s), exp_shifted(x.z, s), exp_shifted(x.w, s));
          if (n >= N) e = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        }
        float4 h, l;
        split_rn(e.x, h.x, l.x);
        split_rn(e.y, h.y, l.y);
        split_rn(e.z, h.z, l.z);
        split_rn(e.w, h.w, l.w);
        const uint32_t off = kmajor_off(nl, q);
        sts_v4(hi + off, h);
        sts_v4(lo + off, l);
      }
    }
    __syncthreads();  // the block is complete
    // copy-out: 32 KB contiguous, 16 bytes per thread and instruction
    float* dst = dst_base + (int64_t)kb * (kPlaneBlockBytes / 4);
#pragma unroll
    for (int i = 0; i < kPlaneBlockBytes / (256 * 16); ++i) {
      const int off = (i * 256 + t) * 16;
      stg_v4(dst + off / 4, lds_v4(hi + off));
    }
    __syncthreads();  // read out before the next block is assembled
  }
}

// B with n contiguous and K <= kStripeMaxK: one CTA (256 threads) per (batch, 128-column tile,
// 32-column quarter) holds its whole column stripe (K x 32 values) in shared memory, so that B is
// read from HBM once: the stripe is loaded, its column extremes taken (a log-domain B), and the
// quarter's rows of every stage written (rows 32q .. 32q+31 of a K-major tile are the 4 KB at
// 4096q of its hi and of its lo part).  Same values as b_planes_kernel.
constexpr int kStripeMaxK = 512;
constexpr int kStripePitch = 33;  // floats per stripe row: conflict-free column reads
__host__ __device__ constexpr int stripe_smem_bytes(int k) {
  return ((k + kBK - 1) / kBK) * kBK * kStripePitch * 4 + 8 * 32 * 4 + 32 * 4;
}

template <bool LOG>
__global__ void __launch_bounds__(256) b_planes_stripe_kernel(const float* __restrict__ b, int64_t b_sb, int64_t b_sk,
                                                              int N, int K, int tiles_n, int shift_min,
                                                              float* __restrict__ planes, float* __restrict__ shift_out) {
  extern __shared__ __align__(16) float stripe[];  // [k_pad][kStripePitch], then red[8][32], colshift[32]
  const int num_kb = (K + kBK - 1) / kBK;
  const int k_pad = num_kb * kBK;
  float* red = stripe + k_pad * kStripePitch;
  float* colshift = red + 8 * 32;
  const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
  const int quarter = blockIdx.x & 3;
  const int nt = (blockIdx.x >> 2) % tiles_n;
  const int64_t bb = (blockIdx.x >> 2) / tiles_n;
  const int c0 = nt * kPlaneN + 32 * quarter;  // first column of the stripe
  const float* base = b + bb * b_sb;
  const bool is_min = shift_min != 0;
  const float fill = LOG ? -INFINITY : 0.0f;

  // -------- the stripe: 16-byte loads, lanes 8j .. 8j+7 read row (4 * it + j), 8 rows in flight per thread
  {
    const int q4 = lane & 7, rsub = lane >> 3;
    const int c = c0 + 4 * q4;
    const bool cv = c < N;  // N % 4 == 0: the quad is whole or absent
#pragma unroll 8
    for (int k = 4 * warp + rsub; k < k_pad; k += 32) {
      float4 v = make_float4(fill, fill, fill, fill);
      if (cv && k < K) v = ldg_v4(base + (int64_t)k * b_sk + c);
      float* row = stripe + k * kStripePitch + 4 * q4;
      row[0] = v.x;
      row[1] = v.y;
      row[2] = v.z;
      row[3] = v.w;
    }
  }
  __syncthreads();
  // -------- column extremes over k (rows past K hold the fill and do not enter)
  if (LOG) {
    float e = is_min ? INFINITY : -INFINITY;
    for (int k = warp; k < K; k += 8) e = extreme(e, stripe[k * kStripePitch + lane], is_min);
    red[warp * 32 + lane] = e;
    __syncthreads();
    if (t < 32) {
      float x = red[t];
#pragma unroll
      for (int w = 1; w < 8; ++w) x = extreme(x, red[w * 32 + t], is_min);
      colshift[t] = x;
      if (c0 + t < N) shift_out[bb * N + c0 + t] = x;
    }
    __syncthreads();
  }
  // -------- the quarter's rows of every stage: thread t writes chunk (row j = t >> 3, k quad t & 7)
  const int j = t >> 3, kq = t & 7;
  const bool col_valid = c0 + j < N;
  const float s = LOG ? colshift[j] : 0.0f;
  const int nl = 32 * quarter + j;
  float* blocks = planes + ((bb * tiles_n + nt) * (int64_t)num_kb) * (kPlaneBlockBytes / 4);
  const uint32_t off = kmajor_off(nl, kq) / 4;  // floats, within the hi (or lo) tile
#pragma unroll 4
  for (int kb = 0; kb < num_kb; ++kb) {
    const float* src = stripe + (kb * kBK + 4 * kq) * kStripePitch + j;
    float e[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float x = src[i * kStripePitch];
      e[i] = LOG ? exp_shifted(x, s) : x;
      if (!col_valid) e[i] = 0.0f;  // a column past N (its shift is a fill value)
    }
    float4 h, l;
    split_rn(e[0], h.x, l.x);
    split_rn(e[1], h.y, l.y);
    split_rn(e[2], h.z, l.z);
    split_rn(e[3], h.w, l.w);
    float* blk = blocks + (int64_t)kb * (kPlaneBlockBytes / 4);
    stg_v4(blk + off, h);
    stg_v4(blk + kPlaneBlockBytes / 8 + off, l);
  }
}

template <int BN, int AMODE, int ASRC, bool B_KMAJ, int BSRC, int TJ>
__global__ void __launch_bounds__(Cfg<BN, ASRC, BSRC>::kThreads, 1)
    lse_gemm_kernel(const __grid_constant__ Params p, const __grid_constant__ CUtensorMap tmap_a,
                    const __grid_constant__ CUtensorMap tmap_a2, const __grid_constant__ CUtensorMap tmap_b) {
  using C = Cfg<BN, ASRC, BSRC>;
  using ARowT = ARow<AMODE, TJ>;
  static_assert(C::kFits, "shared memory configuration");
  static_assert(AMODE != kATucker || ASRC == kALdg, "the Tucker operand is generated from global loads");
  static_assert(BSRC != kBPlanes || (BN == 128 && B_KMAJ && !a_gathered(ASRC)), "prepared B: 128-column K-major stages");
  // two MMA issuers with prepared B: the MMA warp (main products) and kCorrMmaWarp (correction
  // products).  (A second issuer in a warp of its own beside busy B warps measured slower.)
  constexpr bool kTwoMma = BSRC == kBPlanes;
  static_assert(!kTwoMma || C::kDrainGroups == 1, "two MMA issuers with one drain group");
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  float* running = (float*)(smem + C::kOffRun);    // [BN][128], column-major
  float* shifts = (float*)(smem + C::kOffShift);   // [2 slots][s1, s2][128 rows]
  uint64_t* bars = (uint64_t*)(smem + C::kOffBar);
  uint64_t* full = bars;                        // [kStages], one arrival per A and B warp
  uint64_t* empty = full + kStages;             // [kStages], tcgen05.commit
  uint64_t* chunk_full = empty + kStages;       // [2], tcgen05.commit
  uint64_t* chunk_empty = chunk_full + 2;       // [2], drain warps
  uint64_t* corr_empty = chunk_empty + 2;       // [kCorrBufs], drain warps
  uint64_t* shift_full = corr_empty + 2;        // [2], A warps
  uint64_t* shift_empty = shift_full + 2;       // [2], drain warps
  uint64_t* a_full = shift_empty + 2;           // [4], TMA transactions
  uint64_t* a_empty = a_full + 4;               // [4], A warps
  uint64_t* b_full = a_empty + 4;               // [4], TMA transactions
  uint64_t* b_empty = b_full + 4;               // [4], B warps
  uint64_t* drain = b_empty + 4;                // [1], teardown
  uint64_t* corr_full = drain + 1;              // [kCorrBufs], the correction MMAs of a tile (two issuers)
  uint32_t* tmem_slot = (uint32_t*)(corr_full + 2);
  volatile int* abort_flag = (volatile int*)(tmem_slot + 1);
  // the A / B ring barriers the producer armed, drained at wind-down after an abort
  ArmedCopies* a_copies = (ArmedCopies*)(tmem_slot + 2);
  ArmedCopies* b_copies = a_copies + 1;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      // prepared B: the stage's B half comes through b_full / b_empty instead
      mbar_init(&full[s], BSRC == kBPlanes ? kAWarps : kAWarps + kBWarps);
      mbar_init(&empty[s], kTwoMma ? 2 : 1);
    }
    for (int c = 0; c < 2; ++c) {
      mbar_init(&chunk_full[c], 1);
      mbar_init(&chunk_empty[c], kDrainWarps);
      mbar_init(&shift_full[c], kAWarps);
      mbar_init(&shift_empty[c], kDrainWarps);
    }
    for (int s = 0; s < 4; ++s) {
      mbar_init(&a_full[s], 1);
      mbar_init(&a_empty[s], kAWarps);
      mbar_init(&b_full[s], 1);
      mbar_init(&b_empty[s], BSRC == kBPlanes ? 2 : kBWarps);  // prepared B: both MMA issuers' commits
    }
    for (int c = 0; c < C::kCorrBufs; ++c) mbar_init(&corr_empty[c], kDrainWarps);
    mbar_init(drain, kTwoMma ? 2 : 1);
    for (int c = 0; c < 2; ++c) mbar_init(&corr_full[c], 1);
    *abort_flag = 0;
    *a_copies = *b_copies = ArmedCopies{0u, 0u};
    fence_mbarrier_init();
  }
  if (warp == kMmaWarp) tmem_alloc<C::kTmemCols>(tmem_slot);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t smem_base = smem_u32(smem);

  // One thread's MMA issue loop.  kMmaAll: per 8-wide k-step main += A_hi*B_hi and
  // corr += A_hi*B_lo + A_lo*B_hi.  With two issuers, kMmaMain issues the main products (and owns
  // the chunk hand-over) and kMmaCorr the correction products (its tile hand-over through
  // corr_full); the stage barriers then count one commit of each.
  auto mma_issue = [&](int role) {
    constexpr uint32_t idesc = idesc_tf32(kBM, BN, false, !B_KMAJ);
    // K-major B advances 32 bytes per 8-element k-step inside the swizzle
    // row; MN-major B advances two 4-row groups (1024 bytes).
    constexpr uint32_t b_lbo = B_KMAJ ? 16 : 4096, b_sbo = B_KMAJ ? 1024 : 512, b_step = B_KMAJ ? 32 : 1024;
    constexpr uint32_t b_lay = B_KMAJ ? kLayoutSW128 : kLayoutSW128Base32B;
    const bool do_main = role != kMmaCorr, do_corr = role != kMmaMain;
    uint32_t it = 0, gc = 0, tl = 0;
    bool ok = true;
    for (int tile = blockIdx.x; tile < p.num_tiles && ok; tile += gridDim.x, ++tl) {
      const uint32_t cbuf = tl % C::kCorrBufs;
      if (do_corr && !mbar_wait(&corr_empty[cbuf], ((tl / C::kCorrBufs) & 1) ^ 1, kSiteMmaCorr, abort_flag)) {
        ok = false;
        break;
      }
      const uint32_t d_corr = tmem + C::kTmemCorr + cbuf * BN;
      uint32_t d_main = 0;
      for (int kb = 0; kb < p.num_kb; ++kb, ++it) {
        const int kc = kb % kChunkKB;
        if (do_main && kc == 0) {
          const uint32_t cb = gc & 1;
          if (!mbar_wait(&chunk_empty[cb], ((gc >> 1) & 1) ^ 1, kSiteMmaChunk, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          d_main = tmem + C::kTmemMain + cb * BN;
        }
        const uint32_t s = it % kStages;
        const uint32_t ph = (it / kStages) & 1;
        if (kb == 0) XE_TILE_TRACE(tl, 12);
        if (!mbar_wait(&full[s], ph, kSiteMmaFull, abort_flag)) {
          ok = false;
          break;
        }
        // prepared B: its own deeper ring of bulk-copied stages
        const uint32_t bs = BSRC == kBPlanes ? it % C::kBStages : s;
        if (BSRC == kBPlanes && !mbar_wait(&b_full[bs], (it / C::kBStages) & 1, kSiteMmaFull, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        if (kb == 0) XE_TILE_TRACE(tl, 13);
        const uint32_t a_hi = tmem + C::kTmemA + 64 * s, a_lo = a_hi + 32;
        const uint32_t b_hi = smem_base + C::kOffB + bs * C::kStageBytes, b_lo = b_hi + C::kBTile;
#pragma unroll
        for (int kk = 0; kk < kBK / 8; ++kk) {
          const uint64_t dbh = smem_desc(b_hi + kk * b_step, b_lbo, b_sbo, b_lay);
          if (do_main) umma_tf32_ts(d_main, a_hi + kk * 8, dbh, idesc, (kc | kk) != 0);
          if (do_corr) {
            const uint64_t dbl = smem_desc(b_lo + kk * b_step, b_lbo, b_sbo, b_lay);
            umma_tf32_ts(d_corr, a_hi + kk * 8, dbl, idesc, (kb | kk) != 0);
            umma_tf32_ts(d_corr, a_lo + kk * 8, dbh, idesc, 1);
          }
        }
        umma_commit(&empty[s]);
        if (BSRC == kBPlanes) umma_commit(&b_empty[bs]);
        if (do_main && (kc == kChunkKB - 1 || kb == p.num_kb - 1)) {
          umma_commit(&chunk_full[gc & 1]);
          ++gc;
        }
        if (role == kMmaCorr && kb == p.num_kb - 1) umma_commit(&corr_full[cbuf]);
        if (kb == 0 || kb == 8 || kb == p.num_kb - 1) XE_TILE_TRACE(tl, kb == 0 ? 6 : kb == 8 ? 7 : 8);
      }
    }
    // All issued MMAs must finish before TMEM is released.
    umma_commit(drain);
    mbar_wait(drain, 0, kSiteGemmDrain, abort_flag, /*honor_abort=*/false);
  };

  if (warp < kAWarps) {
    // ------------------------------------------------------------ A rows
    const int r = warp * 32 + lane;  // warp w may access TMEM lanes 32w..32w+31
    const uint32_t lane_bits = (uint32_t)(warp * 32) << 16;
    const bool is_min = p.shift_min != 0;
    const float fill = (AMODE == kALinear) ? 0.0f : -INFINITY;
    ARowT a;
    uint32_t it = 0, ait = 0, tl = 0;
    bool ok = true;
    for (int tile = blockIdx.x; tile < p.num_tiles && ok; tile += gridDim.x, ++tl) {
      int bb, mt, nt;
      decode_tile(p, tile, bb, mt, nt);
      const int m = mt * kBM + r;
      // -------- row shifts
      float s1 = 0.0f, s2 = 0.0f;
      float cur[32], nxt[32];
      bool preloaded = false;  // global-load source: both k-blocks of the tile already in cur / nxt
      if (AMODE == kATucker) {
        a.tucker_row(p, bb, m, true);
        s1 = a.sl;
        s2 = a.shift;
      } else {
        a.set_row(p, bb, m);
        if (AMODE == kALog) {
          if (p.shift_a) {
            a.shift = a.valid ? __ldg(p.shift_a + (int64_t)bb * p.sa_sb + (int64_t)m * p.sa_sm) : 0.0f;
          } else if (ASRC != kALdg) {
            // every k-block of this tile is staged (num_kb <= kAStages): scan them.  A row of
            // at most two k-blocks stays in registers (cur, nxt) and its stages are released here.
            float e = is_min ? INFINITY : -INFINITY;
            const bool keep = C::kDrainGroups == 1 && p.num_kb <= 2;
            XE_SEGMENT_BEGIN(seg_scan);
            for (int kb = 0; kb < p.num_kb; ++kb) {
              const uint32_t sidx = (ait + kb) % C::kAStages;
              if (!mbar_wait(&a_full[sidx], ((ait + kb) / C::kAStages) & 1, kSiteAStaged, abort_flag)) {
                ok = false;  // per lane: the vote after the scan makes it warp-uniform
                break;
              }
              const int kvalid = p.K - kb * kBK;
              const uint32_t stage = smem_base + C::kOffA + sidx * C::kAStageBytes;
              // the k tail is masked with -inf for exp(); it must not enter a min
              if (keep && kb == 0) {
                load_staged_row<ASRC>(stage, r, a.valid, kvalid, fill, cur);
#pragma unroll
                for (int j = 0; j < 32; ++j)
                  if (j < kvalid) e = extreme(e, cur[j], is_min);
              } else if (keep) {
                load_staged_row<ASRC>(stage, r, a.valid, kvalid, fill, nxt);
#pragma unroll
                for (int j = 0; j < 32; ++j)
                  if (j < kvalid) e = extreme(e, nxt[j], is_min);
              } else {
                float v[32];
                load_staged_row<ASRC>(stage, r, a.valid, kvalid, fill, v);
                if (kvalid >= 32) {
#pragma unroll
                  for (int j = 0; j < 32; ++j) e = extreme(e, v[j], is_min);
                } else {
#pragma unroll
                  for (int j = 0; j < 32; ++j)
                    if (j < kvalid) e = extreme(e, v[j], is_min);
                }
              }
            }
            XE_SEGMENT_END(seg_scan, 6);
            // a lane whose wait ran out (ok false) goes on to the vote at the shift slot below
            if (keep) {
              __syncwarp();
              if (lane == 0)
                for (int kb = 0; kb < p.num_kb; ++kb) mbar_arrive(&a_empty[(ait + kb) % C::kAStages]);
              ait += p.num_kb;
              preloaded = true;
            }
            a.shift = a.valid ? e : 0.0f;
          } else if (C::kDrainGroups == 1 && p.num_kb <= 2) {
            // global-load source, one or two k-blocks: load the row once, scan it in registers
            a.load_global(p, 0, cur);
            if (p.num_kb == 2) a.load_global(p, kBK, nxt);
            float e = is_min ? INFINITY : -INFINITY;
#pragma unroll
            for (int j = 0; j < 32; ++j)
              if (j < p.K) e = extreme(e, cur[j], is_min);
            if (p.num_kb == 2) {
#pragma unroll
              for (int j = 0; j < 32; ++j)
                if (kBK + j < p.K) e = extreme(e, nxt[j], is_min);
            }
            a.shift = a.valid ? e : 0.0f;
            preloaded = true;
          } else {
            a.shift = a.valid ? a.scan_extreme(p, is_min) : 0.0f;
          }
          s1 = a.shift;
        }
      }
      // -------- publish the row shifts for the epilogue
      {
        const uint32_t slot = tl & 1;
        if (!mbar_wait_warp(&shift_empty[slot], ((tl >> 1) & 1) ^ 1, kSiteAShiftSlot, abort_flag, ok)) {
          ok = false;
          break;
        }
        shifts[(slot * 2 + 0) * kBM + r] = s1;
        shifts[(slot * 2 + 1) * kBM + r] = s2;
        __syncwarp();
        if (lane == 0) mbar_arrive(&shift_full[slot]);
      }
      // -------- k loop
      if (ASRC == kALdg && !preloaded) a.load_global(p, 0, cur);
      for (int kb = 0; kb < p.num_kb; ++kb, ++it) {
        XE_SEGMENT_BEGIN(seg_load);
        // The staged slot is released only once its values have been used (transformed below):
        // a shared-memory load may still be in flight when the next instruction issues, and the
        // producer's TMA would overwrite the slot.
        int release = -1;
        // per lane, voted on below; after an abort the loads read a stage nobody consumes
        bool staged = true;
        if (ASRC != kALdg && !preloaded) {
          const uint32_t sidx = ait % C::kAStages;
          staged = mbar_wait(&a_full[sidx], (ait / C::kAStages) & 1, kSiteAStaged, abort_flag);
          load_staged_row<ASRC>(smem_base + C::kOffA + sidx * C::kAStageBytes, r, a.valid, p.K - kb * kBK, fill,
                                cur);
          release = (int)sidx;
          ++ait;
        } else if (ASRC == kALdg && kb + 1 < p.num_kb && !preloaded) {
          a.load_global(p, (kb + 1) * kBK, nxt);
        }
        XE_SEGMENT_END(seg_load, 1);
        const uint32_t s = it % kStages;
        const uint32_t ph = (it / kStages) & 1;
        if (!mbar_wait_warp(&empty[s], ph ^ 1, kSiteAStage, abort_flag, staged)) {
          ok = false;
          break;
        }
        tc_fence_after();
        XE_SEGMENT_BEGIN(seg_tr);
        const uint32_t col = tmem + lane_bits + C::kTmemA + 64 * s;
        {
          float hi[16], lo[16];
          a.template transform_half<0>(cur, kb * kBK, hi, lo);
          tmem_st16(col, hi);
          tmem_st16(col + 32, lo);
        }
        {
          float hi[16], lo[16];
          a.template transform_half<1>(cur, kb * kBK, hi, lo);
          tmem_st16(col + 16, hi);
          tmem_st16(col + 48, lo);
        }
        XE_SEGMENT_END(seg_tr, 2);
        XE_SEGMENT_BEGIN(seg_st);
        tmem_wait_st();
        XE_SEGMENT_END(seg_st, 3);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&full[s]);
          if (release >= 0) mbar_arrive(&a_empty[release]);
        }
        if (r == 0 && (kb == 0 || kb == 8)) XE_TILE_TRACE(tl, kb == 0 ? 2 : 3);
        if ((ASRC == kALdg || preloaded) && kb + 1 < p.num_kb) {
#pragma unroll
          for (int j = 0; j < 32; ++j) cur[j] = nxt[j];
        }
      }
    }
  } else if (warp < kAWarps + kBWarps) {
    // ------------------------------------------------------------ B tiles
    // (with prepared B its stages arrive by bulk copy: warp kCorrMmaWarp issues the correction
    // products, the others idle)
    if constexpr (BSRC == kBPlanes) {
      if (warp == kCorrMmaWarp && lane == 0) mma_issue(kMmaCorr);
      __syncwarp();
    } else {
    const int t = threadIdx.x - kAWarps * 32;
    using BT = BTile<BN, B_KMAJ, BSRC>;
    BT bt;
    uint32_t it = 0, bit = 0;
    bool ok = true;
    for (int tile = blockIdx.x; tile < p.num_tiles && ok; tile += gridDim.x) {
      int bb, mt, nt;
      decode_tile(p, tile, bb, mt, nt);
      const int n0 = nt * BN;
      bt.begin_tile(p, bb, n0, t);
      float4 cur[BT::kQ], nxt[BT::kQ];
      if (BSRC != kBTma) bt.load(p, bb, n0, 0, t, cur);
      for (int kb = 0; kb < p.num_kb; ++kb, ++it) {
        const bool more = kb + 1 < p.num_kb;
        int release = -1;
        // per lane, voted on below; after an abort the loads read a stage nobody consumes
        bool staged = true;
        if (BSRC == kBTma) {
          const uint32_t sidx = bit % C::kBRawStages;
          staged = mbar_wait(&b_full[sidx], (bit / C::kBRawStages) & 1, kSiteBStage, abort_flag);
          bt.load_staged(p, smem_base + C::kOffBRaw + sidx * C::kBRawBytes, n0, kb * kBK, t, cur);
          release = (int)sidx;  // released after the values are used (see the A rows)
          ++bit;
        } else if (more) {
          bt.load(p, bb, n0, (kb + 1) * kBK, t, nxt);
        }
        const uint32_t s = it % kStages;
        const uint32_t ph = (it / kStages) & 1;
        // per lane; after an abort the stores below only write this CTA's own stage
        const bool ready = mbar_wait(&empty[s], ph ^ 1, kSiteBStage, abort_flag) && staged;
        const uint32_t st = smem_base + C::kOffB + s * C::kStageBytes;
        XE_SEGMENT_BEGIN(seg_b);
        bt.store(p, st, st + C::kBTile, t, cur);
        XE_SEGMENT_END(seg_b, 4);
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&full[s]);
          if (release >= 0) mbar_arrive(&b_empty[release]);
        }
        // a timeout seen by any lane ends the warp's loop for all of them; voted after the arrival
        // (after an abort it only hands on a stage that nobody uses), off the tensor core's path
        if (!__all_sync(0xffffffffu, ready)) {
          ok = false;
          break;
        }
        if (t == 0 && (kb == 0 || kb == 8)) XE_TILE_TRACE(it / p.num_kb, kb == 0 ? 4 : 5);
        if (BSRC != kBTma && more) {
#pragma unroll
          for (int i = 0; i < BT::kQ; ++i) cur[i] = nxt[i];
        }
      }
    }
    }
  } else if (warp == kMmaWarp) {
    // ------------------------------------------------------------ MMA issue
    if (lane == 0) mma_issue(kTwoMma ? kMmaMain : kMmaAll);
    __syncwarp();
  } else if (warp < kProducerWarp || warp > kProducerWarp) {
    // ------------------------------------------------------------ drain + epilogue
    const int q = warp & 3;  // TMEM lane quadrant of this warp
    const int r = q * 32 + lane;
    const uint32_t lane_bits = (uint32_t)(q * 32) << 16;
    // Each drain warp owns TMEM lanes (rows) 32q..32q+31 from the accumulator
    // to the copy-out, so the drain warps never wait for one another.
    const int group = warp > kProducerWarp ? 1 : 0;
    uint32_t gc = 0, tl = 0, ob = 0;
    bool ok = true;
    const int chunks = (p.num_kb + kChunkKB - 1) / kChunkKB;
    // Two groups split the tiles when every tile is a single chunk: the tile's chunk
    // buffer, correction buffer, shift slot and staging buffer all alternate with it.
    // Otherwise group 0 takes every tile.
    const bool split = C::kDrainGroups == 2 && chunks == 1;
    if (group == 1 && !split) ok = false;
    for (int tile = blockIdx.x; tile < p.num_tiles && ok; tile += gridDim.x, ++tl) {
      if (split && (int)(tl & 1) != group) continue;
      if (split) {
        gc = tl;
        ob = group;
      }
      int bb, mt, nt;
      decode_tile(p, tile, bb, mt, nt);
      const int m0 = mt * kBM;
      const int n0 = nt * BN;
      // column shifts of a log-domain B: loaded now, so that their latency passes while the tile's
      // MMAs run; copied to shared memory in the epilogue
      float csv[BN / 32];
#pragma unroll
      for (int i = 0; i < BN / 32; ++i) {
        const int c = lane + 32 * i;
        csv[i] = (p.shift_b && n0 + c < p.N) ? __ldg(p.shift_b + (int64_t)bb * p.sb_sb + (int64_t)(n0 + c) * p.sb_sn)
                                              : 0.0f;
      }
      // -------- chunks: running[col][row] (+)= main chunk, for all but the last chunk;
      // the epilogue reads the last chunk and the correction straight from TMEM.
      for (int c = 0; c < chunks - 1; ++c, ++gc) {
        const uint32_t cb = gc & 1;
        if (!mbar_wait_warp(&chunk_full[cb], (gc >> 1) & 1, kSiteDrainChunk, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        XE_SEGMENT_BEGIN(seg_dr);
#pragma unroll 1
        for (int sl = 0; sl < BN / 32; ++sl) {
          float v[32];
          tmem_ld32(tmem + lane_bits + C::kTmemMain + cb * BN + sl * 32, v);
          tmem_wait_ld();
          float* run = running + sl * 32 * kBM + r;
#pragma unroll
          for (int j = 0; j < 32; ++j) run[j * kBM] = (c == 0) ? v[j] : run[j * kBM] + v[j];
        }
        XE_SEGMENT_END(seg_dr, 5);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&chunk_empty[cb]);
        if (r == 0 && c == 0) XE_TILE_TRACE(tl, 9);
      }
      if (!ok) break;
      const bool direct = chunks == 1;
      const uint32_t dcb = gc & 1;  // the last (or only) chunk
      if (!mbar_wait_warp(&chunk_full[dcb], (gc >> 1) & 1, kSiteDrainChunk, abort_flag)) break;
      // two MMA issuers: the correction products of the tile complete on their own barrier
      if (kTwoMma && !mbar_wait_warp(&corr_full[tl % C::kCorrBufs], (tl / C::kCorrBufs) & 1, kSiteDrainChunk,
                                     abort_flag))
        break;
      tc_fence_after();
      if (r == 0) XE_TILE_TRACE(tl, 10);
      ++gc;
      // -------- epilogue from shared memory, overlapping the next tile's MMAs
      // The row shifts (from the A warps) and the column shifts, into this warp's own slice of
      // shared memory.  With the two-pass form below this comes after the tile's TMEM columns
      // are released, off the path of the next tile's first MMAs.
      const uint32_t slot = tl & 1;
      float* cshift = p.shift_b ? (float*)(smem + C::kOffColShift) + (group * 4 + q) * BN : nullptr;
      float s1 = 0.0f, s2 = 0.0f;
      auto take_shifts = [&]() -> bool {
        XE_SEGMENT_BEGIN(seg_ep);
        const bool shifted = mbar_wait(&shift_full[slot], (tl >> 1) & 1, kSiteDrainShift, abort_flag);
        s1 = shifts[(slot * 2 + 0) * kBM + r];
        s2 = shifts[(slot * 2 + 1) * kBM + r];
        if (!__all_sync(0xffffffffu, shifted)) return false;  // the warp's reconvergence, and a timeout seen by all lanes
        if (lane == 0) mbar_arrive(&shift_empty[slot]);
        if (cshift) {
          __syncwarp();  // the previous tile's reads of cshift are done
#pragma unroll
          for (int i = 0; i < BN / 32; ++i) cshift[lane + 32 * i] = csv[i];
          __syncwarp();
        }
        XE_SEGMENT_END(seg_ep, 7);
        return true;
      };
      // The tile's TMEM columns (the last chunk and the correction) are read out first, summed
      // with the running sum of the earlier chunks into `running`, and released at once: the next
      // tile's MMAs (its correction buffer is this one when there is a single one) then run while
      // this tile's logs and copy-out do.  Same sums in the same order as the one-pass form below.
      const bool two_pass = !split && C::kRunningBytes > 0;
      if (!two_pass && !take_shifts()) break;
      if (two_pass) {
#pragma unroll 1
        for (int sl = 0; sl < BN / 32; ++sl) {
          float* run = running + sl * 32 * kBM + r;
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            float v[16], w[16];
            tmem_ld16(tmem + lane_bits + C::kTmemMain + dcb * BN + sl * 32 + 16 * h, v);
            tmem_ld16(tmem + lane_bits + C::kTmemCorr + (tl % C::kCorrBufs) * BN + sl * 32 + 16 * h, w);
            tmem_wait_ld();
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              const float t = direct ? v[j] : run[(16 * h + j) * kBM] + v[j];
              // an overflowed main term carries the result; its correction is NaN
              run[(16 * h + j) * kBM] = isinf(t) ? t : t + w[j];
            }
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&chunk_empty[dcb]);
          mbar_arrive(&corr_empty[tl % C::kCorrBufs]);
        }
        if (!take_shifts()) break;
      }
      float* cbase = p.c + (int64_t)bb * p.c_sb;
#pragma unroll 1
      for (int sl = 0; sl < BN / 32; ++sl) {
        const float* run = running + sl * 32 * kBM + r;  // this row's 32 sums of the slice
        // every warp stages and copies out its own 32 rows: warp-level ordering suffices
        if (C::kOutBufs == 1 || split) __syncwarp();  // this buffer's previous copy-out is done
        // Staging as [128 rows][32 cols], 16-byte chunks swizzled by (row & 7): row r at
        // stage + r * 128 in a separate buffer, or, in place, at the 128 bytes that hold the
        // running sums of column (32 sl + r % 32), rows 32q .. 32q+31 (this warp's own rows):
        // slice base + (r % 32) * 512 + q * 128.
        uint32_t stage = 0, srow = 0;
        float sums[32];  // in place: the whole slice is read before its bytes are reused
        if constexpr (C::kStageInPlace) {
          stage = smem_base + C::kOffRun + sl * 32 * kBM * 4;
          srow = stage + lane * 512 + q * 128;
#pragma unroll
          for (int j = 0; j < 32; ++j) sums[j] = run[j * kBM];
          __syncwarp();
        } else {
          stage = smem_base + C::kOffOutAligned + (ob % (C::kOutBufs > 0 ? C::kOutBufs : 1)) * C::kOutBytes;
          srow = stage + r * 128;
        }
        if (!split) ++ob;
        XE_SEGMENT_BEGIN(seg_e1);
        // 16 columns at a time: sums (TMEM main + correction, or the running sum), log and
        // shifts in the reference's order, staging
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          float out[16];
          if (C::kStageInPlace) {
#pragma unroll
            for (int j = 0; j < 16; ++j) out[j] = sums[16 * h + j];
          } else if (two_pass) {
#pragma unroll
            for (int j = 0; j < 16; ++j) out[j] = run[(16 * h + j) * kBM];
          } else {
            // the last chunk (plus the running sum of the earlier ones) and the correction
            float v[16], w[16];
            tmem_ld16(tmem + lane_bits + C::kTmemMain + dcb * BN + sl * 32 + 16 * h, v);
            tmem_ld16(tmem + lane_bits + C::kTmemCorr + (tl % C::kCorrBufs) * BN + sl * 32 + 16 * h, w);
            tmem_wait_ld();
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              const float t = direct ? v[j] : run[(16 * h + j) * kBM] + v[j];
              // an overflowed main term carries the result; its correction is NaN
              out[j] = isinf(t) ? t : t + w[j];
            }
            if (sl == BN / 32 - 1 && h == 1) {  // every TMEM column of this tile has been read
              tc_fence_before();
              __syncwarp();
              if (lane == 0) {
                mbar_arrive(&chunk_empty[dcb]);
                mbar_arrive(&corr_empty[tl % C::kCorrBufs]);
              }
            }
          }
          if (!p.raw_out) {
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              float o = fast_log(out[j]);
              if (AMODE != kALinear) o += s1;
              if (AMODE == kATucker) o += s2;
              out[j] = o;
            }
            if (cshift) {
#pragma unroll
              for (int j = 0; j < 16; ++j) out[j] += cshift[sl * 32 + 16 * h + j];
            }
          }
#pragma unroll
          for (int j = 0; j < 4; ++j)
            sts_v4(srow + (((4 * h + j) ^ (r & 7)) << 4), make_float4(out[4 * j], out[4 * j + 1], out[4 * j + 2], out[4 * j + 3]));
        }
        XE_SEGMENT_END(seg_e1, 8);
        XE_SEGMENT_BEGIN(seg_e3);
        __syncwarp();
        XE_SEGMENT_END(seg_e3, 10);
        XE_SEGMENT_BEGIN(seg_e4);
        // coalesced copy-out: each warp writes 32 rows, 4 rows (512 B) per instruction
        const int chunk = lane & 7;
        const int n = n0 + sl * 32 + 4 * chunk;
        // byte offset of a staged row of this warp (see the staging layout above)
        auto row_off = [&](int row) -> uint32_t {
          return C::kStageInPlace ? (uint32_t)((row & 31) * 512 + q * 128) : (uint32_t)(row * 128);
        };
        if (p.c_vec && m0 + kBM <= p.M && n0 + sl * 32 + 32 <= p.N) {
          // interior slice: every row and column in bounds, 16-byte stores
#pragma unroll
          for (int it = 0; it < 8; ++it) {
            const int row = q * 32 + 4 * it + (lane >> 3);
            stg_v4(cbase + (int64_t)(m0 + row) * p.c_sm + n, lds_v4(stage + row_off(row) + ((chunk ^ (row & 7)) << 4)));
          }
          XE_SEGMENT_END(seg_e4, 11);
          continue;
        }
#pragma unroll 1
        for (int it = 0; it < 8; ++it) {
          const int row = q * 32 + 4 * it + (lane >> 3);
          const int m = m0 + row;
          if (m >= p.M || n >= p.N) continue;
          const float4 val = lds_v4(stage + row_off(row) + ((chunk ^ (row & 7)) << 4));
          float* dst = cbase + (int64_t)m * p.c_sm;
          if (p.c_vec && n + 4 <= p.N) {
            stg_v4(dst + n, val);
          } else {
            dst[(int64_t)n * p.c_sn] = val.x;
            if (n + 1 < p.N) dst[(int64_t)(n + 1) * p.c_sn] = val.y;
            if (n + 2 < p.N) dst[(int64_t)(n + 2) * p.c_sn] = val.z;
            if (n + 3 < p.N) dst[(int64_t)(n + 3) * p.c_sn] = val.w;
          }
        }
        XE_SEGMENT_END(seg_e4, 11);
      }
      // in place: the copy-out's reads come before the next tile's running sums are written
      if (C::kStageInPlace) __syncwarp();
      if (r == 0) XE_TILE_TRACE(tl, 11);
    }
  } else if (a_gathered(ASRC)) {
    // ------------------------------------------------------------ gather producer (whole warp)
    // Row r of a tile is table row pixels[m, var[bb]] of fold bb (kAGather2: plus row
    // pixels[m, var[bb + g_pair]] of fold bb + g_pair, staged in the second tile of the
    // stage).  tmap_a views the table as (folds * states) rows of K, 128-byte swizzled boxes
    // of one row x 32 k.  Lane l issues the tile::gather4 loads of rows 4l..4l+3 (512 bytes
    // at stage + 512 l: the swizzled layout the A warps read); lane 0 arms a_full with the
    // stage's bytes first.  The pixel values of the next tile are loaded while this tile's
    // rows are in flight.  B tiles come through TMA from lane 0.
    constexpr int kRows = ASRC == kAGather2 ? 2 : 1;
    // pixel values of rows 4*lane .. 4*lane+3 of a tile (-1: row past M)
    auto load_states = [&](int tile, int (&st)[kRows][4]) {
      int bb, mt, nt;
      decode_tile(p, tile, bb, mt, nt);
#pragma unroll
      for (int h = 0; h < kRows; ++h) {
        const int64_t fold = (int64_t)bb + h * p.g_pair;
        int64_t v = p.g_var ? (int64_t)__ldg(p.g_var + fold) : fold;
        if (v < 0 || v >= p.g_stride) {
          record_bad_index(kSiteGemmGatherState);
          v = 0;
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int m = mt * kBM + lane * 4 + i;
          st[h][i] = m < p.M ? (int)__ldg(p.g_pixels + (int64_t)m * p.g_stride + v) : -1;
        }
      }
    };
    uint32_t ait = 0, bit = 0;
    bool ok = true;
    int st[kRows][4];
    if ((int)blockIdx.x < p.num_tiles) load_states(blockIdx.x, st);
    for (int tile = blockIdx.x; tile < p.num_tiles && ok; tile += gridDim.x) {
      int bb, mt, nt;
      decode_tile(p, tile, bb, mt, nt);
      // table rows (fold * states + state; the host checks they fit in 32 bits); a row past M
      // loads its fold's first row, which the A warps mask
      int row[kRows][4];
#pragma unroll
      for (int h = 0; h < kRows; ++h)
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          int state = st[h][i] < 0 ? 0 : st[h][i];
          if (state >= p.g_states) {
            record_bad_index(kSiteGemmGatherState);
            state = p.g_states - 1;
          }
          row[h][i] = (bb + h * (int)p.g_pair) * p.g_states + state;
        }
      const bool have_next = tile + (int)gridDim.x < p.num_tiles;
      if (have_next) load_states(tile + gridDim.x, st);
      XE_SEGMENT_BEGIN(seg_prod);
      for (int kb = 0; kb < p.num_kb; ++kb) {
        const uint32_t sidx = ait % C::kAStages;
        bool armed = true;
        if (lane == 0) {
          armed = mbar_wait(&a_empty[sidx], ((ait / C::kAStages) & 1) ^ 1, kSiteProducer, abort_flag);
          if (armed) {
            mbar_expect_tx(&a_full[sidx], C::kAStageBytes);
            a_copies->note(sidx, ait / C::kAStages);
          }
        }
        if (__shfl_sync(0xffffffffu, armed ? 1 : 0, 0) == 0) {  // the warp leaves together
          ok = false;
          break;
        }
        const uint32_t dst = smem_base + C::kOffA + sidx * C::kAStageBytes + lane * 512;
#pragma unroll
        for (int h = 0; h < kRows; ++h)
          tma_gather4(dst + h * kATileBytes, &tmap_a, kb * kBK, row[h][0], row[h][1], row[h][2], row[h][3],
                      &a_full[sidx]);
        ++ait;
        if (BSRC == kBTma && lane == 0) {
          const uint32_t bidx = bit % C::kBRawStages;
          if (!mbar_wait(&b_empty[bidx], ((bit / C::kBRawStages) & 1) ^ 1, kSiteProducer, abort_flag)) {
            ok = false;
          } else {
            const uint32_t bdst = smem_base + C::kOffBRaw + bidx * C::kBRawBytes;
            mbar_expect_tx(&b_full[bidx], C::kBRawBytes);
            b_copies->note(bidx, bit / C::kBRawStages);
            if (B_KMAJ)
              tma_load_3d(bdst, &tmap_b, kb * kBK, nt * BN, bb, &b_full[bidx]);
            else
              tma_load_3d(bdst, &tmap_b, nt * BN, kb * kBK, bb, &b_full[bidx]);
            ++bit;
          }
        }
        ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
      }
      XE_SEGMENT_END(seg_prod, 12);
    }
  } else if ((ASRC != kALdg || BSRC == kBTma || BSRC == kBPlanes) && lane == 0) {
    // ------------------------------------------------------------ TMA producer
    uint32_t ait = 0, bit = 0;
    bool ok = true;
    for (int tile = blockIdx.x; tile < p.num_tiles && ok; tile += gridDim.x) {
      int bb, mt, nt;
      decode_tile(p, tile, bb, mt, nt);
      for (int kb = 0; kb < p.num_kb; ++kb) {
        if (ASRC != kALdg) {
          const uint32_t sidx = ait % C::kAStages;
          if (!mbar_wait(&a_empty[sidx], ((ait / C::kAStages) & 1) ^ 1, kSiteProducer, abort_flag)) {
            ok = false;
            break;
          }
          const uint32_t dst = smem_base + C::kOffA + sidx * C::kAStageBytes;
          mbar_expect_tx(&a_full[sidx], C::kAStageBytes);
          a_copies->note(sidx, ait / C::kAStages);
          tma_load_3d(dst, &tmap_a, kb * kBK, mt * kBM, bb, &a_full[sidx]);
          if (ASRC == kATma2) tma_load_3d(dst + kATileBytes, &tmap_a2, kb * kBK, mt * kBM, bb, &a_full[sidx]);
          if (kb == 0 || kb == 8) XE_TILE_TRACE(ait / p.num_kb, kb == 0 ? 0 : 1);
          ++ait;
        }
        if (BSRC == kBTma) {
          const uint32_t sidx = bit % C::kBRawStages;
          if (!mbar_wait(&b_empty[sidx], ((bit / C::kBRawStages) & 1) ^ 1, kSiteProducer, abort_flag)) {
            ok = false;
            break;
          }
          const uint32_t dst = smem_base + C::kOffBRaw + sidx * C::kBRawBytes;
          mbar_expect_tx(&b_full[sidx], C::kBRawBytes);
          b_copies->note(sidx, bit / C::kBRawStages);
          if (B_KMAJ)
            tma_load_3d(dst, &tmap_b, kb * kBK, nt * BN, bb, &b_full[sidx]);
          else
            tma_load_3d(dst, &tmap_b, nt * BN, kb * kBK, bb, &b_full[sidx]);
          ++bit;
        }
        if (BSRC == kBPlanes) {
          // the prepared stage (hi and lo tiles) of this (bb, nt, kb): one 32 KB bulk copy
          const uint32_t sidx = bit % C::kBStages;
          if (!mbar_wait(&b_empty[sidx], ((bit / C::kBStages) & 1) ^ 1, kSiteProducer, abort_flag)) {
            ok = false;
            break;
          }
          const uint32_t dst = smem_base + C::kOffB + sidx * C::kStageBytes;
          mbar_expect_tx(&b_full[sidx], C::kStageBytes);
          b_copies->note(sidx, bit / C::kBStages);
          bulk_load(dst, p.b_planes + (((int64_t)bb * p.tiles_n + nt) * p.num_kb + kb) * (C::kStageBytes / 4),
                    C::kStageBytes, &b_full[sidx]);
          ++bit;
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (*abort_flag) {  // uniform: every thread has passed its last wait
    a_copies->drain(a_full, abort_flag);
    b_copies->drain(b_full, abort_flag);
    __syncthreads();
  }
  tc_fence_after();
  if (warp == kMmaWarp) tmem_dealloc<C::kTmemCols>(tmem);
}

}  // namespace gemm
}  // namespace xe
