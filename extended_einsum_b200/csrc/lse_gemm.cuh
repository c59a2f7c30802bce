// Log-space batched contraction on the sm_100a tensor cores.
//
//   C[b,m,n] = log( sum_k exp(A[b,m,k]-sA[b,m]) * exp(B[b,k,n]-sB[b,n]) ) + sA[b,m] + sB[b,n]
//
// This is the arithmetic that _append_logspace_einsum
// (backend_translation/translate.py:686-750) spreads over ~16 backend calls
// for a binary contraction, fused into one persistent kernel:
//
//   transform warps (8)  global fp32 tile -> exp(x - shift) (or the linear
//                        value) -> TF32 hi/lo split -> 128B-swizzled UMMA
//                        tiles in shared memory (generic-proxy stores)
//   MMA warp (1 thread)  three tcgen05.mma kind::tf32 per k-step:
//                        hi*hi into the main TMEM accumulator and
//                        hi*lo + lo*hi into a separate correction accumulator
//   epilogue warps (4)   tcgen05.ld -> log(main + corr) + shifts -> global
//
// Stages are handed over with mbarriers (full: transform -> MMA, empty:
// tcgen05.commit -> transform); accumulators are double-buffered in TMEM when
// they fit, so the epilogue of one tile overlaps the main loop of the next.
// Every wait is bounded (xe_common.cuh).
#pragma once

#include "xe_common.cuh"

namespace xe {
namespace gemm {

constexpr int kBM = 128;  // UMMA M (cta_group::1)
constexpr int kBK = 32;   // fp32 elements per 128-byte swizzle row
constexpr int kTransformWarps = 8;
constexpr int kTransformThreads = kTransformWarps * 32;
constexpr int kMmaWarp = kTransformWarps;  // warp 8
constexpr int kEpiWarp0 = kMmaWarp + 1;    // warps 9..12
constexpr int kEpiWarps = 4;
constexpr int kThreads = (kTransformWarps + 1 + kEpiWarps) * 32;  // 416

struct Params {
  const float* a;
  const float* a2;
  int64_t a_sb, a_sm, a_sk;
  const float* b;
  int64_t b_sb, b_sk, b_sn;
  float* c;
  int64_t c_sb, c_sm, c_sn;
  const float* shift_a;  // [batch*M]; nullptr when A is linear
  const float* shift_b;  // [batch*N]; nullptr when B is linear
  int batch, M, N, K;
  int tiles_m, tiles_n, num_tiles, num_kb;
  int c_vec;  // output rows may be written with 16-byte stores
};

__host__ __device__ constexpr int pow2_at_least(int x) {
  int p = 32;
  while (p < x) p <<= 1;
  return p;
}

template <int BN, bool SPLIT_ACC>
struct Cfg {
  static constexpr int kATile = kBM * kBK * 4;  // bytes, one of hi/lo
  static constexpr int kBTile = BN * kBK * 4;
  static constexpr int kStageBytes = 2 * kATile + 2 * kBTile;
  static constexpr int kStages = (BN >= 256) ? 2 : (BN >= 128 ? 3 : 4);
  static constexpr int kAccCols = SPLIT_ACC ? 2 * BN : BN;
  static constexpr int kNumAcc = (2 * kAccCols <= 512) ? 2 : 1;
  static constexpr int kTmemCols = pow2_at_least(kNumAcc * kAccCols);
  // shared memory: [1024 alignment slack][stages][barriers]
  static constexpr int kBarrierBytes = 256;
  static constexpr int kSmemBytes = 1024 + kStages * kStageBytes + kBarrierBytes;
  static_assert(kTmemCols <= 512, "accumulators exceed TMEM");
  static_assert(BN % 32 == 0 && BN >= 32 && BN <= 256, "BN");
};

// Byte offset of the 16-byte chunk holding elements (row, 4q..4q+3) of a
// K-major tile (rows x 32 fp32, 128-byte rows, 8-row swizzle atoms).
__device__ __forceinline__ uint32_t kmajor_off(int row, int q) {
  return (uint32_t)((row >> 3) * 1024 + (row & 7) * 128 + ((q ^ (row & 7)) << 4));
}
// Byte offset of the 16-byte chunk holding elements (k, 4q..4q+3) of an
// MN-major tile (32 k-rows x MN, 32-element swizzle atoms stacked every 4096 B).
__device__ __forceinline__ uint32_t mnmajor_off(int k, int q) {
  return (uint32_t)((q >> 3) * 4096 + (k >> 3) * 1024 + (k & 7) * 128 + (((q & 7) ^ (k & 7)) << 4));
}

__device__ __forceinline__ float lse_prologue(float x, float s, bool linear) {
  return linear ? x : expf(x - s);
}

__device__ __forceinline__ void split_store(uint32_t hi_addr, uint32_t lo_addr, float4 e) {
  float4 h, l;
  split_tf32(e.x, h.x, l.x);
  split_tf32(e.y, h.y, l.y);
  split_tf32(e.z, h.z, l.z);
  split_tf32(e.w, h.w, l.w);
  sts_v4(hi_addr, h);
  sts_v4(lo_addr, l);
}

// Loads four elements p[0], p[s], p[2s], p[3s] with per-element masks.
template <bool VEC>
__device__ __forceinline__ float4 load_quad(const float* p, int64_t s, int valid, float fill) {
  float4 v;
  if (VEC) {
    if (valid >= 4) {
      v = ldg_nc_v4(p);
    } else {
      v = make_float4(fill, fill, fill, fill);
    }
  } else {
    v.x = valid > 0 ? ldg_nc(p) : fill;
    v.y = valid > 1 ? ldg_nc(p + s) : fill;
    v.z = valid > 2 ? ldg_nc(p + 2 * s) : fill;
    v.w = valid > 3 ? ldg_nc(p + 3 * s) : fill;
  }
  return v;
}

__device__ __forceinline__ float4 add4(float4 a, float4 b) {
  return make_float4(a.x + b.x, a.y + b.y, a.z + b.z, a.w + b.w);
}

// Number of valid elements among idx, idx+1, idx+2, idx+3 (clamped to 0..4).
__device__ __forceinline__ int quad_valid(int idx, int limit) {
  int v = limit - idx;
  return v < 0 ? 0 : (v > 4 ? 4 : v);
}

template <int BN, bool A_KMAJ, bool B_KMAJ, bool VEC>
struct Loader {
  // A fragment: 4 float4 per transform thread; B fragment: BN/32 float4.
  static constexpr int kAQ = 4;
  static constexpr int kBQ = BN / 32;

  // ---- A ----
  // K-major: thread t covers k-quad t%8 of rows t/8 + 32*i.
  // MN-major: thread t covers m-quad t%32 of k-rows t/32 + 8*i.
  __device__ static void load_a(const Params& p, int bb, int m0, int k0, int t, float4 (&ra)[kAQ]) {
    const bool lin = p.shift_a == nullptr;
    const float fill = lin ? 0.0f : -INFINITY;
    const float* base = p.a + (int64_t)bb * p.a_sb;
    const float* base2 = p.a2 ? p.a2 + (int64_t)bb * p.a_sb : nullptr;
#pragma unroll
    for (int i = 0; i < kAQ; ++i) {
      int m, k, valid;
      int64_t off, step;
      if (A_KMAJ) {
        m = m0 + (t >> 3) + 32 * i;
        k = k0 + 4 * (t & 7);
        valid = (m < p.M) ? quad_valid(k, p.K) : 0;
        off = (int64_t)m * p.a_sm + (int64_t)k * p.a_sk;
        step = p.a_sk;
      } else {
        k = k0 + (t >> 5) + 8 * i;
        m = m0 + 4 * (t & 31);
        valid = (k < p.K) ? quad_valid(m, p.M) : 0;
        off = (int64_t)k * p.a_sk + (int64_t)m * p.a_sm;
        step = p.a_sm;
      }
      float4 v = load_quad<VEC>(base + off, step, valid, fill);
      if (base2) v = add4(v, load_quad<VEC>(base2 + off, step, valid, 0.0f));
      ra[i] = v;
    }
  }

  __device__ static void load_a_shift(const Params& p, int bb, int m0, int t, float (&sa)[4]) {
    if (p.shift_a == nullptr) {
#pragma unroll
      for (int i = 0; i < 4; ++i) sa[i] = 0.0f;
      return;
    }
    const float* s = p.shift_a + (int64_t)bb * p.M;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      int m = A_KMAJ ? m0 + (t >> 3) + 32 * i : m0 + 4 * (t & 31) + i;
      sa[i] = (m < p.M) ? __ldg(s + m) : 0.0f;
    }
  }

  __device__ static void store_a(const Params& p, uint32_t hi, uint32_t lo, int t, const float4 (&ra)[kAQ],
                                 const float (&sa)[4]) {
    const bool lin = p.shift_a == nullptr;
#pragma unroll
    for (int i = 0; i < kAQ; ++i) {
      float4 e;
      uint32_t off;
      if (A_KMAJ) {
        const float s = sa[i];
        e = make_float4(lse_prologue(ra[i].x, s, lin), lse_prologue(ra[i].y, s, lin), lse_prologue(ra[i].z, s, lin),
                        lse_prologue(ra[i].w, s, lin));
        off = kmajor_off((t >> 3) + 32 * i, t & 7);
      } else {
        e = make_float4(lse_prologue(ra[i].x, sa[0], lin), lse_prologue(ra[i].y, sa[1], lin),
                        lse_prologue(ra[i].z, sa[2], lin), lse_prologue(ra[i].w, sa[3], lin));
        off = mnmajor_off((t >> 5) + 8 * i, t & 31);
      }
      split_store(hi + off, lo + off, e);
    }
  }

  // ---- B ----
  // MN-major: thread t covers n-quad t%(BN/4) of k-rows t/(BN/4) + (1024/BN)*i.
  // K-major: thread t covers k-quad t%8 of n-rows t/8 + 32*i.
  static constexpr int kQPR = BN / 4;
  static constexpr int kRPP = kTransformThreads / kQPR;

  __device__ static void load_b(const Params& p, int bb, int n0, int k0, int t, float4 (&rb)[kBQ]) {
    const bool lin = p.shift_b == nullptr;
    const float fill = lin ? 0.0f : -INFINITY;
    const float* base = p.b + (int64_t)bb * p.b_sb;
#pragma unroll
    for (int i = 0; i < kBQ; ++i) {
      int n, k, valid;
      int64_t off, step;
      if (B_KMAJ) {
        n = n0 + (t >> 3) + 32 * i;
        k = k0 + 4 * (t & 7);
        valid = (n < p.N) ? quad_valid(k, p.K) : 0;
        off = (int64_t)n * p.b_sn + (int64_t)k * p.b_sk;
        step = p.b_sk;
      } else {
        k = k0 + t / kQPR + kRPP * i;
        n = n0 + 4 * (t % kQPR);
        valid = (k < p.K) ? quad_valid(n, p.N) : 0;
        off = (int64_t)k * p.b_sk + (int64_t)n * p.b_sn;
        step = p.b_sn;
      }
      rb[i] = load_quad<VEC>(base + off, step, valid, fill);
    }
  }

  // B shifts: K-major -> one per n-row (kBQ values); MN-major -> 4 per quad.
  static constexpr int kBS = B_KMAJ ? kBQ : 4;
  __device__ static void load_b_shift(const Params& p, int bb, int n0, int t, float (&sb)[kBS]) {
    if (p.shift_b == nullptr) {
#pragma unroll
      for (int i = 0; i < kBS; ++i) sb[i] = 0.0f;
      return;
    }
    const float* s = p.shift_b + (int64_t)bb * p.N;
#pragma unroll
    for (int i = 0; i < kBS; ++i) {
      int n = B_KMAJ ? n0 + (t >> 3) + 32 * i : n0 + 4 * (t % kQPR) + i;
      sb[i] = (n < p.N) ? __ldg(s + n) : 0.0f;
    }
  }

  __device__ static void store_b(const Params& p, uint32_t hi, uint32_t lo, int t, const float4 (&rb)[kBQ],
                                 const float (&sb)[kBS]) {
    const bool lin = p.shift_b == nullptr;
#pragma unroll
    for (int i = 0; i < kBQ; ++i) {
      float4 e;
      uint32_t off;
      if (B_KMAJ) {
        const float s = sb[i];
        e = make_float4(lse_prologue(rb[i].x, s, lin), lse_prologue(rb[i].y, s, lin), lse_prologue(rb[i].z, s, lin),
                        lse_prologue(rb[i].w, s, lin));
        off = kmajor_off((t >> 3) + 32 * i, t & 7);
      } else {
        e = make_float4(lse_prologue(rb[i].x, sb[0], lin), lse_prologue(rb[i].y, sb[1], lin),
                        lse_prologue(rb[i].z, sb[2], lin), lse_prologue(rb[i].w, sb[3], lin));
        off = mnmajor_off(t / kQPR + kRPP * i, t % kQPR);
      }
      split_store(hi + off, lo + off, e);
    }
  }
};

__device__ __forceinline__ void decode_tile(const Params& p, int tile, int& bb, int& mt, int& nt) {
  nt = tile % p.tiles_n;
  int rest = tile / p.tiles_n;
  mt = rest % p.tiles_m;
  bb = rest / p.tiles_m;
}

template <int BN, bool A_KMAJ, bool B_KMAJ, bool VEC, bool SPLIT_ACC>
__global__ void __launch_bounds__(kThreads, 1) lse_gemm_kernel(const Params p) {
  using C = Cfg<BN, SPLIT_ACC>;
  using L = Loader<BN, A_KMAJ, B_KMAJ, VEC>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint64_t* bars = (uint64_t*)(smem + C::kStages * C::kStageBytes);
  uint64_t* full = bars;                         // [kStages]
  uint64_t* empty = full + C::kStages;           // [kStages]
  uint64_t* acc_full = empty + C::kStages;       // [kNumAcc]
  uint64_t* acc_empty = acc_full + C::kNumAcc;   // [kNumAcc]
  uint64_t* drain = acc_empty + C::kNumAcc;      // [1]
  uint32_t* tmem_slot = (uint32_t*)(drain + 1);
  volatile int* abort_flag = (volatile int*)(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::kStages; ++s) {
      mbar_init(&full[s], kTransformWarps);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < C::kNumAcc; ++a) {
      mbar_init(&acc_full[a], 1);
      mbar_init(&acc_empty[a], kEpiWarps);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbarrier_init();
  }
  if (warp == kMmaWarp) tmem_alloc<C::kTmemCols>(tmem_slot);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const uint32_t smem_base = smem_u32(smem);

  if (warp < kTransformWarps) {
    // ------------------------------------------------------------ transform
    const int t = threadIdx.x;
    uint32_t it = 0;
    bool ok = true;
    for (int tile = blockIdx.x; tile < p.num_tiles && ok; tile += gridDim.x) {
      int bb, mt, nt;
      decode_tile(p, tile, bb, mt, nt);
      const int m0 = mt * kBM, n0 = nt * BN;
      float sa[4];
      float sb[L::kBS];
      L::load_a_shift(p, bb, m0, t, sa);
      L::load_b_shift(p, bb, n0, t, sb);
      float4 ra[L::kAQ], rb[L::kBQ];
      L::load_a(p, bb, m0, 0, t, ra);
      L::load_b(p, bb, n0, 0, t, rb);
      for (int kb = 0; kb < p.num_kb; ++kb, ++it) {
        float4 na[L::kAQ], nb[L::kBQ];
        const bool more = kb + 1 < p.num_kb;
        if (more) {
          L::load_a(p, bb, m0, (kb + 1) * kBK, t, na);
          L::load_b(p, bb, n0, (kb + 1) * kBK, t, nb);
        }
        const uint32_t s = it % C::kStages;
        const uint32_t ph = (it / C::kStages) & 1;
        if (!mbar_wait(&empty[s], ph ^ 1, kSiteGemmEmpty, abort_flag)) {
          ok = false;
          break;
        }
        const uint32_t st = smem_base + s * C::kStageBytes;
        L::store_a(p, st, st + C::kATile, t, ra, sa);
        L::store_b(p, st + 2 * C::kATile, st + 2 * C::kATile + C::kBTile, t, rb, sb);
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&full[s]);
        if (more) {
#pragma unroll
          for (int i = 0; i < L::kAQ; ++i) ra[i] = na[i];
#pragma unroll
          for (int i = 0; i < L::kBQ; ++i) rb[i] = nb[i];
        }
      }
    }
  } else if (warp == kMmaWarp) {
    // ------------------------------------------------------------ MMA issue
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_tf32(kBM, BN, !A_KMAJ, !B_KMAJ);
      // K-major tiles advance 32 bytes per 8-element k-step inside the
      // swizzle row; MN-major tiles advance one 8-row group (1024 bytes).
      constexpr uint32_t a_lbo = A_KMAJ ? 16 : 4096, a_sbo = 1024, a_step = A_KMAJ ? 32 : 1024;
      constexpr uint32_t b_lbo = B_KMAJ ? 16 : 4096, b_sbo = 1024, b_step = B_KMAJ ? 32 : 1024;
      uint32_t it = 0, tl = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < p.num_tiles && ok; tile += gridDim.x, ++tl) {
        const uint32_t acc = tl % C::kNumAcc;
        const uint32_t acc_ph = (tl / C::kNumAcc) & 1;
        if (!mbar_wait(&acc_empty[acc], acc_ph ^ 1, kSiteGemmAccEmpty, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_main = tmem_base + acc * C::kAccCols;
        const uint32_t d_corr = SPLIT_ACC ? d_main + BN : d_main;
        for (int kb = 0; kb < p.num_kb; ++kb, ++it) {
          const uint32_t s = it % C::kStages;
          const uint32_t ph = (it / C::kStages) & 1;
          if (!mbar_wait(&full[s], ph, kSiteGemmFull, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t st = smem_base + s * C::kStageBytes;
          const uint32_t a_hi = st, a_lo = st + C::kATile;
          const uint32_t b_hi = st + 2 * C::kATile, b_lo = b_hi + C::kBTile;
#pragma unroll
          for (int kk = 0; kk < kBK / 8; ++kk) {
            const uint64_t dah = smem_desc_sw128(a_hi + kk * a_step, a_lbo, a_sbo);
            const uint64_t dal = smem_desc_sw128(a_lo + kk * a_step, a_lbo, a_sbo);
            const uint64_t dbh = smem_desc_sw128(b_hi + kk * b_step, b_lbo, b_sbo);
            const uint64_t dbl = smem_desc_sw128(b_lo + kk * b_step, b_lbo, b_sbo);
            const uint32_t first = (kb | kk) != 0;
            umma_tf32(d_main, dah, dbh, idesc, first);
            if (SPLIT_ACC) {
              umma_tf32(d_corr, dah, dbl, idesc, first);
            } else {
              umma_tf32(d_corr, dah, dbl, idesc, 1);
            }
            umma_tf32(d_corr, dal, dbh, idesc, 1);
          }
          umma_commit(&empty[s]);
        }
        if (ok) umma_commit(&acc_full[acc]);
      }
      // All issued MMAs must finish before TMEM is released.
      umma_commit(drain);
      mbar_wait(drain, 0, kSiteGemmDrain, abort_flag, /*honor_abort=*/false);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;  // TMEM lane quadrant this warp may access
    const int row = q * 32 + lane;
    uint32_t tl = 0;
    for (int tile = blockIdx.x; tile < p.num_tiles; tile += gridDim.x, ++tl) {
      int bb, mt, nt;
      decode_tile(p, tile, bb, mt, nt);
      const int m = mt * kBM + row;
      const int n0 = nt * BN;
      const uint32_t acc = tl % C::kNumAcc;
      const uint32_t acc_ph = (tl / C::kNumAcc) & 1;
      if (!mbar_wait(&acc_full[acc], acc_ph, kSiteGemmAccFull, abort_flag)) break;
      tc_fence_after();
      const float sa = (p.shift_a && m < p.M) ? __ldg(p.shift_a + (int64_t)bb * p.M + m) : 0.0f;
      const float* sbp = p.shift_b ? p.shift_b + (int64_t)bb * p.N : nullptr;
      float* crow = p.c + (int64_t)bb * p.c_sb + (int64_t)m * p.c_sm;
      const uint32_t t_main = tmem_base + ((uint32_t)(q * 32) << 16) + acc * C::kAccCols;
#pragma unroll 1
      for (int ch = 0; ch < BN / 32; ++ch) {
        float vm[32], vc[32];
        tmem_ld32(t_main + ch * 32, vm);
        if (SPLIT_ACC) tmem_ld32(t_main + BN + ch * 32, vc);
        tmem_wait_ld();
        const int nb = n0 + ch * 32;
        if (m < p.M && nb < p.N) {
          float out[32];
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            float v = SPLIT_ACC ? vm[j] + vc[j] : vm[j];
            float r = logf(v);
            if (p.shift_a) r += sa;
            if (sbp) {
              const int n = nb + j;
              r += (n < p.N) ? __ldg(sbp + n) : 0.0f;
            }
            out[j] = r;
          }
          if (p.c_vec && nb + 32 <= p.N) {
#pragma unroll
            for (int j = 0; j < 32; j += 4) stg_v4(crow + nb + j, make_float4(out[j], out[j + 1], out[j + 2], out[j + 3]));
          } else {
#pragma unroll
            for (int j = 0; j < 32; ++j)
              if (nb + j < p.N) crow[(int64_t)(nb + j) * p.c_sn] = out[j];
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[acc]);
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == kMmaWarp) tmem_dealloc<C::kTmemCols>(tmem_base);
}

}  // namespace gemm
}  // namespace xe
