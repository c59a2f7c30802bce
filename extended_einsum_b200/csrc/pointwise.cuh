// Memory-bound kernels of the log-space path: per-operand shift reduction,
// softmax, log-space broadcast addition, categorical gather.  All of them
// stream fp32 with 16-byte accesses where the layout allows it.
#pragma once

#include "xe_common.cuh"

namespace xe {

// torch.amax / torch.amin propagate NaN; so does PTX max.NaN / min.NaN.
template <bool MAXMODE>
__device__ __forceinline__ float nan_extreme(float a, float b) {
  float r;
  if (MAXMODE)
    asm("max.NaN.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
  else
    asm("min.NaN.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
  return r;
}

template <bool MAXMODE>
__device__ __forceinline__ float extreme_identity() {
  return MAXMODE ? -INFINITY : INFINITY;
}

// ---------------------------------------------------------------------------
// Shift reduction over k, rows gathered per warp (k contiguous or general
// stride).  out[b*rows + r] = extreme_k x[b,r,k] (+ x2).
template <bool MAXMODE, bool VEC>
__global__ void __launch_bounds__(256) shift_rows_warp(const float* __restrict__ x, const float* __restrict__ x2,
                                                       int64_t sb, int64_t sr, int64_t sk, int64_t batch,
                                                       int64_t rows, int64_t k, float* __restrict__ out) {
  const int64_t gw = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (gw >= batch * rows) return;
  const int64_t b = gw / rows, r = gw - b * rows;
  const int64_t base = b * sb + r * sr;
  const float* p = x + base;
  const float* p2 = x2 ? x2 + base : nullptr;
  float acc = extreme_identity<MAXMODE>();
  if (VEC) {
    for (int64_t kk = 4 * lane; kk < k; kk += 128) {
      float4 v = ldg_nc_v4(p + kk);
      if (p2) {
        float4 w = ldg_nc_v4(p2 + kk);
        v.x += w.x; v.y += w.y; v.z += w.z; v.w += w.w;
      }
      acc = nan_extreme<MAXMODE>(acc, nan_extreme<MAXMODE>(nan_extreme<MAXMODE>(v.x, v.y), nan_extreme<MAXMODE>(v.z, v.w)));
    }
  } else {
    for (int64_t kk = lane; kk < k; kk += 32) {
      float v = ldg_nc(p + kk * sk);
      if (p2) v += ldg_nc(p2 + kk * sk);
      acc = nan_extreme<MAXMODE>(acc, v);
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc = nan_extreme<MAXMODE>(acc, __shfl_xor_sync(0xffffffffu, acc, o));
  if (lane == 0) out[gw] = acc;
}

// Shift reduction over k when the rows are the contiguous axis (sr == 1):
// block = 32 row-quads x 8 k-slices; grid = (ceil(rows/128), batch).
template <bool MAXMODE, bool VEC>
__global__ void __launch_bounds__(256) shift_rows_colwise(const float* __restrict__ x, const float* __restrict__ x2,
                                                          int64_t sb, int64_t sk, int64_t rows, int64_t k,
                                                          float* __restrict__ out) {
  __shared__ float4 red[8][32];
  const int64_t b = blockIdx.y;
  const int64_t r0 = ((int64_t)blockIdx.x * 32 + threadIdx.x) * 4;
  const int ks = threadIdx.y;
  const float* p = x + b * sb + r0;
  const float* p2 = x2 ? x2 + b * sb + r0 : nullptr;
  const float id = extreme_identity<MAXMODE>();
  float4 acc = make_float4(id, id, id, id);
  const int64_t valid = rows - r0;
  if (valid > 0) {
    for (int64_t kk = ks; kk < k; kk += 8) {
      float4 v;
      if (VEC) {
        v = ldg_nc_v4(p + kk * sk);
        if (p2) {
          float4 w = ldg_nc_v4(p2 + kk * sk);
          v.x += w.x; v.y += w.y; v.z += w.z; v.w += w.w;
        }
      } else {
        const float* q = p + kk * sk;
        const float* q2 = p2 ? p2 + kk * sk : nullptr;
        v.x = ldg_nc(q) + (q2 ? ldg_nc(q2) : 0.0f);
        v.y = valid > 1 ? ldg_nc(q + 1) + (q2 ? ldg_nc(q2 + 1) : 0.0f) : id;
        v.z = valid > 2 ? ldg_nc(q + 2) + (q2 ? ldg_nc(q2 + 2) : 0.0f) : id;
        v.w = valid > 3 ? ldg_nc(q + 3) + (q2 ? ldg_nc(q2 + 3) : 0.0f) : id;
      }
      acc.x = nan_extreme<MAXMODE>(acc.x, v.x);
      acc.y = nan_extreme<MAXMODE>(acc.y, v.y);
      acc.z = nan_extreme<MAXMODE>(acc.z, v.z);
      acc.w = nan_extreme<MAXMODE>(acc.w, v.w);
    }
  }
  red[ks][threadIdx.x] = acc;
  __syncthreads();
  if (ks == 0 && valid > 0) {
#pragma unroll
    for (int j = 1; j < 8; ++j) {
      float4 v = red[j][threadIdx.x];
      acc.x = nan_extreme<MAXMODE>(acc.x, v.x);
      acc.y = nan_extreme<MAXMODE>(acc.y, v.y);
      acc.z = nan_extreme<MAXMODE>(acc.z, v.z);
      acc.w = nan_extreme<MAXMODE>(acc.w, v.w);
    }
    float* o = out + b * rows + r0;
    o[0] = acc.x;
    if (valid > 1) o[1] = acc.y;
    if (valid > 2) o[2] = acc.z;
    if (valid > 3) o[3] = acc.w;
  }
}

// ---------------------------------------------------------------------------
// Softmax.  torch's CPU softmax (the reference executor) computes
// exp(x - max) * (1 / sum); the same formula is used here.
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = nan_extreme<true>(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Block-wide reduction for blocks of kThreads (multiple of 32).
template <int kThreads, bool IS_MAX>
__device__ __forceinline__ float block_reduce(float v, float* scratch) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  v = IS_MAX ? warp_max(v) : warp_sum(v);
  if (kThreads == 32) return v;
  __syncthreads();
  if (lane == 0) scratch[warp] = v;
  __syncthreads();
  float r = (lane < kThreads / 32) ? scratch[lane] : (IS_MAX ? -INFINITY : 0.0f);
  r = IS_MAX ? warp_max(r) : warp_sum(r);
  return r;
}

// Row softmax with the whole row in registers: kThreads threads per row,
// each holding kQ float4 (row length <= kThreads*kQ*4; tail masked).
// kThreads == 32 processes blockDim.x/32 rows per block (one per warp).
template <int kThreads, int kQ, bool VEC>
__global__ void __launch_bounds__(kThreads == 32 ? 256 : kThreads)
    softmax_rows_reg(const float* __restrict__ x, float* __restrict__ y, int64_t rows, int64_t len, int log_out) {
  __shared__ float scratch[32];
  int64_t row;
  int tid;
  if (kThreads == 32) {
    row = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    tid = threadIdx.x & 31;
    if (row >= rows) return;
  } else {
    row = blockIdx.x;
    tid = threadIdx.x;
  }
  const float* px = x + row * len;
  float* py = y + row * len;
  float4 v[kQ];
  float m = -INFINITY;
#pragma unroll
  for (int q = 0; q < kQ; ++q) {
    const int64_t i = 4 * ((int64_t)q * kThreads + tid);
    if (VEC) {
      v[q] = (i < len) ? ldg_nc_v4(px + i) : make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
    } else {
      v[q].x = (i < len) ? ldg_nc(px + i) : -INFINITY;
      v[q].y = (i + 1 < len) ? ldg_nc(px + i + 1) : -INFINITY;
      v[q].z = (i + 2 < len) ? ldg_nc(px + i + 2) : -INFINITY;
      v[q].w = (i + 3 < len) ? ldg_nc(px + i + 3) : -INFINITY;
    }
    m = nan_extreme<true>(m, nan_extreme<true>(nan_extreme<true>(v[q].x, v[q].y), nan_extreme<true>(v[q].z, v[q].w)));
  }
  m = block_reduce<kThreads, true>(m, scratch);
  float s = 0.0f;
#pragma unroll
  for (int q = 0; q < kQ; ++q) {
    const int64_t i = 4 * ((int64_t)q * kThreads + tid);
    // masked lanes are skipped (they hold -inf)
    const float ex = (i < len) ? expf(v[q].x - m) : 0.0f;
    const float ey = (i + 1 < len) ? expf(v[q].y - m) : 0.0f;
    const float ez = (i + 2 < len) ? expf(v[q].z - m) : 0.0f;
    const float ew = (i + 3 < len) ? expf(v[q].w - m) : 0.0f;
    s += (ex + ey) + (ez + ew);
  }
  if (kThreads != 32) __syncthreads();
  s = block_reduce<kThreads, false>(s, scratch);
  const float inv = 1.0f / s;
  // log softmax = x - (max + log(sum))
  const float lse = m + logf(s);
#pragma unroll
  for (int q = 0; q < kQ; ++q) {
    const int64_t i = 4 * ((int64_t)q * kThreads + tid);
    float4 o;
    if (log_out) {
      o = make_float4(v[q].x - lse, v[q].y - lse, v[q].z - lse, v[q].w - lse);
    } else {
      o = make_float4(expf(v[q].x - m) * inv, expf(v[q].y - m) * inv, expf(v[q].z - m) * inv,
                      expf(v[q].w - m) * inv);
    }
    if (VEC) {
      if (i < len) stg_v4(py + i, o);
    } else {
      if (i < len) py[i] = o.x;
      if (i + 1 < len) py[i + 1] = o.y;
      if (i + 2 < len) py[i + 2] = o.z;
      if (i + 3 < len) py[i + 3] = o.w;
    }
  }
}

// Short rows (len <= 4 * G <= 64, 16-byte aligned): G lanes per row, one float4 each, so that a
// warp holds 32 / G rows (the circuit's sum-layer weights are rows of 64).  The arithmetic is
// softmax_rows_reg<32, 1>'s: the lanes it leaves at -inf add exact zeros to its sums, and its
// butterfly over 32 lanes combines the G live lanes in this kernel's order, so the results are
// the same bit for bit.
template <int G>
__global__ void __launch_bounds__(256) softmax_rows_group(const float* __restrict__ x, float* __restrict__ y,
                                                          int64_t rows, int64_t len, int log_out) {
  static_assert(G >= 1 && G <= 16 && (G & (G - 1)) == 0, "G");
  const int64_t row = ((int64_t)blockIdx.x * 256 + threadIdx.x) / G;
  const int lane = threadIdx.x % G;
  // the lanes of this row's group (groups never straddle a warp)
  const unsigned gmask = (G == 32 ? 0xffffffffu : ((1u << G) - 1u)) << ((threadIdx.x & 31) / G * G);
  if (row >= rows) return;  // whole groups leave together
  const float* px = x + row * len;
  float* py = y + row * len;
  const int64_t i = 4 * lane;
  const float4 v = i < len ? ldg_nc_v4(px + i) : make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
  float m = nan_extreme<true>(nan_extreme<true>(v.x, v.y), nan_extreme<true>(v.z, v.w));
#pragma unroll
  for (int o = G / 2; o > 0; o >>= 1) m = nan_extreme<true>(m, __shfl_xor_sync(gmask, m, o));
  const float ex = i < len ? expf(v.x - m) : 0.0f;
  const float ey = i + 1 < len ? expf(v.y - m) : 0.0f;
  const float ez = i + 2 < len ? expf(v.z - m) : 0.0f;
  const float ew = i + 3 < len ? expf(v.w - m) : 0.0f;
  float s = (ex + ey) + (ez + ew);
#pragma unroll
  for (int o = G / 2; o > 0; o >>= 1) s += __shfl_xor_sync(gmask, s, o);
  const float inv = 1.0f / s;
  const float lse = m + logf(s);
  if (i < len) {
    float4 o;
    if (log_out)
      o = make_float4(v.x - lse, v.y - lse, v.z - lse, v.w - lse);
    else
      o = make_float4(expf(v.x - m) * inv, expf(v.y - m) * inv, expf(v.z - m) * inv, expf(v.w - m) * inv);
    stg_v4(py + i, o);
  }
}

// Softmax over the middle axis of (outer, len, inner) when one outer slice (len x inner values,
// at most kSlabMaxFloats) fits in shared memory and inner divides 256: one CTA per outer index
// stages the slice with coalesced 16-byte loads, 256 / inner threads reduce each column
// (max, then the sum of exp(x - max)), and the outputs leave coalesced.  The categorical input
// table of a circuit (variables, 256 states, units) normalises over its states this way.
constexpr int kSlabMaxFloats = 24576;  // 96 KB
__global__ void __launch_bounds__(256) softmax_slab(const float* __restrict__ x, float* __restrict__ y, int64_t len,
                                                    int inner, int log_out) {
  extern __shared__ __align__(16) float slab[];  // [len][inner], then [256] partials, [2][inner] stats
  float* part = slab + len * inner;
  float* stat_m = part + 256;
  float* stat_s = stat_m + inner;
  const int t = threadIdx.x;
  const int64_t n = len * inner;  // a multiple of 4
  const float* px = x + blockIdx.x * n;
  float* py = y + blockIdx.x * n;
  for (int64_t i = 4 * t; i < n; i += 1024) *(float4*)(slab + i) = ldg_nc_v4(px + i);
  __syncthreads();
  const int c = t % inner, p = t / inner, P = 256 / inner;
  float m = -INFINITY;
  for (int64_t a = p; a < len; a += P) m = nan_extreme<true>(m, slab[a * inner + c]);
  part[t] = m;
  __syncthreads();
  if (t < inner) {
    float mm = part[t];
    for (int q = 1; q < P; ++q) mm = nan_extreme<true>(mm, part[q * inner + t]);
    stat_m[t] = mm;
  }
  __syncthreads();
  m = stat_m[c];
  float sum = 0.0f;
  for (int64_t a = p; a < len; a += P) sum += expf(slab[a * inner + c] - m);
  part[t] = sum;
  __syncthreads();
  if (t < inner) {
    float ss = part[t];
    for (int q = 1; q < P; ++q) ss += part[q * inner + t];
    stat_s[t] = ss;
  }
  __syncthreads();
  for (int64_t i = 4 * t; i < n; i += 1024) {
    const float4 v = *(const float4*)(slab + i);
    const int c0 = (int)(i % inner);  // inner % 4 == 0: the quad lies in one row
    float r[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float mj = stat_m[c0 + j], sj = stat_s[c0 + j];
      r[j] = log_out ? r[j] - (mj + logf(sj)) : expf(r[j] - mj) * (1.0f / sj);
    }
    stg_v4(py + i, make_float4(r[0], r[1], r[2], r[3]));
  }
}

// Row softmax for 16384 < len <= 32768 (16-byte aligned rows): persistent CTAs of 1024
// threads, one row in registers (8 float4 per thread, the element mapping and arithmetic of
// softmax_rows_reg<1024, 8>, so the results are identical) while a bulk copy brings the
// CTA's next row into shared memory.  softmax_rows_reg holds one row per SM with its load
// latency exposed; here the next row's transfer overlaps the reductions and stores.
template <int kQ>
__global__ void __launch_bounds__(1024, 1)
    softmax_rows_prefetch(const float* __restrict__ x, float* __restrict__ y, int64_t rows, int64_t len, int log_out) {
  constexpr int kThreads = 1024;
  extern __shared__ __align__(16) uint8_t row_buf[];  // len floats
  __shared__ float scratch[32];
  __shared__ uint64_t full;
  __shared__ int abort_flag;
  const int tid = threadIdx.x;
  const uint32_t buf = smem_u32(row_buf);
  const uint32_t bytes = (uint32_t)(len * 4);
  ArmedCopies copies{0u, 0u};  // thread 0's last row copy, drained after an abort
  uint32_t fetches = 0;
  // the row's bulk copy, in pieces of at most 32 KB (16-byte multiples)
  auto fetch = [&](int64_t row) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(&full)), "r"(bytes) : "memory");
    copies.note(0, fetches++);
    for (uint32_t off = 0; off < bytes; off += 32768) {
      const uint32_t piece = bytes - off < 32768 ? bytes - off : 32768;
      asm volatile(
          "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(buf + off),
          "l"(x + row * len + off / 4), "r"(piece), "r"(smem_u32(&full))
          : "memory");
    }
  };
  if (tid == 0) {
    mbar_init(&full, 1);
    abort_flag = 0;
    fence_mbarrier_init();
  }
  __syncthreads();
  if (tid == 0 && (int64_t)blockIdx.x < rows) fetch(blockIdx.x);
  uint32_t phase = 0;
  for (int64_t row = blockIdx.x; row < rows; row += gridDim.x, phase ^= 1) {
    // the block leaves together (block barriers follow) if any thread's wait ran out
    if (!__syncthreads_and(mbar_wait(&full, phase, kSiteSoftmax, &abort_flag))) break;
    float4 v[kQ];
    float m = -INFINITY;
#pragma unroll
    for (int q = 0; q < kQ; ++q) {
      const int64_t i = 4 * ((int64_t)q * kThreads + tid);
      if (i < len) {
        asm volatile("ld.shared.v4.f32 {%0,%1,%2,%3}, [%4];"
                     : "=f"(v[q].x), "=f"(v[q].y), "=f"(v[q].z), "=f"(v[q].w)
                     : "r"(buf + (uint32_t)(i * 4)));
      } else {
        v[q] = make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
      }
      m = nan_extreme<true>(m, nan_extreme<true>(nan_extreme<true>(v[q].x, v[q].y), nan_extreme<true>(v[q].z, v[q].w)));
    }
    m = block_reduce<kThreads, true>(m, scratch);  // its barriers also order every read of the buffer
    if (tid == 0 && row + gridDim.x < rows) {
      fence_proxy_async_smem();
      fetch(row + gridDim.x);
    }
    float s = 0.0f;
#pragma unroll
    for (int q = 0; q < kQ; ++q) {
      const int64_t i = 4 * ((int64_t)q * kThreads + tid);
      const float ex = (i < len) ? expf(v[q].x - m) : 0.0f;
      const float ey = (i + 1 < len) ? expf(v[q].y - m) : 0.0f;
      const float ez = (i + 2 < len) ? expf(v[q].z - m) : 0.0f;
      const float ew = (i + 3 < len) ? expf(v[q].w - m) : 0.0f;
      s += (ex + ey) + (ez + ew);
    }
    __syncthreads();
    s = block_reduce<kThreads, false>(s, scratch);
    const float inv = 1.0f / s;
    const float lse = m + logf(s);
    float* py = y + row * len;
#pragma unroll
    for (int q = 0; q < kQ; ++q) {
      const int64_t i = 4 * ((int64_t)q * kThreads + tid);
      float4 o;
      if (log_out) {
        o = make_float4(v[q].x - lse, v[q].y - lse, v[q].z - lse, v[q].w - lse);
      } else {
        o = make_float4(expf(v[q].x - m) * inv, expf(v[q].y - m) * inv, expf(v[q].z - m) * inv,
                        expf(v[q].w - m) * inv);
      }
      if (i < len) stg_v4(py + i, o);
    }
    __syncthreads();  // scratch is reused by the next row's reductions
  }
  // after an abort the next row's copy may still be landing in this CTA's shared memory
  if (*(volatile int*)&abort_flag && tid == 0) copies.drain(&full, &abort_flag);
}

// Softmax of rows too long for registers: one block per row, three streaming
// passes (max, sum, write).
__global__ void __launch_bounds__(1024) softmax_rows_stream(const float* __restrict__ x, float* __restrict__ y,
                                                            int64_t len, int log_out) {
  __shared__ float scratch[32];
  const float* px = x + (int64_t)blockIdx.x * len;
  float* py = y + (int64_t)blockIdx.x * len;
  float m = -INFINITY;
  for (int64_t i = threadIdx.x; i < len; i += 1024) m = nan_extreme<true>(m, ldg_nc(px + i));
  m = block_reduce<1024, true>(m, scratch);
  float s = 0.0f;
  for (int64_t i = threadIdx.x; i < len; i += 1024) s += expf(ldg_nc(px + i) - m);
  __syncthreads();
  s = block_reduce<1024, false>(s, scratch);
  const float inv = 1.0f / s, lse = m + logf(s);
  for (int64_t i = threadIdx.x; i < len; i += 1024) {
    const float v = ldg_nc(px + i);
    py[i] = log_out ? v - lse : expf(v - m) * inv;
  }
}

// Softmax over a strided middle axis: one thread per (outer, inner) fibre,
// consecutive threads on consecutive inner positions (coalesced).
__global__ void __launch_bounds__(256) softmax_strided(const float* __restrict__ x, float* __restrict__ y,
                                                       int64_t outer, int64_t len, int64_t inner, int log_out) {
  const int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (g >= outer * inner) return;
  const int64_t o = g / inner, in = g - o * inner;
  const float* px = x + o * len * inner + in;
  float* py = y + o * len * inner + in;
  float m = -INFINITY;
  for (int64_t a = 0; a < len; ++a) m = nan_extreme<true>(m, ldg_nc(px + a * inner));
  float s = 0.0f;
  for (int64_t a = 0; a < len; ++a) s += expf(ldg_nc(px + a * inner) - m);
  const float inv = 1.0f / s, lse = m + logf(s);
  for (int64_t a = 0; a < len; ++a) {
    const float v = ldg_nc(px + a * inner);
    py[a * inner] = log_out ? v - lse : expf(v - m) * inv;
  }
}

// ---------------------------------------------------------------------------
// Log-space broadcast addition (contraction-free einsum / multiply).
struct NdShape {
  int64_t shape[6];
  int64_t as[6];
  int64_t bs[6];
  int ndim;
};

__global__ void __launch_bounds__(256) log_add_nd(const float* __restrict__ a, const float* __restrict__ b,
                                                  float* __restrict__ y, NdShape s, int64_t total, float sign) {
  for (int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; g < total; g += (int64_t)gridDim.x * blockDim.x) {
    int64_t rem = g, oa = 0, ob = 0;
    for (int d = s.ndim - 1; d >= 0; --d) {
      const int64_t idx = rem % s.shape[d];
      rem /= s.shape[d];
      oa += idx * s.as[d];
      ob += idx * s.bs[d];
    }
    y[g] = a[oa] + sign * b[ob];
  }
}

__global__ void __launch_bounds__(256) log_add_contig4(const float4* __restrict__ a, const float4* __restrict__ b,
                                                       float4* __restrict__ y, int64_t n4, float sign) {
  for (int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; g < n4; g += (int64_t)gridDim.x * blockDim.x) {
    float4 u, v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.f32 {%0,%1,%2,%3}, [%4];"
                 : "=f"(u.x), "=f"(u.y), "=f"(u.z), "=f"(u.w)
                 : "l"(a + g));
    asm volatile("ld.global.nc.L1::no_allocate.v4.f32 {%0,%1,%2,%3}, [%4];"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                 : "l"(b + g));
    y[g] = make_float4(u.x + sign * v.x, u.y + sign * v.y, u.z + sign * v.z, u.w + sign * v.w);
  }
}

// ---------------------------------------------------------------------------
// Categorical gather: y[f,b,:] = table[f, pixels[b*ps + var[f]], :].
// One thread per float4 of an output row (units % 4 == 0 on this path).
__global__ void __launch_bounds__(256) categorical_gather4(const float* __restrict__ table,
                                                           const uint8_t* __restrict__ pixels, int64_t ps,
                                                           const int32_t* __restrict__ var_of_fold,
                                                           float* __restrict__ y, int64_t folds, int64_t states,
                                                           int64_t units, int64_t batch) {
  const int64_t uq = units >> 2;
  const int64_t total = folds * batch * uq;
  for (int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; g < total; g += (int64_t)gridDim.x * blockDim.x) {
    const int64_t q = g % uq;
    const int64_t row = g / uq;  // f*batch + b
    const int64_t f = row / batch, b = row - f * batch;
    int64_t v = var_of_fold ? (int64_t)__ldg(var_of_fold + f) : f;
    if (v < 0 || v >= ps) {
      record_bad_index(kSiteGatherState);
      v = 0;
    }
    int64_t s = (int64_t)__ldg(pixels + b * ps + v);
    if (s >= states) {
      record_bad_index(kSiteGatherState);
      s = states - 1;
    }
    const float4 t = ldg_nc_v4(table + (f * states + s) * units + 4 * q);
    stg_v4(y + row * units + 4 * q, t);
  }
}

__global__ void __launch_bounds__(256) categorical_gather1(const float* __restrict__ table,
                                                           const uint8_t* __restrict__ pixels, int64_t ps,
                                                           const int32_t* __restrict__ var_of_fold,
                                                           float* __restrict__ y, int64_t folds, int64_t states,
                                                           int64_t units, int64_t batch) {
  const int64_t total = folds * batch * units;
  for (int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; g < total; g += (int64_t)gridDim.x * blockDim.x) {
    const int64_t u = g % units;
    const int64_t row = g / units;
    const int64_t f = row / batch, b = row - f * batch;
    int64_t v = var_of_fold ? (int64_t)__ldg(var_of_fold + f) : f;
    if (v < 0 || v >= ps) {
      record_bad_index(kSiteGatherState);
      v = 0;
    }
    int64_t s = (int64_t)__ldg(pixels + b * ps + v);
    if (s >= states) {
      record_bad_index(kSiteGatherState);
      s = states - 1;
    }
    y[g] = __ldg(table + (f * states + s) * units + u);
  }
}

// Backward of the categorical gather: dt[f + off, pixels[b, var[f + off]], :] += g[f, b, :].
// One CTA per (fold, slice of the batch): the fold's (states, units) slice is accumulated in
// shared memory (one warp per sample row, lanes over the units), then added to global memory
// once.  g is (folds, batch, units) contiguous.  Bad indices are clamped and reported as in the
// forward gather.
__device__ __forceinline__ int64_t scatter_variable(const int32_t* var_of_fold, int64_t fold, int64_t ps) {
  int64_t v = var_of_fold ? (int64_t)__ldg(var_of_fold + fold) : fold;
  if (v < 0 || v >= ps) {
    record_bad_index(kSiteGatherState);
    v = 0;
  }
  return v;
}

__device__ __forceinline__ int64_t scatter_state(const uint8_t* pixels, int64_t b, int64_t ps, int64_t v, int64_t states) {
  int64_t s = (int64_t)__ldg(pixels + b * ps + v);
  if (s >= states) {
    record_bad_index(kSiteGatherState);
    s = states - 1;
  }
  return s;
}

__global__ void __launch_bounds__(256) categorical_scatter_smem(const float* __restrict__ g,
                                                                const uint8_t* __restrict__ pixels, int64_t ps,
                                                                const int32_t* __restrict__ var_of_fold,
                                                                float* __restrict__ dt, int64_t states, int64_t units,
                                                                int64_t batch, int64_t off, int64_t b_chunk) {
  extern __shared__ float acc[];  // states * units
  const int64_t f = blockIdx.x;
  const int64_t slice = states * units;
  for (int64_t i = threadIdx.x; i < slice; i += blockDim.x) acc[i] = 0.0f;
  __syncthreads();
  const int64_t v = scatter_variable(var_of_fold, f + off, ps);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t b0 = (int64_t)blockIdx.y * b_chunk;
  const int64_t b1 = b0 + b_chunk < batch ? b0 + b_chunk : batch;
  for (int64_t b = b0 + warp; b < b1; b += blockDim.x >> 5) {
    const int64_t st = scatter_state(pixels, b, ps, v, states);
    const float* row = g + (f * batch + b) * units;
    float* dst = acc + st * units;
    for (int64_t u = lane; u < units; u += 32) atomicAdd(dst + u, __ldg(row + u));
  }
  __syncthreads();
  float* out = dt + (f + off) * slice;
  for (int64_t i = threadIdx.x; i < slice; i += blockDim.x) {
    const float a = acc[i];
    if (a != 0.0f) atomicAdd(out + i, a);
  }
}

// The same with global atomics only, for a (states, units) slice larger than shared memory.
__global__ void __launch_bounds__(256) categorical_scatter_global(const float* __restrict__ g,
                                                                  const uint8_t* __restrict__ pixels, int64_t ps,
                                                                  const int32_t* __restrict__ var_of_fold,
                                                                  float* __restrict__ dt, int64_t folds,
                                                                  int64_t states, int64_t units, int64_t batch,
                                                                  int64_t off) {
  const int64_t total = folds * batch * units;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t u = i % units;
    const int64_t row = i / units;
    const int64_t f = row / batch, b = row - f * batch;
    const int64_t v = scatter_variable(var_of_fold, f + off, ps);
    const int64_t st = scatter_state(pixels, b, ps, v, states);
    atomicAdd(dt + ((f + off) * states + st) * units + u, __ldg(g + i));
  }
}


// ---------------------------------------------------------------------------
// Log-space reduction of one operand: y = log(sum_k exp(x - s)) + s with
// s = extreme_k x (two passes over the row; the second hits L1/L2).
template <bool MAXMODE, bool VEC>
__global__ void __launch_bounds__(256) lse_rows_warp(const float* __restrict__ x, int64_t sb, int64_t sr, int64_t sk,
                                                     int64_t batch, int64_t rows, int64_t k, float* __restrict__ y) {
  const int64_t gw = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (gw >= batch * rows) return;
  const int64_t b = gw / rows, r = gw - b * rows;
  const float* p = x + b * sb + r * sr;
  float m = extreme_identity<MAXMODE>();
  if (VEC) {
    for (int64_t kk = 4 * lane; kk < k; kk += 128) {
      const float4 v = ldg_nc_v4(p + kk);
      m = nan_extreme<MAXMODE>(m, nan_extreme<MAXMODE>(nan_extreme<MAXMODE>(v.x, v.y), nan_extreme<MAXMODE>(v.z, v.w)));
    }
  } else {
    for (int64_t kk = lane; kk < k; kk += 32) m = nan_extreme<MAXMODE>(m, ldg_nc(p + kk * sk));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = nan_extreme<MAXMODE>(m, __shfl_xor_sync(0xffffffffu, m, o));
  float s = 0.0f;
  if (VEC) {
    for (int64_t kk = 4 * lane; kk < k; kk += 128) {
      const float4 v = ldg_nc_v4(p + kk);
      s += (expf(v.x - m) + expf(v.y - m)) + (expf(v.z - m) + expf(v.w - m));
    }
  } else {
    for (int64_t kk = lane; kk < k; kk += 32) s += expf(ldg_nc(p + kk * sk) - m);
  }
  s = warp_sum(s);
  if (lane == 0) y[gw] = logf(s) + m;
}

// Same reduction when the rows are the unit-stride axis (sr == 1).
template <bool MAXMODE>
__global__ void __launch_bounds__(256) lse_rows_colwise(const float* __restrict__ x, int64_t sb, int64_t sk,
                                                        int64_t rows, int64_t k, float* __restrict__ y) {
  __shared__ float red[8][32];
  const int64_t b = blockIdx.y;
  const int64_t r = (int64_t)blockIdx.x * 32 + threadIdx.x;
  const int ks = threadIdx.y;
  const bool valid = r < rows;
  const float* p = x + b * sb + r;
  float m = extreme_identity<MAXMODE>();
  if (valid)
    for (int64_t kk = ks; kk < k; kk += 8) m = nan_extreme<MAXMODE>(m, ldg_nc(p + kk * sk));
  red[ks][threadIdx.x] = m;
  __syncthreads();
  m = red[0][threadIdx.x];
#pragma unroll
  for (int j = 1; j < 8; ++j) m = nan_extreme<MAXMODE>(m, red[j][threadIdx.x]);
  __syncthreads();
  float s = 0.0f;
  if (valid)
    for (int64_t kk = ks; kk < k; kk += 8) s += expf(ldg_nc(p + kk * sk) - m);
  red[ks][threadIdx.x] = s;
  __syncthreads();
  if (ks == 0 && valid) {
    float t = 0.0f;
#pragma unroll
    for (int j = 0; j < 8; ++j) t += red[j][threadIdx.x];
    y[b * rows + r] = logf(t) + m;
  }
}

// ---------------------------------------------------------------------------
// Scalar extreme of one or two contiguous arrays (single block; these are the
// small tensors of log-space +/-), combined as extreme(extreme(a), extreme(b)).
template <bool MAXMODE>
__global__ void __launch_bounds__(1024) global_extreme2(const float* __restrict__ a, int64_t na,
                                                        const float* __restrict__ b, int64_t nb,
                                                        float* __restrict__ out) {
  __shared__ float scratch[32];
  float ma = extreme_identity<MAXMODE>(), mb = extreme_identity<MAXMODE>();
  for (int64_t i = threadIdx.x; i < na; i += 1024) ma = nan_extreme<MAXMODE>(ma, ldg_nc(a + i));
  for (int64_t i = threadIdx.x; i < nb; i += 1024) mb = nan_extreme<MAXMODE>(mb, ldg_nc(b + i));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    ma = nan_extreme<MAXMODE>(ma, __shfl_xor_sync(0xffffffffu, ma, o));
    mb = nan_extreme<MAXMODE>(mb, __shfl_xor_sync(0xffffffffu, mb, o));
  }
  __shared__ float scratch_b[32];
  if (lane == 0) {
    scratch[warp] = ma;
    scratch_b[warp] = mb;
  }
  __syncthreads();
  if (warp == 0) {
    ma = scratch[lane];
    mb = scratch_b[lane];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      ma = nan_extreme<MAXMODE>(ma, __shfl_xor_sync(0xffffffffu, ma, o));
      mb = nan_extreme<MAXMODE>(mb, __shfl_xor_sync(0xffffffffu, mb, o));
    }
    if (lane == 0) out[0] = nan_extreme<MAXMODE>(ma, mb);
  }
}

// y = log(exp(a - m) +/- exp(b - m)) + m with m = *shift, broadcast strides.
__global__ void __launch_bounds__(256) log_add_exp_nd(const float* __restrict__ a, const float* __restrict__ b,
                                                      float* __restrict__ y, NdShape s, int64_t total,
                                                      const float* __restrict__ shift, int subtract) {
  const float m = __ldg(shift);
  for (int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; g < total; g += (int64_t)gridDim.x * blockDim.x) {
    int64_t rem = g, oa = 0, ob = 0;
    for (int d = s.ndim - 1; d >= 0; --d) {
      const int64_t idx = rem % s.shape[d];
      rem /= s.shape[d];
      oa += idx * s.as[d];
      ob += idx * s.bs[d];
    }
    const float ea = expf(a[oa] - m), eb = expf(b[ob] - m);
    y[g] = logf(subtract ? ea - eb : ea + eb) + m;
  }
}

// ---------------------------------------------------------------------------
// Domain conversions.
template <int OP>
__global__ void __launch_bounds__(256) unary_map(const float* __restrict__ x, float* __restrict__ y, int64_t n) {
  for (int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; g < n; g += (int64_t)gridDim.x * blockDim.x) {
    const float v = x[g];
    y[g] = OP == 0 ? expf(v) : logf(v);
  }
}

template <int OP>
__global__ void __launch_bounds__(256) unary_map4(const float4* __restrict__ x, float4* __restrict__ y, int64_t n4) {
  for (int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; g < n4; g += (int64_t)gridDim.x * blockDim.x) {
    const float4 v = x[g];
    y[g] = OP == 0 ? make_float4(expf(v.x), expf(v.y), expf(v.z), expf(v.w))
                   : make_float4(logf(v.x), logf(v.y), logf(v.z), logf(v.w));
  }
}

// ---------------------------------------------------------------------------
// Scaled stability modes (sum / max / min fibre normalisation).  A value is
// a pair (normalized, log_scale) with raw = normalized * exp(log_scale) and
// one scale per last-axis fibre; these kernels are its glue.

// Elementwise ops over up to three broadcast operands (strides may be 0).
enum ElementwiseOp : int {
  kOpAdd = 0,       // a + b
  kOpSub = 1,       // a - b
  kOpMul = 2,       // a * b
  kOpDiv = 3,       // a / b
  kOpMax = 4,       // maximum(a, b), NaN-propagating
  kOpMin = 5,       // minimum(a, b), NaN-propagating
  kOpMulExp = 6,    // a * exp(b)            (a scaled pair back to raw)
  kOpLogAdd = 7,    // log(a) + b            (log of a scaled pair)
  kOpRescale = 8,   // a * exp(b - c)        (a pair brought to the common scale c)
  kNumElementwiseOps = 9
};

struct NdShape3 {
  int64_t shape[6];
  int64_t as[6];
  int64_t bs[6];
  int64_t cs[6];
  int ndim;
};

template <int OP>
__device__ __forceinline__ float elementwise_apply(float a, float b, float c) {
  if (OP == kOpAdd) return a + b;
  if (OP == kOpSub) return a - b;
  if (OP == kOpMul) return a * b;
  if (OP == kOpDiv) return a / b;
  if (OP == kOpMax) return (isnan(a) || a > b) ? a : b;
  if (OP == kOpMin) return (isnan(a) || a < b) ? a : b;
  if (OP == kOpMulExp) return a * expf(b);
  if (OP == kOpLogAdd) return logf(a) + b;
  return a * expf(b - c);
}

template <int OP>
__global__ void __launch_bounds__(256) elementwise_nd(const float* __restrict__ a, const float* __restrict__ b,
                                                      const float* __restrict__ c, float* __restrict__ y, NdShape3 s,
                                                      int64_t total) {
  for (int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; g < total; g += (int64_t)gridDim.x * blockDim.x) {
    int64_t rem = g, oa = 0, ob = 0, oc = 0;
    for (int d = s.ndim - 1; d >= 0; --d) {
      const int64_t idx = rem % s.shape[d];
      rem /= s.shape[d];
      oa += idx * s.as[d];
      ob += idx * s.bs[d];
      oc += idx * s.cs[d];
    }
    y[g] = elementwise_apply<OP>(a[oa], b ? b[ob] : 0.0f, c ? c[oc] : 0.0f);
  }
}

// One warp per row of the last axis: the index arithmetic of the leading axes
// is done once per row, the row itself is streamed (coalesced where the last
// axis is contiguous, a broadcast scale read once per row where its stride is 0).
template <int OP>
__global__ void __launch_bounds__(256) elementwise_rows(const float* __restrict__ a, const float* __restrict__ b,
                                                        const float* __restrict__ c, float* __restrict__ y, NdShape3 s,
                                                        int64_t rows, int64_t n) {
  const int lane = threadIdx.x & 31;
  const int last = s.ndim - 1;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  for (int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); row < rows; row += warps) {
    int64_t rem = row, oa = 0, ob = 0, oc = 0;
    for (int d = last - 1; d >= 0; --d) {
      const int64_t idx = rem % s.shape[d];
      rem /= s.shape[d];
      oa += idx * s.as[d];
      ob += idx * s.bs[d];
      oc += idx * s.cs[d];
    }
    float* py = y + row * n;
    for (int64_t j = lane; j < n; j += 32)
      py[j] = elementwise_apply<OP>(a[oa + j * s.as[last]], b ? b[ob + j * s.bs[last]] : 0.0f,
                                    c ? c[oc + j * s.cs[last]] : 0.0f);
  }
}

// All three operands dense and 16-byte aligned (same shape, no broadcast).
template <int OP>
__global__ void __launch_bounds__(256) elementwise_contig4(const float4* __restrict__ a, const float4* __restrict__ b,
                                                           const float4* __restrict__ c, float4* __restrict__ y,
                                                           int64_t n4) {
  for (int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; g < n4; g += (int64_t)gridDim.x * blockDim.x) {
    const float4 u = a[g];
    const float4 v = b ? b[g] : make_float4(0.f, 0.f, 0.f, 0.f);
    const float4 w = c ? c[g] : make_float4(0.f, 0.f, 0.f, 0.f);
    y[g] = make_float4(elementwise_apply<OP>(u.x, v.x, w.x), elementwise_apply<OP>(u.y, v.y, w.y),
                       elementwise_apply<OP>(u.z, v.z, w.z), elementwise_apply<OP>(u.w, v.w, w.w));
  }
}

// Leading (non-fibre) axes of a strided tensor: row index -> element offset.
struct RowIndexer {
  int64_t shape[6];
  int64_t stride[6];
  int ndim;
  __device__ __forceinline__ int64_t offset(int64_t row) const {
    int64_t off = 0;
    for (int d = ndim - 1; d >= 0; --d) {
      const int64_t idx = row % shape[d];
      row /= shape[d];
      off += idx * stride[d];
    }
    return off;
  }
};

// Fibre statistics and the normalised fibre, one warp per fibre.
enum FiberKind : int {
  kFiberSum = 0,  // total = sum;  normalized = x / total; log_scale = log(total)
  kFiberMax = 1,  // total = max;  same
  kFiberMin = 2,  // total = min;  same
  kFiberExp = 3,  // exp of a raw fibre: log_scale = max x; normalized = exp(x - log_scale)
  kFiberLse = 4,  // exp of a log-domain fibre, sum-normalised: log_scale = logsumexp x; normalized = exp(x - log_scale)
};

template <int KIND>
__global__ void __launch_bounds__(256) fiber_rows(const float* __restrict__ x, RowIndexer ri, int64_t rows, int64_t n,
                                                  int64_t sn, float* __restrict__ normalized,
                                                  float* __restrict__ log_scale) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  for (int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); row < rows; row += warps) {
    const float* px = x + ri.offset(row);
    float acc = KIND == kFiberSum ? 0.0f : (KIND == kFiberMin ? INFINITY : -INFINITY);
    for (int64_t j = lane; j < n; j += 32) {
      const float v = px[j * sn];
      if (KIND == kFiberSum) acc += v;
      else acc = nan_extreme<KIND != kFiberMin>(acc, v);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float other = __shfl_xor_sync(0xffffffffu, acc, o);
      acc = KIND == kFiberSum ? acc + other : nan_extreme<KIND != kFiberMin>(acc, other);
    }
    float total = acc;
    if (KIND == kFiberLse) {
      float s = 0.0f;
      for (int64_t j = lane; j < n; j += 32) s += expf(px[j * sn] - acc);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
      total = isinf(acc) ? acc : acc + logf(s);
    }
    float* py = normalized + row * n;
    for (int64_t j = lane; j < n; j += 32) {
      const float v = px[j * sn];
      py[j] = (KIND == kFiberExp || KIND == kFiberLse) ? expf(v - total) : v / total;
    }
    if (lane == 0) log_scale[row] = (KIND == kFiberExp || KIND == kFiberLse) ? total : logf(total);
  }
}

// Plain reduction over k of a (batch, rows, k) strided view: sum, max or min.
template <int KIND>
__global__ void __launch_bounds__(256) reduce_rows(const float* __restrict__ x, int64_t sb, int64_t sr, int64_t sk,
                                                   int64_t batch, int64_t rows, int64_t k, float* __restrict__ y) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  for (int64_t g = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); g < batch * rows; g += warps) {
    const float* px = x + (g / rows) * sb + (g % rows) * sr;
    float acc = KIND == kFiberSum ? 0.0f : (KIND == kFiberMin ? INFINITY : -INFINITY);
    for (int64_t j = lane; j < k; j += 32) {
      const float v = px[j * sk];
      if (KIND == kFiberSum) acc += v;
      else acc = nan_extreme<KIND != kFiberMin>(acc, v);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float other = __shfl_xor_sync(0xffffffffu, acc, o);
      acc = KIND == kFiberSum ? acc + other : nan_extreme<KIND != kFiberMin>(acc, other);
    }
    if (lane == 0) y[g] = acc;
  }
}

// The same reduction when the outputs of a batch entry are contiguous (sr == 1, rows <= 256) and
// k is strided (a leading axis): one 1024-thread block per batch entry, thread t on column
// t % rows and on the k-slice t / rows (k = slice, slice + S, ... for S = 1024 / rows slices), so
// that a warp's loads cover consecutive columns; the S partials of a column are then combined in
// slice order (deterministic).
template <int KIND>
__global__ void __launch_bounds__(1024) reduce_cols(const float* __restrict__ x, int64_t sb, int64_t sk, int64_t rows,
                                                    int64_t k, float* __restrict__ y) {
  __shared__ float part[1024];
  const int64_t bb = blockIdx.x;
  const int c = (int)(threadIdx.x % rows);
  const int slice = (int)(threadIdx.x / rows);
  const int slices = (int)(1024 / rows);
  float acc = KIND == kFiberSum ? 0.0f : (KIND == kFiberMin ? INFINITY : -INFINITY);
  if (slice < slices) {
    const float* px = x + bb * sb + c;
#pragma unroll 8
    for (int64_t j = slice; j < k; j += slices) {
      const float v = __ldg(px + j * sk);
      if (KIND == kFiberSum) acc += v;
      else acc = nan_extreme<KIND != kFiberMin>(acc, v);
    }
  }
  part[threadIdx.x] = acc;
  __syncthreads();
  if (threadIdx.x < rows) {
    float r = part[threadIdx.x];
    for (int s2 = 1; s2 < slices; ++s2) {
      const float v = part[s2 * rows + threadIdx.x];
      r = KIND == kFiberSum ? r + v : nan_extreme<KIND != kFiberMin>(r, v);
    }
    y[bb * rows + threadIdx.x] = r;
  }
}

// y (cols, rows) = x (rows, cols)^T for bytes, x with row stride s_row: 32 x 32 tiles through
// shared memory, 32 consecutive bytes per warp access on both sides.
__global__ void __launch_bounds__(256) transpose_u8(const uint8_t* __restrict__ x, int64_t rows, int64_t cols,
                                                    int64_t s_row, uint8_t* __restrict__ y) {
  __shared__ uint8_t tile[32][33];
  const int64_t r0 = (int64_t)blockIdx.y * 32, c0 = (int64_t)blockIdx.x * 32;
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int64_t r = r0 + ty + 8 * i, c = c0 + tx;
    if (r < rows && c < cols) tile[ty + 8 * i][tx] = x[r * s_row + c];
  }
  __syncthreads();
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int64_t c = c0 + ty + 8 * i, r = r0 + tx;
    if (r < rows && c < cols) y[c * rows + r] = tile[tx][ty + 8 * i];
  }
}

}  // namespace xe
