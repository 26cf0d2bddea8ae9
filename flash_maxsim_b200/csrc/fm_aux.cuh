// Training backward, INT8 quantisation and the bounded-wait self test.
//
// Backward of MaxSim given the forward's argmax a[n, b, q] (token index of the
// row maximum, -1 for an empty document):
//   dQ[n, q, :] = sum_b g[n, b] * D[b, a[n, b, q], :]
//   dD[b, t, :] = sum_{(n, q): a[n, b, q] == t} g[n, b] * Q[n, q, :]
// Same result as the reference's `_maxsim_bwd_dQ_kernel` /
// `_maxsim_bwd_dD_kernel` (flash_maxsim/flash_maxsim.py:153-188), but
// deterministic: every output row is accumulated in fp32 in a fixed order by
// exactly one warp (no atomics), then rounded to fp16 once.
//
// quantize: per-token affine uint8 exactly as flash_maxsim/flash_maxsim_quant.py:11-28
// (fp32 min/max, scale = max((max - min) / 255, 1e-8), u = clamp(rint((x - min) / scale)),
// IEEE division, round-half-even), scale and min rounded to fp16.
#pragma once

#include <cstdint>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include "fm_ptx.cuh"

namespace fm {

constexpr int kBwdThreads = 256;
constexpr int kMaxSeg = 8;  // 256-element segments per row => d <= 2048

// 8 consecutive fp16 -> fp32 accumulate with weight g
__device__ __forceinline__ void fma8(float (&acc)[8], const uint4 raw, float g) {
  const __half2* h = reinterpret_cast<const __half2*>(&raw);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float2 f = __half22float2(h[j]);
    acc[2 * j] = fmaf(g, f.x, acc[2 * j]);
    acc[2 * j + 1] = fmaf(g, f.y, acc[2 * j + 1]);
  }
}

__device__ __forceinline__ uint4 pack8(const float (&acc)[8]) {
  uint4 r;
  __half2* h = reinterpret_cast<__half2*>(&r);
#pragma unroll
  for (int j = 0; j < 4; ++j) h[j] = __floats2half2_rn(acc[2 * j], acc[2 * j + 1]);
  return r;
}

// dQ: grid (Nq, ceil(Lq / 8)), 8 warps; warp = one query row, lanes span d
// (8 fp16 per lane per 256-element segment).  Loops over documents in order.
__global__ void __launch_bounds__(kBwdThreads) maxsim_bwd_dq_kernel(
    const __half* __restrict__ D, const int32_t* __restrict__ am, const float* __restrict__ g,
    __half* __restrict__ dQ, int Nq, int B, int Lq, int Ld, int d, int shared) {
  const int n = blockIdx.x;
  const int q = blockIdx.y * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (q >= Lq) return;
  const int nseg = (d + 255) / 256;
  float acc[kMaxSeg][8];
#pragma unroll
  for (int s = 0; s < kMaxSeg; ++s)
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[s][j] = 0.f;

  for (int b0 = 0; b0 < B; b0 += 32) {
    const int bl = b0 + lane;
    int t = -1;
    float gv = 0.f;
    if (bl < B) {
      const size_t pair = static_cast<size_t>(n) * B + bl;
      t = __ldg(am + pair * Lq + q);
      gv = __ldg(g + pair);
    }
    const int nb = min(32, B - b0);
    for (int i = 0; i < nb; ++i) {
      const int ti = __shfl_sync(0xffffffffu, t, i);
      const float gi = __shfl_sync(0xffffffffu, gv, i);
      if (ti < 0) continue;
      const size_t doc = shared ? static_cast<size_t>(b0 + i) : static_cast<size_t>(n) * B + b0 + i;
      const __half* row = D + (doc * Ld + ti) * static_cast<size_t>(d);
#pragma unroll
      for (int s = 0; s < kMaxSeg; ++s) {
        if (s < nseg) {
          const int k = s * 256 + lane * 8;
          if (k < d) fma8(acc[s], __ldg(reinterpret_cast<const uint4*>(row + k)), gi);
        }
      }
    }
  }
  __half* out = dQ + (static_cast<size_t>(n) * Lq + q) * d;
#pragma unroll
  for (int s = 0; s < kMaxSeg; ++s) {
    if (s < nseg) {
      const int k = s * 256 + lane * 8;
      if (k < d) *reinterpret_cast<uint4*>(out + k) = pack8(acc[s]);
    }
  }
}

// dD: one CTA per document.  The (query, row) entries that picked a token of
// this document are bucketed by token with a stable counting sort in shared
// memory, then each warp writes whole token rows (zeros for untouched rows).
// Shared memory: cnt[Ld + 1] + order[Nq * Lq] ints + g[Nq] floats.
__global__ void __launch_bounds__(kBwdThreads) maxsim_bwd_dd_kernel(
    const __half* __restrict__ Q, const int32_t* __restrict__ am, const float* __restrict__ g,
    __half* __restrict__ dD, int Nq, int B, int Lq, int Ld, int d) {
  extern __shared__ int sm_i[];
  const int b = blockIdx.x;
  const int E = Nq * Lq;
  int* cnt = sm_i;                     // Ld + 1
  int* order = sm_i + (Ld + 1);        // E
  float* gs = reinterpret_cast<float*>(order + E);  // Nq
  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;

  for (int t = tid; t <= Ld; t += kBwdThreads) cnt[t] = 0;
  for (int n = tid; n < Nq; n += kBwdThreads) gs[n] = __ldg(g + static_cast<size_t>(n) * B + b);
  __syncthreads();
  auto entry_tok = [&](int e) -> int {
    const int n = e / Lq, q = e - (e / Lq) * Lq;
    const int t = __ldg(am + (static_cast<size_t>(n) * B + b) * Lq + q);
    return (t >= 0 && t < Ld) ? t : -1;
  };
  for (int e = tid; e < E; e += kBwdThreads) {
    const int t = entry_tok(e);
    if (t >= 0) atomicAdd(&cnt[t], 1);
  }
  __syncthreads();
  // exclusive scan of cnt[0..Ld] by warp 0 (each lane a contiguous range)
  if (warp == 0) {
    const int per = (Ld + 1 + 31) / 32;
    const int lo = lane * per, hi = min(Ld + 1, lo + per);
    int s = 0;
    for (int t = lo; t < hi; ++t) s += cnt[t];
    int incl = s;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int v = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += v;
    }
    int run = incl - s;
    for (int t = lo; t < hi; ++t) {
      const int c = cnt[t];
      cnt[t] = run;
      run += c;
    }
    __syncwarp();
    // stable scatter: entries in increasing order, ties by lane order
    for (int e0 = 0; e0 < E; e0 += 32) {
      const int e = e0 + lane;
      const int t = (e < E) ? entry_tok(e) : -1;
      const unsigned grp = __match_any_sync(0xffffffffu, t);
      if (t >= 0) {
        const int rank = __popc(grp & ((1u << lane) - 1u));
        order[cnt[t] + rank] = e;
      }
      __syncwarp();
      if (t >= 0 && lane == __ffs(grp) - 1) cnt[t] += __popc(grp);
      __syncwarp();
    }
  }
  __syncthreads();
  // bucket t = [t == 0 ? 0 : cnt[t-1], cnt[t])
  const int nseg = (d + 255) / 256;
  for (int t = warp; t < Ld; t += kBwdThreads / 32) {
    const int beg = t == 0 ? 0 : cnt[t - 1];
    const int end = cnt[t];
    __half* out = dD + (static_cast<size_t>(b) * Ld + t) * d;
    for (int s = 0; s < nseg; ++s) {
      const int k = s * 256 + lane * 8;
      float acc[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[j] = 0.f;
      for (int p = beg; p < end; ++p) {
        const int e = order[p];
        const int n = e / Lq;
        if (k < d)
          fma8(acc, __ldg(reinterpret_cast<const uint4*>(Q + static_cast<size_t>(e) * d + k)), gs[n]);
      }
      if (k < d) *reinterpret_cast<uint4*>(out + k) = pack8(acc);
    }
  }
}

// 8 consecutive elements of a row as fp32 (exact widening)
__device__ __forceinline__ void load8(const __half* p, float (&f)[8]) {
  const uint4 raw = __ldg(reinterpret_cast<const uint4*>(p));
  const __half2* h = reinterpret_cast<const __half2*>(&raw);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float2 v = __half22float2(h[j]);
    f[2 * j] = v.x;
    f[2 * j + 1] = v.y;
  }
}
__device__ __forceinline__ void load8(const float* p, float (&f)[8]) {
  const float4 a = __ldg(reinterpret_cast<const float4*>(p));
  const float4 b = __ldg(reinterpret_cast<const float4*>(p + 4));
  f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w;
  f[4] = b.x; f[5] = b.y; f[6] = b.z; f[7] = b.w;
}
__device__ __forceinline__ void load8(const __nv_bfloat16* p, float (&f)[8]) {
  const uint4 raw = __ldg(reinterpret_cast<const uint4*>(p));
  const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    f[2 * j] = __uint_as_float(w[j] << 16);
    f[2 * j + 1] = __uint_as_float(w[j] & 0xffff0000u);
  }
}

// One warp per token row.  d % 8 == 0; lanes hold 8 consecutive elements per
// 256-element segment.  T = __half, float or __nv_bfloat16 (the reference
// widens any input to fp32 before its min/max, so every type is quantised
// from its own exact fp32 value).
template <typename T>
__global__ void __launch_bounds__(256) quantize_int8_kernel(const T* __restrict__ D,
                                                            uint8_t* __restrict__ U,
                                                            __half* __restrict__ scales,
                                                            __half* __restrict__ mins, int64_t rows,
                                                            int d) {
  const int64_t row = static_cast<int64_t>(blockIdx.x) * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const T* src = D + row * d;
  const int nseg = (d + 255) / 256;
  float v[kMaxSeg][8];
  float mn = INFINITY, mx = -INFINITY;
#pragma unroll
  for (int s = 0; s < kMaxSeg; ++s) {
    const int k = s * 256 + lane * 8;
    if (s < nseg && k < d) {
      load8(src + k, v[s]);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        mn = fminf(mn, v[s][j]);
        mx = fmaxf(mx, v[s][j]);
      }
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, o));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  }
  float scale = __fdiv_rn(__fsub_rn(mx, mn), 255.0f);
  if (scale < 1e-8f) scale = 1e-8f;
  uint8_t* dst = U + row * d;
#pragma unroll
  for (int s = 0; s < kMaxSeg; ++s) {
    const int k = s * 256 + lane * 8;
    if (s < nseg && k < d) {
      uint32_t w[2] = {0u, 0u};
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        float u = rintf(__fdiv_rn(__fsub_rn(v[s][j], mn), scale));
        u = fminf(fmaxf(u, 0.f), 255.f);
        w[j >> 2] |= static_cast<uint32_t>(u) << (8 * (j & 3));
      }
      *reinterpret_cast<uint2*>(dst + k) = make_uint2(w[0], w[1]);
    }
  }
  if (lane == 0) {
    scales[row] = __float2half_rn(scale);
    mins[row] = __float2half_rn(mn);
  }
}

// Waits on an mbarrier that nothing ever arrives at; the bounded wait must
// give up after timeout_ns and record FM_ERR_TIMEOUT_SELFTEST.
__global__ void wait_selftest_kernel(int* status, uint64_t timeout_ns) {
  __shared__ __align__(8) uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    mbar_init(smem_u32(&bar), 1);
    abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    WaitCtl ctl{&abort_flag, status, timeout_ns};
    mbar_wait(smem_u32(&bar), 0, ctl, FM_ERR_TIMEOUT_SELFTEST);
  }
}

}  // namespace fm
