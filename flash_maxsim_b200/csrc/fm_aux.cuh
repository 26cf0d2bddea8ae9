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

// dQ partial sums: grid (ceil(Nq * Lq / 8) row tiles, nsplit document ranges);
// warp = one query row (n, q), lanes span d (8 fp16 per lane per 256-element
// segment).  Documents of the range are visited in order, eight gathers in
// flight (four for d > 512).  With nsplit == 1 the row is written as fp16 directly; otherwise
// the fp32 partial goes to ws[split][row][d] and maxsim_bwd_dq_reduce adds
// the splits in order.  blockIdx.x (row tiles) varies fastest, so the CTAs
// that run together read the same document range (L2-resident).
template <int NSEG>
__global__ void __launch_bounds__(kBwdThreads) maxsim_bwd_dq_kernel(
    const __half* __restrict__ D, const int32_t* __restrict__ am, const float* __restrict__ g,
    __half* __restrict__ dQ, float* __restrict__ ws, int Nq, int B, int Lq, int Ld, int d,
    int docs_per_split) {
  const int row = blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  const int rows = Nq * Lq;
  if (row >= rows) return;
  const int n = row / Lq, q = row - n * Lq;
  const int b_lo = blockIdx.y * docs_per_split;
  const int b_hi = min(B, b_lo + docs_per_split);
  constexpr int nseg = NSEG;
  float acc[NSEG][8];
#pragma unroll
  for (int s = 0; s < NSEG; ++s)
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[s][j] = 0.f;

  for (int b0 = b_lo; b0 < b_hi; b0 += 32) {
    const int bl = b0 + lane;
    int t = -1;
    float gv = 0.f;
    if (bl < b_hi) {
      const size_t pair = static_cast<size_t>(n) * B + bl;
      t = __ldg(am + pair * Lq + q);
      gv = __ldg(g + pair);
    }
    const int nb = min(32, b_hi - b0);
    constexpr int U = NSEG <= 2 ? 8 : 4;  // gathers in flight per lane
    for (int i = 0; i < nb; i += U) {
      uint4 raw[U][NSEG];
      float gi[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int ti = __shfl_sync(0xffffffffu, t, (i + u) & 31);
        gi[u] = __shfl_sync(0xffffffffu, gv, (i + u) & 31);
        const bool use = (i + u < nb) && ti >= 0 && ti < Ld;  // out-of-range entries count for nothing
        if (!use) gi[u] = 0.f;
        const __half* rowp = D + (static_cast<size_t>(b0 + i + u) * Ld + (use ? ti : 0)) * static_cast<size_t>(d);
#pragma unroll
        for (int s = 0; s < NSEG; ++s) {
          const int k = s * 256 + lane * 8;
          raw[u][s] = (use && s < nseg && k < d) ? __ldg(reinterpret_cast<const uint4*>(rowp + k))
                                                 : make_uint4(0, 0, 0, 0);
        }
      }
#pragma unroll
      for (int u = 0; u < U; ++u)
#pragma unroll
        for (int s = 0; s < NSEG; ++s)
          if (s < nseg) fma8(acc[s], raw[u][s], gi[u]);
    }
  }
  if (gridDim.y == 1) {
    __half* out = dQ + static_cast<size_t>(row) * d;
#pragma unroll
    for (int s = 0; s < NSEG; ++s) {
      const int k = s * 256 + lane * 8;
      if (s < nseg && k < d) *reinterpret_cast<uint4*>(out + k) = pack8(acc[s]);
    }
  } else {
    float* out = ws + (static_cast<size_t>(blockIdx.y) * rows + row) * d;
#pragma unroll
    for (int s = 0; s < NSEG; ++s) {
      const int k = s * 256 + lane * 8;
      if (s < nseg && k < d) {
        *reinterpret_cast<float4*>(out + k) = make_float4(acc[s][0], acc[s][1], acc[s][2], acc[s][3]);
        *reinterpret_cast<float4*>(out + k + 4) = make_float4(acc[s][4], acc[s][5], acc[s][6], acc[s][7]);
      }
    }
  }
}

// dQ[row][k] = sum over splits (in order) of ws[split][row][k], rounded to fp16.
__global__ void __launch_bounds__(256) maxsim_bwd_dq_reduce(const float* __restrict__ ws,
                                                            __half* __restrict__ dQ, int64_t n8, int nsplit) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * 256 + threadIdx.x;  // group of 8 elements
  if (i >= n8) return;
  float acc[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) acc[j] = 0.f;
  for (int s = 0; s < nsplit; ++s) {
    const float4* p = reinterpret_cast<const float4*>(ws + (static_cast<int64_t>(s) * n8 + i) * 8);
    const float4 x = __ldg(p), y = __ldg(p + 1);
    acc[0] += x.x; acc[1] += x.y; acc[2] += x.z; acc[3] += x.w;
    acc[4] += y.x; acc[5] += y.y; acc[6] += y.z; acc[7] += y.w;
  }
  *reinterpret_cast<uint4*>(dQ + i * 8) = pack8(acc);
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

// dD, one CTA per document, every warp busy in every phase.  The (query,
// row) entries e that picked a token of this document are bucketed by token
// with a stable counting sort: warp w counts the tokens of its slice of
// entries (slices in entry order), the counts become offsets in (token,
// warp) order, and each warp scatters its slice in order -- so every bucket
// lists its entries in ascending e, the same fixed summation order as the
// single-warp sort.  Then each warp streams the entries of a contiguous,
// entry-balanced range of tokens (see the accumulation below) and writes
// whole token rows (zeros for untouched tokens).
// Shared memory: cnt[8][Ld + 1] + base[Ld + 2] + order[Nq * Lq] ints,
// g of each sorted entry [Nq * Lq] and g[Nq] floats.
constexpr int kDdWarps = kBwdThreads / 32;
__host__ __device__ constexpr size_t dd2_smem_bytes(int Nq, int Lq, int Ld) {
  return (static_cast<size_t>(kDdWarps) * (Ld + 1) + (Ld + 2) + 2 * static_cast<size_t>(Nq) * Lq) * 4 +
         static_cast<size_t>(Nq) * 4;
}

__global__ void __launch_bounds__(kBwdThreads) maxsim_bwd_dd2_kernel(
    const __half* __restrict__ Q, const int32_t* __restrict__ am, const float* __restrict__ g,
    __half* __restrict__ dD, int Nq, int B, int Lq, int Ld, int d) {
  extern __shared__ int sm_i[];
  const int b = blockIdx.x;
  const int E = Nq * Lq;
  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  int* cnt = sm_i;                                  // [kDdWarps][Ld + 1]
  int* base = cnt + kDdWarps * (Ld + 1);            // [Ld + 2]
  int* order = base + (Ld + 2);                     // [E]
  float* gsort = reinterpret_cast<float*>(order + E);  // [E] g of each sorted entry
  float* gs = gsort + E;                            // [Nq]

  for (int i = tid; i < kDdWarps * (Ld + 1); i += kBwdThreads) cnt[i] = 0;
  for (int n = tid; n < Nq; n += kBwdThreads) gs[n] = __ldg(g + static_cast<size_t>(n) * B + b);
  __syncthreads();
  // entry e = n * Lq + q; lanes walk their entries 32 apart with (n, q)
  // advanced incrementally (no division per entry)
  auto entry_tok = [&](int n, int q) -> int {
    const int t = __ldg(am + (static_cast<size_t>(n) * B + b) * Lq + q);
    return (t >= 0 && t < Ld) ? t : -1;
  };
  auto advance = [&](int& n, int& q) {
    q += 32;
    while (q >= Lq) {
      q -= Lq;
      ++n;
    }
  };
  const int e_lo = static_cast<int>(static_cast<int64_t>(E) * warp / kDdWarps);
  const int e_hi = static_cast<int>(static_cast<int64_t>(E) * (warp + 1) / kDdWarps);
  int* mycnt = cnt + warp * (Ld + 1);
  {
    int n = (e_lo + lane) / Lq, q = e_lo + lane - n * Lq;
    for (int e = e_lo + lane; e < e_hi; e += 32) {
      const int t = entry_tok(n, q);
      if (t >= 0) atomicAdd(&mycnt[t], 1);
      advance(n, q);
    }
  }
  __syncthreads();
  // per token: offsets of the warps' runs inside the token's bucket; the
  // bucket sizes go to base[t]
  for (int t = tid; t < Ld; t += kBwdThreads) {
    int run = 0;
#pragma unroll
    for (int w = 0; w < kDdWarps; ++w) {
      const int c = cnt[w * (Ld + 1) + t];
      cnt[w * (Ld + 1) + t] = run;
      run += c;
    }
    base[t] = run;
  }
  __syncthreads();
  // exclusive scan of base[0..Ld) into base[0..Ld] (warp 0, contiguous lane ranges)
  if (warp == 0) {
    const int per = (Ld + 31) / 32;
    const int lo = lane * per, hi = min(Ld, lo + per);
    int s = 0;
    for (int t = lo; t < hi; ++t) s += base[t];
    int incl = s;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int v = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += v;
    }
    int run = incl - s;
    for (int t = lo; t < hi; ++t) {
      const int c = base[t];
      base[t] = run;
      run += c;
    }
    if (lane == 31) base[Ld] = incl;
  }
  __syncthreads();
  // stable scatter of each warp's slice, in entry order
  int sn = (e_lo + lane) / Lq, sq = e_lo + lane - sn * Lq;
  for (int e0 = e_lo; e0 < e_hi; e0 += 32) {
    const int e = e0 + lane;
    const int t = (e < e_hi) ? entry_tok(sn, sq) : -1;
    const unsigned grp = __match_any_sync(0xffffffffu, t);
    if (t >= 0) {
      const int rank = __popc(grp & ((1u << lane) - 1u));
      order[base[t] + mycnt[t] + rank] = e;
      gsort[base[t] + mycnt[t] + rank] = gs[sn];
    }
    advance(sn, sq);
    __syncwarp();
    if (t >= 0 && lane == __ffs(grp) - 1) mycnt[t] += __popc(grp);
    __syncwarp();
  }
  __syncthreads();
  // Accumulation: the tokens that hold entries, [0, t_end), are cut into 8
  // contiguous ranges with about equal entry counts (whole tokens); each warp
  // streams its range's entries in order with eight gathers in flight across
  // token boundaries, writing each token row as it completes (zero rows
  // included).  Tokens [t_end, Ld) hold no entry: all warps write their zero
  // rows in turn.  Each token's sum keeps the ascending entry order.
  const int etot = base[Ld];
  auto lower_bound = [&](int v) {  // first token t with base[t] >= v (base is non-decreasing)
    int lo = 0, hi = Ld;
    while (lo < hi) {
      const int mid = (lo + hi) >> 1;
      if (base[mid] < v) lo = mid + 1;
      else hi = mid;
    }
    return lo;
  };
  const int t_end = lower_bound(etot);  // tokens past the last one that has an entry
  const int t_lo = warp == 0 ? 0 : min(lower_bound(static_cast<int>(static_cast<int64_t>(etot) * warp / kDdWarps)), t_end);
  const int t_hi = warp == kDdWarps - 1 ? t_end
                                        : min(lower_bound(static_cast<int>(static_cast<int64_t>(etot) * (warp + 1) / kDdWarps)), t_end);
  const int nseg = (d + 255) / 256;
  constexpr int U = 8;
  for (int s = 0; s < nseg; ++s) {
    const int k = s * 256 + lane * 8;
    const bool kin = k < d;
    __half* out0 = dD + static_cast<size_t>(b) * Ld * d + k;
    float acc[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[j] = 0.f;
    int t = t_lo;
    const int p_end = t_hi > t_lo ? base[t_hi] : base[t_lo];
    for (int p0 = t_hi > t_lo ? base[t_lo] : p_end; p0 < p_end; p0 += U) {
      uint4 raw[U];
      float gv[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const bool in = p0 + u < p_end;
        const int e = in ? order[p0 + u] : 0;
        gv[u] = in ? gsort[p0 + u] : 0.f;
        raw[u] = (in && kin) ? __ldg(reinterpret_cast<const uint4*>(Q + static_cast<size_t>(e) * d + k))
                             : make_uint4(0, 0, 0, 0);
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int pp = p0 + u;
        if (pp >= p_end) break;
        while (pp >= base[t + 1]) {  // token t is complete
          if (kin) *reinterpret_cast<uint4*>(out0 + static_cast<size_t>(t) * d) = pack8(acc);
#pragma unroll
          for (int j = 0; j < 8; ++j) acc[j] = 0.f;
          ++t;
        }
        fma8(acc, raw[u], gv[u]);
      }
    }
    for (; t < t_hi; ++t) {  // the range's last token, and any empty ones before it
      if (kin) *reinterpret_cast<uint4*>(out0 + static_cast<size_t>(t) * d) = pack8(acc);
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[j] = 0.f;
    }
    const uint4 z = make_uint4(0, 0, 0, 0);
    for (int tz = t_end + warp; tz < Ld; tz += kDdWarps)
      if (kin) *reinterpret_cast<uint4*>(out0 + static_cast<size_t>(tz) * d) = z;
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
// Index-time normalisation (NORM = true): every row is first divided by
// max(||x||_2, 1e-12) (F.normalize's rule) with the norm summed in a fixed
// order -- per lane x*x over its elements in order (no fused multiply-add),
// then an xor butterfly over the row's lanes -- and an IEEE square root and
// division, so the result is reproducible bit for bit on the host.
template <int LPR, int NSEG>
__device__ __forceinline__ float row_inv_norm_sq(const float (&v)[NSEG][8], int nseg, int l, int d) {
  float s = 0.f;
#pragma unroll
  for (int g = 0; g < NSEG; ++g) {
    const int k = (g * LPR + l) * 8;
    if (g < nseg && k < d) {
#pragma unroll
      for (int j = 0; j < 8; ++j) s = __fadd_rn(s, __fmul_rn(v[g][j], v[g][j]));
    }
  }
#pragma unroll
  for (int o = LPR / 2; o > 0; o >>= 1) s = __fadd_rn(s, __shfl_xor_sync(0xffffffffu, s, o));
  return s;
}

template <typename T, int LPR, int NR, bool NORM = false>
__global__ void __launch_bounds__(256) quantize_int8_kernel(const T* __restrict__ D,
                                                            uint8_t* __restrict__ U,
                                                            __half* __restrict__ scales,
                                                            __half* __restrict__ mins, int64_t rows,
                                                            int d) {
  // LPR lanes per row (8 elements each per segment), 32 / LPR rows per warp at
  // a time and NR such row sets per warp, all loaded before any is converted
  // (enough bytes in flight to stream HBM)
  constexpr int RPW = 32 / LPR;
  constexpr int SEG = NR > 1 ? 1 : kMaxSeg;  // several row sets only when a row fits one segment
  const int lane = threadIdx.x & 31;
  const int sub = lane / LPR, l = lane % LPR;
  const int64_t row0 = (static_cast<int64_t>(blockIdx.x) * 8 + (threadIdx.x >> 5)) * RPW * NR + sub;
  const int nseg = (d + LPR * 8 - 1) / (LPR * 8);
  float v[NR][SEG][8];
  float mn[NR], mx[NR];
#pragma unroll
  for (int r = 0; r < NR; ++r) {
    const int64_t row = row0 + r * RPW;
    mn[r] = INFINITY;
    mx[r] = -INFINITY;
    const T* src = D + (row < rows ? row : 0) * d;
#pragma unroll
    for (int s = 0; s < SEG; ++s) {
      const int k = (s * LPR + l) * 8;
      if (row < rows && s < nseg && k < d) load8(src + k, v[r][s]);
    }
  }
  if (NORM) {
#pragma unroll
    for (int r = 0; r < NR; ++r) {
      const float den = fmaxf(__fsqrt_rn(row_inv_norm_sq<LPR, SEG>(v[r], nseg, l, d)), 1e-12f);
#pragma unroll
      for (int s = 0; s < SEG; ++s)
#pragma unroll
        for (int j = 0; j < 8; ++j) v[r][s][j] = __fdiv_rn(v[r][s][j], den);
    }
  }
#pragma unroll
  for (int r = 0; r < NR; ++r) {
    const bool live = row0 + r * RPW < rows;
#pragma unroll
    for (int s = 0; s < SEG; ++s) {
      const int k = (s * LPR + l) * 8;
      if (live && s < nseg && k < d) {
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          mn[r] = fminf(mn[r], v[r][s][j]);
          mx[r] = fmaxf(mx[r], v[r][s][j]);
        }
      }
    }
#pragma unroll
    for (int o = LPR / 2; o > 0; o >>= 1) {  // within the row's lanes
      mn[r] = fminf(mn[r], __shfl_xor_sync(0xffffffffu, mn[r], o));
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], o));
    }
  }
#pragma unroll
  for (int r = 0; r < NR; ++r) {
    const int64_t row = row0 + r * RPW;
    if (row >= rows) continue;
    float scale = __fdiv_rn(__fsub_rn(mx[r], mn[r]), 255.0f);
    if (scale < 1e-8f) scale = 1e-8f;
    uint8_t* dst = U + row * d;
    // u = rint((x - min) / scale) with the IEEE quotient, as the reference
    // does. The product with the rounded reciprocal is within 2 ulp (< 5e-5
    // here, the quotient is <= 255) of the exact quotient, and rint only
    // depends on which side of k + 0.5 the quotient lies: where the product is
    // within 1e-4 of a half-integer the exact quotient is computed instead, so
    // the codes equal the division's everywhere.
    const float inv = __frcp_rn(scale);
#pragma unroll
    for (int s = 0; s < SEG; ++s) {
      const int k = (s * LPR + l) * 8;
      if (s < nseg && k < d) {
        uint32_t w[2] = {0u, 0u};
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const float num = __fsub_rn(v[r][s][j], mn[r]);
          float q = __fmul_rn(num, inv);
          if (fabsf(__fsub_rn(__fsub_rn(q, floorf(q)), 0.5f)) < 1e-4f) q = __fdiv_rn(num, scale);
          float u = rintf(q);
          u = fminf(fmaxf(u, 0.f), 255.f);
          w[j >> 2] |= static_cast<uint32_t>(u) << (8 * (j & 3));
        }
        *reinterpret_cast<uint2*>(dst + k) = make_uint2(w[0], w[1]);
      }
    }
    if (l == 0) {
      scales[row] = __float2half_rn(scale);
      mins[row] = __float2half_rn(mn[r]);
    }
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
