// Top-k selection of MaxSim scores per query, sm_100a.
//
// Rerankers keep the k best documents of each query (the reference's demo
// and benchmark call `scores.topk(k)` on the full score matrix,
// examples/demo.py:126-134, benchmarks/bench.py:36).  Here the selection is
// split in two stages that never sort the [Nq, B] matrix:
//
//  1. per part: the k best (score, document) pairs of each query among the
//     documents of one part.  The forward kernels do this in their own tail
//     (part = CTA, over the documents that CTA scored, while the scores are
//     still in L2); for score matrices from other kernels
//     `topk_partial_kernel` does it over contiguous document ranges.
//  2. `topk_merge_kernel`: one CTA per query merges the parts' candidates.
//
// Order: score descending, then document id ascending (ties never depend on
// the schedule, so the result is deterministic and equals a stable sort).
// A warp selects in k rounds: when its candidates fit in registers (up to 256)
// each lane sorts its own, and every round takes the best lane head with two
// single-instruction warp reductions; larger candidate sets are re-read each
// round ("best candidate after the previous pick").  No atomics.
#pragma once

#include <cstdint>
#include <cuda_fp16.h>

namespace fm {

constexpr int kTopkThreads = 256;
constexpr int kTopkMaxK = 1024;

struct TopkArgs {
  int k;             // 0: no selection
  int parts;         // candidate parts per query (the forward's grid)
  float* cand_s;     // [Nq][parts][k]
  int32_t* cand_b;   // [Nq][parts][k] document ids, -1 = none
};

struct TopkCand {
  float s;
  int b;  // < 0: no candidate
};

// Order-preserving map of a (non-NaN) float to a nonzero unsigned key:
// larger floats give larger keys; -inf maps above 0.
__device__ __forceinline__ unsigned tk_key(float s) {
  const unsigned u = __float_as_uint(s == 0.f ? 0.f : s);  // -0 and +0 tie
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float tk_unkey(unsigned k) {
  return __uint_as_float((k & 0x80000000u) ? (k & 0x7fffffffu) : ~k);
}

// (s, b) comes before (bs, bb) in the output order
__device__ __forceinline__ bool tk_before(float s, int b, float bs, int bb) {
  return s > bs || (s == bs && b < bb);
}

// One warp selects the k best of `count` candidates get(p), p < count, and
// lane 0 writes them in order to out_s / out_b (score -inf, id -1 where fewer
// than k candidates exist).  NaN scores are never selected.  The first
// NR * 32 candidates are held in registers; larger counts are re-read per
// round through get().
template <int NR, class Get>
__device__ __forceinline__ void warp_topk(int count, int k, Get get, float* out_s, int32_t* out_b, int lane) {
  float rs[NR];
  int rb[NR];
  const bool in_regs = count <= NR * 32;
  if (in_regs) {
#pragma unroll
    for (int i = 0; i < NR; ++i) {
      const int p = i * 32 + lane;
      TopkCand c{0.f, -1};
      if (p < count) c = get(p);
      rs[i] = c.s;
      rb[i] = (c.s == c.s) ? c.b : -1;  // NaN scores are never selected
    }
    // each lane sorts its candidates best first (odd-even transposition;
    // empty entries last), then every round takes the best lane head and
    // only the winning lane moves on: no per-round scan of the registers
#pragma unroll
    for (int pass = 0; pass < NR; ++pass) {
#pragma unroll
      for (int i = pass & 1; i + 1 < NR; i += 2) {
        const bool sw = rb[i + 1] >= 0 && (rb[i] < 0 || tk_before(rs[i + 1], rb[i + 1], rs[i], rb[i]));
        const float ts = rs[i];
        const int tb = rb[i];
        rs[i] = sw ? rs[i + 1] : rs[i];
        rb[i] = sw ? rb[i + 1] : rb[i];
        rs[i + 1] = sw ? ts : rs[i + 1];
        rb[i + 1] = sw ? tb : rb[i + 1];
      }
    }
    int r = 0;
    for (; r < k; ++r) {
      const unsigned key = rb[0] >= 0 ? tk_key(rs[0]) : 0u;
      const unsigned kmax = __reduce_max_sync(0xffffffffu, key);
      if (kmax == 0u) break;
      const unsigned id = (key == kmax) ? static_cast<unsigned>(rb[0]) : 0xffffffffu;
      const int bmin = static_cast<int>(__reduce_min_sync(0xffffffffu, id));
      if (lane == 0) {
        out_s[r] = tk_unkey(kmax);
        out_b[r] = bmin;
      }
      if (key == kmax && rb[0] == bmin) {
#pragma unroll
        for (int i = 0; i + 1 < NR; ++i) {
          rs[i] = rs[i + 1];
          rb[i] = rb[i + 1];
        }
        rb[NR - 1] = -1;
      }
    }
    if (lane == 0)
      for (; r < k; ++r) {
        out_s[r] = -INFINITY;
        out_b[r] = -1;
      }
    return;
  }
  float ps = INFINITY;  // previous pick; every candidate comes after (+inf, -1)
  int pb = -1;
  int r = 0;
  for (; r < k; ++r) {
    float bs = 0.f;
    int bb = -1;
    auto consider = [&](float s, int b) {
      if (b < 0 || s != s) return;
      if (!(s < ps || (s == ps && b > pb))) return;  // already picked
      if (bb < 0 || tk_before(s, b, bs, bb)) {
        bs = s;
        bb = b;
      }
    };
    if (in_regs) {
#pragma unroll
      for (int i = 0; i < NR; ++i) consider(rs[i], rb[i]);
    } else {
      for (int p = lane; p < count; p += 32) {
        const TopkCand c = get(p);
        consider(c.s, c.b);
      }
    }
    // warp winner with two single-instruction reductions: the largest score
    // (as an order-preserving unsigned key; 0 = no candidate), then the
    // smallest document id among the lanes holding it
    const unsigned key = bb >= 0 ? tk_key(bs) : 0u;
    const unsigned kmax = __reduce_max_sync(0xffffffffu, key);
    if (kmax == 0u) break;
    const unsigned id = (key == kmax) ? static_cast<unsigned>(bb) : 0xffffffffu;
    bb = static_cast<int>(__reduce_min_sync(0xffffffffu, id));
    bs = tk_unkey(kmax);
    if (lane == 0) {
      out_s[r] = bs;
      out_b[r] = bb;
    }
    ps = bs;
    pb = bb;
  }
  if (lane == 0)
    for (; r < k; ++r) {
      out_s[r] = -INFINITY;
      out_b[r] = -1;
    }
}

// Stage 1 over a score matrix: CTA (n, part) selects the k best documents of
// query n in document range [B * part / parts, B * (part + 1) / parts); each
// warp takes a slice, warp 0 merges the warps' picks from shared memory.
// Shared memory: 8 * k * 8 bytes.
__global__ void __launch_bounds__(kTopkThreads) topk_partial_kernel(const float* __restrict__ scores, int B,
                                                                     TopkArgs t) {
  extern __shared__ __align__(16) uint8_t tk_smem[];
  const int n = blockIdx.x, part = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  constexpr int W = kTopkThreads / 32;
  float* ws = reinterpret_cast<float*>(tk_smem);
  int32_t* wb = reinterpret_cast<int32_t*>(ws + W * t.k);
  const int64_t lo = static_cast<int64_t>(B) * part / t.parts;
  const int64_t hi = static_cast<int64_t>(B) * (part + 1) / t.parts;
  const int64_t span = hi - lo;
  const int wlo = static_cast<int>(lo + span * warp / W), whi = static_cast<int>(lo + span * (warp + 1) / W);
  const float* row = scores + static_cast<size_t>(n) * B;
  warp_topk<8>(whi - wlo, t.k, [&](int p) { return TopkCand{__ldg(row + wlo + p), wlo + p}; },
               ws + warp * t.k, wb + warp * t.k, lane);
  __syncthreads();
  if (warp == 0) {
    const size_t o = (static_cast<size_t>(n) * t.parts + part) * t.k;
    warp_topk<8>(W * t.k, t.k, [&](int p) { return TopkCand{ws[p], wb[p]}; }, t.cand_s + o, t.cand_b + o, lane);
  }
}

// Stage 2: one CTA per query merges parts * k candidates into the final k,
// written as fp32 scores and int64 document ids (id_offset added: the first
// document of this shard).  Shared memory: (8 + 1) * k * 8 bytes.
__global__ void __launch_bounds__(kTopkThreads) topk_merge_kernel(TopkArgs t, float* __restrict__ out_s,
                                                                   int64_t* __restrict__ out_i, int64_t id_offset) {
  extern __shared__ __align__(16) uint8_t tk_smem[];
  asm volatile("griddepcontrol.wait;" ::: "memory");  // the candidates' writer has completed
  const int n = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  constexpr int W = kTopkThreads / 32;
  float* ws = reinterpret_cast<float*>(tk_smem);       // [W * k] per-warp picks
  int32_t* wb = reinterpret_cast<int32_t*>(ws + W * t.k);
  float* fs = reinterpret_cast<float*>(wb + W * t.k);  // [k] final picks
  int32_t* fb = reinterpret_cast<int32_t*>(fs + t.k);
  const int total = t.parts * t.k;
  const int wlo = total * warp / W, whi = total * (warp + 1) / W;
  const float* cs = t.cand_s + static_cast<size_t>(n) * total;
  const int32_t* cb = t.cand_b + static_cast<size_t>(n) * total;
  warp_topk<8>(whi - wlo, t.k, [&](int p) { return TopkCand{cs[wlo + p], cb[wlo + p]}; }, ws + warp * t.k,
               wb + warp * t.k, lane);
  __syncthreads();
  if (warp == 0) warp_topk<8>(W * t.k, t.k, [&](int p) { return TopkCand{ws[p], wb[p]}; }, fs, fb, lane);
  __syncthreads();
  for (int r = threadIdx.x; r < t.k; r += kTopkThreads) {
    const int b = fb[r];
    out_s[static_cast<size_t>(n) * t.k + r] = fs[r];
    out_i[static_cast<size_t>(n) * t.k + r] = b >= 0 ? id_offset + b : -1;
  }
}

}  // namespace fm
