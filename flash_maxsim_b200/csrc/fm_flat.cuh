// Batched shared-document MaxSim over a flat token stream, sm_100a.
//
//   score[n, b] = sum_q max_{t < Ld} <Q[n, q], D[b, t]>      (all documents of length Ld)
//
// Same result as the reference's `_maxsim_fwd_kernel` on shared documents
// (flash_maxsim/flash_maxsim.py:83-146, launched by flash_maxsim_batched at
// flash_maxsim.py:233-250) when no per-document lengths are given.
//
// Why a flat stream: a tcgen05.mma of M = 128, K = 16 occupies the tensor
// pipe for max(~96, N / 2) cycles, so only N >= 192 runs at full rate, and
// cutting each document into its own chunks (300 tokens -> 160 + 140) pays
// for padding and small N.  Here the [B, Ld, d] documents are read as one
// [B * Ld, d] token matrix and cut into chunks of CT = 192 tokens regardless
// of document boundaries; every MMA has N = CT.
//
//  * Each CTA owns a contiguous range of whole documents (no document is split
//    across CTAs).  An item is G = 2 consecutive chunks resident in shared
//    memory.  For each 128-row query block (M-block, both K atoms in one
//    32 KB stage, two stages) the MMA thread multiplies chunk 0 into TMEM slot
//    0 and commits it, then chunk 1 into slot 1: the epilogue drains one slot
//    while the tensor core fills the other.
//  * TMEM lane = query row, column = token.  The two epilogue warps of a lane
//    quarter split a chunk's 32-column pieces (even / odd) and reduce each
//    document segment of the chunk (segments end where documents end, every
//    Ld tokens) to a per-row maximum.  The even warp hands its segment maxima
//    to the odd warp through shared memory and an mbarrier; the odd warp
//    merges them, closes the documents that end in the chunk (row maxima
//    summed over the warp's 32 rows = one query row group, into a per-item
//    table) and carries the open document's running maximum, kept per
//    (M-block, row) in spare TMEM columns, into the next chunk and item.
//  * When every M-block of an item is done, the documents that end inside it
//    are scored (row-group sums added in a fixed order) and written.
//  * Queries with more than 128 row groups are processed in spans of whole
//    queries; every span streams the documents again (the pass stays bound by
//    the tensor pipe).
//
// Warp roles: 0 = document TMA producer, 1 = MMA issuer + TMEM owner,
// 2..5 = epilogue (even pieces), 6 = query TMA producer, 7..10 = epilogue
// (odd pieces, merge, carry).  Every wait is a bounded mbarrier wait.
#pragma once

#include <cuda.h>
#include <cstdint>
#include <cuda_fp16.h>
#include "fm_fwd.cuh"
#include "fm_ptx.cuh"

namespace fm {

constexpr int kFlatThreads = 11 * 32;
constexpr int kFlatG = 2;         // chunks per item
constexpr int kFlatCT = 192;      // tokens per chunk (MMA N)
constexpr int kFlatTS = 2;        // TMEM accumulator slots (a ring over all chunks)
constexpr int kFlatMaxJb = 32;    // M-blocks per span (128 row groups)
constexpr int kFlatSeg = 3;       // document segments per chunk (Ld >= CT / 2)
constexpr int kFlatDocSlots = 3;  // documents that can end inside one item (Ld >= 2 CT / 3)
constexpr uint32_t kFlatCarryCol = kFlatTS * kFlatCT;  // TMEM columns of the per-(M-block, row) carry
constexpr int kFlatXch = 8;       // segment-exchange buffers (chunks in flight between the two warps)

struct FlatArgs {
  float* scores;  // [Nq, B]
  int* status;
  uint64_t timeout_ns;
  int B, Ld, Nq, Lq, d;
  int atoms;    // 64-element K atoms (1 or 2)
  int nd;       // document slots
  int Gq;       // row groups (32 rows) per query
  int R;        // row groups in total (Nq * Gq)
  int span_rg;  // row groups per span (a multiple of Gq, <= 128)
  uint32_t off_q, off_d, off_rows, off_xch, off_bar, d_slot_bytes;
  int dbg;
};

__device__ __forceinline__ void flat_drain(uint32_t bar, uint32_t parity, const FlatArgs& a) {
  const uint64_t t0 = globaltimer_ns();
  while (!mbar_try_wait(bar, parity)) {
    if (globaltimer_ns() - t0 > a.timeout_ns) {
      record_status(a.status, FM_ERR_TIMEOUT_DRAIN);
      break;
    }
  }
}

// max of m and v[j] over lo <= j < hi (runtime bounds)
__device__ __forceinline__ float range_max32(const float (&v)[32], int lo, int hi, float m) {
#pragma unroll
  for (int j = 0; j < 32; ++j) m = fmaxf(m, (j >= lo && j < hi) ? v[j] : -INFINITY);
  return m;
}

__device__ __forceinline__ float full_max32(const float (&v)[32], float m) {
  float a0 = fmax3(m, v[0], v[1]);
  float a1 = fmax3(v[2], v[3], v[4]);
  float a2 = fmax3(v[5], v[6], v[7]);
  float a3 = fmax3(v[8], v[9], v[10]);
  float a4 = fmax3(v[11], v[12], v[13]);
  float a5 = fmax3(v[14], v[15], v[16]);
  float a6 = fmax3(v[17], v[18], v[19]);
  float a7 = fmax3(v[20], v[21], v[22]);
  float a8 = fmax3(v[23], v[24], v[25]);
  float a9 = fmax3(v[26], v[27], v[28]);
  float a10 = fmax3(v[29], v[30], v[31]);
  a0 = fmax3(a0, a1, a2);
  a3 = fmax3(a3, a4, a5);
  a6 = fmax3(a6, a7, a8);
  a9 = fmaxf(a9, a10);
  return fmaxf(fmax3(a0, a3, a6), a9);
}

// Fold one 32-column piece (columns [c0, c0 + nv) of the chunk) into the
// segment maxima: segment 0 = [0, e0), segment 1 = [e0, e1), segment 2 =
// [e1, ncols), where nb of the document ends e0 < e1 lie inside the chunk.
// A piece holds at most one document end (Ld >= 128).  Common case: the
// whole piece lies in one segment (one max tree); otherwise one masked pass
// splits it at the document end (and drops columns past the chunk's end).
__device__ __forceinline__ void fold_piece(const float (&v)[32], int c0, int nv, int e0, int e1, int nb,
                                           float& m0, float& m1, float& m2) {
  const int end = c0 + nv;
  int bpos = 32;  // first column of the right part
  if (nb >= 1 && e0 > c0 && e0 < end) bpos = e0 - c0;
  if (nb >= 2 && e1 > c0 && e1 < end) bpos = e1 - c0;
  const int seg = (nb >= 1 && c0 >= e0 ? 1 : 0) + (nb >= 2 && c0 >= e1 ? 1 : 0);  // segment of column 0
  float lo, hi = -INFINITY;
  if (bpos == 32 && nv == 32) {
    lo = full_max32(v, -INFINITY);
  } else {
    lo = -INFINITY;
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      lo = fmaxf(lo, (j < bpos && j < nv) ? v[j] : -INFINITY);
      hi = fmaxf(hi, (j >= bpos && j < nv) ? v[j] : -INFINITY);
    }
  }
  if (seg == 0) {
    m0 = fmaxf(m0, lo);
    m1 = fmaxf(m1, hi);
  } else if (seg == 1) {
    m1 = fmaxf(m1, lo);
    m2 = fmaxf(m2, hi);
  } else {
    m2 = fmaxf(m2, lo);
  }
}

__global__ void __launch_bounds__(kFlatThreads, 1)
    maxsim_flat_kernel(const __grid_constant__ CUtensorMap tmap_q, const __grid_constant__ CUtensorMap tmap_d,
                       const FlatArgs a) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const uint32_t sbase = smem_u32(smem);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  // barriers: d_full[nd] d_empty[nd] q_full[2] q_empty[2] t_full[kFlatTS] t_empty[kFlatTS]
  //           x_full[kFlatXch][4] item[2] drain
  const uint32_t bar0 = sbase + a.off_bar;
  auto d_full = [&](int i) { return bar0 + 8u * i; };
  auto d_empty = [&](int i) { return bar0 + 8u * (a.nd + i); };
  const uint32_t bq0 = bar0 + 8u * (2 * a.nd);
  auto q_full = [&](int i) { return bq0 + 8u * i; };
  auto q_empty = [&](int i) { return bq0 + 8u * (2 + i); };
  auto t_full = [&](int i) { return bq0 + 8u * (4 + i); };
  auto t_empty = [&](int i) { return bq0 + 8u * (4 + kFlatTS + i); };
  constexpr int kXb = 4 + 2 * kFlatTS;
  auto x_full = [&](int k, int q) { return bq0 + 8u * (kXb + 4 * k + q); };
  auto item_bar = [&](int i) { return bq0 + 8u * (kXb + 4 * kFlatXch + i); };
  const uint32_t drain = bq0 + 8u * (kXb + 4 * kFlatXch + 2);
  uint8_t* ctl_area = smem + a.off_bar + 8 * (2 * a.nd + kXb + 4 * kFlatXch + 3);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(ctl_area);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(ctl_area + 8);
  WaitCtl ctl{abort_flag, a.status, a.timeout_ns};

  if (threadIdx.x == 0) {
    for (int i = 0; i < a.nd; ++i) {
      mbar_init(d_full(i), 1);
      mbar_init(d_empty(i), 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(q_full(i), 1);
      mbar_init(q_empty(i), 1);
      mbar_init(item_bar(i), 8);
    }
    for (int i = 0; i < kFlatTS; ++i) {
      mbar_init(t_full(i), 1);
      mbar_init(t_empty(i), 8);  // both epilogue warps of every lane quarter
    }
    for (int k = 0; k < kFlatXch; ++k)
      for (int q = 0; q < 4; ++q) mbar_init(x_full(k, q), 1);
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), 512);
    tmem_relinquish();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmap_q);
    tma_prefetch_desc(&tmap_d);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  grid_dep_wait();
  grid_dep_launch();
  const uint32_t tmem_base = *tmem_slot;

  // this CTA's documents and token range
  const int d_lo = static_cast<int>((static_cast<int64_t>(a.B) * blockIdx.x) / gridDim.x);
  const int d_hi = static_cast<int>((static_cast<int64_t>(a.B) * (blockIdx.x + 1)) / gridDim.x);
  const int T0 = d_lo * a.Ld, T1 = d_hi * a.Ld;
  constexpr int item_tokens = kFlatG * kFlatCT;
  const int n_items = (T1 - T0 + item_tokens - 1) / item_tokens;
  const int n_spans = (a.R + a.span_rg - 1) / a.span_rg;
  const uint32_t q_stage = a.atoms * 16384u;

  if (warp == 0) {
    // ===================== document producer =====================
    if (lane == 0) {
      const uint64_t pol = l2_policy_evict_first();
      const uint32_t tx = a.atoms * kFlatCT * 128u;
      Ring r;
      int issued = 0;
      bool ok = true;
      for (int sp = 0; sp < n_spans && ok; ++sp) {
        for (int it = 0; it < n_items && ok; ++it) {
          const int I0 = T0 + it * item_tokens;
          const int cn = min(kFlatG, (T1 - I0 + kFlatCT - 1) / kFlatCT);
          for (int c = 0; c < cn; ++c) {
            if (!mbar_wait(d_empty(r.idx), r.phase ^ 1u, ctl, FM_ERR_TIMEOUT_DEMPTY)) {
              ok = false;
              break;
            }
            mbar_expect_tx(d_full(r.idx), tx);
            const uint32_t dst = sbase + a.off_d + r.idx * a.d_slot_bytes;
            for (int at = 0; at < a.atoms; ++at)
              tma_load_3d(dst + at * kFlatCT * 128, &tmap_d, at * 64, I0 + c * kFlatCT, 0, d_full(r.idx), pol);
            r.next(a.nd);
            ++issued;
          }
        }
      }
      for (int i = 0; i < a.nd && i < issued; ++i) {
        if (--r.idx < 0) {
          r.idx = a.nd - 1;
          r.phase ^= 1u;
        }
        flat_drain(d_full(r.idx), r.phase, a);
      }
    }
  } else if (warp == 6) {
    // ===================== query producer =====================
    if (lane == 0) {
      const uint64_t pol = l2_policy_evict_last();
      Ring r;
      int issued = 0;
      bool ok = true;
      for (int sp = 0; sp < n_spans && ok; ++sp) {
        const int rg0 = sp * a.span_rg;
        const int nmb = (min(a.span_rg, a.R - rg0) + 3) / 4;
        for (int it = 0; it < n_items && ok; ++it) {
          for (int jb = 0; jb < nmb; ++jb) {
            if (!mbar_wait(q_empty(r.idx), r.phase ^ 1u, ctl, FM_ERR_TIMEOUT_QEMPTY)) {
              ok = false;
              break;
            }
            mbar_expect_tx(q_full(r.idx), q_stage);
            for (int at = 0; at < a.atoms; ++at)
              tma_load_3d(sbase + a.off_q + r.idx * 32768u + at * 16384u, &tmap_q, at * 64, (rg0 + 4 * jb) * 32,
                          0, q_full(r.idx), pol);
            r.next(2);
            ++issued;
          }
        }
      }
      for (int i = 0; i < 2 && i < issued; ++i) {
        if (--r.idx < 0) {
          r.idx = 1;
          r.phase ^= 1u;
        }
        flat_drain(q_full(r.idx), r.phase, a);
      }
    }
  } else if (warp == 1) {
    // ===================== MMA issuer =====================
    if (lane == 0) {
      const uint32_t idesc = idesc_f16_f32(128, kFlatCT);
      constexpr uint32_t d_atom = kFlatCT * 8u;  // one K atom of a document slot, 16-byte units
      const int ksteps = a.atoms * 4;
      const bool skip_mma = FM_DBG(a, 2);
      Ring dr, qr, tr;
      bool ok = true;
      FM_TR_DECL;
      for (int sp = 0; sp < n_spans && ok; ++sp) {
        const int rg0 = sp * a.span_rg;
        const int nmb = (min(a.span_rg, a.R - rg0) + 3) / 4;
        for (int it = 0; it < n_items && ok; ++it) {
          const int I0 = T0 + it * item_tokens;
          const int cn = min(kFlatG, (T1 - I0 + kFlatCT - 1) / kFlatCT);
          uint64_t ddesc0 = 0, ddesc1 = 0;
          {
            Ring r = dr;
            for (int c = 0; c < cn; ++c) {
              if (!mbar_wait(d_full(r.idx), r.phase, ctl, FM_ERR_TIMEOUT_DFULL)) {
                ok = false;
                break;
              }
              const uint64_t dd = smem_desc_sw128(sbase + a.off_d + r.idx * a.d_slot_bytes);
              if (c == 0) ddesc0 = dd; else ddesc1 = dd;
              r.next(a.nd);
            }
          }
          if (!ok) break;
          tc_fence_after();
          for (int jb = 0; jb < nmb && ok; ++jb) {
            FM_TR(0, 5);
            if (!mbar_wait(q_full(qr.idx), qr.phase, ctl, FM_ERR_TIMEOUT_QFULL)) {
              ok = false;
              break;
            }
            FM_TR(0, 6);
            tc_fence_after();
            const uint64_t qdesc = smem_desc_sw128(sbase + a.off_q + qr.idx * 32768u);
            for (int c = 0; c < cn; ++c) {
              FM_TR(0, 1);
              if (!mbar_wait(t_empty(tr.idx), tr.phase ^ 1u, ctl, FM_ERR_TIMEOUT_TEMPTY)) {
                ok = false;
                break;
              }
              FM_TR(0, 2);
              tc_fence_after();
              const uint64_t dd = c ? ddesc1 : ddesc0;
              const uint32_t tacc = tmem_base + tr.idx * kFlatCT;
              if (!skip_mma) {
#pragma unroll
                for (int kk = 0; kk < 8; ++kk) {
                  if (kk < ksteps)
                    tc_mma_f16(tacc, qdesc + (kk >> 2) * (16384u >> 4) + (kk & 3) * 2u,
                               dd + (kk >> 2) * d_atom + (kk & 3) * 2u, idesc, kk > 0 ? 1u : 0u);
                }
              }
              FM_TR(0, 3);
              tc_commit(t_full(tr.idx));
              tr.next(kFlatTS);
            }
            if (!ok) break;
            tc_commit(q_empty(qr.idx));
            qr.next(2);
          }
          if (!ok) break;
          for (int c = 0; c < cn; ++c) {
            tc_commit(d_empty(dr.idx));
            dr.next(a.nd);
          }
        }
      }
      tc_commit(drain);
      flat_drain(drain, 0, a);
    }
  } else {
    // ===================== epilogue =====================
    const int set = warp >= 7 ? 1 : 0;  // 0: even pieces, 1: odd pieces + merge + carry
    const int sub = warp & 3;           // TMEM lane quarter
    const int et = set * 128 + (threadIdx.x & 127);
    const uint32_t lane_base = static_cast<uint32_t>(sub * 32) << 16;
    float* rows = reinterpret_cast<float*>(smem + a.off_rows);  // [2][kFlatDocSlots][128]
    float* xch = reinterpret_cast<float*>(smem + a.off_xch);    // [kFlatXch][4 quarters][kFlatSeg][32]
    const bool skip_epi = FM_DBG(a, 1);
    Ring tr;
    uint32_t xph = 0u;
    int kc = 0;  // chunk counter (selects the exchange buffer)
    bool ok = true;
    FM_TR_DECL;
    const int tch = warp == 2 ? 1 : (warp == 7 ? 2 : 7);
    int ibuf = 0;
    uint32_t iph = 0u;  // bit b: phase parity of item barrier b
    for (int sp = 0; sp < n_spans && ok; ++sp) {
      const int rg0 = sp * a.span_rg;
      const int srg = min(a.span_rg, a.R - rg0);  // row groups of this span
      const int nmb = (srg + 3) / 4;
      for (int it = 0; it < n_items && ok; ++it) {
        const int I0 = T0 + it * item_tokens;
        const int I1 = min(T1, I0 + item_tokens);
        const int cn = (I1 - I0 + kFlatCT - 1) / kFlatCT;
        const int e_first = I0 / a.Ld;  // first document that can end in this item
        float* rb = rows + ibuf * kFlatDocSlots * 128;
        for (int jb = 0; jb < nmb && ok; ++jb) {
          const int lrg = 4 * jb + sub;  // row group within the span
          const bool active = lrg < srg;
          const uint32_t carry_addr = tmem_base + lane_base + kFlatCarryCol + jb;
          float carry = -INFINITY;
          if (set == 1 && it > 0) {
            carry = tmem_ld1(carry_addr);
            tmem_wait_ld();
          }
          for (int c = 0; c < cn; ++c, ++kc) {
            FM_TR(tch, 1);
            if (!mbar_wait(t_full(tr.idx), tr.phase, ctl, FM_ERR_TIMEOUT_TFULL)) {
              ok = false;
              break;
            }
            FM_TR(tch, 2);
            tc_fence_after();
            const int tok0 = I0 + c * kFlatCT;
            const int ncols = min(kFlatCT, I1 - tok0);
            // documents ending in this chunk: at chunk columns e0 (, e1); nb of them
            const int e_a = tok0 / a.Ld;  // document open at the chunk's first column
            const int e0 = (e_a + 1) * a.Ld - tok0;
            const int e1 = e0 + a.Ld;
            const int nb = e0 > ncols ? 0 : (e1 > ncols ? 1 : 2);
            float m0 = -INFINITY, m1 = -INFINITY, m2 = -INFINITY;
            const uint32_t taddr = tmem_base + lane_base + tr.idx * kFlatCT;
            {
              // this warp's pieces: set, set + 2, set + 4 (32 columns each)
              const int np = (ncols + 31) >> 5;
              for (int p = set; p < np; p += 4) {  // two loads in flight
                const bool two = p + 2 < np;
                float v[32], w[32];
                tmem_ld32(taddr + 32 * p, v);
                if (two) tmem_ld32(taddr + 32 * (p + 2), w);
                tmem_wait_ld();
                if (!skip_epi) {
                  fold_piece(v, 32 * p, min(32, ncols - 32 * p), e0, e1, nb, m0, m1, m2);
                  if (two) fold_piece(w, 32 * (p + 2), min(32, ncols - 32 * (p + 2)), e0, e1, nb, m0, m1, m2);
                }
              }
              FM_TR(tch, 3);
              // the accumulator slot is free once its columns are in registers
              tc_fence_before();
              __syncwarp();
              if (lane == 0) mbar_arrive(t_empty(tr.idx));
              tr.next(kFlatTS);
            }
            FM_TR(tch, 4);
            const int xb = kc & (kFlatXch - 1);
            float* xq = xch + ((xb * 4 + sub) * kFlatSeg) * 32 + lane;
            if (set == 0) {
              // hand the segment maxima to the odd-piece warp of this quarter
              xq[0] = m0;
              if (nb >= 1) xq[32] = m1;
              if (nb >= 2) xq[64] = m2;
              __syncwarp();
              if (lane == 0) mbar_arrive(x_full(xb, sub));
            } else {
              if (!mbar_wait(x_full(xb, sub), (xph >> xb) & 1u, ctl, FM_ERR_TIMEOUT_TFULL)) {
                ok = false;
                break;
              }
              xph ^= 1u << xb;
              FM_TR(tch, 5);
              m0 = fmaxf(m0, xq[0]);
              if (nb >= 1) m1 = fmaxf(m1, xq[32]);
              if (nb >= 2) m2 = fmaxf(m2, xq[64]);
              // close the documents that end in this chunk; carry the open one
              float open = fmaxf(carry, m0);
              if (nb >= 1) {
                const float t0 = warp_sum(active ? open : 0.f);
                if (lane == 0 && active) rb[(e_a - e_first) * 128 + lrg] = t0;
                open = m1;
                if (nb >= 2) {
                  const float t1 = warp_sum(active ? open : 0.f);
                  if (lane == 0 && active) rb[(e_a + 1 - e_first) * 128 + lrg] = t1;
                  open = m2;
                }
              }
              carry = open;
              FM_TR(tch, 6);
            }
          }
          if (!ok) break;
          if (set == 1) {
            tmem_st1(carry_addr, carry);
            tmem_wait_st();
          }
        }
        // every document ending in this item has all its row-group sums: score them
        // (every epilogue warp arrives, also after a failed wait)
        __syncwarp();
        if (lane == 0) mbar_arrive(item_bar(ibuf));
        if (!ok) break;
        if (!mbar_wait(item_bar(ibuf), (iph >> ibuf) & 1u, ctl, FM_ERR_TIMEOUT_TFULL)) {
          ok = false;
          break;
        }
        iph ^= 1u << ibuf;
        const int e_end = I1 / a.Ld;  // documents [e_first, e_end) end in this item
        const int nq0 = rg0 / a.Gq, nqs = srg / a.Gq;
        for (int x = et; x < (e_end - e_first) * nqs; x += 256) {
          const int i = x / nqs;
          const int n = x - i * nqs;
          float s = 0.f;
          for (int g = 0; g < a.Gq; ++g) s += rb[i * 128 + n * a.Gq + g];
          a.scores[static_cast<size_t>(nq0 + n) * a.B + e_first + i] = s;
        }
        ibuf ^= 1;
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 512);
  }
}

}  // namespace fm
