// Dense fp16 MaxSim for one short query (Lq <= 64, d <= 128), sm_100a.
//
//   score[b] = sum_q max_{t < len_b} <Q[q], D[b, t]>
//
// Same result as the reference's `_maxsim_fwd_kernel` with Nq = 1
// (flash_maxsim/flash_maxsim.py:24-77, launched by flash_maxsim() at
// flash_maxsim.py:221-230), organised for a pass that is bound by HBM:
//
//  * The document is the M operand.  TMA copies a chunk of CT consecutive
//    tokens (all K atoms) from HBM into 128-byte-swizzled shared memory and
//    the tensor core multiplies each 128-token half against the whole query,
//    which is the N operand (N = 32 per 32 query rows, loaded once per CTA).
//    The short query is therefore never replicated over 128 MMA rows, and one
//    chunk costs CT/128 x d/16 small MMAs instead of a 128-row query block
//    per 32 rows.
//  * TMEM lane = token, column = query row.  Each epilogue thread owns one
//    token of every chunk it takes and keeps a running max per query row over
//    its tokens (tokens past the document are masked).  At the end of a
//    document a 31-shuffle butterfly leaves lane j with the max of query row j
//    over the warp's tokens, and the last warp of the document to finish
//    combines the warps' maxima and writes the score.
//  * Documents go to CTAs round robin; chunks never span two documents, so
//    the TMA box of a document's last chunk reads only the document's rows
//    (rows past Ld are zero-filled by the copy engine, not read).
//
// Warp roles: 0 = producer (query once, then document chunks), 1 = MMA issuer
// and TMEM owner, 2..2+EW-1 = epilogue (two warps per TMEM lane quarter when
// EW = 8, taking alternate chunks).
#pragma once

#include <cuda.h>
#include <cstdint>
#include <cuda_fp16.h>
#include "fm_fwd.cuh"
#include "fm_ptx.cuh"

namespace fm {

__host__ __device__ constexpr int q1_threads(int epi_warps) { return (2 + epi_warps) * 32; }
constexpr int kQ1Xch = 8;  // per-document exchange slots of the epilogue

struct Q1Args {
  const int32_t* lengths;  // [B] or null
  const int32_t* cu;       // packed documents: [B + 1] token offsets into D [T, d], or null
  float* scores;           // [B]
  int* status;
  uint64_t timeout_ns;
  int B, Lq, Ld, d;
  int N;                   // MMA N = 32 x GQ query rows
  int atoms;               // 64-element K atoms (ceil(d / 64))
  int nu;                  // document ring slots
  int nts;                 // TMEM slots (CT / 128 halves of N columns each)
  uint32_t off_q, off_u, off_misc, off_bar, u_slot_bytes;
  const int32_t* sp_idx;    // sparse scoring: [B, K] query-row indices (negative ones wrap), else null
  int K;                   // indices per document (sparse scoring)
  int sparse;              // 1: score[b] = sum_k rowmax[idx[b, k]]
  int dbg;  // tuning builds (FM_TUNING) only: bits that switch off parts of the work
  TopkArgs topk;           // k > 0: per-CTA top-k candidates in the tail
};

__device__ __forceinline__ int q1_len(const Q1Args& a, int b) {
  int len = a.cu ? __ldg(a.cu + b + 1) - __ldg(a.cu + b) : (a.lengths ? __ldg(a.lengths + b) : a.Ld);
  return len < 0 ? 0 : (len > a.Ld ? a.Ld : len);
}

// Max over the 32 lanes of v[j] for every j; afterwards lane j's v[0] holds
// column j's maximum.  Lanes with bit o set keep the upper half at offset o.
__device__ __forceinline__ float q1_butterfly_max32(float (&v)[32], int lane) {
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) {
    const bool up = (lane & o) != 0;
#pragma unroll
    for (int i = 0; i < o; ++i) {
      const float send = up ? v[i] : v[i + o];
      const float keep = up ? v[i + o] : v[i];
      v[i] = fmaxf(keep, __shfl_xor_sync(0xffffffffu, send, o));
    }
  }
  return v[0];
}

__device__ __forceinline__ void q1_drain(uint32_t bar, uint32_t parity, const Q1Args& a) {
  const uint64_t t0 = globaltimer_ns();
  while (!mbar_try_wait(bar, parity)) {
    if (globaltimer_ns() - t0 > a.timeout_ns) {
      record_status(a.status, FM_ERR_TIMEOUT_DRAIN);
      break;
    }
  }
}

template <int GQ, int EW, int CT>
__global__ void __launch_bounds__(q1_threads(EW), 1)
    maxsim_q1_kernel(const __grid_constant__ CUtensorMap tmap_q, const __grid_constant__ CUtensorMap tmap_d,
                     const Q1Args a) {
  constexpr int NH = CT / 128;  // 128-token MMA halves per chunk
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const uint32_t sbase = smem_u32(smem);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  // barriers: u_full[nu] u_empty[nu] t_full[nts] t_empty[nts] q_full drain
  const uint32_t bar0 = sbase + a.off_bar;
  auto u_full = [&](int i) { return bar0 + 8u * i; };
  auto u_empty = [&](int i) { return bar0 + 8u * (a.nu + i); };
  auto t_full = [&](int i) { return bar0 + 8u * (2 * a.nu + i); };
  auto t_empty = [&](int i) { return bar0 + 8u * (2 * a.nu + a.nts + i); };
  const uint32_t q_full = bar0 + 8u * (2 * a.nu + 2 * a.nts);
  const uint32_t drain = q_full + 8u;
  uint8_t* ctl_area = smem + a.off_bar + 8 * (2 * a.nu + 2 * a.nts + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(ctl_area);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(ctl_area + 8);
  WaitCtl ctl{abort_flag, a.status, a.timeout_ns};

  float* xch = reinterpret_cast<float*>(smem + a.off_misc);        // [kQ1Xch docs][EW warps][GQ][32]
  int* cnt = reinterpret_cast<int*>(xch + kQ1Xch * EW * GQ * 32);  // [kQ1Xch] arrivals
  volatile int* done = cnt + kQ1Xch;                               // [kQ1Xch] combined generations
  float* rowmax_s = reinterpret_cast<float*>(cnt + 2 * kQ1Xch);   // [EW][32 GQ] sparse scoring

  if (threadIdx.x == 0) {
    for (int i = 0; i < a.nu; ++i) {
      mbar_init(u_full(i), 1);   // producer's expect_tx arrival + transaction bytes
      mbar_init(u_empty(i), 1);  // MMA commit
    }
    for (int i = 0; i < a.nts; ++i) {
      mbar_init(t_full(i), 1);
      mbar_init(t_empty(i), 4);  // the four warps (one per lane quarter) that take the chunk
    }
    mbar_init(q_full, 1);
    mbar_init(drain, 1);
    *abort_flag = 0;
    for (int i = 0; i < kQ1Xch; ++i) {
      cnt[i] = 0;
      done[i] = 0;
    }
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
  // the prologue above may overlap the previous kernel in the stream; inputs
  // are read only after it has completed
  grid_dep_wait();
  grid_dep_launch();
  const uint32_t tmem_base = *tmem_slot;
  const int w0 = blockIdx.x, wstep = gridDim.x;
  const uint32_t ts_stride = NH * a.N;  // TMEM columns per slot

  if (warp == 0) {
    // ===================== producer =====================
    if (lane == 0) {
      const uint64_t pol = l2_policy_evict_first();
      const uint64_t pol_q = l2_policy_evict_last();
      // the query, once: one box of N rows per K atom (rows past Lq read as zero)
      mbar_expect_tx(q_full, a.atoms * a.N * 128u);
      for (int at = 0; at < a.atoms; ++at)
        tma_load_3d(sbase + a.off_q + at * a.N * 128, &tmap_q, at * 64, 0, 0, q_full, pol_q);
      const uint32_t tx = a.atoms * CT * 128u;
      Ring ur;
      int issued = 0;
      bool ok = true;
      for (int b = w0; b < a.B && ok; b += wstep) {
        const int nch = (q1_len(a, b) + CT - 1) / CT;
        for (int c = 0; c < nch; ++c) {
          if (!mbar_wait(u_empty(ur.idx), ur.phase ^ 1u, ctl, FM_ERR_TIMEOUT_UEMPTY)) {
            ok = false;
            break;
          }
          mbar_expect_tx(u_full(ur.idx), tx);
          const uint32_t dst = sbase + a.off_u + ur.idx * a.u_slot_bytes;
          const int row = (a.cu ? __ldg(a.cu + b) : 0) + c * CT;  // packed: row of a [T, d] map
          const int zc = a.cu ? 0 : b;
          for (int at = 0; at < a.atoms; ++at)
            tma_load_3d(dst + at * CT * 128, &tmap_d, at * 64, row, zc, u_full(ur.idx), pol);
          ur.next(a.nu);
          ++issued;
        }
      }
      for (int i = 0; i < a.nu && i < issued; ++i) {
        if (--ur.idx < 0) {
          ur.idx = a.nu - 1;
          ur.phase ^= 1u;
        }
        q1_drain(u_full(ur.idx), ur.phase, a);
      }
      q1_drain(q_full, 0, a);
    }
  } else if (warp == 1) {
    // ===================== MMA issuer =====================
    if (lane == 0) {
      // A = document half (M = 128 tokens), B = query (N rows), both K-major fp16
      const uint32_t idesc = idesc_f16_f32(128, a.N);
      const uint64_t bq = smem_desc_sw128(sbase + a.off_q);
      const uint32_t q_atom = a.N * 8u;  // one K atom of the query, 16-byte units
      const uint32_t d_atom = CT * 8u;   // one K atom of a chunk
      const int ksteps = a.atoms * 4;    // K = 16 per MMA, 4 per 64-element atom
      Ring ur, tr;
      bool ok = mbar_wait(q_full, 0, ctl, FM_ERR_TIMEOUT_QFULL);
      tc_fence_after();
      for (int b = w0; b < a.B && ok; b += wstep) {
        const int nch = (q1_len(a, b) + CT - 1) / CT;
        for (int c = 0; c < nch; ++c) {
          if (!mbar_wait(u_full(ur.idx), ur.phase, ctl, FM_ERR_TIMEOUT_UFULL)) { ok = false; break; }
          if (!mbar_wait(t_empty(tr.idx), tr.phase ^ 1u, ctl, FM_ERR_TIMEOUT_TEMPTY)) { ok = false; break; }
          tc_fence_after();
          const uint64_t ad = smem_desc_sw128(sbase + a.off_u + ur.idx * a.u_slot_bytes);
          const uint32_t tacc = tmem_base + tr.idx * ts_stride;
          if (!FM_DBG(a, 2)) {
#pragma unroll
            for (int hb = 0; hb < NH; ++hb) {  // rows [128 hb, 128 hb + 128) of the chunk
              const uint64_t ah = ad + hb * (128u * 128u >> 4);
#pragma unroll
              for (int kk = 0; kk < 8; ++kk) {
                if (kk < ksteps)
                  tc_mma_f16(tacc + hb * a.N, ah + (kk >> 2) * d_atom + (kk & 3) * 2u,
                             bq + (kk >> 2) * q_atom + (kk & 3) * 2u, idesc, kk > 0 ? 1u : 0u);
              }
            }
          }
          tc_commit(t_full(tr.idx));
          tc_commit(u_empty(ur.idx));
          tr.next(a.nts);
          ur.next(a.nu);
        }
      }
      tc_commit(drain);
      q1_drain(drain, 0, a);
    }
  } else {
    // ===================== epilogue =====================
    const int sub = warp & 3;  // TMEM lane quarter = tokens [32 sub, 32 sub + 32) of each half
    // EW == 8: the two warps of a lane quarter own alternate TMEM slots (the
    // slot count is even), so every use of a slot is read by the same warp and
    // no warp ever waits on a slot barrier more than one phase ahead
    const int half = (EW == 8) ? (warp - 2) / 4 : 0;
    const uint32_t lane_base = static_cast<uint32_t>(sub * 32) << 16;
    const int tok_in_half = sub * 32 + lane;
    Ring tr;
    int dloc = 0;
    int kglob = 0;  // chunk counter of this CTA
    bool ok = true;
    for (int b = w0; b < a.B && ok; b += wstep, ++dloc) {
      const int len = q1_len(a, b);
      const int nch = (len + CT - 1) / CT;
      // running max per query row over this thread's tokens; lanes are reduced per document
      float rmax[32 * GQ];
#pragma unroll
      for (int j = 0; j < 32 * GQ; ++j) rmax[j] = -INFINITY;
      for (int c = 0; c < nch; ++c, ++kglob) {
        if (EW == 8 && (tr.idx & 1) != half) {  // the other warp of this lane quarter reads it
          tr.next(a.nts);
          continue;
        }
        if (!mbar_wait(t_full(tr.idx), tr.phase, ctl, FM_ERR_TIMEOUT_TFULL)) { ok = false; break; }
        tc_fence_after();
        const int tok0 = c * CT;
        const bool full = tok0 + CT <= len;  // whole chunk valid (warp-uniform)
        const uint32_t th = tmem_base + lane_base + tr.idx * ts_stride;
        const bool v0ok = tok0 + tok_in_half < len;
        const bool v1ok = tok0 + 128 + tok_in_half < len;
#pragma unroll
        for (int g = 0; g < GQ; ++g) {
          float v0[32], v1[32];
          tmem_ld32(th + g * 32, v0);
          if (NH == 2) tmem_ld32(th + a.N + g * 32, v1);
          tmem_wait_ld();
          if (!FM_DBG(a, 1)) {
            if (full) {
#pragma unroll
              for (int j = 0; j < 32; ++j)
                rmax[g * 32 + j] = NH == 2 ? fmax3(rmax[g * 32 + j], v0[j], v1[j]) : fmaxf(rmax[g * 32 + j], v0[j]);
            } else {
#pragma unroll
              for (int j = 0; j < 32; ++j) {
                const float x0 = v0ok ? v0[j] : -INFINITY;
                const float x1 = (NH == 2 && v1ok) ? v1[j] : -INFINITY;
                rmax[g * 32 + j] = fmax3(rmax[g * 32 + j], x0, x1);
              }
            }
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(t_empty(tr.idx));
        tr.next(a.nts);
      }
      if (!ok) break;
      float acc[GQ];
#pragma unroll
      for (int g = 0; g < GQ; ++g) {
        float v[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = rmax[g * 32 + j];
        acc[g] = q1_butterfly_max32(v, lane);
      }
      // --- combine the warps of this document: the last one to arrive sums ---
      const int slot = dloc % kQ1Xch;
      const int gen = dloc / kQ1Xch;
      // a warp can run ahead (short or empty documents): wait until the slot's
      // previous document has been combined
      if (gen > 0) {
        const uint64_t t0 = globaltimer_ns();
        while (done[slot] < gen) {
          if (*abort_flag) { ok = false; break; }
          if (globaltimer_ns() - t0 > a.timeout_ns) {
            *abort_flag = 1;
            record_status(a.status, FM_ERR_TIMEOUT_TFULL);
            ok = false;
            break;
          }
        }
        if (!ok) break;
        __threadfence_block();
      }
      const int ew = warp - 2;
#pragma unroll
      for (int g = 0; g < GQ; ++g) xch[((slot * EW + ew) * GQ + g) * 32 + lane] = acc[g];
      __syncwarp();
      int old = 0;
      if (lane == 0) {
        __threadfence_block();
        old = atomicAdd(&cnt[slot], 1);
      }
      old = __shfl_sync(0xffffffffu, old, 0);
      if (old == EW - 1) {
        __threadfence_block();
        float tot = 0.f;
        float* rm = rowmax_s + ew * 32 * GQ;
#pragma unroll
        for (int g = 0; g < GQ; ++g) {
          float mm = -INFINITY;
          for (int w = 0; w < EW; ++w) mm = fmaxf(mm, xch[((slot * EW + w) * GQ + g) * 32 + lane]);
          tot += (g * 32 + lane < a.Lq) ? mm : 0.f;
          rm[g * 32 + lane] = mm;
        }
        if (a.sparse) {
          // score = sum over the document's K query-row indices of their row maxima
          // (flash_maxsim/flash_maxsim_sparse.py:60-80); an empty document scores
          // 0 when K == 0 and -inf otherwise
          __syncwarp();
          tot = 0.f;
          if (len == 0) {
            tot = (a.K == 0 || lane != 0) ? 0.f : -INFINITY;
          } else {
            const int32_t* ip = a.sp_idx + static_cast<size_t>(b) * a.K;
            for (int k = lane; k < a.K; k += 32) {
              int q = __ldg(ip + k);
              if (q < 0) q += a.Lq;
              if (q < 0 || q >= a.Lq) {
                record_status(a.status, FM_ERR_BAD_INDEX);
                continue;
              }
              tot += rm[q];
            }
          }
        }
        tot = warp_sum(tot);
        if (lane == 0) {
          a.scores[b] = tot;
          cnt[slot] = 0;
          __threadfence_block();
          done[slot] = gen + 1;
        }
        __syncwarp();
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 512);
  }
  if (a.topk.k > 0 && warp == 2 && !*abort_flag) {
    // Top-k tail: the k best of the documents this CTA scored (w0, w0 + wstep,
    // ...), read back from the scores it just wrote (plain loads).
    const int count = (a.B - w0 + wstep - 1) / wstep;
    const size_t o = static_cast<size_t>(blockIdx.x) * a.topk.k;
    warp_topk<8>(count, a.topk.k,
                 [&](int p) {
                   const int b = w0 + p * wstep;
                   return TopkCand{a.scores[b], b};
                 },
                 a.topk.cand_s + o, a.topk.cand_b + o, lane);
  }
}

}  // namespace fm
