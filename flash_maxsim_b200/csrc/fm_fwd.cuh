// MaxSim forward kernel for sm_100a (B200).
//
//   score[n, b] = sum_{q < Lq} max_{t < len_b} <Q[n, q, :], D[b, t, :]>
//
// The same computation as the reference's `_maxsim_fwd_kernel`
// (flash_maxsim/flash_maxsim.py:83-146), its INT8 variant
// (flash_maxsim/flash_maxsim_quant.py:52-98) and its sparse variant
// (flash_maxsim/flash_maxsim_sparse.py:42-91), organised for Blackwell:
//
//  * Work item = one document (shared docs: scored against every query;
//    per-query docs: one (query, doc) pair).  Persistent CTAs stride over
//    work items.
//  * A document is split into chunks of C tokens (C <= 256, multiple of 16).
//    A group of G chunks is kept resident in a shared-memory ring (D ring,
//    filled by TMA from HBM, 128-byte swizzle, OOB rows zero-filled).
//  * Query rows are packed into 128-row "M-blocks" of four 32-row row groups
//    (one row group = 32 consecutive tokens of one query, rows past Lq are
//    TMA zero-fill).  M-blocks stream from L2 through a Q ring.
//  * tcgen05.mma (M=128, N=C, K=16, fp16 in, fp32 accumulate) computes
//    S = Qblock . Dchunk^T straight into TMEM: lane = query row,
//    column = doc token.  TMEM holds a ring of accumulator slots, so the
//    epilogue drains one slot while the tensor core fills the next.
//  * The epilogue (4 warps, one TMEM lane per thread) takes the running max
//    of its row over the valid columns (tokens >= len are skipped), keeps it
//    across chunks in registers and across chunk groups in shared memory,
//    then reduces rows of the same query with warp shuffles.  The similarity
//    matrix never leaves the SM.
//  * When a work item only needs one or two row groups (single-query scoring)
//    the row groups are replicated across the four TMEM lane quarters and the
//    four epilogue warps split the columns between them, so the epilogue
//    never limits an HBM-bound stream.
//
// Warp roles: 0 = D producer (TMA), 1 = MMA issuer + TMEM owner,
// 2..5 = epilogue, 6 = Q producer (TMA), 7..10 = INT8 converters (INT8 only).
#pragma once

#include <cuda.h>
#include <cstdint>
#include <cuda_fp16.h>
#include "fm_ptx.cuh"

namespace fm {

enum FwdMode : int { MODE_DENSE = 0, MODE_SPARSE = 1, MODE_INT8 = 2 };

constexpr int kEpiWarp0 = 2;
constexpr int kQProdWarp = 6;
constexpr int kConvWarp0 = 7;
constexpr int kThreadsF16 = 7 * 32;
constexpr int kThreadsI8 = 11 * 32;

struct FwdArgs {
  const int32_t* lengths;    // [n_docs] valid tokens per doc, or null (all Ld)
  float* scores;             // [Nq, B] (dense), [B] (sparse / int8)
  int32_t* argmax;           // [Nq*B, Lq] or null
  const int32_t* sp_idx;     // sparse: [B, K]
  const __half* q;           // Q, [Nq, Lq, d] contiguous (INT8 uses it for row sums)
  const __half* scales;      // INT8: [B, Ld]
  const __half* mins;        // INT8: [B, Ld]
  int* status;               // status word (global)
  uint64_t timeout_ns;
  int Nq, B, Lq, Ld, d, K;
  int shared;                // 1: every doc against every query
  int n_work;                // number of work items
  int Gq;                    // row groups per query = ceil(Lq / 32)
  int R;                     // row groups per work item
  int C;                     // tokens per chunk (MMA N)
  int G;                     // chunks per resident group
  int nd;                    // D ring slots (chunks)
  int nq;                    // Q ring stages
  int nu;                    // INT8 staging slots
  int nk;                    // Q stages per M-block (K split)
  int kq_atoms;              // 64-element K atoms per Q stage
  int d_atoms;               // 64-element K atoms per token in smem (nk * kq_atoms)
  int d_atoms_real;          // atoms that hold data (ceil(d / 64)); the rest stay zero
  int RS;                    // row groups per span when a doc needs >1 group
  int rep;                   // lane-quarter replication (1, 2 or 4)
  int q_resident;            // Q loaded once for the whole launch
  int nts;                   // TMEM accumulator slots
  int ts_stride;             // TMEM columns per slot
  int rowbuf;                // floats in the per-doc row buffer
  uint32_t off_q, off_d, off_u, off_state, off_rows, off_xch, off_qsum, off_bar;
  uint32_t q_stage_bytes, d_slot_bytes, u_slot_bytes;
};

// Schedule of one work item, computed identically by every role.
struct Item {
  int doc;      // index of the doc in D (flattened for per-query docs)
  int b;        // score column
  int n_lo;     // first query of the item
  int nqi;      // queries in the item
  int rg_lo;    // first row group
  int rg_hi;    // one past the last row group
  int len;      // valid tokens (clamped to [0, Ld])
  int nch;      // chunks
  int ngr;      // chunk groups
  int span;     // row groups per span
};

__device__ __forceinline__ Item make_item(const FwdArgs& a, int w) {
  Item it;
  if (a.shared) {
    it.doc = w;
    it.b = w;
    it.n_lo = 0;
    it.nqi = a.Nq;
    it.rg_lo = 0;
    it.rg_hi = a.Nq * a.Gq;
  } else {
    const int n = w / a.B;
    it.doc = w;
    it.b = w - n * a.B;
    it.n_lo = n;
    it.nqi = 1;
    it.rg_lo = n * a.Gq;
    it.rg_hi = it.rg_lo + a.Gq;
  }
  int len = a.lengths ? __ldg(a.lengths + it.doc) : a.Ld;
  len = len < 0 ? 0 : (len > a.Ld ? a.Ld : len);
  it.len = len;
  it.nch = (len + a.C - 1) / a.C;
  it.ngr = (it.nch + a.G - 1) / a.G;
  it.span = (it.ngr > 1) ? a.RS : (it.rg_hi - it.rg_lo);
  return it;
}

// M-blocks in a span of row groups [s0, s1)
__device__ __forceinline__ int span_mblocks(const FwdArgs& a, int s0, int s1) {
  return a.rep > 1 ? 1 : (s1 - s0 + 3) / 4;
}

struct SmemBars {
  uint32_t base;
  int nq, nd, nts, nu;
  __device__ uint32_t q_full(int i) const { return base + 8u * i; }
  __device__ uint32_t q_empty(int i) const { return base + 8u * (nq + i); }
  __device__ uint32_t d_full(int i) const { return base + 8u * (2 * nq + i); }
  __device__ uint32_t d_empty(int i) const { return base + 8u * (2 * nq + nd + i); }
  __device__ uint32_t t_full(int i) const { return base + 8u * (2 * nq + 2 * nd + i); }
  __device__ uint32_t t_empty(int i) const { return base + 8u * (2 * nq + 2 * nd + nts + i); }
  __device__ uint32_t u_full(int i) const { return base + 8u * (2 * nq + 2 * nd + 2 * nts + i); }
  __device__ uint32_t u_empty(int i) const {
    return base + 8u * (2 * nq + 2 * nd + 2 * nts + nu + i);
  }
  __device__ uint32_t drain() const { return base + 8u * (2 * nq + 2 * nd + 2 * nts + 2 * nu); }
  __device__ uint32_t end() const { return drain() + 8u; }
};

// -------------------------------------------------------------------------
// epilogue helpers
// -------------------------------------------------------------------------
template <bool ARGMAX>
struct RowAcc {
  float m;
  int idx;
  __device__ __forceinline__ void init() {
    m = -INFINITY;
    idx = 0;
  }
  __device__ __forceinline__ void merge(float mv, int iv) {
    if (ARGMAX) {
      if (mv > m || (mv == m && iv < idx)) {
        m = mv;
        idx = iv;
      }
    } else {
      m = fmaxf(m, mv);
    }
  }
};

// Max (and first argmax) of one 32-column piece; nv valid columns.
template <bool ARGMAX>
__device__ __forceinline__ void piece_max(const float (&v)[32], int nv, int col0, RowAcc<ARGMAX>& acc) {
  if (ARGMAX) {
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      if (i < nv && v[i] > acc.m) {
        acc.m = v[i];
        acc.idx = col0 + i;
      }
    }
  } else {
    if (nv == 32) {
      float a0 = fmax3(v[0], v[1], v[2]);
      float a1 = fmax3(v[3], v[4], v[5]);
      float a2 = fmax3(v[6], v[7], v[8]);
      float a3 = fmax3(v[9], v[10], v[11]);
      float a4 = fmax3(v[12], v[13], v[14]);
      float a5 = fmax3(v[15], v[16], v[17]);
      float a6 = fmax3(v[18], v[19], v[20]);
      float a7 = fmax3(v[21], v[22], v[23]);
      float a8 = fmax3(v[24], v[25], v[26]);
      float a9 = fmax3(v[27], v[28], v[29]);
      float b0 = fmax3(a0, a1, a2);
      float b1 = fmax3(a3, a4, a5);
      float b2 = fmax3(a6, a7, a8);
      float b3 = fmax3(a9, v[30], v[31]);
      acc.m = fmax3(acc.m, fmax3(b0, b1, b2), b3);
    } else {
      float m = acc.m;
#pragma unroll
      for (int i = 0; i < 32; ++i)
        if (i < nv) m = fmaxf(m, v[i]);
      acc.m = m;
    }
  }
}

__device__ __forceinline__ float warp_sum(float x) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
  return x;
}

// -------------------------------------------------------------------------
// the kernel
// -------------------------------------------------------------------------
template <int MODE, bool ARGMAX>
__global__ void __launch_bounds__(MODE == MODE_INT8 ? kThreadsI8 : kThreadsF16, 1)
    maxsim_fwd_kernel(const __grid_constant__ CUtensorMap tmap_q,
                      const __grid_constant__ CUtensorMap tmap_d, const FwdArgs a) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // 1024-byte alignment of the operand rings (required by the 128 B swizzle)
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const uint32_t sbase = smem_u32(smem);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  SmemBars bars;
  bars.base = sbase + a.off_bar;
  bars.nq = a.nq;
  bars.nd = a.nd;
  bars.nts = a.nts;
  bars.nu = (MODE == MODE_INT8) ? a.nu : 0;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + a.off_bar + (bars.end() - bars.base));
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + a.off_bar + (bars.end() - bars.base) + 8);
  WaitCtl ctl{abort_flag, a.status, a.timeout_ns};

  if (threadIdx.x == 0) {
    for (int i = 0; i < a.nq; ++i) {
      mbar_init(bars.q_full(i), 1);
      mbar_init(bars.q_empty(i), 1);
    }
    for (int i = 0; i < a.nd; ++i) {
      mbar_init(bars.d_full(i), MODE == MODE_INT8 ? 128 : 1);
      mbar_init(bars.d_empty(i), 1);
    }
    for (int i = 0; i < a.nts; ++i) {
      mbar_init(bars.t_full(i), 1);
      mbar_init(bars.t_empty(i), 4);
    }
    if (MODE == MODE_INT8) {
      for (int i = 0; i < a.nu; ++i) {
        mbar_init(bars.u_full(i), 1);
        mbar_init(bars.u_empty(i), 128);
      }
    }
    mbar_init(bars.drain(), 1);
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
  // Zero the Q ring and the K-padding atoms of every D slot once: padded
  // atoms are never loaded, so the tensor core always multiplies finite
  // values by exact zeros there.
  {
    uint4* qz = reinterpret_cast<uint4*>(smem + a.off_q);
    const int nq16 = a.nq * a.q_stage_bytes / 16;
    for (int i = threadIdx.x; i < nq16; i += blockDim.x) qz[i] = make_uint4(0, 0, 0, 0);
    const int pad16 = (a.d_atoms - a.d_atoms_real) * a.C * 128 / 16;
    for (int s = 0; s < a.nd && pad16 > 0; ++s) {
      uint4* dz = reinterpret_cast<uint4*>(smem + a.off_d + s * a.d_slot_bytes +
                                           a.d_atoms_real * a.C * 128);
      for (int i = threadIdx.x; i < pad16; i += blockDim.x) dz[i] = make_uint4(0, 0, 0, 0);
    }
    fence_proxy_async_smem();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const int w0 = blockIdx.x;
  const int wstep = gridDim.x;

  if (warp == 0) {
    // ===================== D producer =====================
    if (lane == 0) {
      const uint64_t pol = l2_policy_evict_first();
      int dcnt = 0;
      bool ok = true;
      for (int w = w0; w < a.n_work && ok; w += wstep) {
        const Item it = make_item(a, w);
        for (int s0 = it.rg_lo; s0 < it.rg_hi && ok; s0 += it.span) {
          for (int g = 0; g < it.ngr && ok; ++g) {
            const int c0 = g * a.G;
            const int cn = min(a.G, it.nch - c0);
            for (int c = 0; c < cn; ++c) {
              if (MODE == MODE_INT8) {
                const int slot = dcnt % a.nu;
                const uint32_t ph = (dcnt / a.nu) & 1;
                if (!mbar_wait(bars.u_empty(slot), ph ^ 1, ctl, FM_ERR_TIMEOUT_UEMPTY)) { ok = false; break; }
                mbar_expect_tx(bars.u_full(slot), a.d_atoms_real * a.C * 64u);
                const uint32_t dst = sbase + a.off_u + slot * a.u_slot_bytes;
                for (int at = 0; at < a.d_atoms_real; ++at)
                  tma_load_3d(dst + at * a.C * 64, &tmap_d, at * 64, (c0 + c) * a.C, it.doc,
                              bars.u_full(slot), pol);
              } else {
                const int slot = dcnt % a.nd;
                const uint32_t ph = (dcnt / a.nd) & 1;
                if (!mbar_wait(bars.d_empty(slot), ph ^ 1, ctl, FM_ERR_TIMEOUT_DEMPTY)) { ok = false; break; }
                mbar_expect_tx(bars.d_full(slot), a.d_atoms_real * a.C * 128u);
                const uint32_t dst = sbase + a.off_d + slot * a.d_slot_bytes;
                for (int at = 0; at < a.d_atoms_real; ++at)
                  tma_load_3d(dst + at * a.C * 128, &tmap_d, at * 64, (c0 + c) * a.C, it.doc,
                              bars.d_full(slot), pol);
              }
              ++dcnt;
            }
          }
        }
      }
      // Wait (bounded) for the last load issued into every slot to land so
      // no bulk copy is in flight when the CTA exits.
      const int nslots = (MODE == MODE_INT8) ? a.nu : a.nd;
      for (int i = 0; i < nslots && i < dcnt; ++i) {
        const int k = dcnt - 1 - i;
        const int slot = (MODE == MODE_INT8) ? k % a.nu : k % a.nd;
        const uint32_t ph = (MODE == MODE_INT8) ? (k / a.nu) & 1 : (k / a.nd) & 1;
        const uint32_t bar = (MODE == MODE_INT8) ? bars.u_full(slot) : bars.d_full(slot);
        const uint64_t t0 = globaltimer_ns();
        while (!mbar_try_wait(bar, ph)) {
          if (globaltimer_ns() - t0 > a.timeout_ns) {
            record_status(a.status, FM_ERR_TIMEOUT_DRAIN);
            break;
          }
        }
      }
    }
  } else if (warp == kQProdWarp) {
    // ===================== Q producer =====================
    if (lane == 0) {
      const uint64_t pol = l2_policy_evict_last();
      int qcnt = 0;
      bool ok = true;
      for (int w = w0; w < a.n_work && ok; w += wstep) {
        const Item it = make_item(a, w);
        if (it.nch == 0) continue;
        for (int s0 = it.rg_lo; s0 < it.rg_hi && ok; s0 += it.span) {
          const int s1 = min(it.rg_hi, s0 + it.span);
          const int nmb = span_mblocks(a, s0, s1);
          for (int g = 0; g < it.ngr && ok; ++g) {
            for (int jb = 0; jb < nmb && ok; ++jb) {
              for (int ks = 0; ks < a.nk; ++ks) {
                if (a.q_resident && qcnt > 0) break;
                const int slot = qcnt % a.nq;
                const uint32_t ph = (qcnt / a.nq) & 1;
                if (!mbar_wait(bars.q_empty(slot), ph ^ 1, ctl, FM_ERR_TIMEOUT_QEMPTY)) { ok = false; break; }
                int nload = 0;
                for (int sub = 0; sub < 4; ++sub) {
                  const int rg = (a.rep > 1) ? s0 + sub / a.rep : s0 + 4 * jb + sub;
                  if (rg < s1) ++nload;
                }
                const int at_hi = min(a.kq_atoms, a.d_atoms_real - ks * a.kq_atoms);
                mbar_expect_tx(bars.q_full(slot), nload * at_hi * 4096u);
                const uint32_t dst = sbase + a.off_q + slot * a.q_stage_bytes;
                for (int sub = 0; sub < 4; ++sub) {
                  const int rg = (a.rep > 1) ? s0 + sub / a.rep : s0 + 4 * jb + sub;
                  if (rg >= s1) continue;
                  const int qn = rg / a.Gq;
                  const int qy = (rg - qn * a.Gq) * 32;
                  for (int at = 0; at < at_hi; ++at)
                    tma_load_3d(dst + at * 16384 + sub * 4096, &tmap_q, (ks * a.kq_atoms + at) * 64,
                                qy, qn, bars.q_full(slot), pol);
                }
                ++qcnt;
              }
            }
          }
        }
      }
      for (int i = 0; i < a.nq && i < qcnt; ++i) {
        const int k = qcnt - 1 - i;
        const uint64_t t0 = globaltimer_ns();
        while (!mbar_try_wait(bars.q_full(k % a.nq), (k / a.nq) & 1)) {
          if (globaltimer_ns() - t0 > a.timeout_ns) {
            record_status(a.status, FM_ERR_TIMEOUT_DRAIN);
            break;
          }
        }
      }
    }
  } else if (warp == 1) {
    // ===================== MMA issuer =====================
    if (lane == 0) {
      const uint32_t idesc = idesc_f16_f32(128, a.C);
      const int ksteps = a.kq_atoms * 4;  // K=16 steps per Q stage
      int dcnt = 0, qcnt = 0, tcnt = 0;
      bool ok = true;
      for (int w = w0; w < a.n_work && ok; w += wstep) {
        const Item it = make_item(a, w);
        if (it.nch == 0) continue;
        for (int s0 = it.rg_lo; s0 < it.rg_hi && ok; s0 += it.span) {
          const int s1 = min(it.rg_hi, s0 + it.span);
          const int nmb = span_mblocks(a, s0, s1);
          for (int g = 0; g < it.ngr && ok; ++g) {
            const int c0 = g * a.G;
            const int cn = min(a.G, it.nch - c0);
            for (int c = 0; c < cn && ok; ++c) {
              const int k = dcnt + c;
              if (!mbar_wait(bars.d_full(k % a.nd), (k / a.nd) & 1, ctl, FM_ERR_TIMEOUT_DFULL)) ok = false;
            }
            if (!ok) break;
            tc_fence_after();
            for (int jb = 0; jb < nmb && ok; ++jb) {
              if (a.nk == 1) {
                const int qslot = a.q_resident ? 0 : qcnt % a.nq;
                const uint32_t qph = a.q_resident ? 0 : (qcnt / a.nq) & 1;
                if (!mbar_wait(bars.q_full(qslot), qph, ctl, FM_ERR_TIMEOUT_QFULL)) { ok = false; break; }
                tc_fence_after();
                const uint32_t qaddr = sbase + a.off_q + qslot * a.q_stage_bytes;
                for (int c = 0; c < cn; ++c) {
                  const int ts = tcnt % a.nts;
                  if (!mbar_wait(bars.t_empty(ts), ((tcnt / a.nts) & 1) ^ 1, ctl, FM_ERR_TIMEOUT_TEMPTY)) { ok = false; break; }
                  tc_fence_after();
                  const uint32_t daddr = sbase + a.off_d + ((dcnt + c) % a.nd) * a.d_slot_bytes;
                  const uint32_t tacc = tmem_base + ts * a.ts_stride;
                  for (int kk = 0; kk < ksteps; ++kk) {
                    const int at = kk >> 2, sub = kk & 3;
                    const uint64_t adesc = smem_desc_sw128(qaddr + at * 16384 + sub * 32);
                    const uint64_t bdesc = smem_desc_sw128(daddr + at * a.C * 128 + sub * 32);
                    tc_mma_f16(tacc, adesc, bdesc, idesc, kk > 0 ? 1u : 0u);
                  }
                  tc_commit(bars.t_full(ts));
                  ++tcnt;
                }
                if (!ok) break;
                if (!a.q_resident) tc_commit(bars.q_empty(qslot));
                ++qcnt;
              } else {
                // K split over several Q stages: every chunk slot of this
                // M-block stays live until the last stage.
                for (int c = 0; c < cn && ok; ++c) {
                  const int t = tcnt + c;
                  if (!mbar_wait(bars.t_empty(t % a.nts), ((t / a.nts) & 1) ^ 1, ctl, FM_ERR_TIMEOUT_TEMPTY)) ok = false;
                }
                if (!ok) break;
                tc_fence_after();
                for (int ks = 0; ks < a.nk && ok; ++ks) {
                  const int qslot = qcnt % a.nq;
                  if (!mbar_wait(bars.q_full(qslot), (qcnt / a.nq) & 1, ctl, FM_ERR_TIMEOUT_QFULL)) { ok = false; break; }
                  tc_fence_after();
                  const uint32_t qaddr = sbase + a.off_q + qslot * a.q_stage_bytes;
                  for (int c = 0; c < cn; ++c) {
                    const uint32_t daddr = sbase + a.off_d + ((dcnt + c) % a.nd) * a.d_slot_bytes;
                    const uint32_t tacc = tmem_base + ((tcnt + c) % a.nts) * a.ts_stride;
                    for (int kk = 0; kk < ksteps; ++kk) {
                      const int at = kk >> 2, sub = kk & 3;
                      const uint64_t adesc = smem_desc_sw128(qaddr + at * 16384 + sub * 32);
                      const uint64_t bdesc =
                          smem_desc_sw128(daddr + (ks * a.kq_atoms + at) * a.C * 128 + sub * 32);
                      tc_mma_f16(tacc, adesc, bdesc, idesc, (ks > 0 || kk > 0) ? 1u : 0u);
                    }
                  }
                  tc_commit(bars.q_empty(qslot));
                  ++qcnt;
                }
                if (!ok) break;
                for (int c = 0; c < cn; ++c) tc_commit(bars.t_full((tcnt + c) % a.nts));
                tcnt += cn;
              }
            }
            if (!ok) break;
            for (int c = 0; c < cn; ++c) tc_commit(bars.d_empty((dcnt + c) % a.nd));
            dcnt += cn;
          }
        }
      }
      // make sure every MMA issued by this thread has completed before the
      // TMEM is released
      tc_commit(bars.drain());
      const uint64_t t0 = globaltimer_ns();
      while (!mbar_try_wait(bars.drain(), 0)) {
        if (globaltimer_ns() - t0 > a.timeout_ns) {
          record_status(a.status, FM_ERR_TIMEOUT_DRAIN);
          break;
        }
      }
    }
  } else if (warp >= kEpiWarp0 && warp < kEpiWarp0 + 4) {
    // ===================== epilogue =====================
    const int et = threadIdx.x - kEpiWarp0 * 32;  // 0..127
    const int sub = warp & 3;                      // TMEM lane quarter
    const uint32_t lane_base = static_cast<uint32_t>(sub * 32) << 16;
    float* state_m = reinterpret_cast<float*>(smem + a.off_state);
    int* state_i = reinterpret_cast<int*>(smem + a.off_state + (a.RS / 4) * 128 * 4);
    float* rows = reinterpret_cast<float*>(smem + a.off_rows);
    float* xch_m = reinterpret_cast<float*>(smem + a.off_xch);
    int* xch_i = reinterpret_cast<int*>(smem + a.off_xch + 128 * 4);
    const int rep = a.rep;
    const int part = sub % rep;
    const int ppc = (a.C + 31) / 32;  // 32-column pieces per chunk

    float* qsum_s = reinterpret_cast<float*>(smem + a.off_qsum);
    if (MODE == MODE_INT8) {
      // INT8: sum_k Q[q, k] of every query row (single query), fixed order
      for (int q = et; q < a.Gq * 32; q += 128) {
        float s = 0.f;
        if (q < a.Lq) {
          const __half* qr = a.q + static_cast<size_t>(q) * a.d;
          for (int k = 0; k < a.d; ++k) s += __half2float(qr[k]);
        }
        qsum_s[q] = s;
      }
      named_bar_sync(1, 128);
    }
    int tcnt = 0;
    bool ok = true;
    for (int w = w0; w < a.n_work && ok; w += wstep) {
      const Item it = make_item(a, w);
      if (it.nch == 0) {
        // empty document: every query row has max = -inf
        if (MODE == MODE_DENSE) {
          for (int i = et; i < it.nqi; i += 128)
            a.scores[static_cast<size_t>(it.n_lo + i) * a.B + it.b] = -INFINITY;
        } else if (et == 0) {
          a.scores[it.b] = (MODE == MODE_SPARSE && a.K == 0) ? 0.f : -INFINITY;
        }
        if (ARGMAX) {
          for (int i = et; i < it.nqi * a.Lq; i += 128) {
            const int n = it.n_lo + i / a.Lq;
            const int q = i - (i / a.Lq) * a.Lq;
            a.argmax[(static_cast<size_t>(n) * a.B + it.b) * a.Lq + q] = -1;
          }
        }
        continue;
      }
      for (int s0 = it.rg_lo; s0 < it.rg_hi && ok; s0 += it.span) {
        const int s1 = min(it.rg_hi, s0 + it.span);
        const int nmb = span_mblocks(a, s0, s1);
        for (int g = 0; g < it.ngr && ok; ++g) {
          const int c0 = g * a.G;
          const int cn = min(a.G, it.nch - c0);
          for (int jb = 0; jb < nmb && ok; ++jb) {
            const int rg = (rep > 1) ? s0 + sub / rep : s0 + 4 * jb + sub;
            const bool active = rg < s1;
            const int qrow = (rg % a.Gq) * 32 + lane;
            const float qsum = (MODE == MODE_INT8 && active) ? qsum_s[qrow] : 0.f;
            RowAcc<ARGMAX> acc;
            acc.init();
            for (int c = 0; c < cn; ++c) {
              const int ts = tcnt % a.nts;
              if (!mbar_wait(bars.t_full(ts), (tcnt / a.nts) & 1, ctl, FM_ERR_TIMEOUT_TFULL)) { ok = false; break; }
              tc_fence_after();
              if (active) {
                const int tok0 = (c0 + c) * a.C;
                const int valid = min(a.C, it.len - tok0);
                const int npieces = (valid + 31) >> 5;
                const uint32_t taddr = tmem_base + lane_base + ts * a.ts_stride;
                // piece p of this chunk belongs to part ((c*ppc + p) % rep)
                int p = 0;
                if (rep > 1) {
                  const int first = (c * ppc) % rep;
                  p = (part - first + rep) % rep;
                }
                for (; p < npieces; p += rep) {
                  float v[32];
                  tmem_ld32(taddr + p * 32, v);
                  tmem_wait_ld();
                  const int nv = min(32, valid - p * 32);
                  if (MODE == MODE_INT8) {
                    const size_t tb = static_cast<size_t>(it.b) * a.Ld + tok0 + p * 32;
                    const int col = lane < nv ? lane : 0;
                    const float sc = __half2float(a.scales[tb + col]);
                    const float mn = __half2float(a.mins[tb + col]);
#pragma unroll
                    for (int i = 0; i < 32; ++i) {
                      const float s_i = __shfl_sync(0xffffffffu, sc, i);
                      const float m_i = __shfl_sync(0xffffffffu, mn, i);
                      v[i] = fmaf(s_i, v[i], m_i * qsum);
                    }
                  }
                  piece_max<ARGMAX>(v, nv, tok0 + p * 32, acc);
                }
              }
              tc_fence_before();
              __syncwarp();
              if (lane == 0) mbar_arrive(bars.t_empty(ts));
              ++tcnt;
            }
            if (!ok) break;
            // combine across chunk groups
            if (it.ngr > 1) {
              const int si = jb * 128 + sub * 32 + lane;
              if (g == 0) {
                state_m[si] = acc.m;
                if (ARGMAX) state_i[si] = acc.idx;
              } else {
                RowAcc<ARGMAX> prev;
                prev.m = state_m[si];
                prev.idx = ARGMAX ? state_i[si] : 0;
                prev.merge(acc.m, acc.idx);
                acc = prev;
                if (g < it.ngr - 1) {
                  state_m[si] = acc.m;
                  if (ARGMAX) state_i[si] = acc.idx;
                }
              }
            }
            if (g == it.ngr - 1) {
              if (rep > 1) {
                xch_m[sub * 32 + lane] = acc.m;
                if (ARGMAX) xch_i[sub * 32 + lane] = acc.idx;
              } else {
                const bool rv = active && qrow < a.Lq;
                if (MODE == MODE_SPARSE) {
                  if (rv) rows[qrow] = acc.m;
                } else {
                  const float tot = warp_sum(rv ? acc.m : 0.f);
                  if (lane == 0 && active) rows[rg - it.rg_lo] = tot;
                }
                if (ARGMAX && rv) {
                  const int n = rg / a.Gq;
                  a.argmax[(static_cast<size_t>(n) * a.B + it.b) * a.Lq + qrow] = acc.idx;
                }
              }
            }
          }
        }
      }
      if (!ok) break;
      // ---- per-doc finalisation (epilogue warps only) ----
      named_bar_sync(1, 128);
      if (rep > 1) {
        if (part == 0) {
          RowAcc<ARGMAX> acc;
          acc.m = xch_m[sub * 32 + lane];
          acc.idx = ARGMAX ? xch_i[sub * 32 + lane] : 0;
          for (int r = 1; r < rep; ++r)
            acc.merge(xch_m[(sub + r) * 32 + lane], ARGMAX ? xch_i[(sub + r) * 32 + lane] : 0);
          const int rg = it.rg_lo + sub / rep;
          const int qrow = (rg % a.Gq) * 32 + lane;
          const bool rv = rg < it.rg_hi && qrow < a.Lq;
          if (MODE == MODE_SPARSE) {
            if (rv) rows[qrow] = acc.m;
          } else {
            const float tot = warp_sum(rv ? acc.m : 0.f);
            if (lane == 0 && rg < it.rg_hi) rows[rg - it.rg_lo] = tot;
          }
          if (ARGMAX && rv) {
            const int n = rg / a.Gq;
            a.argmax[(static_cast<size_t>(n) * a.B + it.b) * a.Lq + qrow] = acc.idx;
          }
        }
        named_bar_sync(1, 128);
      }
      if (MODE == MODE_SPARSE) {
        // score = sum_k rowmax[idx[b, k]] in a fixed order
        if (warp == kEpiWarp0) {
          float s = 0.f;
          const int32_t* ip = a.sp_idx + static_cast<size_t>(it.b) * a.K;
          for (int k = lane; k < a.K; k += 32) {
            int q = __ldg(ip + k);
            if (q < 0) q += a.Lq;
            if (q < 0 || q >= a.Lq) {
              record_status(a.status, FM_ERR_BAD_INDEX);
              continue;
            }
            s += rows[q];
          }
          s = warp_sum(s);
          if (lane == 0) a.scores[it.b] = s;
        }
      } else {
        for (int i = et; i < it.nqi; i += 128) {
          float s = 0.f;
          for (int gq = 0; gq < a.Gq; ++gq) s += rows[i * a.Gq + gq];
          a.scores[static_cast<size_t>(it.n_lo + i) * a.B + it.b] = s;
        }
      }
      named_bar_sync(1, 128);
    }
  } else if (MODE == MODE_INT8 && warp >= kConvWarp0 && warp < kConvWarp0 + 4) {
    // ===================== INT8 converters =====================
    // uint8 staging slot (64-byte rows per 64-element atom, no swizzle) ->
    // fp16 128-byte-swizzled operand slot.  u is converted exactly
    // (0x6400 | u is the fp16 value 1024 + u; subtracting 1024 leaves u);
    // the per-token affine map scale * u + min is applied in the epilogue.
    const int ct = threadIdx.x - kConvWarp0 * 32;  // 0..127
    int ucnt = 0;
    bool ok = true;
    const int n16 = a.d_atoms_real * a.C * 4;  // 16-byte pieces of one u8 chunk
    const __half2 k1024 = __floats2half2_rn(1024.f, 1024.f);
    for (int w = w0; w < a.n_work && ok; w += wstep) {
      const Item it = make_item(a, w);
      for (int s0 = it.rg_lo; s0 < it.rg_hi && ok; s0 += it.span) {
        for (int g = 0; g < it.ngr && ok; ++g) {
          const int cn = min(a.G, it.nch - g * a.G);
          for (int c = 0; c < cn; ++c) {
            const int uslot = ucnt % a.nu;
            const int dslot = ucnt % a.nd;
            if (!mbar_wait(bars.u_full(uslot), (ucnt / a.nu) & 1, ctl, FM_ERR_TIMEOUT_UFULL)) { ok = false; break; }
            if (!mbar_wait(bars.d_empty(dslot), ((ucnt / a.nd) & 1) ^ 1, ctl, FM_ERR_TIMEOUT_DEMPTY)) { ok = false; break; }
            const uint8_t* src = smem + a.off_u + uslot * a.u_slot_bytes;
            uint8_t* dst = smem + a.off_d + dslot * a.d_slot_bytes;
            for (int i = ct; i < n16; i += 128) {
              const int at = i / (a.C * 4);
              const int rem = i - at * (a.C * 4);
              const int row = rem >> 2;
              const int ch = rem & 3;
              const uint4 u = *reinterpret_cast<const uint4*>(src + at * a.C * 64 + row * 64 + ch * 16);
              uint32_t hv[8];
              const uint32_t wds[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
              for (int j = 0; j < 4; ++j) {
                uint32_t lo = __byte_perm(wds[j], 0x64646464u, 0x5140);
                uint32_t hi = __byte_perm(wds[j], 0x64646464u, 0x7362);
                __half2 hlo = __hsub2(*reinterpret_cast<__half2*>(&lo), k1024);
                __half2 hhi = __hsub2(*reinterpret_cast<__half2*>(&hi), k1024);
                hv[2 * j] = *reinterpret_cast<uint32_t*>(&hlo);
                hv[2 * j + 1] = *reinterpret_cast<uint32_t*>(&hhi);
              }
              uint8_t* rowp = dst + at * a.C * 128 + row * 128;
              const int j0 = (2 * ch) ^ (row & 7);
              const int j1 = (2 * ch + 1) ^ (row & 7);
              *reinterpret_cast<uint4*>(rowp + j0 * 16) = make_uint4(hv[0], hv[1], hv[2], hv[3]);
              *reinterpret_cast<uint4*>(rowp + j1 * 16) = make_uint4(hv[4], hv[5], hv[6], hv[7]);
            }
            fence_proxy_async_smem();
            mbar_arrive(bars.d_full(dslot));
            mbar_arrive(bars.u_empty(uslot));
            ++ucnt;
          }
        }
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
