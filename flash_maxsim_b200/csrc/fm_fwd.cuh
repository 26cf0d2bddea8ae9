// MaxSim forward kernel for sm_100a (B200).
//
//   score[n, b] = sum_{q < Lq} max_{t < len_b} <Q[n, q, :], D[b, t, :]>
//
// The same computation as the reference's `_maxsim_fwd_kernel`
// (flash_maxsim/flash_maxsim.py:83-146), its INT8 variant
// (flash_maxsim/flash_maxsim_quant.py:52-98) and its sparse variant
// (flash_maxsim/flash_maxsim_sparse.py:42-91), organised for Blackwell:
//
//  * Work item = one document, or a group of up to kMaxGroupDocs consecutive
//    documents when every document of the group fits in shared memory at
//    once (shared docs).  Persistent CTAs stride over work items.
//  * A document is split into chunks of C tokens (C <= 256, multiple of 16).
//    The chunks of an item (or of one chunk group of a long document) stay
//    resident in a shared-memory ring (D ring, filled by TMA from HBM,
//    128-byte swizzle, OOB rows zero-filled).
//  * Query rows are packed into 128-row "M-blocks" of four 32-row row groups
//    (one row group = 32 consecutive tokens of one query, rows past Lq are
//    TMA zero-fill).  M-blocks stream from L2 through a Q ring, and each one
//    is used for every resident chunk of the item before it is released, so
//    grouping short documents cuts the L2 -> SM query traffic per flop.
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
//  * The single MMA-issuing thread does as little bookkeeping as possible:
//    ring positions advance incrementally (no division), descriptors are a
//    base plus constant offsets, and per-item state is scalar.
//
// Warp roles: 0 = D producer (TMA), 1 = MMA issuer + TMEM owner,
// 2..5 = epilogue, 6 = Q producer (TMA), 7..10 = INT8 converters (INT8 only).
#pragma once

#include <cuda.h>
#include <cstdint>
#include <cuda_fp16.h>
#include "fm_ptx.cuh"
#include "fm_topk.cuh"

namespace fm {

enum FwdMode : int { MODE_DENSE = 0, MODE_SPARSE = 1, MODE_INT8 = 2 };

constexpr int kEpiWarp0 = 2;   // epilogue warps 2..5
constexpr int kQProdWarp = 6;
constexpr int kEpiWarp1 = 7;   // second epilogue set 7..10 (fp16 modes): odd query blocks
constexpr int kConvWarp0 = 7;  // INT8 converters 7..10
constexpr int kMmaWarp2 = 11;  // second MMA issuer (fp16 modes, K in one query stage)
constexpr int kThreadsF16 = 12 * 32;
constexpr int kThreadsI8 = 11 * 32;
constexpr int kMaxGroupDocs = 8;

struct FwdArgs {
  const int32_t* lengths;    // [n_docs] valid tokens per doc, or null (all Ld)
  const int32_t* cu;         // packed documents: [n_docs + 1] token offsets into D [T, d], or null
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
  int gd;                    // documents per work item (shared dense docs)
  int n_work;                // number of work items
  int Gq;                    // row groups per query = ceil(Lq / 32)
  int R;                     // row groups per document
  int C;                     // tokens per chunk (MMA N)
  int G;                     // chunk slots of one resident group
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
  int q_flat;                // Lq % 32 == 0: an M-block is 128 consecutive rows of Q
  int mma2;                  // 1: two MMA issuers (warps 1 and 11) take alternate chunks
  int dbg;  // tuning builds (FM_TUNING) only: bits that switch off parts of the work
  int nts;                   // TMEM accumulator slots
  int ts_stride;             // TMEM columns per slot
  int rowbuf;                // floats in the per-item row buffer
  uint32_t off_q, off_d, off_u, off_sc, off_state, off_rows, off_xch, off_qsum, off_bar;
  uint32_t q_stage_bytes, d_slot_bytes, u_slot_bytes;
  TopkArgs topk;             // k > 0 (dense shared docs): per-CTA top-k candidates in the tail
};

// Position in a ring of n slots: slot index and the parity of the current lap.
struct Ring {
  int idx = 0;
  uint32_t phase = 0;
  __device__ __forceinline__ void next(int n) {
    if (++idx == n) {
      idx = 0;
      phase ^= 1u;
    }
  }
};

__device__ __forceinline__ int doc_len(const FwdArgs& a, int doc) {
  int len = a.cu ? __ldg(a.cu + doc + 1) - __ldg(a.cu + doc) : (a.lengths ? __ldg(a.lengths + doc) : a.Ld);
  return len < 0 ? 0 : (len > a.Ld ? a.Ld : len);
}

// Schedule of one work item, computed identically by every role.  Scalar
// fields only; per-document lengths of a group are re-read when needed.
struct Item {
  int d0;        // first document (index into D, flattened for per-query docs)
  int b0;        // score column of the first document
  int ndocs;     // documents in the item (consecutive)
  int len0;      // valid tokens of the first document
  int nch0;      // chunks of the first document
  int nch_total; // chunks of the whole item
  int n_lo;      // first query of the item
  int nqi;       // queries of the item
  int rg_lo;     // first row group
  int rg_hi;     // one past the last row group
  int ngr;       // chunk groups (> 1 only for one long document)
  int span;      // row groups per span
};

__device__ __forceinline__ Item make_item(const FwdArgs& a, int w) {
  Item it;
  if (a.shared) {
    it.d0 = w * a.gd;
    it.b0 = it.d0;
    it.ndocs = min(a.gd, a.B - it.d0);
    it.n_lo = 0;
    it.nqi = a.Nq;
    it.rg_lo = 0;
    it.rg_hi = a.Nq * a.Gq;
  } else {
    const int n = w / a.B;
    it.d0 = w;
    it.b0 = w - n * a.B;
    it.ndocs = 1;
    it.n_lo = n;
    it.nqi = 1;
    it.rg_lo = n * a.Gq;
    it.rg_hi = it.rg_lo + a.Gq;
  }
  it.len0 = doc_len(a, it.d0);
  it.nch0 = (it.len0 + a.C - 1) / a.C;
  it.nch_total = it.nch0;
  for (int i = 1; i < it.ndocs; ++i) it.nch_total += (doc_len(a, it.d0 + i) + a.C - 1) / a.C;
  if (it.ndocs == 1) {
    it.ngr = (it.nch0 + a.G - 1) / a.G;
  } else {
    it.ngr = it.nch_total > 0 ? 1 : 0;
  }
  it.span = (it.ngr > 1) ? a.RS : (it.rg_hi - it.rg_lo);
  return it;
}

// Chunks of chunk group g (a long single document is split in groups of G).
__device__ __forceinline__ int group_chunks(const FwdArgs& a, const Item& it, int g) {
  return it.ndocs == 1 ? min(a.G, it.nch0 - g * a.G) : it.nch_total;
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
  // INT8: per-token scale/min staging of D slot i released by the epilogue
  __device__ uint32_t s_empty(int i) const {
    return base + 8u * (2 * nq + 2 * nd + 2 * nts + 2 * nu + i);
  }
  __device__ uint32_t drain() const {
    return base + 8u * (2 * nq + 2 * nd + 2 * nts + 2 * nu + (nu ? nd : 0));
  }
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

// One 32-column piece in the epilogue: INT8 affine map (scale * acc +
// min * rowsum(q), per-token scale/min staged in shared memory as float2 by
// the converter warps; `sm` points at this piece's first column) if needed,
// then the running max.
template <int MODE, bool ARGMAX>
__device__ __forceinline__ void epi_piece(float (&v)[32], int nv, int col0, const float2* sm,
                                          float qsum, RowAcc<ARGMAX>& acc) {
  if (MODE == MODE_INT8) {
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      const float2 sc = sm[i];
      v[i] = fmaf(sc.x, v[i], sc.y * qsum);
    }
  }
  piece_max<ARGMAX>(v, nv, col0, acc);
}

// Row max over the first `valid` columns of one accumulator slot, plain fp16
// scoring (no argmax, no INT8 map), 32-column pieces first, first + step, ...
// (step 2 when two warps share a lane quarter): full pieces two per TMEM wait,
// ragged tail masked with -inf.  Compact on purpose: the epilogue is
// latency-bound, so its instruction count sets its speed.
__device__ __forceinline__ void chunk_max_plain(uint32_t taddr, int valid, RowAcc<false>& acc, int first,
                                                int step) {
  const int nfull = valid >> 5;
  int q = first;
  for (; q + step < nfull; q += 2 * step) {
    float v0[32], v1[32];
    tmem_ld32(taddr + q * 32, v0);
    tmem_ld32(taddr + (q + step) * 32, v1);
    tmem_wait_ld();
    piece_max<false>(v0, 32, 0, acc);
    piece_max<false>(v1, 32, 0, acc);
  }
  for (; q * 32 < valid; q += step) {
    float v0[32];
    tmem_ld32(taddr + q * 32, v0);
    tmem_wait_ld();
    const int rem = valid - q * 32;
    if (rem < 32) {
#pragma unroll
      for (int i = 0; i < 32; ++i) v0[i] = i < rem ? v0[i] : -INFINITY;
    }
    piece_max<false>(v0, 32, 0, acc);
  }
}

__device__ __forceinline__ float warp_sum(float x) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
  return x;
}

// Bounded wait for the last phase of `bar` used by a ring position (drain
// before exit); records FM_ERR_TIMEOUT_DRAIN when it gives up.
__device__ __forceinline__ void drain_wait(uint32_t bar, uint32_t parity, const FwdArgs& a) {
  const uint64_t t0 = globaltimer_ns();
  while (!mbar_try_wait(bar, parity)) {
    if (globaltimer_ns() - t0 > a.timeout_ns) {
      record_status(a.status, FM_ERR_TIMEOUT_DRAIN);
      break;
    }
  }
}

// -------------------------------------------------------------------------
// the kernel
// -------------------------------------------------------------------------
template <int MODE, bool ARGMAX>
__global__ void __launch_bounds__(MODE == MODE_INT8 ? kThreadsI8 : kThreadsF16, 1)
    maxsim_fwd_kernel(const __grid_constant__ CUtensorMap tmap_q,
                      const __grid_constant__ CUtensorMap tmap_q2,
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
      mbar_init(bars.q_empty(i), a.mma2 ? 2 : 1);  // a commit from every MMA issuer
    }
    for (int i = 0; i < a.nd; ++i) {
      mbar_init(bars.d_full(i), MODE == MODE_INT8 ? 128 : 1);
      mbar_init(bars.d_empty(i), a.mma2 ? 2 : 1);
    }
    for (int i = 0; i < a.nts; ++i) {
      mbar_init(bars.t_full(i), 1);
      // every epilogue warp that reads the slot releases it
      mbar_init(bars.t_empty(i), (MODE != MODE_INT8 && a.rep == 1) ? 8 : 4);
    }
    if (MODE == MODE_INT8) {
      for (int i = 0; i < a.nu; ++i) {
        mbar_init(bars.u_full(i), 1);
        mbar_init(bars.u_empty(i), 128);
      }
      for (int i = 0; i < a.nd; ++i) mbar_init(bars.s_empty(i), 4);
    }
    mbar_init(bars.drain(), a.mma2 ? 2 : 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), 512);
    tmem_relinquish();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmap_q);
    tma_prefetch_desc(&tmap_q2);
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
  FM_PROF_T0(pk0);

  if (warp == 0) {
    // ===================== D producer =====================
    if (lane == 0) {
      const uint64_t pol = l2_policy_evict_first();
      const int nslots = (MODE == MODE_INT8) ? a.nu : a.nd;
      const uint32_t tx = a.d_atoms_real * a.C * ((MODE == MODE_INT8) ? 64u : 128u);
      const uint32_t slot_bytes = (MODE == MODE_INT8) ? a.u_slot_bytes : a.d_slot_bytes;
      const uint32_t atom_bytes = a.C * ((MODE == MODE_INT8) ? 64u : 128u);
      const uint32_t ring_base = sbase + ((MODE == MODE_INT8) ? a.off_u : a.off_d);
      Ring r;
      int issued = 0;
      bool ok = true;
      FM_TR_DECL;
      for (int w = w0; w < a.n_work && ok; w += wstep) {
        const Item it = make_item(a, w);
        for (int s0 = it.rg_lo; s0 < it.rg_hi && ok; s0 += it.span) {
          for (int g = 0; g < it.ngr && ok; ++g) {
            for (int i = 0; i < it.ndocs && ok; ++i) {
              const int doc = it.d0 + i;
              int cb = 0, ce;
              if (it.ndocs == 1) {
                cb = g * a.G;
                ce = min(it.nch0, cb + a.G);
              } else {
                ce = (doc_len(a, doc) + a.C - 1) / a.C;
              }
              for (int c = cb; c < ce; ++c) {
                const uint32_t empty = (MODE == MODE_INT8) ? bars.u_empty(r.idx) : bars.d_empty(r.idx);
                const uint32_t full = (MODE == MODE_INT8) ? bars.u_full(r.idx) : bars.d_full(r.idx);
                FM_TR(4, 1);
                if (!mbar_wait(empty, r.phase ^ 1u, ctl,
                               MODE == MODE_INT8 ? FM_ERR_TIMEOUT_UEMPTY : FM_ERR_TIMEOUT_DEMPTY)) {
                  ok = false;
                  break;
                }
                FM_TR(4, 2);
                mbar_expect_tx(full, tx);
                const uint32_t dst = ring_base + r.idx * slot_bytes;
                // padded documents: (token, doc) of a [docs, Ld, d] map; packed
                // documents: row cu[doc] + token of a [T, d] map (rows of the next
                // document past the end are masked by the epilogue)
                const int row = (a.cu ? __ldg(a.cu + doc) : 0) + c * a.C;
                const int zc = a.cu ? 0 : doc;
                for (int at = 0; at < a.d_atoms_real; ++at)
                  tma_load_3d(dst + at * atom_bytes, &tmap_d, at * 64, row, zc, full, pol);
                FM_TR(4, 3);
                r.next(nslots);
                ++issued;
              }
            }
          }
        }
      }
      // Wait (bounded) for the last load issued into every slot to land so
      // no bulk copy is in flight when the CTA exits.
      for (int i = 0; i < nslots && i < issued; ++i) {
        if (--r.idx < 0) {
          r.idx = nslots - 1;
          r.phase ^= 1u;
        }
        drain_wait((MODE == MODE_INT8) ? bars.u_full(r.idx) : bars.d_full(r.idx), r.phase, a);
      }
    }
  } else if (warp == kQProdWarp) {
    // ===================== Q producer =====================
    if (lane == 0) {
      const uint64_t pol = l2_policy_evict_last();
      Ring r;
      int issued = 0;
      bool ok = true;
      FM_TR_DECL;
      for (int w = w0; w < a.n_work && ok; w += wstep) {
        const Item it = make_item(a, w);
        if (it.nch_total == 0) continue;
        for (int s0 = it.rg_lo; s0 < it.rg_hi && ok; s0 += it.span) {
          const int s1 = min(it.rg_hi, s0 + it.span);
          const int nmb = span_mblocks(a, s0, s1);
          for (int g = 0; g < it.ngr && ok; ++g) {
            for (int jb = 0; jb < nmb && ok; ++jb) {
              for (int ks = 0; ks < a.nk; ++ks) {
                if (a.q_resident && issued > 0) break;
                FM_TR(3, 1);
                if (!mbar_wait(bars.q_empty(r.idx), r.phase ^ 1u, ctl, FM_ERR_TIMEOUT_QEMPTY)) {
                  ok = false;
                  break;
                }
                FM_TR(3, 2);
                const int at_hi = min(a.kq_atoms, a.d_atoms_real - ks * a.kq_atoms);
                const uint32_t dst = sbase + a.off_q + r.idx * a.q_stage_bytes;
                const uint32_t full = bars.q_full(r.idx);
                if (a.q_flat && a.rep == 1) {
                  // one 128-row box per K atom (rows past the span are loaded but unused)
                  mbar_expect_tx(full, at_hi * 16384u);
                  for (int at = 0; at < at_hi; ++at)
                    tma_load_3d(dst + at * 16384, &tmap_q2, (ks * a.kq_atoms + at) * 64,
                                (s0 + 4 * jb) * 32, 0, full, pol);
                } else {
                  int nload = 0;
                  for (int sub = 0; sub < 4; ++sub) {
                    const int rg = (a.rep > 1) ? s0 + sub / a.rep : s0 + 4 * jb + sub;
                    if (rg < s1) ++nload;
                  }
                  mbar_expect_tx(full, nload * at_hi * 4096u);
                  for (int sub = 0; sub < 4; ++sub) {
                    const int rg = (a.rep > 1) ? s0 + sub / a.rep : s0 + 4 * jb + sub;
                    if (rg >= s1) continue;
                    const int qn = rg / a.Gq;
                    const int qy = (rg - qn * a.Gq) * 32;
                    for (int at = 0; at < at_hi; ++at)
                      tma_load_3d(dst + at * 16384 + sub * 4096, &tmap_q, (ks * a.kq_atoms + at) * 64,
                                  qy, qn, full, pol);
                  }
                }
                r.next(a.nq);
                ++issued;
              }
            }
          }
        }
      }
      for (int i = 0; i < a.nq && i < issued; ++i) {
        if (--r.idx < 0) {
          r.idx = a.nq - 1;
          r.phase ^= 1u;
        }
        drain_wait(bars.q_full(r.idx), r.phase, a);
      }
    }
  } else if (warp == 1 || (MODE != MODE_INT8 && warp == kMmaWarp2 && a.mma2)) {
    // ===================== MMA issuer(s) =====================
    // With a.mma2 two threads (warps 1 and 11) issue: each owns alternate TMEM
    // slots (and so the chunks that land in them), so one issues while the
    // other waits or commits; both follow the same ring positions and both
    // commit the query stage, document slot and drain barriers (counts of 2).
    if (lane == 0) {
      const int me = warp == 1 ? 0 : 1;
      const uint32_t idesc = idesc_f16_f32(128, a.C);
      const int ksteps = a.kq_atoms * 4;  // K=16 steps per Q stage (4 or 8)
      const uint32_t b_atom = a.C * 8u;    // one K atom of a D slot, in 16-byte units
      const bool skip_mma = FM_DBG(a, 2);
      [[maybe_unused]] const int ich = me == 0 ? 0 : 5;  // trace channel of this issuer (FM_TRACE)
      Ring dr, qr, tr;
      bool ok = true;
      FM_TR_DECL;
      for (int w = w0; w < a.n_work && ok; w += wstep) {
        const Item it = make_item(a, w);
        if (it.nch_total == 0) continue;
        for (int s0 = it.rg_lo; s0 < it.rg_hi && ok; s0 += it.span) {
          const int s1 = min(it.rg_hi, s0 + it.span);
          const int nmb = span_mblocks(a, s0, s1);
          for (int g = 0; g < it.ngr && ok; ++g) {
            const int cn = group_chunks(a, it, g);
            {
              Ring r = dr;
              FM_TR(ich, 8);
              for (int c = 0; c < cn; ++c) {
                if (!mbar_wait(bars.d_full(r.idx), r.phase, ctl, FM_ERR_TIMEOUT_DFULL)) {
                  ok = false;
                  break;
                }
                r.next(a.nd);
              }
              FM_TR(ich, 9);
            }
            if (!ok) break;
            tc_fence_after();
            for (int jb = 0; jb < nmb && ok; ++jb) {
              if (a.nk == 1) {
                const int qslot = a.q_resident ? 0 : qr.idx;
                const uint32_t qph = a.q_resident ? 0u : qr.phase;
                FM_TR(ich, 5);
                if (!(FM_DBG(a, 1024) && qr.phase) && !(FM_DBG(a, 256) && mbar_test_wait(bars.q_full(qslot), qph)) &&
                    !mbar_wait(bars.q_full(qslot), qph, ctl, FM_ERR_TIMEOUT_QFULL)) {
                  ok = false;
                  break;
                }
                FM_TR(ich, 6);
                tc_fence_after();
                const uint64_t adesc = smem_desc_sw128(sbase + a.off_q + qslot * a.q_stage_bytes);
                Ring r = dr;
                for (int c = 0; c < cn; ++c) {
                  // slots alternate between the issuers: every use of a slot is issued
                  // (and its release awaited) by the same thread, so no issuer ever
                  // waits on a slot barrier more than one phase ahead
                  if (a.mma2 && (tr.idx & 1) != me) {  // the other issuer's slot
                    tr.next(a.nts);
                    r.next(a.nd);
                    continue;
                  }
                  FM_TR(ich, 1);
                  if (!FM_DBG(a, 512) && !(FM_DBG(a, 256) && mbar_test_wait(bars.t_empty(tr.idx), tr.phase ^ 1u)) &&
                      !mbar_wait(bars.t_empty(tr.idx), tr.phase ^ 1u, ctl, FM_ERR_TIMEOUT_TEMPTY)) {
                    ok = false;
                    break;
                  }
                  FM_TR(ich, 2);
                  tc_fence_after();
                  const uint64_t bdesc = smem_desc_sw128(sbase + a.off_d + r.idx * a.d_slot_bytes);
                  const uint32_t tacc = tmem_base + tr.idx * a.ts_stride;
                  FM_PROF_T0(pm0);
                  if (!skip_mma) {
#pragma unroll
                    for (int kk = 0; kk < 8; ++kk) {
                      if (kk < ksteps) {
                        // +32 bytes per K=16 step inside a 128-byte atom, next atom after 4
                        const uint64_t ao = (kk >> 2) * (16384u >> 4) + (kk & 3) * 2u;
                        const uint64_t bo = (kk >> 2) * b_atom + (kk & 3) * 2u;
                        tc_mma_f16(tacc, adesc + ao, bdesc + bo, idesc, kk > 0 ? 1u : 0u);
                      }
                    }
                  }
                  FM_PROF_ADD(20, pm0);
                  FM_TR(ich, 3);
                  tc_commit(bars.t_full(tr.idx));
                  FM_TR(ich, 4);
                  tr.next(a.nts);
                  r.next(a.nd);
                }
                if (!ok) break;
                if (!a.q_resident) {
                  tc_commit(bars.q_empty(qr.idx));
                  qr.next(a.nq);
                }
                FM_TR(ich, 7);
              } else {
                // K split over several Q stages (single-document items only):
                // every chunk slot of this M-block stays live until the last stage.
                // (with two issuers each handles the chunks in its own slots)
                {
                  Ring t = tr;
                  for (int c = 0; c < cn; ++c) {
                    if (a.mma2 && (t.idx & 1) != me) {
                      t.next(a.nts);
                      continue;
                    }
                    if (!mbar_wait(bars.t_empty(t.idx), t.phase ^ 1u, ctl, FM_ERR_TIMEOUT_TEMPTY)) {
                      ok = false;
                      break;
                    }
                    t.next(a.nts);
                  }
                }
                if (!ok) break;
                tc_fence_after();
                for (int ks = 0; ks < a.nk && ok; ++ks) {
                  if (!mbar_wait(bars.q_full(qr.idx), qr.phase, ctl, FM_ERR_TIMEOUT_QFULL)) {
                    ok = false;
                    break;
                  }
                  tc_fence_after();
                  const uint64_t adesc = smem_desc_sw128(sbase + a.off_q + qr.idx * a.q_stage_bytes);
                  Ring r = dr, t = tr;
                  for (int c = 0; c < cn; ++c) {
                    const uint64_t bdesc = smem_desc_sw128(sbase + a.off_d + r.idx * a.d_slot_bytes) +
                                           ks * a.kq_atoms * b_atom;
                    const uint32_t tacc = tmem_base + t.idx * a.ts_stride;
                    if (!skip_mma && !(a.mma2 && (t.idx & 1) != me)) {
#pragma unroll
                      for (int kk = 0; kk < 8; ++kk) {
                        if (kk < ksteps) {
                          const uint64_t ao = (kk >> 2) * (16384u >> 4) + (kk & 3) * 2u;
                          const uint64_t bo = (kk >> 2) * b_atom + (kk & 3) * 2u;
                          tc_mma_f16(tacc, adesc + ao, bdesc + bo, idesc, (ks > 0 || kk > 0) ? 1u : 0u);
                        }
                      }
                    }
                    r.next(a.nd);
                    t.next(a.nts);
                  }
                  tc_commit(bars.q_empty(qr.idx));
                  qr.next(a.nq);
                }
                if (!ok) break;
                for (int c = 0; c < cn; ++c) {
                  if (!(a.mma2 && (tr.idx & 1) != me)) tc_commit(bars.t_full(tr.idx));
                  tr.next(a.nts);
                }
              }
            }
            if (!ok) break;
            for (int c = 0; c < cn; ++c) {
              tc_commit(bars.d_empty(dr.idx));
              dr.next(a.nd);
            }
          }
        }
      }
      // make sure every MMA issued by this thread has completed before the
      // TMEM is released
      tc_commit(bars.drain());
      drain_wait(bars.drain(), 0, a);
    }
  } else if ((warp >= kEpiWarp0 && warp < kEpiWarp0 + 4) ||
             (MODE != MODE_INT8 && warp >= kEpiWarp1 && warp < kEpiWarp1 + 4)) {
    // ===================== epilogue =====================
    // fp16 modes run two sets of four warps (one warp per TMEM lane quarter in
    // each set), so every scheduler has two epilogue warps to switch between.
    // Without column replication (rep == 1) both warps of a lane quarter read
    // every chunk, taking alternate 32-column pieces, and merge their row maxima
    // per (M-block, document) through a double-buffered exchange and a 64-thread
    // barrier per quarter.  With replication (rep > 1) the second set idles.
    constexpr int EW = (MODE == MODE_INT8) ? 4 : 8;
    const int half = warp >= kEpiWarp1 ? 1 : 0;
    const bool pair = EW == 8 && a.rep == 1;        // two warps per lane quarter split columns
    const bool idle = EW == 8 && a.rep > 1 && half == 1;
    const int pstep = pair ? 2 : 1;
    const int pfirst = pair ? half : 0;
    float* xp_m = reinterpret_cast<float*>(smem + a.off_xch + 128 * 8);  // [2 buffers][128]
    int* xp_i = reinterpret_cast<int*>(smem + a.off_xch + 128 * 8 + 2 * 128 * 4);
    int xbuf = 0;
    const int et = half ? 128 + threadIdx.x - kEpiWarp1 * 32 : threadIdx.x - kEpiWarp0 * 32;  // 0..32*EW-1
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
    const bool skip_epi = FM_DBG(a, 1);

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
      named_bar_sync(1, 32 * EW);
    }
    Ring tr, er;
    bool ok = true;
    FM_TR_DECL;
    const int tch = warp == kEpiWarp0 ? 1 : (warp == kEpiWarp1 ? 2 : 7);
    for (int w = w0; w < a.n_work && ok; w += wstep) {
      const Item it = make_item(a, w);
      if (it.nch_total == 0) {
        // only empty documents: every query row has max = -inf
        for (int i = 0; i < it.ndocs; ++i) {
          const int b = it.b0 + i;
          if (MODE == MODE_DENSE) {
            for (int n = et; n < it.nqi; n += 32 * EW)
              a.scores[static_cast<size_t>(it.n_lo + n) * a.B + b] = -INFINITY;
          } else if (et == 0) {
            a.scores[b] = (MODE == MODE_SPARSE && a.K == 0) ? 0.f : -INFINITY;
          }
          if (ARGMAX) {
            for (int e = et; e < it.nqi * a.Lq; e += 32 * EW) {
              const int n = it.n_lo + e / a.Lq;
              const int q = e - (e / a.Lq) * a.Lq;
              a.argmax[(static_cast<size_t>(n) * a.B + b) * a.Lq + q] = -1;
            }
          }
        }
        continue;
      }
      for (int s0 = it.rg_lo; s0 < it.rg_hi && ok && !idle; s0 += it.span) {
        const int s1 = min(it.rg_hi, s0 + it.span);
        const int nmb = span_mblocks(a, s0, s1);
        for (int g = 0; g < it.ngr && ok; ++g) {
          for (int jb = 0; jb < nmb && ok; ++jb) {
            Ring sr = er;  // INT8: D-ring position of the group's first chunk
            const int rg = (rep > 1) ? s0 + sub / rep : s0 + 4 * jb + sub;
            const bool active = rg < s1;
            const int qrow = (rg % a.Gq) * 32 + lane;
            const float qsum = (MODE == MODE_INT8 && active) ? qsum_s[qrow] : 0.f;
            for (int i = 0; i < it.ndocs && ok; ++i) {
              int cb = 0, ce, len;
              if (it.ndocs == 1) {
                cb = g * a.G;
                ce = min(it.nch0, cb + a.G);
                len = it.len0;
              } else {
                len = doc_len(a, it.d0 + i);
                ce = (len + a.C - 1) / a.C;
              }
              const int b = it.b0 + i;
              RowAcc<ARGMAX> acc;
              acc.init();
              for (int c = cb; c < ce; ++c) {
                const float2* scs = nullptr;
                if (MODE == MODE_INT8) {
                  // the slot's scales were written before its d_full arrival; the slot
                  // cannot be refilled before this warp releases it (s_empty)
                  if (!mbar_wait(bars.d_full(sr.idx), sr.phase, ctl, FM_ERR_TIMEOUT_DFULL)) {
                    ok = false;
                    break;
                  }
                  scs = reinterpret_cast<const float2*>(smem + a.off_sc) + sr.idx * a.C;
                  sr.next(a.nd);
                }
                FM_TR(tch, 1);
                if (!mbar_wait(bars.t_full(tr.idx), tr.phase, ctl, FM_ERR_TIMEOUT_TFULL)) {
                  ok = false;
                  break;
                }
                FM_TR(tch, 2);
                tc_fence_after();
                FM_PROF_T0(pe0);
                if (MODE != MODE_INT8 && !ARGMAX && rep == 1) {
                  if (active && !skip_epi)
                    chunk_max_plain(tmem_base + lane_base + tr.idx * a.ts_stride,
                                    min(a.C, len - c * a.C), *reinterpret_cast<RowAcc<false>*>(&acc),
                                    pfirst, pstep);
                } else if (active && !skip_epi) {
                  const int tok0 = c * a.C;
                  const int valid = min(a.C, len - tok0);
                  const int npieces = (valid + 31) >> 5;
                  const uint32_t taddr = tmem_base + lane_base + tr.idx * a.ts_stride;
                  // piece p of this chunk belongs to part ((c * ppc + p) % nparts)
                  const int nparts = rep > 1 ? rep : pstep;
                  const int mypart = rep > 1 ? part : pfirst;
                  int p = 0;
                  if (nparts > 1) {
                    const int first = (c * ppc) % nparts;
                    p = (mypart - first + nparts) % nparts;
                  }
                  // two TMEM loads in flight per wait
                  for (; p < npieces; p += 2 * nparts) {
                    const int p1 = p + nparts;
                    const bool two = p1 < npieces;
                    float v0[32], v1[32];

                    tmem_ld32(taddr + p * 32, v0);
                    if (two) tmem_ld32(taddr + p1 * 32, v1);
                    tmem_wait_ld();

                    epi_piece<MODE, ARGMAX>(v0, min(32, valid - p * 32), tok0 + p * 32, scs + p * 32,
                                            qsum, acc);
                    if (two)
                      epi_piece<MODE, ARGMAX>(v1, min(32, valid - p1 * 32), tok0 + p1 * 32, scs + p1 * 32,
                                              qsum, acc);
                  }
                }
                FM_PROF_ADD(22 + sub, pe0);
                tc_fence_before();
                __syncwarp();
                FM_TR(tch, 3);
                if (lane == 0) mbar_arrive(bars.t_empty(tr.idx));
                tr.next(a.nts);
              }
              if (!ok) break;
              if (pair) {
                // merge the two column halves of each row: set 1 hands over, set 0 goes on
                if (half == 1) {
                  xp_m[xbuf * 128 + sub * 32 + lane] = acc.m;
                  if (ARGMAX) xp_i[xbuf * 128 + sub * 32 + lane] = acc.idx;
                }
                FM_TR(tch, 5);
                named_bar_sync(2 + sub, 64);
                FM_TR(tch, 6);
                if (half == 0)
                  acc.merge(xp_m[xbuf * 128 + sub * 32 + lane], ARGMAX ? xp_i[xbuf * 128 + sub * 32 + lane] : 0);
                xbuf ^= 1;
                if (half == 1) continue;
              }
              FM_PROF_T0(pf0);
              // combine across chunk groups (single-document items)
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
                    if (lane == 0 && active) rows[i * a.R + rg - it.rg_lo] = tot;
                  }
                  if (ARGMAX && rv) {
                    const int n = rg / a.Gq;
                    a.argmax[(static_cast<size_t>(n) * a.B + b) * a.Lq + qrow] = ce > 0 ? acc.idx : -1;
                  }
                }
              }
              FM_PROF_ADD(28, pf0);
            }
          }
          if (MODE == MODE_INT8 && ok) {
            // release the group's scale staging (after its last M-block)
            const int cn = group_chunks(a, it, g);
            for (int c = 0; c < cn; ++c) {
              if (lane == 0) mbar_arrive(bars.s_empty(er.idx));
              er.next(a.nd);
            }
          }
        }
      }
      if (!ok) break;
      // ---- per-item finalisation (epilogue warps only) ----
      FM_PROF_T0(pi0);
      named_bar_sync(1, 32 * EW);
      FM_PROF_ADD(29, pi0);
      if (rep > 1) {
        // single-document items: combine the column parts of each row
        if (part == 0 && half == 0) {
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
            a.argmax[(static_cast<size_t>(n) * a.B + it.b0) * a.Lq + qrow] = acc.idx;
          }
        }
        named_bar_sync(1, 32 * EW);
      }
      if (MODE == MODE_SPARSE) {
        // score = sum_k rowmax[idx[b, k]] in a fixed order
        if (warp == kEpiWarp0) {
          float s = 0.f;
          const int32_t* ip = a.sp_idx + static_cast<size_t>(it.b0) * a.K;
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
          if (lane == 0) a.scores[it.b0] = s;
        }
      } else {
        for (int e = et; e < it.ndocs * it.nqi; e += 32 * EW) {
          const int i = e / it.nqi;
          const int n = e - i * it.nqi;
          float s = 0.f;
          for (int gq = 0; gq < a.Gq; ++gq) s += rows[i * a.R + n * a.Gq + gq];
          a.scores[static_cast<size_t>(it.n_lo + n) * a.B + it.b0 + i] = s;
        }
      }
      FM_PROF_T0(pi1);
      named_bar_sync(1, 32 * EW);
      FM_PROF_ADD(30, pi1);
      FM_PROF_ADD(31, pi0);
    }
  } else if (MODE == MODE_INT8 && warp >= kConvWarp0 && warp < kConvWarp0 + 4) {
    // ===================== INT8 converters =====================
    // uint8 staging slot (64-byte rows per 64-element atom, no swizzle) ->
    // fp16 128-byte-swizzled operand slot holding 1024 + u (0x6400 | u, exact);
    // the per-token affine map is applied in the epilogue.
    const int ct = threadIdx.x - kConvWarp0 * 32;  // 0..127
    Ring ur, dr;
    bool ok = true;
    for (int w = w0; w < a.n_work && ok; w += wstep) {
      const Item it = make_item(a, w);
      for (int s0 = it.rg_lo; s0 < it.rg_hi && ok; s0 += it.span) {
        for (int g = 0; g < it.ngr && ok; ++g) {
          // single-document items (INT8 scores one query against each doc)
          const int cb = g * a.G, ce = min(it.nch0, cb + a.G);
          for (int c = cb; c < ce; ++c) {
            if (!mbar_wait(bars.u_full(ur.idx), ur.phase, ctl, FM_ERR_TIMEOUT_UFULL)) { ok = false; break; }
            if (!mbar_wait(bars.d_empty(dr.idx), dr.phase ^ 1u, ctl, FM_ERR_TIMEOUT_DEMPTY)) { ok = false; break; }
            if (!mbar_wait(bars.s_empty(dr.idx), dr.phase ^ 1u, ctl, FM_ERR_TIMEOUT_DEMPTY)) { ok = false; break; }
            const uint8_t* src = smem + a.off_u + ur.idx * a.u_slot_bytes;
            uint8_t* dst = smem + a.off_d + dr.idx * a.d_slot_bytes;
            // per-token (scale, min - 1024 * scale) of this chunk as fp32 pairs: the
            // operand holds 1024 + u (fp16 0x6400 | u, exact), so
            // scale * <q, 1024 + u> + (min - 1024 * scale) * sum(q) = <q, scale * u + min>
            float2* scs = reinterpret_cast<float2*>(smem + a.off_sc) + dr.idx * a.C;
            const size_t tb = static_cast<size_t>(it.b0) * a.Ld + static_cast<size_t>(c) * a.C;
            for (int t = ct; t < a.C; t += 128) {
              float sv = 0.f, mv = 0.f;
              if (c * a.C + t < it.len0) {
                sv = __half2float(a.scales[tb + t]);
                mv = __half2float(a.mins[tb + t]);
              }
              scs[t] = make_float2(sv, fmaf(-1024.f, sv, mv));
            }
            // lane -> (row, 16-byte column) of a 64-byte uint8 row; 32 rows per pass,
            // four passes unrolled for independent shared-memory loads
            const int ch = ct & 3;
            const int r0 = ct >> 2;
            for (int at = 0; at < a.d_atoms_real; ++at) {
              const uint8_t* s_at = src + at * a.C * 64 + ch * 16;
              uint8_t* d_at = dst + at * a.C * 128;
              for (int rb = 0; rb < a.C; rb += 128) {
                uint4 u[4];
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                  const int row = rb + r0 + 32 * k;
                  if (row < a.C) u[k] = *reinterpret_cast<const uint4*>(s_at + row * 64);
                }
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                  const int row = rb + r0 + 32 * k;
                  if (row < a.C) {
                    const uint32_t wds[4] = {u[k].x, u[k].y, u[k].z, u[k].w};
                    uint32_t hv[8];
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                      hv[2 * j] = __byte_perm(wds[j], 0x64646464u, 0x5140);
                      hv[2 * j + 1] = __byte_perm(wds[j], 0x64646464u, 0x7362);
                    }
                    uint8_t* rowp = d_at + row * 128;
                    const int sw = row & 7;
                    *reinterpret_cast<uint4*>(rowp + (((2 * ch) ^ sw) << 4)) = make_uint4(hv[0], hv[1], hv[2], hv[3]);
                    *reinterpret_cast<uint4*>(rowp + (((2 * ch + 1) ^ sw) << 4)) = make_uint4(hv[4], hv[5], hv[6], hv[7]);
                  }
                }
              }
            }
            fence_proxy_async_smem();
            mbar_arrive(bars.d_full(dr.idx));
            mbar_arrive(bars.u_empty(ur.idx));
            ur.next(a.nu);
            dr.next(a.nd);
          }
        }
      }
    }
  }

  if (threadIdx.x == 0) FM_PROF_ADD(27, pk0);
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 512);
  }
  if (MODE == MODE_DENSE && !ARGMAX && a.topk.k > 0 && a.shared && !*abort_flag) {
    // Top-k tail: every warp takes queries in turn and selects the k best of the
    // documents this CTA scored (work items w0, w0 + wstep, ...; gd documents
    // each), read back from the score matrix this CTA just wrote (L2-resident;
    // plain loads, the data is not read-only during the kernel).
    const int nwarps = blockDim.x >> 5;
    const int count = ((a.n_work - w0 + wstep - 1) / wstep) * a.gd;
    for (int n = warp; n < a.Nq; n += nwarps) {
      const float* row = a.scores + static_cast<size_t>(n) * a.B;
      const size_t o = (static_cast<size_t>(n) * a.topk.parts + blockIdx.x) * a.topk.k;
      warp_topk<24>(count, a.topk.k,
                    [&](int p) {
                      const int j = p / a.gd;
                      const int b = (w0 + j * wstep) * a.gd + (p - j * a.gd);
                      return b < a.B ? TopkCand{row[b], b} : TopkCand{0.f, -1};
                    },
                    a.topk.cand_s + o, a.topk.cand_b + o, lane);
    }
  }
}

}  // namespace fm
