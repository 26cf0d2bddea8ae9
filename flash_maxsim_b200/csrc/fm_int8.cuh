// INT8 fused-dequant MaxSim for one short query (Lq <= 64), sm_100a.
//
//   score[b] = sum_q max_{t < len_b} sum_k Q[q,k] * (u[b,t,k] * scale[b,t] + min[b,t])
//
// Same result as the reference's `_maxsim_int8_kernel`
// (flash_maxsim/flash_maxsim_quant.py:52-98) measured against maxsim_naive on
// dequantize_int8(D), organised for Blackwell:
//
//  * The uint8 codes are never converted.  TMA copies a 128-token chunk
//    straight from HBM into 128-byte-swizzled shared memory, and the tensor
//    core multiplies it as unsigned 8-bit integers (tcgen05.mma kind::i8,
//    s32 accumulate) with the chunk as the M=128 operand.
//  * The fp16 query is split once per CTA into two signed 8-bit parts,
//    q = alpha * (h + l / 256) with alpha = max|q| / 127 per query row
//    (|q - alpha * (h + l / 256)| <= alpha / 512).  Both parts are the N
//    operand (N = 64 for Lq <= 32: 32 rows of h, then 32 rows of l), so one
//    MMA pass gives <h,u> and <l,u> for every (token, query row) pair without
//    replicating the short query over 128 rows.
//  * TMEM lane = token, column = query row (x2 parts).  Each epilogue thread
//    owns one token: it applies, in fp32,
//      S[t, q] = scale_t * alpha_q * (256 <h,u> + <l,u>) / 256 + min_t * sum_k Q[q, k]
//    (256 <h,u> + <l,u> is an exact integer), masks tokens past the document,
//    and at the end of a document one warp reduction per query row
//    (redux.sync.max.f32) leaves lane j with the max over the warp's tokens
//    for query row j.  Per-token scale/min arrive by bulk copy with the chunk.
//
// Warp roles: 0 = producer (TMA + bulk copies), 1 = MMA issuer + TMEM owner,
// 2.. = epilogue (also build the split query), (a second MMA issuer with 8
// epilogue warps), last = combiner: the epilogue warps hand each document's
// per-warp row maxima over through an mbarrier-guarded exchange slot and go
// on to the next document; the combiner takes the maximum over warps, sums the
// query rows and writes the score.
#pragma once

#include <cuda.h>
#include <cstdint>
#include <cuda_fp16.h>
#include "fm_fwd.cuh"
#include "fm_ptx.cuh"

namespace fm {

// two warps + 4 or 8 epilogue warps (8: two per TMEM lane quarter taking
// alternate chunks, so every scheduler has two independent epilogue warps)
// (with 8 epilogue warps a second MMA issuer follows them: warp 10), then the
// combiner warp that sums each document's row maxima
__host__ __device__ constexpr int i8_combiner_warp(int epi_warps) { return 2 + epi_warps + (epi_warps == 8 ? 1 : 0); }
__host__ __device__ constexpr int i8_threads(int epi_warps) { return (i8_combiner_warp(epi_warps) + 1) * 32; }
#ifndef FM_I8_TOKENS
#define FM_I8_TOKENS 256
#endif
constexpr int kI8Tokens = FM_I8_TOKENS;  // tokens per chunk (one TMA box)
constexpr int kI8Half = 128;             // tokens per MMA (M)
constexpr int kI8Halves = kI8Tokens / kI8Half;  // M blocks per chunk
constexpr int kI8Xch = 8;       // per-document exchange slots of the epilogue

struct Int8Args {
  const int32_t* lengths;  // [B] or null
  float* scores;           // [B]
  const __half* q;         // [Lq, d]
  const __half* scales;    // [B, Ld]
  const __half* mins;      // [B, Ld]
  int* status;
  uint64_t timeout_ns;
  int B, Lq, Ld, d;
  int N;                   // MMA N = 2 parts x 32 x GQ
  int atoms;               // 128-element K atoms (ceil(d / 128))
  int nu;                  // uint8 ring slots
  int nts;                 // TMEM slots (two halves of N columns each)
  size_t sc_total_bytes;   // bytes of the scales tensor (B * Ld * 2)
  uint32_t sc_slot_bytes;  // fp16 scale span + min span of one chunk
  uint32_t off_q, off_u, off_sc, off_misc, off_bar, u_slot_bytes;
  int dbg;  // tuning builds (FM_TUNING) only: bits that switch off parts of the work
};

__device__ __forceinline__ int i8_len(const Int8Args& a, int b) {
  int len = a.lengths ? __ldg(a.lengths + b) : a.Ld;
  return len < 0 ? 0 : (len > a.Ld ? a.Ld : len);
}

// Max over the 32 lanes of v[j] for every j; afterwards lane j's v[0] holds
// column j's maximum.  Lanes with bit o set keep the upper half at offset o.
// (The FP8 kernel's per-document reduction.)
__device__ __forceinline__ float butterfly_max32(float (&v)[32], int lane) {
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

__device__ __forceinline__ void spin_drain(uint32_t bar, uint32_t parity, const Int8Args& a) {
  const uint64_t t0 = globaltimer_ns();
  while (!mbar_try_wait(bar, parity)) {
    if (globaltimer_ns() - t0 > a.timeout_ns) {
      record_status(a.status, FM_ERR_TIMEOUT_DRAIN);
      break;
    }
  }
}

template <int GQ, int EW>
__global__ void __launch_bounds__(i8_threads(EW), 1)
    maxsim_int8_kernel(const __grid_constant__ CUtensorMap tmap_u, const Int8Args a) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const uint32_t sbase = smem_u32(smem);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  // barriers: u_full[nu] u_empty[nu] t_full[nts] t_empty[nts] q_ready drain x_full[kI8Xch] x_empty[kI8Xch]
  const uint32_t bar0 = sbase + a.off_bar;
  auto u_full = [&](int i) { return bar0 + 8u * i; };
  auto u_empty = [&](int i) { return bar0 + 8u * (a.nu + i); };
  auto t_full = [&](int i) { return bar0 + 8u * (2 * a.nu + i); };
  auto t_empty = [&](int i) { return bar0 + 8u * (2 * a.nu + a.nts + i); };
  const uint32_t q_ready = bar0 + 8u * (2 * a.nu + 2 * a.nts);
  const uint32_t drain = q_ready + 8u;
  auto x_full = [&](int i) { return drain + 8u + 8u * i; };
  auto x_empty = [&](int i) { return drain + 8u + 8u * (kI8Xch + i); };
  uint8_t* ctl_area = smem + a.off_bar + 8 * (2 * a.nu + 2 * a.nts + 2 + 2 * kI8Xch);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(ctl_area);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(ctl_area + 8);
  WaitCtl ctl{abort_flag, a.status, a.timeout_ns};

  float* a256_s = reinterpret_cast<float*>(smem + a.off_misc);  // [64] alpha / 256 per query row
  float* qsum_s = a256_s + 64;                                   // [64]
  float* xch = qsum_s + 64;                                      // [kI8Xch docs][EW warps][GQ][32]

  if (threadIdx.x == 0) {
    for (int i = 0; i < a.nu; ++i) {
      mbar_init(u_full(i), 1);       // producer's expect_tx arrival + transaction bytes
      mbar_init(u_empty(i), 1 + 4);  // MMA commit + the four epilogue warps of the chunk
    }
    for (int i = 0; i < a.nts; ++i) {
      mbar_init(t_full(i), 1);
      mbar_init(t_empty(i), 4);
    }
    mbar_init(q_ready, EW);
    mbar_init(drain, EW == 8 ? 2 : 1);  // every MMA issuer commits
    for (int i = 0; i < kI8Xch; ++i) {
      mbar_init(x_full(i), EW);  // every epilogue warp's row maxima of the document
      mbar_init(x_empty(i), 1);  // the combiner has read the slot
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), 512);
    tmem_relinquish();
  }
  if (warp == 0 && lane == 0) tma_prefetch_desc(&tmap_u);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const int w0 = blockIdx.x, wstep = gridDim.x;

  if (warp == 0) {
    // ===================== producer =====================
    if (lane == 0) {
      FM_TR_DECL;
      const uint64_t pol = l2_policy_evict_first();
      const uint32_t tx = a.atoms * kI8Tokens * 128u;
      Ring ur;
      int issued = 0;
      bool ok = true;
      for (int b = w0; b < a.B && ok; b += wstep) {
        const int len = i8_len(a, b);
        const int nch = (len + kI8Tokens - 1) / kI8Tokens;
        for (int c = 0; c < nch; ++c) {
          FM_TR(4, 1);
          if (!mbar_wait(u_empty(ur.idx), ur.phase ^ 1u, ctl, FM_ERR_TIMEOUT_UEMPTY)) {
            ok = false;
            break;
          }
          FM_TR(4, 2);
          // uint8 tile by TMA; the chunk's fp16 scales and mins by two bulk copies
          // of the enclosing 16-byte-aligned spans (staging: [scales span][mins span])
          const size_t e0 = static_cast<size_t>(b) * a.Ld + static_cast<size_t>(c) * kI8Tokens;
          const size_t byte0 = e0 * 2;
          const size_t lo16 = byte0 & ~static_cast<size_t>(15);
          const uint32_t span =
              static_cast<uint32_t>((byte0 + kI8Tokens * 2 - lo16 + 15) & ~static_cast<size_t>(15));
          const bool bulk_ok = lo16 + span <= a.sc_total_bytes && !FM_DBG(a, 4);
          uint8_t* stage = smem + a.off_sc + ur.idx * a.sc_slot_bytes;
          if (!bulk_ok && !FM_DBG(a, 4)) {
            // the span would run past the end of the tensors: plain loads (last chunk)
            __half* ss = reinterpret_cast<__half*>(stage);
            __half* ms = reinterpret_cast<__half*>(stage + a.sc_slot_bytes / 2);
            const int sh = static_cast<int>((byte0 - lo16) / 2);
            const size_t total = static_cast<size_t>(a.B) * a.Ld;
            for (int t = 0; t < kI8Tokens && e0 + t < total; ++t) {
              ss[sh + t] = a.scales[e0 + t];
              ms[sh + t] = a.mins[e0 + t];
            }
          }
          // this arrival also releases the plain stores above
          mbar_expect_tx(u_full(ur.idx), tx + (bulk_ok ? 2 * span : 0u));
          const uint32_t dst = sbase + a.off_u + ur.idx * a.u_slot_bytes;
          for (int at = 0; at < a.atoms; ++at)
            tma_load_3d(dst + at * kI8Tokens * 128, &tmap_u, at * 128, c * kI8Tokens, b, u_full(ur.idx),
                        pol);
          if (bulk_ok) {
            const uint32_t st = smem_u32(stage);
            bulk_load(st, reinterpret_cast<const uint8_t*>(a.scales) + lo16, span, u_full(ur.idx), pol);
            bulk_load(st + a.sc_slot_bytes / 2, reinterpret_cast<const uint8_t*>(a.mins) + lo16, span,
                      u_full(ur.idx), pol);
          }
          FM_TR(4, 3);
          ur.next(a.nu);
          ++issued;
        }
      }
      for (int i = 0; i < a.nu && i < issued; ++i) {
        if (--ur.idx < 0) {
          ur.idx = a.nu - 1;
          ur.phase ^= 1u;
        }
        spin_drain(u_full(ur.idx), ur.phase, a);
      }
    }
  } else if (warp == 1 || (EW == 8 && warp == 2 + EW)) {
    // ===================== MMA issuer(s) =====================
    // With 8 epilogue warps two threads (warps 1 and 10) issue, each owning
    // alternate TMEM slots; the slot counts (nts, nu) are even, so every use of
    // a TMEM slot and of a staging slot is handled by the same issuer.
    if (lane == 0) {
      const int me = warp == 1 ? 0 : 1;
      [[maybe_unused]] const int ich = me == 0 ? 0 : 5;  // trace channel of this issuer (FM_TRACE)
      FM_TR_DECL;
      // A = uint8 chunk (unsigned, M = 128 tokens), B = split query (signed, N rows)
      const uint32_t idesc = (2u << 4) | (0u << 7) | (1u << 10) |
                             (static_cast<uint32_t>(a.N >> 3) << 17) | (static_cast<uint32_t>(128 >> 4) << 24);
      const uint64_t bq = smem_desc_sw128(sbase + a.off_q);
      const uint32_t q_atom = a.N * 8u;        // one K atom of the query parts, 16-byte units
      const uint32_t u_atom = kI8Tokens * 8u;  // one K atom of a chunk
      Ring ur, tr;
      bool ok = mbar_wait(q_ready, 0, ctl, FM_ERR_TIMEOUT_QFULL);
      tc_fence_after();
      for (int b = w0; b < a.B && ok; b += wstep) {
        const int len = i8_len(a, b);
        const int nch = (len + kI8Tokens - 1) / kI8Tokens;
        for (int c = 0; c < nch; ++c) {
          if (EW == 8 && (tr.idx & 1) != me) {  // the other issuer's slot
            tr.next(a.nts);
            ur.next(a.nu);
            continue;
          }
          // a half with no valid token is neither multiplied nor read by the epilogue
          const int nhalf = min(kI8Halves, (len - c * kI8Tokens + kI8Half - 1) / kI8Half);
          FM_TR(ich, 1);
          if (!mbar_wait(u_full(ur.idx), ur.phase, ctl, FM_ERR_TIMEOUT_UFULL)) { ok = false; break; }
          FM_TR(ich, 2);
          if (!mbar_wait(t_empty(tr.idx), tr.phase ^ 1u, ctl, FM_ERR_TIMEOUT_TEMPTY)) { ok = false; break; }
          FM_TR(ich, 3);
          tc_fence_after();
          FM_PROF_T0(pm0);
          const uint64_t au = smem_desc_sw128(sbase + a.off_u + ur.idx * a.u_slot_bytes);
          const uint32_t tacc = tmem_base + tr.idx * kI8Halves * a.N;
          for (int hb = 0; hb < nhalf; ++hb) {  // rows [128 hb, 128 hb + 128) of the chunk
            const uint64_t ah = au + hb * (kI8Half * 128u >> 4);
            for (int at = 0; at < a.atoms && !FM_DBG(a, 2); ++at) {
#pragma unroll
              for (int kk = 0; kk < 4; ++kk)  // K = 32 bytes per step, 4 steps per 128-byte atom
                tc_mma_i8(tacc + hb * a.N, ah + at * u_atom + kk * 2u, bq + at * q_atom + kk * 2u,
                          idesc, (at | kk) ? 1u : 0u);
            }
          }
          tc_commit(t_full(tr.idx));
          tc_commit(u_empty(ur.idx));
          FM_TR(ich, 4);
          FM_PROF_ADD(20, pm0);
          tr.next(a.nts);
          ur.next(a.nu);
        }
      }
      tc_commit(drain);
      spin_drain(drain, 0, a);
    }
  } else if (warp >= 2 && warp < 2 + EW) {
    // ===================== epilogue =====================
    const int sub = warp & 3;  // TMEM lane quarter = tokens [32 sub, 32 sub + 32) of a chunk
    const int et = threadIdx.x - 64;  // 0 .. 32 EW - 1
    // --- split the query into two signed 8-bit parts: B row r = part * 32 GQ + query row;
    //     one alpha = max|Q| / 127 for the whole query ---
    {
      const int r = et;
      const bool builder = r < a.N;
      const int qrow = builder ? r % (32 * GQ) : 0;
      const int part = builder ? r / (32 * GQ) : 0;
      const bool rv = builder && qrow < a.Lq;
      const __half* qr = a.q + static_cast<size_t>(rv ? qrow : 0) * a.d;
      float amax = 0.f, qs = 0.f;
      if (rv)
        for (int k = 0; k < a.d; ++k) {
          const float v = __half2float(qr[k]);
          amax = fmaxf(amax, fabsf(v));
          qs += v;
        }
      if (builder && part == 0) {
        a256_s[qrow] = amax;  // row max for now
        qsum_s[qrow] = qs;
      }
      named_bar_sync(1, 32 * EW);
      float gmax = 0.f;
      for (int j = 0; j < 32 * GQ; ++j) gmax = fmaxf(gmax, a256_s[j]);
      const float alpha = gmax > 0.f ? gmax / 127.f : 1.f;
      named_bar_sync(1, 32 * EW);
      if (builder && part == 0) a256_s[qrow] = alpha * (1.f / 256.f);
      if (builder) {
        uint8_t* row = smem + a.off_q + r * 128;
        for (int at = 0; at < a.atoms; ++at) {
          for (int c16 = 0; c16 < 8; ++c16) {
            uint32_t w[4] = {0u, 0u, 0u, 0u};
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              const int k = at * 128 + c16 * 16 + j;
              int val = 0;
              if (rv && k < a.d) {
                const float x = __half2float(qr[k]) / alpha;
                int hi = static_cast<int>(rintf(x));
                hi = hi > 127 ? 127 : (hi < -127 ? -127 : hi);
                if (part == 0) {
                  val = hi;
                } else {
                  const int lo = static_cast<int>(rintf((x - static_cast<float>(hi)) * 256.f));
                  val = lo > 127 ? 127 : (lo < -127 ? -127 : lo);
                }
              }
              w[j >> 2] |= (static_cast<uint32_t>(val) & 0xffu) << (8 * (j & 3));
            }
            *reinterpret_cast<uint4*>(row + at * a.N * 128 + ((c16 ^ (r & 7)) << 4)) =
                make_uint4(w[0], w[1], w[2], w[3]);
          }
        }
      }
      fence_proxy_async_smem();
      named_bar_sync(1, 32 * EW);
      if (lane == 0) mbar_arrive(q_ready);
    }
    // query constants (the same for every lane): alpha / 256 and per-row sum_k Q
    const float a256 = a256_s[0];
    float qsm[32 * GQ];
#pragma unroll
    for (int j = 0; j < 32 * GQ; ++j) qsm[j] = qsum_s[j];
    // EW == 8: the two warps of a lane quarter own alternate TMEM slots (the
    // slot count is even), so every use of a slot is read by the same warp and
    // no warp ever waits on a slot barrier more than one phase ahead
    const int half = (EW == 8) ? (warp - 2) / 4 : 0;
    const uint32_t lane_base = static_cast<uint32_t>(sub * 32) << 16;
    const int tok_in_chunk = sub * 32 + lane;
    Ring ur, tr;
    // trace channels (FM_TRACE): 1 and 2 = the two warps of lane quarter 0, 3 = a warp of quarter 2
    [[maybe_unused]] const int ech = sub == 0 ? 1 + half : (sub == 2 && half == 0 ? 3 : 7);
    FM_TR_DECL;
    int dloc = 0;
    int kglob = 0;  // chunk counter of this CTA
    bool ok = true;
    for (int b = w0; b < a.B && ok; b += wstep, ++dloc) {
      const int len = i8_len(a, b);
      const int nch = (len + kI8Tokens - 1) / kI8Tokens;
      // running max per query row over this thread's tokens; lanes are reduced per document
      float rmax[32 * GQ];
#pragma unroll
      for (int j = 0; j < 32 * GQ; ++j) rmax[j] = -INFINITY;
      for (int c = 0; c < nch; ++c, ++kglob) {
        if (EW == 8 && (tr.idx & 1) != half) {  // the other warp of this lane quarter reads it
          tr.next(a.nts);
          ur.next(a.nu);
          continue;
        }
        // u_full also publishes the chunk's scales/mins; the slot is not refilled
        // before this warp releases it below
        if (ech < 7) FM_TR(ech, 1);
        if (!mbar_wait(u_full(ur.idx), ur.phase, ctl, FM_ERR_TIMEOUT_UFULL)) { ok = false; break; }
        if (!mbar_wait(t_full(tr.idx), tr.phase, ctl, FM_ERR_TIMEOUT_TFULL)) { ok = false; break; }
        if (ech < 7) FM_TR(ech, 2);
        tc_fence_after();
        FM_PROF_T0(pe0);
        const size_t byte0 = (static_cast<size_t>(b) * a.Ld + static_cast<size_t>(c) * kI8Tokens) * 2;
        const uint8_t* stage = smem + a.off_sc + ur.idx * a.sc_slot_bytes;
        const bool full = (c + 1) * kI8Tokens <= len;  // whole chunk valid (warp-uniform)
#pragma unroll
        for (int hb = 0; hb < kI8Halves; ++hb) {
          const int tic = hb * kI8Half + tok_in_chunk;
          const bool valid = c * kI8Tokens + tic < len;
          if (!full && !__any_sync(0xffffffffu, valid)) continue;
          const uint32_t th = tmem_base + lane_base + tr.idx * kI8Halves * a.N + hb * a.N;
          const int sh = static_cast<int>((byte0 & 15) >> 1) + tic;
          const float s_t = __half2float(reinterpret_cast<const __half*>(stage)[sh]);
          const float m_t = __half2float(reinterpret_cast<const __half*>(stage + a.sc_slot_bytes / 2)[sh]);
          const float sa = s_t * a256;
#pragma unroll
          for (int g = 0; g < GQ; ++g) {
            uint32_t h[32], l[32];
            tmem_ld32(th + g * 32, reinterpret_cast<float(&)[32]>(h));
            tmem_ld32(th + 32 * GQ + g * 32, reinterpret_cast<float(&)[32]>(l));
            tmem_wait_ld();
            if ((full || valid) && !FM_DBG(a, 1)) {
#pragma unroll
              for (int j = 0; j < 32; ++j) {
                const int hl = static_cast<int>(h[j]) * 256 + static_cast<int>(l[j]);  // exact
                const float sv = fmaf(sa, static_cast<float>(hl), m_t * qsm[g * 32 + j]);
                rmax[g * 32 + j] = fmaxf(rmax[g * 32 + j], sv);
              }
            }
          }
        }
        if (ech < 7) FM_TR(ech, 3);
        FM_PROF_ADD(22 + sub, pe0);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(t_empty(tr.idx));
          mbar_arrive(u_empty(ur.idx));
        }
        tr.next(a.nts);
        ur.next(a.nu);
      }
      if (!ok) break;
      float acc[GQ];
#pragma unroll
      for (int g = 0; g < GQ; ++g) {
        float v[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = rmax[g * 32 + j];
        acc[g] = colmax32(v, lane);
      }
      if (ech < 7) FM_TR(ech, 5);
      // --- hand the row maxima to the combiner: wait until it has read this
      //     exchange slot's previous document (parity of the slot's last use) ---
      const int slot = dloc % kI8Xch;
      const uint32_t xpar = static_cast<uint32_t>(dloc / kI8Xch) & 1u;
      if (!mbar_wait(x_empty(slot), xpar ^ 1u, ctl, FM_ERR_TIMEOUT_TFULL)) break;
      if (ech < 7) FM_TR(ech, 6);
      const int ew = warp - 2;
#pragma unroll
      for (int g = 0; g < GQ; ++g) xch[((slot * EW + ew) * GQ + g) * 32 + lane] = acc[g];
      __syncwarp();
      if (lane == 0) mbar_arrive(x_full(slot));
      if (ech < 7) FM_TR(ech, 7);
    }
  } else if (warp == i8_combiner_warp(EW)) {
    // ===================== combiner =====================
    // lane = query row of a 32-row group: max over the epilogue warps, then the
    // sum over the query's rows (the same order as a one-warp reduction)
    int dloc = 0;
    for (int b = w0; b < a.B; b += wstep, ++dloc) {
      const int slot = dloc % kI8Xch;
      const uint32_t xpar = static_cast<uint32_t>(dloc / kI8Xch) & 1u;
      if (!mbar_wait(x_full(slot), xpar, ctl, FM_ERR_TIMEOUT_TFULL)) break;
      float tot = 0.f;
#pragma unroll
      for (int g = 0; g < GQ; ++g) {
        float mm = -INFINITY;
        for (int w = 0; w < EW; ++w) mm = fmaxf(mm, xch[((slot * EW + w) * GQ + g) * 32 + lane]);
        tot += (g * 32 + lane < a.Lq) ? mm : 0.f;
      }
      tot = warp_sum(tot);
      if (lane == 0) a.scores[b] = tot;
      __syncwarp();
      if (lane == 0) mbar_arrive(x_empty(slot));
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
