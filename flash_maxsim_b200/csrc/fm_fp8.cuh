// FP8 (e4m3) document storage: fused-dequant MaxSim for one short query
// (Lq <= 64, d <= 256), sm_100a.
//
//   score[b] = sum_q max_{t < len_b} scale[b,t] * sum_k Q[q,k] * e4m3(code[b,t,k])
//
// The sibling of the INT8 path (flash_maxsim/flash_maxsim_quant.py:105-142)
// for documents stored as e4m3 codes with one fp32 scale per token
// (x ~= scale_t * code, scale_t = max|x_t| / 448): half the HBM bytes of
// fp16 documents, no per-token min.
//
//  * The e4m3 codes are never converted.  TMA copies a chunk of 256 tokens
//    (128 for 64-row queries) from
//    HBM into 128-byte-swizzled shared memory and the tensor core multiplies
//    it as e4m3 (tcgen05.mma kind::f8f6f4, fp32 accumulate) with the chunk
//    in 128-token halves as the M = 128 operand.
//  * The fp16 query is split once per CTA into three e4m3 parts,
//    Q / alpha ~= h + l + e with h = e4m3(x), l = e4m3(x - h),
//    e = e4m3(x - h - l), x = Q / alpha, alpha = max|Q| / 448 (relative
//    error about 2^-12 per element).  The three parts are one N operand of
//    3 x 32 GQ rows, so one MMA pass gives <h,c>, <l,c>, <e,c> for every
//    (token, query row); e4m3 x e4m3 products are exact in fp32.
//  * TMEM lane = token, column = (part, query row).  Each epilogue thread
//    owns one token: S = scale_t * alpha * (<h,c> + <l,c> + <e,c>), masked
//    past the document, running max per query row; the token's scale is
//    loaded by the thread itself (one coalesced 128-byte row per warp),
//    issued before it waits for the accumulator.  A 31-shuffle butterfly
//    reduces the warp's tokens per query row and the last of the 8 warps of
//    a document writes its score.
//
// Warp roles: 0 = producer (TMA), 1 = MMA issuer + TMEM owner,
// 2..9 = epilogue (two warps per TMEM lane quarter, alternate chunks; they
// also build the split query).
#pragma once

#include <cuda.h>
#include <cstdint>
#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include "fm_aux.cuh"
#include "fm_int8.cuh"
#include "fm_ptx.cuh"
#include "fm_topk.cuh"

namespace fm {

constexpr int kF8Half = 128;    // tokens per MMA (M); a chunk is NH of them (one TMA box per K atom)
constexpr int kF8EW = 8;        // epilogue warps
constexpr int kF8Xch = 8;       // per-document exchange slots of the epilogue
constexpr int kF8Parts = 3;     // e4m3 parts of the query
__host__ __device__ constexpr int f8_threads() { return (2 + kF8EW) * 32; }

struct Fp8Args {
  const int32_t* lengths;  // [B] or null
  float* scores;           // [B]
  const __half* q;         // [Lq, d]
  const float* scales;     // [B, Ld] per-token scales
  int* status;
  uint64_t timeout_ns;
  int B, Lq, Ld, d;
  int N;                   // MMA N = 3 parts x 32 GQ rows
  int atoms;               // 128-element K atoms (ceil(d / 128))
  int nu;                  // chunk ring slots
  int nts;                 // TMEM slots (N columns each; even)
  uint32_t off_q, off_u, off_misc, off_bar, u_slot_bytes;
  TopkArgs topk;           // k > 0: per-CTA top-k candidates in the tail
};

__device__ __forceinline__ int f8_len(const Fp8Args& a, int b) {
  int len = a.lengths ? __ldg(a.lengths + b) : a.Ld;
  return len < 0 ? 0 : (len > a.Ld ? a.Ld : len);
}

// D[tmem] (+)= A[smem] * B[smem]^T, kind::f8f6f4 (e4m3 x e4m3 here), fp32 accumulate.
__device__ __forceinline__ void tc_mma_f8(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Instruction descriptor, kind::f8f6f4: D fp32 [4,6)=1, A and B e4m3 (type 0
// at [7,10) and [10,13)), both K-major, N>>3 at [17,23), M>>4 at [24,29).
__host__ __device__ __forceinline__ uint32_t idesc_e4m3_f32(int M, int N) {
  return (1u << 4) | (static_cast<uint32_t>(N >> 3) << 17) | (static_cast<uint32_t>(M >> 4) << 24);
}

__device__ __forceinline__ float e4m3_round(float x) {
  const __nv_fp8_storage_t c = __nv_cvt_float_to_fp8(x, __NV_SATFINITE, __NV_E4M3);
  return __half2float(__half(__nv_cvt_fp8_to_halfraw(c, __NV_E4M3)));
}
__device__ __forceinline__ uint32_t e4m3_bits(float x) {
  return static_cast<uint32_t>(__nv_cvt_float_to_fp8(x, __NV_SATFINITE, __NV_E4M3));
}

template <int GQ, int NH>
__global__ void __launch_bounds__(f8_threads(), 1)
    maxsim_fp8_kernel(const __grid_constant__ CUtensorMap tmap_u, const Fp8Args a) {
  constexpr int EW = kF8EW;
  constexpr int kF8Tokens = NH * kF8Half;  // tokens per chunk
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const uint32_t sbase = smem_u32(smem);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  // barriers: u_full[nu] u_empty[nu] t_full[nts] t_empty[nts] q_ready drain
  const uint32_t bar0 = sbase + a.off_bar;
  auto u_full = [&](int i) { return bar0 + 8u * i; };
  auto u_empty = [&](int i) { return bar0 + 8u * (a.nu + i); };
  auto t_full = [&](int i) { return bar0 + 8u * (2 * a.nu + i); };
  auto t_empty = [&](int i) { return bar0 + 8u * (2 * a.nu + a.nts + i); };
  const uint32_t q_ready = bar0 + 8u * (2 * a.nu + 2 * a.nts);
  const uint32_t drain = q_ready + 8u;
  uint8_t* ctl_area = smem + a.off_bar + 8 * (2 * a.nu + 2 * a.nts + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(ctl_area);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(ctl_area + 8);
  WaitCtl ctl{abort_flag, a.status, a.timeout_ns};

  float* amax_s = reinterpret_cast<float*>(smem + a.off_misc);    // [64] per query row max|Q|
  float* xch = amax_s + 64;                                        // [kF8Xch docs][EW warps][GQ][32]
  int* cnt = reinterpret_cast<int*>(xch + kF8Xch * EW * GQ * 32);  // [kF8Xch] arrivals
  volatile int* done = cnt + kF8Xch;                               // [kF8Xch] combined generations

  if (threadIdx.x == 0) {
    for (int i = 0; i < a.nu; ++i) {
      mbar_init(u_full(i), 1);   // producer's expect_tx arrival + transaction bytes
      mbar_init(u_empty(i), 1);  // MMA commit
    }
    for (int i = 0; i < a.nts; ++i) {
      mbar_init(t_full(i), 1);
      mbar_init(t_empty(i), 4);  // the four warps (one per lane quarter) that take the chunk
    }
    mbar_init(q_ready, EW);
    mbar_init(drain, 1);
    *abort_flag = 0;
    for (int i = 0; i < kF8Xch; ++i) {
      cnt[i] = 0;
      done[i] = 0;
    }
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
      const uint64_t pol = l2_policy_evict_first();
      const uint32_t tx = a.atoms * kF8Tokens * 128u;
      Ring ur;
      int issued = 0;
      bool ok = true;
      for (int b = w0; b < a.B && ok; b += wstep) {
        const int nch = (f8_len(a, b) + kF8Tokens - 1) / kF8Tokens;
        for (int c = 0; c < nch; ++c) {
          if (!mbar_wait(u_empty(ur.idx), ur.phase ^ 1u, ctl, FM_ERR_TIMEOUT_UEMPTY)) {
            ok = false;
            break;
          }
          mbar_expect_tx(u_full(ur.idx), tx);
          const uint32_t dst = sbase + a.off_u + ur.idx * a.u_slot_bytes;
          for (int at = 0; at < a.atoms; ++at)
            tma_load_3d(dst + at * kF8Tokens * 128, &tmap_u, at * 128, c * kF8Tokens, b, u_full(ur.idx), pol);
          ur.next(a.nu);
          ++issued;
        }
      }
      for (int i = 0; i < a.nu && i < issued; ++i) {
        if (--ur.idx < 0) {
          ur.idx = a.nu - 1;
          ur.phase ^= 1u;
        }
        const uint64_t t0 = globaltimer_ns();
        while (!mbar_try_wait(u_full(ur.idx), ur.phase)) {
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
      // A = e4m3 chunk (M = 128 tokens), B = the three query parts (N rows)
      const uint32_t idesc = idesc_e4m3_f32(128, a.N);
      const uint64_t bq = smem_desc_sw128(sbase + a.off_q);
      const uint32_t q_atom = a.N * 8u;         // one K atom of the query parts, 16-byte units
      const uint32_t u_atom = kF8Tokens * 8u;   // one K atom of a chunk
      Ring ur, tr;
      bool ok = mbar_wait(q_ready, 0, ctl, FM_ERR_TIMEOUT_QFULL);
      tc_fence_after();
      for (int b = w0; b < a.B && ok; b += wstep) {
        const int nch = (f8_len(a, b) + kF8Tokens - 1) / kF8Tokens;
        for (int c = 0; c < nch; ++c) {
          if (!mbar_wait(u_full(ur.idx), ur.phase, ctl, FM_ERR_TIMEOUT_UFULL)) { ok = false; break; }
          if (!mbar_wait(t_empty(tr.idx), tr.phase ^ 1u, ctl, FM_ERR_TIMEOUT_TEMPTY)) { ok = false; break; }
          tc_fence_after();
          const uint64_t au = smem_desc_sw128(sbase + a.off_u + ur.idx * a.u_slot_bytes);
          const uint32_t tacc = tmem_base + tr.idx * (NH * a.N);
          // a 128-token half with no valid token is neither multiplied nor read
          const int nhalf = min(NH, (f8_len(a, b) - c * kF8Tokens + kF8Half - 1) / kF8Half);
          for (int hb = 0; hb < nhalf; ++hb) {
            const uint64_t ah = au + hb * (kF8Half * 128u >> 4);
            for (int at = 0; at < a.atoms; ++at) {
#pragma unroll
              for (int kk = 0; kk < 4; ++kk)  // K = 32 bytes per step, 4 steps per 128-byte atom
                tc_mma_f8(tacc + hb * a.N, ah + at * u_atom + kk * 2u, bq + at * q_atom + kk * 2u, idesc,
                          (at | kk) ? 1u : 0u);
            }
          }
          tc_commit(t_full(tr.idx));
          tc_commit(u_empty(ur.idx));
          tr.next(a.nts);
          ur.next(a.nu);
        }
      }
      tc_commit(drain);
      const uint64_t t0 = globaltimer_ns();
      while (!mbar_try_wait(drain, 0)) {
        if (globaltimer_ns() - t0 > a.timeout_ns) {
          record_status(a.status, FM_ERR_TIMEOUT_DRAIN);
          break;
        }
      }
    }
  } else if (warp >= 2 && warp < 2 + EW) {
    // ===================== epilogue =====================
    const int sub = warp & 3;          // TMEM lane quarter = tokens [32 sub, 32 sub + 32) of a chunk
    const int et = threadIdx.x - 64;   // 0 .. 32 EW - 1
    constexpr int R = 32 * GQ;         // query rows per part
    // --- the split query: B row r = part * R + query row, 128 bytes per K atom ---
    {
      const int qrow = et < R ? et : 0;
      const bool rv = et < R && qrow < a.Lq;
      const __half* qr = a.q + static_cast<size_t>(rv ? qrow : 0) * a.d;
      float amax = 0.f;
      if (rv)
        for (int k = 0; k < a.d; ++k) amax = fmaxf(amax, fabsf(__half2float(qr[k])));
      if (et < R) amax_s[et] = amax;
      named_bar_sync(1, 32 * EW);
      float gmax = 0.f;
      for (int j = 0; j < R; ++j) gmax = fmaxf(gmax, amax_s[j]);
      const float alpha = gmax > 0.f ? gmax / 448.f : 1.f;
      if (et < R) {
        for (int at = 0; at < a.atoms; ++at) {
          for (int c16 = 0; c16 < 8; ++c16) {
            uint32_t w[kF8Parts][4] = {};
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              const int k = at * 128 + c16 * 16 + j;
              float x = (rv && k < a.d) ? __half2float(qr[k]) / alpha : 0.f;
#pragma unroll
              for (int p = 0; p < kF8Parts; ++p) {
                const float h = e4m3_round(x);
                w[p][j >> 2] |= e4m3_bits(x) << (8 * (j & 3));
                x -= h;  // exact: h is x rounded to a coarser grid
              }
            }
#pragma unroll
            for (int p = 0; p < kF8Parts; ++p) {
              const int r = p * R + et;
              uint8_t* row = smem + a.off_q + at * a.N * 128 + r * 128;
              *reinterpret_cast<uint4*>(row + ((c16 ^ (r & 7)) << 4)) = make_uint4(w[p][0], w[p][1], w[p][2], w[p][3]);
            }
          }
        }
      }
      fence_proxy_async_smem();
      named_bar_sync(1, 32 * EW);
      if (et == 0) amax_s[63] = alpha;
      named_bar_sync(1, 32 * EW);
      if (lane == 0) mbar_arrive(q_ready);
    }
    const float alpha = amax_s[63];
    // the two warps of a lane quarter own alternate TMEM slots (nts is even)
    const int half = (warp - 2) / 4;
    const uint32_t lane_base = static_cast<uint32_t>(sub * 32) << 16;
    const int tok = sub * 32 + lane;
    Ring tr;
    int dloc = 0;
    bool ok = true;
    for (int b = w0; b < a.B && ok; b += wstep, ++dloc) {
      const int len = f8_len(a, b);
      const int nch = (len + kF8Tokens - 1) / kF8Tokens;
      float rmax[R];
#pragma unroll
      for (int j = 0; j < R; ++j) rmax[j] = -INFINITY;
      for (int c = 0; c < nch; ++c) {
        if ((tr.idx & 1) != half) {  // the other warp of this lane quarter reads it
          tr.next(a.nts);
          continue;
        }
        // this thread's tokens' scales, loaded before waiting for the accumulator
        float sa[NH];
        bool valid[NH];
#pragma unroll
        for (int hb = 0; hb < NH; ++hb) {
          valid[hb] = c * kF8Tokens + hb * kF8Half + tok < len;
          sa[hb] = valid[hb]
                       ? __ldg(a.scales + static_cast<size_t>(b) * a.Ld + c * kF8Tokens + hb * kF8Half + tok) * alpha
                       : 0.f;
        }
        if (!mbar_wait(t_full(tr.idx), tr.phase, ctl, FM_ERR_TIMEOUT_TFULL)) { ok = false; break; }
        tc_fence_after();
#pragma unroll
        for (int hb = 0; hb < NH; ++hb) {
          if (!__any_sync(0xffffffffu, valid[hb])) continue;  // half not multiplied
          const uint32_t th = tmem_base + lane_base + tr.idx * (NH * a.N) + hb * a.N;
#pragma unroll
          for (int g = 0; g < GQ; ++g) {
            float h[32], l[32], e[32];
            tmem_ld32(th + g * 32, h);
            tmem_ld32(th + R + g * 32, l);
            tmem_ld32(th + 2 * R + g * 32, e);
            tmem_wait_ld();
            if (valid[hb]) {
#pragma unroll
              for (int j = 0; j < 32; ++j)
                rmax[g * 32 + j] = fmaxf(rmax[g * 32 + j], sa[hb] * ((h[j] + l[j]) + e[j]));
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
        acc[g] = butterfly_max32(v, lane);
      }
      // --- combine the warps of this document: the last one to arrive sums ---
      const int slot = dloc % kF8Xch;
      const int gen = dloc / kF8Xch;
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
#pragma unroll
        for (int g = 0; g < GQ; ++g) {
          float mm = -INFINITY;
          for (int w = 0; w < EW; ++w) mm = fmaxf(mm, xch[((slot * EW + w) * GQ + g) * 32 + lane]);
          tot += (g * 32 + lane < a.Lq) ? mm : 0.f;
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
    // the k best of the documents this CTA scored, read back from its scores
    const int count = (a.B - w0 + wstep - 1) / wstep;
    const size_t o = static_cast<size_t>(blockIdx.x) * a.topk.k;
    warp_topk<8>(count, a.topk.k, [&](int p) { return TopkCand{a.scores[w0 + p * wstep], w0 + p * wstep}; },
                 a.topk.cand_s + o, a.topk.cand_b + o, lane);
  }
}

// Per-token e4m3 quantisation: scale = max|x| / 448 (1 for an all-zero
// token), code = e4m3(x / scale) with round-to-nearest-even and saturation
// (|x / scale| <= 448 up to rounding).  A row takes LPR lanes (8 elements
// each per segment, LPR = 8 / 16 / 32 for d <= 64 / 128 / larger, the INT8
// quantiser's layout), loaded once into registers.  With NORM every row is
// first divided by max(||x||_2, 1e-12), the norm summed in the fixed order of
// row_inv_norm_sq.  T = __half, float or __nv_bfloat16.
template <typename T, int LPR, bool NORM = false>
__global__ void __launch_bounds__(256) quantize_fp8_kernel(const T* __restrict__ D, uint8_t* __restrict__ codes,
                                                           float* __restrict__ scales, int64_t rows, int d) {
  constexpr int RPW = 32 / LPR;                       // rows per warp
  constexpr int SEG = LPR == 32 ? kMaxSeg : 1;        // segments per lane (d <= 2048)
  const int lane = threadIdx.x & 31;
  const int sub = lane / LPR, l = lane % LPR;
  const int64_t row = (static_cast<int64_t>(blockIdx.x) * 8 + (threadIdx.x >> 5)) * RPW + sub;
  const bool live = row < rows;
  const int nseg = (d + LPR * 8 - 1) / (LPR * 8);
  const T* src = D + (live ? row : 0) * d;
  float v[SEG][8];
#pragma unroll
  for (int g = 0; g < SEG; ++g) {
    const int k = (g * LPR + l) * 8;
    if (live && g < nseg && k < d) load8(src + k, v[g]);
  }
  if (NORM) {
    const float den = fmaxf(__fsqrt_rn(row_inv_norm_sq<LPR, SEG>(v, nseg, l, d)), 1e-12f);
#pragma unroll
    for (int g = 0; g < SEG; ++g)
#pragma unroll
      for (int j = 0; j < 8; ++j) v[g][j] = __fdiv_rn(v[g][j], den);
  }
  float amax = 0.f;
#pragma unroll
  for (int g = 0; g < SEG; ++g) {
    const int k = (g * LPR + l) * 8;
    if (live && g < nseg && k < d) {
#pragma unroll
      for (int j = 0; j < 8; ++j) amax = fmaxf(amax, fabsf(v[g][j]));
    }
  }
#pragma unroll
  for (int o = LPR / 2; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  if (!live) return;
  const float scale = amax > 0.f ? amax / 448.f : 1.f;
#pragma unroll
  for (int g = 0; g < SEG; ++g) {
    const int k = (g * LPR + l) * 8;
    if (g < nseg && k < d) {
      uint32_t w0 = 0, w1 = 0;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const uint32_t c = e4m3_bits(__fdiv_rn(v[g][j], scale));
        if (j < 4) w0 |= c << (8 * j);
        else w1 |= c << (8 * (j - 4));
      }
      *reinterpret_cast<uint2*>(codes + row * d + k) = make_uint2(w0, w1);
    }
  }
  if (l == 0) scales[row] = scale;
}

}  // namespace fm
