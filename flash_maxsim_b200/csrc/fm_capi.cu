// C ABI of libflashmaxsim_sm100.so: argument checks, launch plans, TMA
// descriptors and kernel launches.  Declarations: include/flash_maxsim_sm100.h.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>

#include "../../include/flash_maxsim_sm100.h"
#include "fm_aux.cuh"
#include "fm_fwd.cuh"
#include "fm_int8.cuh"
#include "fm_q1.cuh"
#include "fm_flat.cuh"
#include "fm_topk.cuh"
#include "fm_fp8.cuh"

// Scratch for fm_maxsim_bwd_noalloc: the dQ partial sums live here instead of
// in caller-provided memory.  Every device that loads this library keeps
// these 16 MiB for the life of the process.  In host code the name below is
// only a host-side handle; the device address comes from
// cudaGetSymbolAddress (see noalloc_scratch()).
constexpr size_t kNoAllocScratchBytes = static_cast<size_t>(16) << 20;
static __device__ __align__(256) float g_fm_noalloc_scratch[kNoAllocScratchBytes / sizeof(float)];

namespace fm {
namespace {

constexpr int kMaxSmem = 232448;        // 227 KB opt-in shared memory per CTA on sm_100
constexpr int kMinSmem = 120 * 1024;    // keeps one CTA per SM (each owns all 512 TMEM columns)
std::atomic<int64_t> g_timeout_ns{2000000000LL};
std::atomic<int> g_flat_kernel{0};  // fm_set_option(FM_OPT_FLAT_KERNEL, 1)

int round_up(int x, int m) { return (x + m - 1) / m * m; }
int cdiv(int x, int m) { return (x + m - 1) / m; }

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

int sm_count() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return -1;
  static int cache[64] = {0};
  if (dev < 64 && cache[dev] > 0) return cache[dev];
  int n = 0;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return -1;
  if (dev < 64) cache[dev] = n;
  return n;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// 3D tiled map over a [n2][n1][n0] tensor, box {b0, b1, 1}
bool make_map_3d(CUtensorMap* m, CUtensorMapDataType dt, int esize, const void* base, uint64_t n0,
                 uint64_t n1, uint64_t n2, uint32_t b0, uint32_t b1, CUtensorMapSwizzle sw) {
  auto fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[3] = {n0, n1, n2};
  cuuint64_t strides[2] = {n0 * esize, n0 * n1 * esize};
  cuuint32_t box[3] = {b0, b1, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(m, dt, 3, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// Plan overrides for tuning sweeps, e.g. FLASH_MAXSIM_TUNE="nd=3,nq=3,gd=2",
// read once per process.  Only tuning builds (-DFM_TUNING, never shipped) read
// the variable: its `dbg` bits switch off MMAs, waits or whole kernels to
// measure what is left, so a default build always uses the fixed plan below.
struct Tune {
  int nd = 0, nq = 0, G = 0, C = 0, dbg = 0, gd = 0, flat = 0;
};
#ifdef FM_TUNING
const Tune& tune() {
  static Tune t;
  static std::once_flag once;
  std::call_once(once, [] {
    const char* e = std::getenv("FLASH_MAXSIM_TUNE");
    if (!e) return;
    const char* p = e;
    while (*p) {
      char key[8];
      int v = 0, n = 0;
      if (std::sscanf(p, "%7[a-zA-Z]=%d%n", key, &v, &n) != 2) break;
      if (!std::strcmp(key, "nd")) t.nd = v;
      if (!std::strcmp(key, "nq")) t.nq = v;
      if (!std::strcmp(key, "G")) t.G = v;
      if (!std::strcmp(key, "C")) t.C = v;
      if (!std::strcmp(key, "dbg")) t.dbg = v;
      if (!std::strcmp(key, "gd")) t.gd = v;
      if (!std::strcmp(key, "flat")) t.flat = v;
      p += n;
      if (*p == ',') ++p;
    }
  });
  return t;
}
#else
constexpr Tune kNoTune{};
constexpr const Tune& tune() { return kNoTune; }
#endif

struct Shape {
  int mode;
  bool argmax;
  int Nq, B, Lq, Ld, d, K;
  int shared;
};

// Choose chunk size, ring depths and shared-memory carve-up for `gd`
// documents per work item.
bool plan_for_gd(const Shape& s, int gd, FwdArgs& a, int& smem_bytes) {
  const bool int8 = s.mode == MODE_INT8;
  a.Nq = s.Nq;
  a.B = s.B;
  a.Lq = s.Lq;
  a.Ld = s.Ld;
  a.d = s.d;
  a.K = s.K;
  a.shared = s.shared;
  a.Gq = cdiv(s.Lq, 32);
  a.R = s.shared ? s.Nq * a.Gq : a.Gq;
  a.gd = gd;
  a.n_work = s.shared ? cdiv(s.B, gd) : s.Nq * s.B;
  a.rep = a.R == 1 ? 4 : (a.R == 2 ? 2 : 1);
  const int atoms = cdiv(s.d, 64);
  a.kq_atoms = std::min(atoms, 2);
  a.nk = cdiv(atoms, a.kq_atoms);
  a.d_atoms = a.nk * a.kq_atoms;
  a.d_atoms_real = atoms;
  // Chunk: the fewest chunks of <= 256 tokens that cover Ld with equal sizes,
  // capped so that one chunk (all K atoms) plus two Q stages fit in shared memory.
  if (s.Ld <= 256) {
    a.C = round_up(std::max(s.Ld, 16), 16);
  } else {
    const int n = cdiv(s.Ld, 256);
    a.C = round_up(cdiv(s.Ld, n), 16);
  }
  {
    const int budget = kMaxSmem - 2 * a.kq_atoms * 16384 - 16 * 1024;
    // fp16: one D slot per chunk; INT8: one fp16 slot plus two uint8 staging slots
    const int per_token = a.d_atoms * (int8 ? 256 : 128);
    const int cap = (budget / per_token) / 16 * 16;
    if (cap < 16) return false;
    a.C = std::min(a.C, cap);
    if (tune().C >= 16 && tune().C % 16 == 0 && tune().C <= std::min(256, cap)) a.C = tune().C;
  }
  // two MMA issuers own alternate TMEM slots, so an odd slot count (3 slots of
  // 160 columns) leaves them unbalanced: 192-token chunks give 2 slots at the
  // same MMA cost (an M=128, K=16 MMA takes the same time for any N <= 192)
  if (!int8 && tune().C == 0 && 512 / round_up(a.C, 32) == 3 && (a.nk == 1 || !s.argmax)) {
    const int cap = ((kMaxSmem - 2 * a.kq_atoms * 16384 - 16 * 1024) / (a.d_atoms * 128)) / 16 * 16;
    if (cap >= 192) a.C = 192;
  }
  a.ts_stride = round_up(a.C, 32);
  a.nts = 512 / a.ts_stride;
  a.q_resident = (s.shared && a.R <= 4 && a.nk == 1) ? 1 : 0;
  a.q_flat = (s.Lq % 32 == 0) ? 1 : 0;
  a.dbg = tune().dbg;
  // two MMA issuers (measured faster everywhere; config 5, argmax with the K
  // split over two query stages: 5.88 vs 6.02 ms per forward)
  a.mma2 = (!int8 && a.nts >= 2 && !(tune().dbg & 4096)) ? 1 : 0;
  a.q_stage_bytes = a.kq_atoms * 16384u;
  a.d_slot_bytes = static_cast<uint32_t>(a.d_atoms) * a.C * 128u;
  a.u_slot_bytes = int8 ? static_cast<uint32_t>(a.d_atoms) * a.C * 64u : 0u;
  a.rowbuf = (s.mode == MODE_SPARSE) ? a.Gq * 32 : gd * a.R;
  const int nch_max = cdiv(s.Ld, a.C);
  const int mb_total = cdiv(a.R, 4);

  const int rows_bytes = round_up(a.rowbuf * 4, 16);
  const int xch_bytes = 128 * 8 + 2 * 128 * 8;  // column-part exchange + double-buffered pair exchange
  const int qsum_bytes = int8 ? round_up(a.Gq * 32 * 4, 16) : 0;
  const int state_per_mb = 128 * 4 * (s.argmax ? 2 : 1);

  const int G_top = gd * nch_max;
  for (int G = G_top; G >= 1; --G) {
    if (gd > 1 && G != G_top) break;  // a document group is always fully resident
    if (a.nk > 1 && G > a.nts) continue;
    if (tune().G > 0 && G != std::min(tune().G, nch_max)) continue;
    const bool multi = G < nch_max;
    // INT8 keeps its read-ahead in the (half-size) uint8 staging ring instead
    const int nd_hi = int8 ? G + 1 : (a.q_resident ? std::max(2 * G, 8) : 2 * G);
    for (int nd = nd_hi; nd >= G; --nd) {
      if (tune().nd > 0 && nd != tune().nd) continue;
      const int nq_hi = a.q_resident ? 1 : 4, nq_lo = a.q_resident ? 1 : 2;
      for (int nq = nq_hi; nq >= nq_lo; --nq) {
        if (tune().nq > 0 && !a.q_resident && nq != tune().nq) continue;
        const int nu_hi = int8 ? 8 : 0, nu_lo = int8 ? 2 : 0;
        for (int nu = nu_hi; nu >= nu_lo; --nu) {
          const int nbars = 2 * nq + 2 * nd + 2 * a.nts + 2 * nu + (int8 ? nd : 0) + 1;
          const int sc_bytes = int8 ? nd * a.C * 8 : 0;
          const int bar_bytes = round_up(nbars * 8 + 16, 16);
          const int base = 1024 + nq * static_cast<int>(a.q_stage_bytes) +
                           nd * static_cast<int>(a.d_slot_bytes) + nu * static_cast<int>(a.u_slot_bytes) +
                           sc_bytes + rows_bytes + xch_bytes + qsum_bytes + bar_bytes;
          if (base > kMaxSmem) continue;
          int state_bytes = 0;
          int RS;
          if (multi && a.rep == 1) {
            const int fit_mb = (kMaxSmem - base) / state_per_mb;
            const int mb = std::min(mb_total, fit_mb);
            if (mb < 1) continue;
            RS = mb * 4;
            state_bytes = mb * state_per_mb;
          } else if (multi) {
            RS = 4;
            state_bytes = state_per_mb;
            if (base + state_bytes > kMaxSmem) continue;
          } else {
            RS = round_up(a.R, 4);
          }
          a.G = G;
          a.nd = nd;
          a.nq = nq;
          a.nu = nu;
          a.RS = RS;
          uint32_t off = 0;
          a.off_q = off;
          off += nq * a.q_stage_bytes;
          a.off_d = off;
          off += nd * a.d_slot_bytes;
          a.off_u = off;
          off += nu * a.u_slot_bytes;
          a.off_sc = off;
          off += sc_bytes;
          a.off_state = off;
          off += state_bytes;
          a.off_rows = off;
          off += rows_bytes;
          a.off_xch = off;
          off += xch_bytes;
          a.off_qsum = off;
          off += qsum_bytes;
          a.off_bar = round_up(off, 16);
          off = a.off_bar + bar_bytes;
          smem_bytes = std::max(static_cast<int>(off) + 1024, kMinSmem);
          return smem_bytes <= kMaxSmem;
        }
      }
    }
  }
  return false;
}

// Documents per work item: each streamed 128-row query block is used for
// every chunk of an item, so short documents are grouped until an item holds
// >= ~512 tokens (below that, delivering query blocks from L2 and the per
// chunk hand-off, not the tensor core, limit the pass).  Falls back to
// smaller groups when a group does not fit in shared memory.
bool make_plan(const Shape& s, FwdArgs& a, int& smem_bytes) {
  int gd = 1;
  if (s.shared && s.mode == MODE_DENSE && s.Nq * cdiv(s.Lq, 32) > 2 && s.d <= 128) {
    const int C0 = s.Ld <= 256 ? round_up(std::max(s.Ld, 16), 16)
                               : round_up(cdiv(s.Ld, cdiv(s.Ld, 256)), 16);
    gd = std::max(1, std::min(kMaxGroupDocs, cdiv(512, cdiv(s.Ld, C0) * C0)));
  }
  if (tune().gd > 0) gd = std::min(tune().gd, kMaxGroupDocs);
  for (; gd >= 1; --gd)
    if (plan_for_gd(s, gd, a, smem_bytes)) return true;
  return false;
}

template <int MODE, bool ARGMAX>
int launch_fwd(const CUtensorMap& tq, const CUtensorMap& tq2, const CUtensorMap& td, const FwdArgs& a,
               int smem, cudaStream_t stream) {
  auto kern = maxsim_fwd_kernel<MODE, ARGMAX>;
  static std::atomic<int> configured_smem{0};
  if (configured_smem.load() < smem) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxSmem) !=
        cudaSuccess)
      return FM_ERR_LAUNCH;
    configured_smem.store(kMaxSmem);
  }
  const int sms = sm_count();
  if (sms <= 0) return FM_ERR_NO_DEVICE;
  const int grid = std::max(1, std::min(a.n_work, sms));
  const int threads = MODE == MODE_INT8 ? kThreadsI8 : kThreadsF16;
  if (a.topk.k > 0 && a.topk.parts != grid) return FM_ERR_ARG;  // set by fwd_common
  kern<<<grid, threads, smem, stream>>>(tq, tq2, td, a);
  return cudaGetLastError() == cudaSuccess ? FM_OK : FM_ERR_LAUNCH;
}

bool q1_ok(const Shape& s);
bool flat_ok(const Shape& s, const int32_t* lengths);
int launch_flat(const Shape& s, const void* Q, const void* D, float* scores, int32_t* status,
                cudaStream_t stream);
int launch_q1(const Shape& s, const void* Q, const void* D, const int32_t* lengths, float* scores,
              const int32_t* sp_idx, int32_t* status, cudaStream_t stream, TopkArgs* topk,
              const int32_t* cu, int64_t T);

// Forward launch for any shape.  `topk` (optional): when the chosen kernel
// selects per-CTA top-k candidates in its tail (one query or shared dense
// documents), topk->parts is set to its grid; otherwise it stays 0.
int fwd_common(const Shape& s, const void* Q, const void* D, const int32_t* lengths, float* scores,
               int32_t* argmax, const int32_t* sp_idx, const void* scales, const void* mins,
               int32_t* status, cudaStream_t stream, TopkArgs* topk = nullptr,
               const int32_t* cu = nullptr, int64_t T = 0) {
  if (!Q || !D || !scores || !status) return FM_ERR_ARG;
  if (s.Nq < 1 || s.B < 0 || s.Lq < 1 || s.Ld < 1 || s.d < 8 || s.d > 2048) return FM_ERR_ARG;
  if (s.d % 8 != 0) return FM_ERR_ARG;
  if (s.mode == MODE_INT8 && s.d % 16 != 0) return FM_ERR_ARG;
  if (!aligned16(Q) || !aligned16(D)) return FM_ERR_ARG;
  if (s.mode == MODE_SPARSE && (s.K < 0 || (s.K > 0 && !sp_idx))) return FM_ERR_ARG;
  if (s.mode == MODE_INT8 && (!scales || !mins)) return FM_ERR_ARG;
  if (s.B == 0) return FM_OK;
  const int64_t n_docs = s.shared ? s.B : static_cast<int64_t>(s.Nq) * s.B;
  if (n_docs > INT32_MAX || static_cast<int64_t>(s.Nq) * s.B > INT32_MAX) return FM_ERR_ARG;

  if (topk) topk->parts = 0;
  if (cu && (s.mode != MODE_DENSE || !s.shared || T < 1 || T >= INT32_MAX)) return FM_ERR_ARG;
  if (q1_ok(s)) return launch_q1(s, Q, D, lengths, scores, sp_idx, status, stream, topk, cu, T);
  if (!topk && !cu && flat_ok(s, lengths)) return launch_flat(s, Q, D, scores, status, stream);

  FwdArgs a{};
  int smem = 0;
  if (!make_plan(s, a, smem)) return FM_ERR_UNSUPPORTED;
  a.lengths = lengths;
  a.cu = cu;
  a.scores = scores;
  a.argmax = argmax;
  a.sp_idx = sp_idx;
  a.q = static_cast<const __half*>(Q);
  a.scales = static_cast<const __half*>(scales);
  a.mins = static_cast<const __half*>(mins);
  a.status = status;
  a.timeout_ns = static_cast<uint64_t>(g_timeout_ns.load());
  a.topk = TopkArgs{0, 0, nullptr, nullptr};
  if (topk && topk->k > 0 && s.mode == MODE_DENSE && !s.argmax && s.shared) {
    const int sms = sm_count();
    if (sms <= 0) return FM_ERR_NO_DEVICE;
    topk->parts = std::max(1, std::min(a.n_work, sms));
    a.topk = *topk;
  }

  CUtensorMap tq, tq2, td;
  const int nq_rows = s.mode == MODE_DENSE ? s.Nq : 1;
  if (!make_map_3d(&tq, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, Q, s.d, s.Lq, nq_rows, 64, 32,
                   CU_TENSOR_MAP_SWIZZLE_128B))
    return FM_ERR_LAUNCH;
  // the same rows as one [Nq * Lq, d] matrix, 128-row boxes
  if (!make_map_3d(&tq2, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, Q, s.d,
                   static_cast<uint64_t>(s.Lq) * nq_rows, 1, 64, 128, CU_TENSOR_MAP_SWIZZLE_128B))
    return FM_ERR_LAUNCH;
  if (s.mode == MODE_INT8) {
    if (!make_map_3d(&td, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, D, s.d, s.Ld, n_docs, 64, a.C,
                     CU_TENSOR_MAP_SWIZZLE_NONE))
      return FM_ERR_LAUNCH;
  } else if (cu) {
    // packed documents: one [T, d] token matrix, rows addressed through cu
    if (!make_map_3d(&td, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, D, s.d, static_cast<uint64_t>(T), 1, 64, a.C,
                     CU_TENSOR_MAP_SWIZZLE_128B))
      return FM_ERR_LAUNCH;
  } else {
    if (!make_map_3d(&td, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, D, s.d, s.Ld, n_docs, 64, a.C,
                     CU_TENSOR_MAP_SWIZZLE_128B))
      return FM_ERR_LAUNCH;
  }
  switch (s.mode) {
    case MODE_DENSE:
      return s.argmax ? launch_fwd<MODE_DENSE, true>(tq, tq2, td, a, smem, stream)
                      : launch_fwd<MODE_DENSE, false>(tq, tq2, td, a, smem, stream);
    case MODE_SPARSE:
      return launch_fwd<MODE_SPARSE, false>(tq, tq2, td, a, smem, stream);
    case MODE_INT8:
      return launch_fwd<MODE_INT8, false>(tq, tq2, td, a, smem, stream);
  }
  return FM_ERR_ARG;
}

// INT8 fast path: uint8 codes straight into kind::i8 MMAs (fm_int8.cuh).
bool int8_fast_ok(int Lq, int d) { return Lq <= 64 && d >= 128 && d <= 256 && d % 16 == 0; }

bool plan_int8_fast(int B, int Lq, int Ld, int d, Int8Args& a, int& smem) {
  a.B = B;
  a.Lq = Lq;
  a.Ld = Ld;
  a.d = d;
  const int gq = cdiv(Lq, 32);
  a.N = 64 * gq;
  a.nts = std::min(16, 512 / (kI8Halves * a.N));  // a slot holds the 128-token halves of a chunk
  if (a.nts % 2) return false;  // the two warps of a lane quarter own alternate slots
  a.atoms = cdiv(d, 128);
  a.u_slot_bytes = a.atoms * kI8Tokens * 128u;
  a.sc_slot_bytes = 2 * round_up(kI8Tokens * 2 + 32, 16);
  const int q_bytes = a.atoms * a.N * 128;
  const int misc = round_up((64 + 64 + kI8Xch * 8 * gq * 32) * 4, 16);
  const int per_slot = static_cast<int>(a.u_slot_bytes + a.sc_slot_bytes) + 16;
  const int fixed = 1024 + round_up(q_bytes, 1024) + misc + (2 * a.nts + 2 + 2 * kI8Xch) * 8 + 32;
  a.nu = std::min(16, (kMaxSmem - fixed) / per_slot);
  if (tune().nd > 0) a.nu = std::min(a.nu, tune().nd);
  a.nu &= ~1;  // even: paired epilogue warps and MMA issuers own alternate slots
  if (a.nu < 2) return false;
  uint32_t off = 0;
  a.off_q = off;
  off += round_up(q_bytes, 1024);
  a.off_u = off;
  off += a.nu * a.u_slot_bytes;
  a.off_sc = off;
  off += a.nu * a.sc_slot_bytes;
  a.off_misc = round_up(off, 16);
  off = a.off_misc + misc;
  a.off_bar = round_up(off, 16);
  off = a.off_bar + (2 * a.nu + 2 * a.nts + 2 + 2 * kI8Xch) * 8 + 32;
  smem = std::max(static_cast<int>(off) + 1024, kMinSmem);
  return smem <= kMaxSmem;
}

template <int GQ, int EW>
int launch_int8_gq(const CUtensorMap& tu, const Int8Args& a, int smem, cudaStream_t stream) {
  static std::atomic<bool> cfg{false};
  if (!cfg.load()) {
    if (cudaFuncSetAttribute(maxsim_int8_kernel<GQ, EW>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             kMaxSmem) != cudaSuccess)
      return FM_ERR_LAUNCH;
    cfg.store(true);
  }
  const int sms = sm_count();
  if (sms <= 0) return FM_ERR_NO_DEVICE;
  maxsim_int8_kernel<GQ, EW><<<std::max(1, std::min(a.B, sms)), i8_threads(EW), smem, stream>>>(tu, a);
  return cudaGetLastError() == cudaSuccess ? FM_OK : FM_ERR_LAUNCH;
}

int launch_int8_fast(const void* Q, const void* Du8, const void* scales, const void* mins,
                     const int32_t* lengths, float* scores, int B, int Lq, int Ld, int d,
                     int32_t* status, cudaStream_t stream) {
  Int8Args a{};
  int smem = 0;
  if (!plan_int8_fast(B, Lq, Ld, d, a, smem)) return FM_ERR_UNSUPPORTED;
  if (!aligned16(scales) || !aligned16(mins)) return FM_ERR_ARG;
  a.lengths = lengths;
  a.scores = scores;
  a.q = static_cast<const __half*>(Q);
  a.scales = static_cast<const __half*>(scales);
  a.mins = static_cast<const __half*>(mins);
  a.status = status;
  a.timeout_ns = static_cast<uint64_t>(g_timeout_ns.load());
  a.sc_total_bytes = static_cast<size_t>(B) * Ld * 2;
  a.dbg = tune().dbg;
  CUtensorMap tu;
  if (!make_map_3d(&tu, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, Du8, d, Ld, B, 128, kI8Tokens,
                   CU_TENSOR_MAP_SWIZZLE_128B))
    return FM_ERR_LAUNCH;
  // 8 epilogue warps for a 32-row query; 4 for 64 rows (register budget)
  return a.N == 64 ? launch_int8_gq<1, 8>(tu, a, smem, stream) : launch_int8_gq<2, 4>(tu, a, smem, stream);
}

// Short-query path (fm_q1.cuh): one query of <= 64 rows and d <= 128 against
// shared documents, the document chunk as the MMA's M operand.
bool q1_ok(const Shape& s) {
  return (s.mode == MODE_DENSE || s.mode == MODE_SPARSE) && !s.argmax && s.Nq == 1 && s.Lq <= 64 &&
         s.d <= 128 && !(tune().dbg & 8);
}

bool plan_q1(const Shape& s, int CT, Q1Args& a, int& smem) {
  a.B = s.B;
  a.Lq = s.Lq;
  a.Ld = s.Ld;
  a.d = s.d;
  a.N = 32 * cdiv(s.Lq, 32);
  a.atoms = cdiv(s.d, 64);
  a.nts = 512 / ((CT / 128) * a.N);
  if (a.nts % 2) return false;  // the two warps of a lane quarter own alternate slots
  a.u_slot_bytes = static_cast<uint32_t>(a.atoms) * CT * 128u;
  const int q_bytes = round_up(a.atoms * a.N * 128, 1024);
  const int ew = 8;
  const int misc = round_up((kQ1Xch * ew * (a.N / 32) * 32) * 4 + 2 * kQ1Xch * 4 + ew * a.N * 4, 16);
  const int fixed = 1024 + q_bytes + misc + (2 * 16 + 2 * a.nts + 2) * 8 + 48;  // bars for up to 16 slots
  a.nu = std::min(16, (kMaxSmem - fixed) / static_cast<int>(a.u_slot_bytes));
  if (tune().nd > 0) a.nu = std::min(a.nu, tune().nd);
  if (a.nu < 2) return false;
  uint32_t off = 0;
  a.off_q = off;
  off += q_bytes;
  a.off_u = off;
  off += a.nu * a.u_slot_bytes;
  a.off_misc = round_up(off, 16);
  off = a.off_misc + misc;
  a.off_bar = round_up(off, 16);
  off = a.off_bar + (2 * a.nu + 2 * a.nts + 2) * 8 + 32;
  smem = std::max(static_cast<int>(off) + 1024, kMinSmem);
  return smem <= kMaxSmem;
}

template <int GQ, int CT>
int launch_q1_t(const CUtensorMap& tq, const CUtensorMap& td, const Q1Args& a, int smem,
                cudaStream_t stream) {
  auto kern = maxsim_q1_kernel<GQ, 8, CT>;
  static std::atomic<bool> cfg{false};
  if (!cfg.load()) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxSmem) != cudaSuccess)
      return FM_ERR_LAUNCH;
    cfg.store(true);
  }
  const int sms = sm_count();
  if (sms <= 0) return FM_ERR_NO_DEVICE;
  cudaLaunchConfig_t cfgl{};
  cfgl.gridDim = dim3(std::max(1, std::min(a.B, sms)));
  cfgl.blockDim = dim3(q1_threads(8));
  cfgl.dynamicSmemBytes = smem;
  cfgl.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfgl.attrs = attr;
  cfgl.numAttrs = (tune().dbg & 128) ? 0 : 1;
  if (cudaLaunchKernelEx(&cfgl, kern, tq, td, a) != cudaSuccess) return FM_ERR_LAUNCH;
  return cudaGetLastError() == cudaSuccess ? FM_OK : FM_ERR_LAUNCH;
}

int launch_q1(const Shape& s, const void* Q, const void* D, const int32_t* lengths, float* scores,
              const int32_t* sp_idx, int32_t* status, cudaStream_t stream, TopkArgs* topk,
              const int32_t* cu, int64_t T) {
  const int CT = tune().C == 256 ? 256 : 128;
  Q1Args a{};
  int smem = 0;
  if (!plan_q1(s, CT, a, smem)) return FM_ERR_UNSUPPORTED;
  a.lengths = lengths;
  a.cu = cu;
  a.scores = scores;
  a.status = status;
  a.timeout_ns = static_cast<uint64_t>(g_timeout_ns.load());
  a.dbg = tune().dbg;
  a.sparse = s.mode == MODE_SPARSE ? 1 : 0;
  a.sp_idx = sp_idx;
  a.K = s.mode == MODE_SPARSE ? s.K : 0;
  a.topk = TopkArgs{0, 0, nullptr, nullptr};
  if (topk && topk->k > 0) {
    const int sms = sm_count();
    if (sms <= 0) return FM_ERR_NO_DEVICE;
    topk->parts = std::max(1, std::min(a.B, sms));  // the grid of launch_q1_t
    a.topk = *topk;
  }
  CUtensorMap tq, td;
  if (!make_map_3d(&tq, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, Q, s.d, s.Lq, 1, 64, a.N,
                   CU_TENSOR_MAP_SWIZZLE_128B))
    return FM_ERR_LAUNCH;
  if (!(cu ? make_map_3d(&td, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, D, s.d, static_cast<uint64_t>(T), 1, 64, CT,
                         CU_TENSOR_MAP_SWIZZLE_128B)
           : make_map_3d(&td, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, D, s.d, s.Ld, s.B, 64, CT,
                         CU_TENSOR_MAP_SWIZZLE_128B)))
    return FM_ERR_LAUNCH;
  if (a.N == 32)
    return CT == 256 ? launch_q1_t<1, 256>(tq, td, a, smem, stream) : launch_q1_t<1, 128>(tq, td, a, smem, stream);
  return CT == 256 ? launch_q1_t<2, 256>(tq, td, a, smem, stream) : launch_q1_t<2, 128>(tq, td, a, smem, stream);
}

// Flat-token path (fm_flat.cuh): shared documents of one length (no lengths
// array, Ld >= 128), whole 32-row query row groups, >= 128 query rows, d <= 128.
bool flat_ok(const Shape& s, const int32_t* lengths) {
  if (s.mode != MODE_DENSE || s.argmax || !s.shared || lengths != nullptr) return false;
  if (s.Lq % 32 != 0 || s.Nq * s.Lq < 128 || s.d > 128 || s.Lq / 32 > 4 * kFlatMaxJb) return false;
  // measured slower than the per-document kernel on B200 so far (the epilogue
  // cannot drain a 192-column chunk within one chunk's MMA time): opt-in only
  if (s.Ld < 128 || !(tune().flat || g_flat_kernel.load())) return false;
  return static_cast<int64_t>(s.B) * s.Ld + 2 * kFlatCT < (static_cast<int64_t>(1) << 31);
}

bool plan_flat(const Shape& s, FlatArgs& a, int& smem) {
  a.B = s.B;
  a.Ld = s.Ld;
  a.Nq = s.Nq;
  a.Lq = s.Lq;
  a.d = s.d;
  a.atoms = cdiv(s.d, 64);
  a.nd = 3;
  a.Gq = s.Lq / 32;
  a.R = s.Nq * a.Gq;
  a.span_rg = a.R <= 4 * kFlatMaxJb ? a.R : (4 * kFlatMaxJb / a.Gq) * a.Gq;
  a.d_slot_bytes = static_cast<uint32_t>(a.atoms) * kFlatCT * 128u;
  uint32_t off = 0;
  a.off_q = off;
  off += 2 * 32768u;
  a.off_d = off;
  off += a.nd * a.d_slot_bytes;
  a.off_rows = off;
  off += 2 * kFlatDocSlots * 128 * 4;
  a.off_xch = off;
  off += kFlatXch * 4 * kFlatSeg * 32 * 4;
  a.off_bar = off;
  off += (2 * a.nd + 4 + 2 * kFlatTS + 4 * kFlatXch + 3) * 8 + 16;
  smem = std::max(static_cast<int>(off) + 1024, kMinSmem);
  return smem <= kMaxSmem;
}

int launch_flat(const Shape& s, const void* Q, const void* D, float* scores, int32_t* status,
                cudaStream_t stream) {
  FlatArgs a{};
  int smem = 0;
  if (!plan_flat(s, a, smem)) return FM_ERR_UNSUPPORTED;
  a.scores = scores;
  a.status = status;
  a.timeout_ns = static_cast<uint64_t>(g_timeout_ns.load());
  a.dbg = tune().dbg;
  CUtensorMap tq, td;
  if (!make_map_3d(&tq, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, Q, s.d, static_cast<uint64_t>(s.Nq) * s.Lq, 1, 64,
                   128, CU_TENSOR_MAP_SWIZZLE_128B))
    return FM_ERR_LAUNCH;
  if (!make_map_3d(&td, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, D, s.d, static_cast<uint64_t>(s.B) * s.Ld, 1, 64,
                   kFlatCT, CU_TENSOR_MAP_SWIZZLE_128B))
    return FM_ERR_LAUNCH;
  static std::atomic<bool> cfg{false};
  if (!cfg.load()) {
    if (cudaFuncSetAttribute(maxsim_flat_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxSmem) !=
        cudaSuccess)
      return FM_ERR_LAUNCH;
    cfg.store(true);
  }
  const int sms = sm_count();
  if (sms <= 0) return FM_ERR_NO_DEVICE;
  cudaLaunchConfig_t cfgl{};
  cfgl.gridDim = dim3(std::max(1, std::min(s.B, sms)));
  cfgl.blockDim = dim3(kFlatThreads);
  cfgl.dynamicSmemBytes = smem;
  cfgl.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfgl.attrs = attr;
  cfgl.numAttrs = (tune().dbg & 128) ? 0 : 1;
  if (cudaLaunchKernelEx(&cfgl, maxsim_flat_kernel, tq, td, a) != cudaSuccess) return FM_ERR_LAUNCH;
  return cudaGetLastError() == cudaSuccess ? FM_OK : FM_ERR_LAUNCH;
}

// FP8 path (fm_fp8.cuh): one query of <= 64 rows, e4m3 documents, d <= 256.
// nh: 128-token halves per chunk (2 for one 32-row query, whose TMEM slots of
// 2 x 96 columns still come in an even number; 1 for 64-row queries).
bool plan_fp8(int B, int Lq, int Ld, int d, int nh, Fp8Args& a, int& smem) {
  a.B = B;
  a.Lq = Lq;
  a.Ld = Ld;
  a.d = d;
  const int gq = cdiv(Lq, 32);
  a.N = kF8Parts * 32 * gq;
  a.nts = (512 / (nh * a.N)) & ~1;  // even: the two warps of a lane quarter own alternate slots
  if (a.nts < 2) return false;
  a.atoms = cdiv(d, 128);
  a.u_slot_bytes = a.atoms * nh * kF8Half * 128u;
  const int q_bytes = round_up(a.atoms * a.N * 128, 1024);
  const int misc = round_up((64 + kF8Xch * kF8EW * gq * 32) * 4 + 2 * kF8Xch * 4, 16);
  const int fixed = 1024 + q_bytes + misc + (2 * 16 + 2 * a.nts + 2) * 8 + 32;
  a.nu = std::min(16, (kMaxSmem - fixed) / static_cast<int>(a.u_slot_bytes));
  if (a.nu < 2) return false;
  uint32_t off = 0;
  a.off_q = off;
  off += q_bytes;
  a.off_u = off;
  off += a.nu * a.u_slot_bytes;
  a.off_misc = round_up(off, 16);
  off = a.off_misc + misc;
  a.off_bar = round_up(off, 16);
  off = a.off_bar + (2 * a.nu + 2 * a.nts + 2) * 8 + 32;
  smem = std::max(static_cast<int>(off) + 1024, kMinSmem);
  return smem <= kMaxSmem;
}

template <int GQ, int NH>
int launch_fp8_gq(const CUtensorMap& tu, const Fp8Args& a, int smem, cudaStream_t stream) {
  static std::atomic<bool> cfg{false};
  if (!cfg.load()) {
    if (cudaFuncSetAttribute(maxsim_fp8_kernel<GQ, NH>, cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxSmem) !=
        cudaSuccess)
      return FM_ERR_LAUNCH;
    cfg.store(true);
  }
  const int sms = sm_count();
  if (sms <= 0) return FM_ERR_NO_DEVICE;
  maxsim_fp8_kernel<GQ, NH><<<std::max(1, std::min(a.B, sms)), f8_threads(), smem, stream>>>(tu, a);
  return cudaGetLastError() == cudaSuccess ? FM_OK : FM_ERR_LAUNCH;
}

int launch_fp8(const void* Q, const void* D8, const float* scales, const int32_t* lengths, float* scores, int B,
               int Lq, int Ld, int d, int32_t* status, cudaStream_t stream, TopkArgs* topk) {
  Fp8Args a{};
  int smem = 0;
  const int nh = Lq <= 32 ? 2 : 1;
  if (!plan_fp8(B, Lq, Ld, d, nh, a, smem)) return FM_ERR_UNSUPPORTED;
  if ((reinterpret_cast<uintptr_t>(scales) & 3u) != 0) return FM_ERR_ARG;
  a.lengths = lengths;
  a.scores = scores;
  a.q = static_cast<const __half*>(Q);
  a.scales = scales;
  a.status = status;
  a.timeout_ns = static_cast<uint64_t>(g_timeout_ns.load());
  a.topk = TopkArgs{0, 0, nullptr, nullptr};
  if (topk && topk->k > 0) {
    const int sms = sm_count();
    if (sms <= 0) return FM_ERR_NO_DEVICE;
    topk->parts = std::max(1, std::min(B, sms));
    a.topk = *topk;
  }
  CUtensorMap tu;
  if (!make_map_3d(&tu, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, D8, d, Ld, B, 128, nh * kF8Half,
                   CU_TENSOR_MAP_SWIZZLE_128B))
    return FM_ERR_LAUNCH;
  return a.N == 96 ? launch_fp8_gq<1, 2>(tu, a, smem, stream) : launch_fp8_gq<2, 1>(tu, a, smem, stream);
}

}  // namespace
}  // namespace fm

using namespace fm;

extern "C" {

int fm_abi_version(void) { return 100; }

const char* fm_status_string(int code) {
  switch (code) {
    case FM_OK: return "ok";
    case FM_ERR_ARG: return "invalid argument";
    case FM_ERR_LAUNCH: return "kernel launch or TMA descriptor error";
    case FM_ERR_TIMEOUT_DFULL: return "device wait timed out: document tile never arrived";
    case FM_ERR_TIMEOUT_DEMPTY: return "device wait timed out: document slot never released";
    case FM_ERR_TIMEOUT_QFULL: return "device wait timed out: query block never arrived";
    case FM_ERR_TIMEOUT_QEMPTY: return "device wait timed out: query stage never released";
    case FM_ERR_TIMEOUT_TFULL: return "device wait timed out: accumulator never committed";
    case FM_ERR_TIMEOUT_TEMPTY: return "device wait timed out: accumulator never drained";
    case FM_ERR_TIMEOUT_UFULL: return "device wait timed out: uint8 tile never arrived";
    case FM_ERR_TIMEOUT_UEMPTY: return "device wait timed out: uint8 slot never released";
    case FM_ERR_TIMEOUT_DRAIN: return "device wait timed out while draining in-flight copies";
    case FM_ERR_TIMEOUT_SELFTEST: return "device wait timed out (self test)";
    case FM_ERR_BAD_INDEX: return "sparse query index out of range";
    case FM_ERR_UNSUPPORTED: return "shape not supported by the sm_100a kernels";
    case FM_ERR_NO_DEVICE: return "no CUDA device";
    case FM_ERR_SCRATCH_TOO_SMALL:
      return "shape needs more dQ workspace than the 16 MiB built-in scratch of fm_maxsim_bwd_noalloc "
             "(two document ranges of Nq * Lq * d fp32 partial sums must fit)";
  }
  return "unknown status";
}

void fm_set_wait_timeout_ns(int64_t ns) { g_timeout_ns.store(ns > 0 ? ns : 2000000000LL); }

int fm_set_option(int option, int value) {
  switch (option) {
    case FM_OPT_FLAT_KERNEL: g_flat_kernel.store(value ? 1 : 0); return FM_OK;
  }
  return FM_ERR_ARG;
}

int fm_fwd_plan_info(int mode, int argmax, int Nq, int B, int Lq, int Ld, int d, int shared_docs,
                     int K, int32_t* out, int n_out) {
  if (!out || n_out < 16 || mode < 0 || mode > 2) return FM_ERR_ARG;
  if (Nq < 1 || B < 0 || Lq < 1 || Ld < 1 || d < 8 || d > 2048) return FM_ERR_ARG;
  Shape s{mode, argmax != 0, Nq, B, Lq, Ld, d, K, shared_docs ? 1 : 0};
  FwdArgs a{};
  int smem = 0;
  if (!make_plan(s, a, smem)) return FM_ERR_UNSUPPORTED;
  const int32_t v[16] = {a.C, a.G, a.nd, a.nq, a.nu, a.nk, a.kq_atoms, a.d_atoms, a.RS, a.rep,
                         a.q_resident, a.nts, a.ts_stride, smem, a.R, a.gd};
  for (int i = 0; i < 16; ++i) out[i] = v[i];
  return FM_OK;
}

int fm_maxsim_fwd(const uint16_t* Q, const uint16_t* D, const int32_t* doc_lengths, float* scores,
                  int32_t* argmax, int Nq, int B, int Lq, int Ld, int d, int shared_docs,
                  int32_t* status, void* stream) {
  Shape s{MODE_DENSE, argmax != nullptr, Nq, B, Lq, Ld, d, 0, shared_docs ? 1 : 0};
  return fwd_common(s, Q, D, doc_lengths, scores, argmax, nullptr, nullptr, nullptr, status,
                    static_cast<cudaStream_t>(stream));
}

int fm_maxsim_packed_fwd(const uint16_t* Q, const uint16_t* D_tokens, const int32_t* cu_seqlens,
                         float* scores, int32_t* argmax, int Nq, int B, int Lq, int max_len, int d,
                         int64_t total_tokens, int32_t* status, void* stream) {
  if (!cu_seqlens) return FM_ERR_ARG;
  Shape s{MODE_DENSE, argmax != nullptr, Nq, B, Lq, max_len, d, 0, 1};
  return fwd_common(s, Q, D_tokens, nullptr, scores, argmax, nullptr, nullptr, nullptr, status,
                    static_cast<cudaStream_t>(stream), nullptr, cu_seqlens, total_tokens);
}

int fm_maxsim_int8_fwd(const uint16_t* Q, const uint8_t* D_u8, const uint16_t* scales,
                       const uint16_t* mins, const int32_t* doc_lengths, float* scores, int B,
                       int Lq, int Ld, int d, int32_t* status, void* stream) {
  if (int8_fast_ok(Lq, d) && tune().dbg != 8) {
    if (!Q || !D_u8 || !scales || !mins || !scores || !status || B < 0 || Ld < 1 || Lq < 1)
      return FM_ERR_ARG;
    if (!aligned16(Q) || !aligned16(D_u8)) return FM_ERR_ARG;
    if (B == 0) return FM_OK;
    return launch_int8_fast(Q, D_u8, scales, mins, doc_lengths, scores, B, Lq, Ld, d, status,
                            static_cast<cudaStream_t>(stream));
  }
  Shape s{MODE_INT8, false, 1, B, Lq, Ld, d, 0, 1};
  return fwd_common(s, Q, D_u8, doc_lengths, scores, nullptr, nullptr, scales, mins, status,
                    static_cast<cudaStream_t>(stream));
}

int fm_maxsim_sparse_fwd(const uint16_t* Q, const uint16_t* D, const int32_t* indices,
                         const int32_t* doc_lengths, float* scores, int B, int K, int Lq, int Ld,
                         int d, int32_t* status, void* stream) {
  Shape s{MODE_SPARSE, false, 1, B, Lq, Ld, d, K, 1};
  return fwd_common(s, Q, D, doc_lengths, scores, nullptr, indices, nullptr, nullptr, status,
                    static_cast<cudaStream_t>(stream));
}

}  // extern "C"

namespace fm {
namespace {
bool topk_smem_ready() {
  static std::once_flag once;
  static bool ok = false;
  std::call_once(once, [] {
    const int bytes = (kTopkThreads / 32 + 1) * kTopkMaxK * 8;
    ok = cudaFuncSetAttribute(topk_partial_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) ==
             cudaSuccess &&
         cudaFuncSetAttribute(topk_merge_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) ==
             cudaSuccess;
  });
  return ok;
}

// Candidate workspace: Nq x parts x k (score, id) pairs, parts <= SM count.
int64_t topk_ws_bytes(int Nq, int k) {
  const int sms = sm_count();
  if (sms <= 0) return -1;
  return static_cast<int64_t>(Nq) * sms * k * 8;
}

// Stage 1 over a score matrix (parts = min(B, SMs)) unless `parts_done`
// candidates already exist, then stage 2.
int topk_finish(const float* scores, int Nq, int B, int k, TopkArgs t, int parts_done, float* top_s,
                int64_t* top_i, int64_t id_offset, cudaStream_t st) {
  if (!topk_smem_ready()) return FM_ERR_LAUNCH;
  const int W = kTopkThreads / 32;
  if (parts_done == 0) {
    const int sms = sm_count();
    if (sms <= 0) return FM_ERR_NO_DEVICE;
    t.parts = std::max(1, std::min(B, sms));
    topk_partial_kernel<<<dim3(Nq, t.parts), kTopkThreads, W * k * 8, st>>>(scores, B, t);
    if (cudaGetLastError() != cudaSuccess) return FM_ERR_LAUNCH;
  } else {
    t.parts = parts_done;
  }
  // programmatic dependent launch: the merge kernel's launch overlaps the
  // tail of the kernel that wrote the candidates; it reads them only after
  // griddepcontrol.wait (that kernel complete, its writes visible)
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(Nq);
  cfg.blockDim = dim3(kTopkThreads);
  cfg.dynamicSmemBytes = (W + 1) * k * 8;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (cudaLaunchKernelEx(&cfg, topk_merge_kernel, t, top_s, top_i, id_offset) != cudaSuccess) return FM_ERR_LAUNCH;
  return cudaGetLastError() == cudaSuccess ? FM_OK : FM_ERR_LAUNCH;
}

bool topk_ws_ok(int Nq, int k, const void* ws, int64_t ws_bytes) {
  const int64_t need = topk_ws_bytes(Nq, k);
  return need > 0 && ws && ws_bytes >= need && aligned16(ws);
}

// Document ranges of the dQ pass: enough CTAs to fill the GPU (>= 2 per SM),
// ranges whose documents fit comfortably in L2 (<= 64 MB), >= 8 docs each.
int dq_splits(int Nq, int B, int Lq, int Ld, int d) {
  const int tiles = cdiv(Nq * Lq, 8);
  const int64_t doc_bytes = static_cast<int64_t>(Ld) * d * 2;
  int ns = std::max(cdiv(296, tiles), static_cast<int>((doc_bytes * B + (64ll << 20) - 1) / (64ll << 20)));
  ns = std::min(ns, std::max(1, B / 8));
  return std::max(1, ns);
}
}  // namespace
}  // namespace fm

extern "C" {

int fm_maxsim_fp8_fwd(const uint16_t* Q, const uint8_t* D_fp8, const float* scales, const int32_t* doc_lengths,
                      float* scores, int B, int Lq, int Ld, int d, int32_t* status, void* stream) {
  if (!Q || !D_fp8 || !scales || !scores || !status || B < 0 || Lq < 1 || Lq > 64 || Ld < 1 || d < 16 ||
      d > 256 || d % 16 != 0)
    return FM_ERR_ARG;
  if (!aligned16(Q) || !aligned16(D_fp8)) return FM_ERR_ARG;
  if (B == 0) return FM_OK;
  return launch_fp8(Q, D_fp8, scales, doc_lengths, scores, B, Lq, Ld, d, status, static_cast<cudaStream_t>(stream),
                    nullptr);
}

int64_t fm_topk_workspace_size(int Nq, int k) {
  if (Nq < 1 || k < 1 || k > kTopkMaxK) return 0;
  const int64_t b = topk_ws_bytes(Nq, k);
  return b > 0 ? b : 0;
}

int fm_maxsim_topk(const uint16_t* Q, const uint16_t* D, const int32_t* doc_lengths, float* scores, int k,
                   float* top_scores, int64_t* top_idx, int Nq, int B, int Lq, int Ld, int d,
                   void* workspace, int64_t workspace_bytes, int32_t* status, void* stream) {
  if (!top_scores || !top_idx || k < 1 || k > kTopkMaxK || B < 1 || k > B || Nq < 1) return FM_ERR_ARG;
  if (!topk_ws_ok(Nq, k, workspace, workspace_bytes)) return FM_ERR_ARG;
  const int64_t cand = static_cast<int64_t>(Nq) * sm_count() * k;
  TopkArgs t{k, 0, static_cast<float*>(workspace), reinterpret_cast<int32_t*>(static_cast<float*>(workspace) + cand)};
  Shape s{MODE_DENSE, false, Nq, B, Lq, Ld, d, 0, 1};
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int rc = fwd_common(s, Q, D, doc_lengths, scores, nullptr, nullptr, nullptr, nullptr, status, st, &t);
  if (rc != FM_OK) return rc;
  return topk_finish(scores, Nq, B, k, t, t.parts, top_scores, top_idx, 0, st);
}

int fm_topk_select(const float* scores, int Nq, int B, int k, int64_t id_offset, float* top_scores,
                   int64_t* top_idx, void* workspace, int64_t workspace_bytes, void* stream) {
  if (!scores || !top_scores || !top_idx || Nq < 1 || B < 1 || k < 1 || k > kTopkMaxK || k > B)
    return FM_ERR_ARG;
  if (!topk_ws_ok(Nq, k, workspace, workspace_bytes)) return FM_ERR_ARG;
  const int64_t cand = static_cast<int64_t>(Nq) * sm_count() * k;
  TopkArgs t{k, 0, static_cast<float*>(workspace), reinterpret_cast<int32_t*>(static_cast<float*>(workspace) + cand)};
  return topk_finish(scores, Nq, B, k, t, 0, top_scores, top_idx, id_offset, static_cast<cudaStream_t>(stream));
}

int fm_topk_merge(const float* cand_scores, const int32_t* cand_ids, int Nq, int parts, int k,
                  float* top_scores, int64_t* top_idx, void* stream) {
  if (!cand_scores || !cand_ids || !top_scores || !top_idx || Nq < 1 || parts < 1 || k < 1 || k > kTopkMaxK)
    return FM_ERR_ARG;
  TopkArgs t{k, parts, const_cast<float*>(cand_scores), const_cast<int32_t*>(cand_ids)};
  return topk_finish(nullptr, Nq, 0, k, t, parts, top_scores, top_idx, 0, static_cast<cudaStream_t>(stream));
}

int64_t fm_maxsim_bwd_workspace_size(int Nq, int B, int Lq, int Ld, int d) {
  if (Nq < 1 || B < 1 || Lq < 1 || Ld < 1 || d < 8) return 0;
  const int ns = dq_splits(Nq, B, Lq, Ld, d);
  return ns > 1 ? static_cast<int64_t>(ns) * Nq * Lq * d * 4 : 0;
}

}  // extern "C"

namespace fm {
namespace {
// The backward with `ns` document ranges for dQ (ns > 1 needs a workspace of
// ns * Nq * Lq * d fp32 values; ns == 1 writes dQ directly).
int bwd_impl(const uint16_t* Q, const uint16_t* D, const int32_t* argmax, const float* grad_scores,
             uint16_t* grad_Q, uint16_t* grad_D, int Nq, int B, int Lq, int Ld, int d, int ns,
             void* workspace, int64_t workspace_bytes, cudaStream_t st) {
  if (!Q || !D || !argmax || !grad_scores || !grad_Q || !grad_D) return FM_ERR_ARG;
  if (Nq < 1 || B < 0 || Lq < 1 || Ld < 1 || d < 8 || d > 2048 || d % 8 != 0) return FM_ERR_ARG;
  if (!aligned16(Q) || !aligned16(D) || !aligned16(grad_Q) || !aligned16(grad_D)) return FM_ERR_ARG;
  const int64_t E = static_cast<int64_t>(Nq) * Lq;
  if (E > 32768) return FM_ERR_UNSUPPORTED;
  const size_t smem = (static_cast<size_t>(Ld) + 1 + E) * 4 + static_cast<size_t>(Nq) * 4;
  if (smem > static_cast<size_t>(kMaxSmem)) return FM_ERR_UNSUPPORTED;
  if (B == 0) {
    // no documents: dQ is zero
    return cudaMemsetAsync(grad_Q, 0, E * d * 2, st) == cudaSuccess ? FM_OK : FM_ERR_LAUNCH;
  }
  ns = std::max(1, std::min(ns, B));
  const int64_t need = ns > 1 ? static_cast<int64_t>(ns) * E * d * 4 : 0;
  if (need > 0 && (!workspace || workspace_bytes < need || !aligned16(workspace))) return FM_ERR_ARG;
  const int per = cdiv(B, ns);
  dim3 gq(cdiv(static_cast<int>(E), 8), ns);
  const __half* Dh = reinterpret_cast<const __half*>(D);
  __half* dQh = reinterpret_cast<__half*>(grad_Q);
  float* ws = static_cast<float*>(workspace);
  if (!(tune().dbg & 32)) {
    const int nseg = cdiv(d, 256);
    if (nseg == 1)
      maxsim_bwd_dq_kernel<1><<<gq, kBwdThreads, 0, st>>>(Dh, argmax, grad_scores, dQh, ws, Nq, B, Lq, Ld, d, per);
    else if (nseg == 2)
      maxsim_bwd_dq_kernel<2><<<gq, kBwdThreads, 0, st>>>(Dh, argmax, grad_scores, dQh, ws, Nq, B, Lq, Ld, d, per);
    else if (nseg <= 4)
      maxsim_bwd_dq_kernel<4><<<gq, kBwdThreads, 0, st>>>(Dh, argmax, grad_scores, dQh, ws, Nq, B, Lq, Ld, d, per);
    else
      maxsim_bwd_dq_kernel<8><<<gq, kBwdThreads, 0, st>>>(Dh, argmax, grad_scores, dQh, ws, Nq, B, Lq, Ld, d, per);
    if (cudaGetLastError() != cudaSuccess) return FM_ERR_LAUNCH;
    if (ns > 1) {
      const int64_t n8 = E * d / 8;
      maxsim_bwd_dq_reduce<<<static_cast<unsigned>((n8 + 255) / 256), 256, 0, st>>>(ws, dQh, n8, ns);
      if (cudaGetLastError() != cudaSuccess) return FM_ERR_LAUNCH;
    }
  }
  static std::atomic<bool> dd_cfg{false};
  if (!dd_cfg.load()) {
    if (cudaFuncSetAttribute(maxsim_bwd_dd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             kMaxSmem) != cudaSuccess ||
        cudaFuncSetAttribute(maxsim_bwd_dd2_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             kMaxSmem) != cudaSuccess)
      return FM_ERR_LAUNCH;
    dd_cfg.store(true);
  }
  // every warp sorts and scatters (per-warp counts) when they fit in shared
  // memory; otherwise the single-sorter kernel (same summation order)
  const size_t smem2 = dd2_smem_bytes(Nq, Lq, Ld);
  if (!(tune().dbg & 16)) {
    if (smem2 <= static_cast<size_t>(kMaxSmem))
      maxsim_bwd_dd2_kernel<<<B, kBwdThreads, smem2, st>>>(
          reinterpret_cast<const __half*>(Q), argmax, grad_scores, reinterpret_cast<__half*>(grad_D), Nq, B, Lq,
          Ld, d);
    else
      maxsim_bwd_dd_kernel<<<B, kBwdThreads, smem, st>>>(
          reinterpret_cast<const __half*>(Q), argmax, grad_scores, reinterpret_cast<__half*>(grad_D), Nq, B, Lq,
          Ld, d);
  }
  return cudaGetLastError() == cudaSuccess ? FM_OK : FM_ERR_LAUNCH;
}

using CtxGetCurrentFn = CUresult (*)(CUcontext*);
CtxGetCurrentFn ctx_get_current_fn() {
  static CtxGetCurrentFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<CtxGetCurrentFn>(p);
  });
  return fn;
}
}  // namespace
}  // namespace fm

extern "C" {

int fm_maxsim_bwd(const uint16_t* Q, const uint16_t* D, const int32_t* argmax,
                  const float* grad_scores, uint16_t* grad_Q, uint16_t* grad_D, int Nq, int B,
                  int Lq, int Ld, int d, void* workspace, int64_t workspace_bytes, void* stream) {
  const int ns = (Nq >= 1 && B >= 1 && Lq >= 1 && Ld >= 1 && d >= 8) ? dq_splits(Nq, B, Lq, Ld, d) : 1;
  return bwd_impl(Q, D, argmax, grad_scores, grad_Q, grad_D, Nq, B, Lq, Ld, d, ns, workspace,
                  workspace_bytes, static_cast<cudaStream_t>(stream));
}

int fm_maxsim_bwd_noalloc(const uint16_t* Q, const uint16_t* D, const int32_t* argmax,
                          const float* grad_scores, uint16_t* grad_Q, uint16_t* grad_D, int Nq,
                          int B, int Lq, int Ld, int d, void* stream) {
  if (Nq < 1 || B < 0 || Lq < 1 || Ld < 1 || d < 8) return FM_ERR_ARG;
  // Fewer dQ document ranges than fm_maxsim_bwd would use when the usual count
  // does not fit the scratch (ranges are still added in order, so the result
  // is deterministic; with one range dQ is written directly, no scratch).
  // The size limit is checked before any pointer is looked at.
  // Shapes whose partial sums do not fit twice are refused: a single range
  // would run every document through one CTA per row tile.
  const int64_t per_range = static_cast<int64_t>(Nq) * Lq * d * 4;
  int ns = B >= 1 ? dq_splits(Nq, B, Lq, Ld, d) : 1;
  if (ns > 1 && static_cast<int64_t>(ns) * per_range > static_cast<int64_t>(kNoAllocScratchBytes)) {
    if (2 * per_range > static_cast<int64_t>(kNoAllocScratchBytes)) return FM_ERR_SCRATCH_TOO_SMALL;
    ns = static_cast<int>(static_cast<int64_t>(kNoAllocScratchBytes) / per_range);
  }
  void* scratch = nullptr;
  if (ns > 1) {
    // Device address of the built-in scratch for the current device, looked up
    // with that device current and cached together with its CUDA context (a
    // new context, e.g. after cudaDeviceReset, reloads the module and moves
    // the array, so the address is looked up again).
    static std::mutex mu;
    static void* addr[64] = {nullptr};
    static CUcontext ctx_of[64] = {nullptr};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return FM_ERR_NO_DEVICE;
    auto get_ctx = ctx_get_current_fn();
    if (!get_ctx) return FM_ERR_LAUNCH;
    CUcontext ctx = nullptr;
    std::lock_guard<std::mutex> lock(mu);
    if (get_ctx(&ctx) != CUDA_SUCCESS) return FM_ERR_LAUNCH;
    if (!addr[dev] || !ctx || ctx_of[dev] != ctx) {
      // the lookup itself makes the device's primary context current if needed
      void* p = nullptr;
      if (cudaGetSymbolAddress(&p, g_fm_noalloc_scratch) != cudaSuccess || !p) return FM_ERR_LAUNCH;
      if (get_ctx(&ctx) != CUDA_SUCCESS || !ctx) return FM_ERR_LAUNCH;
      addr[dev] = p;
      ctx_of[dev] = ctx;
    }
    scratch = addr[dev];
  }
  return bwd_impl(Q, D, argmax, grad_scores, grad_Q, grad_D, Nq, B, Lq, Ld, d, ns, scratch,
                  static_cast<int64_t>(kNoAllocScratchBytes), static_cast<cudaStream_t>(stream));
}

}  // extern "C"

namespace fm {
namespace {
template <bool NORM>
int quantize_int8_impl(const void* D, int dtype, uint8_t* D_u8, uint16_t* scales, uint16_t* mins, int64_t rows,
                       int d, void* stream) {
  if (!D || !D_u8 || !scales || !mins || rows < 0 || d < 8 || d > 2048 || d % 8 != 0)
    return FM_ERR_ARG;
  if (!aligned16(D) || (reinterpret_cast<uintptr_t>(D_u8) & 7u)) return FM_ERR_ARG;
  if (rows == 0) return FM_OK;
  // lanes per row: 8 elements each, a power of two, up to a warp; rows that
  // fit one segment are handled 4 row sets per warp
  const int lpr = d <= 64 ? 8 : (d <= 128 ? 16 : 32);
  const int nr = d <= 256 ? 4 : 1;
  const int64_t rows_per_block = 8 * (32 / lpr) * nr;
  const int64_t blocks = (rows + rows_per_block - 1) / rows_per_block;
  if (blocks > INT32_MAX) return FM_ERR_ARG;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const unsigned nb = static_cast<unsigned>(blocks);
  __half* sc = reinterpret_cast<__half*>(scales);
  __half* mn = reinterpret_cast<__half*>(mins);
  auto launch = [&](auto tag) {
    using T = decltype(tag);
    const T* src = static_cast<const T*>(D);
    if (lpr == 8) quantize_int8_kernel<T, 8, 4, NORM><<<nb, 256, 0, st>>>(src, D_u8, sc, mn, rows, d);
    else if (lpr == 16) quantize_int8_kernel<T, 16, 4, NORM><<<nb, 256, 0, st>>>(src, D_u8, sc, mn, rows, d);
    else if (nr == 4) quantize_int8_kernel<T, 32, 4, NORM><<<nb, 256, 0, st>>>(src, D_u8, sc, mn, rows, d);
    else quantize_int8_kernel<T, 32, 1, NORM><<<nb, 256, 0, st>>>(src, D_u8, sc, mn, rows, d);
  };
  switch (dtype) {
    case FM_DTYPE_F16: launch(__half{}); break;
    case FM_DTYPE_F32: launch(float{}); break;
    case FM_DTYPE_BF16: launch(__nv_bfloat16{}); break;
    default:
      return FM_ERR_ARG;
  }
  return cudaGetLastError() == cudaSuccess ? FM_OK : FM_ERR_LAUNCH;
}

template <bool NORM>
int quantize_fp8_impl(const void* D, int dtype, uint8_t* D_fp8, float* scales, int64_t rows, int d, void* stream) {
  if (!D || !D_fp8 || !scales || rows < 0 || d < 8 || d > 2048 || d % 8 != 0) return FM_ERR_ARG;
  if (!aligned16(D) || (reinterpret_cast<uintptr_t>(D_fp8) & 7u)) return FM_ERR_ARG;
  if (rows == 0) return FM_OK;
  const int lpr = d <= 64 ? 8 : (d <= 128 ? 16 : 32);
  const int64_t rows_per_block = 8 * (32 / lpr);
  const int64_t blocks = (rows + rows_per_block - 1) / rows_per_block;
  if (blocks > INT32_MAX) return FM_ERR_ARG;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const unsigned nb = static_cast<unsigned>(blocks);
  auto launch = [&](auto tag) {
    using T = decltype(tag);
    const T* src = static_cast<const T*>(D);
    if (lpr == 8) quantize_fp8_kernel<T, 8, NORM><<<nb, 256, 0, st>>>(src, D_fp8, scales, rows, d);
    else if (lpr == 16) quantize_fp8_kernel<T, 16, NORM><<<nb, 256, 0, st>>>(src, D_fp8, scales, rows, d);
    else quantize_fp8_kernel<T, 32, NORM><<<nb, 256, 0, st>>>(src, D_fp8, scales, rows, d);
  };
  switch (dtype) {
    case FM_DTYPE_F16: launch(__half{}); break;
    case FM_DTYPE_F32: launch(float{}); break;
    case FM_DTYPE_BF16: launch(__nv_bfloat16{}); break;
    default:
      return FM_ERR_ARG;
  }
  return cudaGetLastError() == cudaSuccess ? FM_OK : FM_ERR_LAUNCH;
}
}  // namespace
}  // namespace fm

extern "C" {

int fm_quantize_int8(const void* D, int dtype, uint8_t* D_u8, uint16_t* scales, uint16_t* mins, int64_t rows,
                     int d, void* stream) {
  return quantize_int8_impl<false>(D, dtype, D_u8, scales, mins, rows, d, stream);
}

int fm_normalize_quantize_int8(const void* D, int dtype, uint8_t* D_u8, uint16_t* scales, uint16_t* mins,
                               int64_t rows, int d, void* stream) {
  return quantize_int8_impl<true>(D, dtype, D_u8, scales, mins, rows, d, stream);
}

int fm_quantize_fp8(const void* D, int dtype, uint8_t* D_fp8, float* scales, int64_t rows, int d, void* stream) {
  return quantize_fp8_impl<false>(D, dtype, D_fp8, scales, rows, d, stream);
}

int fm_normalize_quantize_fp8(const void* D, int dtype, uint8_t* D_fp8, float* scales, int64_t rows, int d,
                              void* stream) {
  return quantize_fp8_impl<true>(D, dtype, D_fp8, scales, rows, d, stream);
}

#ifdef FM_PROFILE
// profiling builds only: copy (and optionally clear) the wait/section counters
int fm_prof_read(unsigned long long* out, int reset) {
  if (cudaMemcpyFromSymbol(out, g_fm_prof, sizeof(unsigned long long) * 32) != cudaSuccess)
    return FM_ERR_LAUNCH;
  if (reset) {
    const unsigned long long z[32] = {0};
    if (cudaMemcpyToSymbol(g_fm_prof, z, sizeof(z)) != cudaSuccess) return FM_ERR_LAUNCH;
  }
  return FM_OK;
}
#endif

#ifdef FM_TRACE
int fm_trace_read(unsigned long long* out, int reset) {
  if (cudaMemcpyFromSymbol(out, g_fm_trace, sizeof(unsigned long long) * 8 * 4096) != cudaSuccess)
    return FM_ERR_LAUNCH;
  if (reset) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_fm_trace) != cudaSuccess) return FM_ERR_LAUNCH;
    if (cudaMemset(p, 0, sizeof(unsigned long long) * 8 * 4096) != cudaSuccess) return FM_ERR_LAUNCH;
  }
  return FM_OK;
}
#endif

int fm_wait_selftest(int32_t* status, int64_t timeout_ns, void* stream) {
  if (!status || timeout_ns <= 0) return FM_ERR_ARG;
  wait_selftest_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(
      status, static_cast<uint64_t>(timeout_ns));
  return cudaGetLastError() == cudaSuccess ? FM_OK : FM_ERR_LAUNCH;
}

}  // extern "C"
