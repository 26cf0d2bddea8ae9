/*
 * flash_maxsim_sm100.h -- C ABI of libflashmaxsim_sm100.so, the B200 (sm_100a)
 * MaxSim scoring kernels.
 *
 * Plain C: device pointers, sizes and a CUDA stream handle (cudaStream_t
 * passed as void*). fp16 tensors are passed as uint16_t bit patterns. Every
 * tensor is dense, row-major and contiguous, with 16-byte-aligned base
 * addresses. The library allocates nothing: the caller owns every buffer.
 * Calls are asynchronous on `stream` and re-entrant.
 *
 * Return value: 0 on success, otherwise an FM_ERR_* code for an argument or
 * launch error detected on the host. Device-side failures (a bounded wait that
 * ran out of time, a sparse index out of range) are written into the caller's
 * device status word `status` (first error wins; 0 = OK); read it after the
 * stream has been synchronised. fm_status_string() names every code.
 *
 * Each entry point replaces one launch site of the reference (roipony/flash-maxsim
 * 0.1.0, Triton kernels), cited per function.
 */
#ifndef FLASH_MAXSIM_SM100_H
#define FLASH_MAXSIM_SM100_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* status / error codes */
#define FM_OK 0
#define FM_ERR_ARG 1
#define FM_ERR_LAUNCH 2
/* device-side bounded waits that ran out of time (10..18) */
#define FM_ERR_TIMEOUT_DFULL 10
#define FM_ERR_TIMEOUT_DEMPTY 11
#define FM_ERR_TIMEOUT_QFULL 12
#define FM_ERR_TIMEOUT_QEMPTY 13
#define FM_ERR_TIMEOUT_TFULL 14
#define FM_ERR_TIMEOUT_TEMPTY 15
#define FM_ERR_TIMEOUT_UFULL 16
#define FM_ERR_TIMEOUT_UEMPTY 17
#define FM_ERR_TIMEOUT_DRAIN 18
#define FM_ERR_TIMEOUT_SELFTEST 19
#define FM_ERR_BAD_INDEX 20
#define FM_ERR_UNSUPPORTED 21
#define FM_ERR_NO_DEVICE 22
#define FM_ERR_SCRATCH_TOO_SMALL 23

/* ABI version of this header (major * 100 + minor). */
int fm_abi_version(void);

/* Human-readable name of a status / error code. */
const char* fm_status_string(int code);

/* Limit, in nanoseconds, of every device-side wait (default 2e9). */
void fm_set_wait_timeout_ns(int64_t ns);

/*
 * Process-wide options (returns FM_ERR_ARG for an unknown option).
 * FM_OPT_FLAT_KERNEL = 1 routes shared-document batches without doc_lengths
 * (Ld >= 128, Lq % 32 == 0, d <= 128) to the flat-token kernel, which cuts
 * the token matrix into fixed chunks across document boundaries (no MMA
 * columns spent on chunk padding); 0 (default) keeps the per-document kernel.
 * Both give the same scores. No counterpart in the reference.
 */
#define FM_OPT_FLAT_KERNEL 1
int fm_set_option(int option, int value);

/*
 * Launch plan the forward entry points would use for a shape (host only, no
 * device needed). mode: 0 dense, 1 sparse, 2 INT8. Writes 16 ints to `out`:
 * chunk tokens C, chunks per resident group G, D ring slots, Q ring stages,
 * INT8 staging slots, Q stages per M-block, K atoms per Q stage, K atoms per
 * token, row groups per span, lane-quarter replication, Q resident flag, TMEM
 * slots, TMEM columns per slot, dynamic shared memory bytes, row groups per
 * document, documents per work item. The plan is that of the general forward
 * kernel; one query of <= 64 rows with d <= 128 (dense or sparse) and the INT8
 * shapes of fm_maxsim_int8_fwd's fast path run dedicated kernels instead.
 * No counterpart in the reference (its Triton autotuner picks tile
 * sizes at run time, flash_maxsim/flash_maxsim.py:15-81).
 */
int fm_fwd_plan_info(int mode, int argmax, int Nq, int B, int Lq, int Ld, int d, int shared_docs,
                     int K, int32_t* out, int n_out);

/*
 * MaxSim forward, fp16 inputs, fp32 scores.
 *   scores[n * B + b] = sum_{q<Lq} max_{t<len(doc)} <Q[n,q,:], D[doc,t,:]>
 * shared_docs = 1: D is [B, Ld, d], doc = b, every query scores every doc.
 * shared_docs = 0: D is [Nq, B, Ld, d], doc = n * B + b.
 * doc_lengths: NULL (all Ld) or int32 per doc ([B] shared, [Nq*B] otherwise);
 *   values are clamped to [0, Ld]; an empty doc scores -inf.
 * argmax: NULL, or int32 [Nq*B, Lq] receiving the first token index of each
 *   row maximum (-1 for an empty doc).
 * Q: [Nq, Lq, d] fp16; d % 8 == 0, d <= 2048.
 * Replaces the `_launch_fwd` -> `_maxsim_fwd_kernel` launch
 *   (flash_maxsim/flash_maxsim.py:195-208, kernel :83-146), used by
 *   flash_maxsim (:221-230), flash_maxsim_batched (:233-250) and the
 *   training forward (:255-263).
 */
int fm_maxsim_fwd(const uint16_t* Q, const uint16_t* D, const int32_t* doc_lengths,
                  float* scores, int32_t* argmax, int Nq, int B, int Lq, int Ld, int d,
                  int shared_docs, int32_t* status, void* stream);

/*
 * MaxSim forward over packed (unpadded) documents: document b is rows
 * [cu_seqlens[b], cu_seqlens[b+1]) of D_tokens [total_tokens, d] fp16, so a
 * ragged batch needs no padding in host or device memory.
 *   scores[n * B + b] = sum_{q<Lq} max_{cu[b] <= t < cu[b+1]} <Q[n,q,:], D_tokens[t,:]>
 * cu_seqlens: int32 [B + 1], non-decreasing, cu[0] >= 0, cu[B] <= total_tokens.
 * max_len: an upper bound of every document's length (longer documents are
 *   cut to max_len tokens, as doc_lengths > Ld are clamped to Ld); it sizes
 *   the launch plan. An empty document scores -inf.
 * argmax: NULL, or int32 [Nq*B, Lq] (token index within the document).
 * Q: [Nq, Lq, d] fp16, shared by every document. Same kernels as
 * fm_maxsim_fwd (the TMA box of a chunk starts at the document's first row).
 * No counterpart in the reference, whose callers pad ragged documents to
 * [B, Ld, d] with doc_lengths (examples/demo.py:55-69).
 */
int fm_maxsim_packed_fwd(const uint16_t* Q, const uint16_t* D_tokens, const int32_t* cu_seqlens,
                         float* scores, int32_t* argmax, int Nq, int B, int Lq, int max_len, int d,
                         int64_t total_tokens, int32_t* status, void* stream);

/*
 * Fused dequantise + MaxSim, single query.
 *   scores[b] = sum_q max_t sum_k Q[q,k] * (u[b,t,k] * scale[b,t] + min[b,t])
 * D_u8: [B, Ld, d] uint8 (d % 16 == 0), scales/mins: [B, Ld] fp16.
 * Replaces `_maxsim_int8_kernel` launched by flash_maxsim_int8
 *   (flash_maxsim/flash_maxsim_quant.py:105-142, kernel :52-98).
 */
int fm_maxsim_int8_fwd(const uint16_t* Q, const uint8_t* D_u8, const uint16_t* scales,
                       const uint16_t* mins, const int32_t* doc_lengths, float* scores, int B,
                       int Lq, int Ld, int d, int32_t* status, void* stream);

/*
 * FP8 document storage: e4m3 codes [B, Ld, d] (d % 16 == 0, d <= 256) with
 * one fp32 scale per token [B, Ld], single query of Lq <= 64 rows.
 *   scores[b] = sum_q max_{t<len(b)} sum_k Q[q,k] * scale[b,t] * e4m3(D_fp8[b,t,k])
 * Half the bytes of fp16 documents. The sibling of fm_maxsim_int8_fwd
 * (which replaces flash_maxsim/flash_maxsim_quant.py:105-142); the reference
 * has no FP8 format.
 * fm_quantize_fp8: rows of d elements of type `dtype` (FM_DTYPE_*) ->
 *   scale = max|x| / 448 (1 for an all-zero row), code = e4m3(x / scale),
 *   round-to-nearest-even, saturating; D_fp8 [rows, d] bytes, scales fp32 [rows].
 */
int fm_maxsim_fp8_fwd(const uint16_t* Q, const uint8_t* D_fp8, const float* scales, const int32_t* doc_lengths,
                      float* scores, int B, int Lq, int Ld, int d, int32_t* status, void* stream);
int fm_quantize_fp8(const void* D, int dtype, uint8_t* D_fp8, float* scales, int64_t rows, int d, void* stream);

/*
 * Sparse MaxSim: per document b, only the K query rows indices[b, :] count
 * (duplicates count twice, negative indices wrap like torch indexing).
 *   scores[b] = sum_{k<K} max_{t<len(b)} <Q[indices[b,k],:], D[b,t,:]>
 * Q: [Lq, d], D: [B, Ld, d], indices: int32 [B, K].
 * Replaces `_sparse_maxsim_kernel` launched by flash_maxsim_sparse
 *   (flash_maxsim/flash_maxsim_sparse.py:98-140, kernel :42-91).
 */
int fm_maxsim_sparse_fwd(const uint16_t* Q, const uint16_t* D, const int32_t* indices,
                         const int32_t* doc_lengths, float* scores, int B, int K, int Lq,
                         int Ld, int d, int32_t* status, void* stream);

/*
 * Top-k documents per query (score descending, then document id ascending;
 * deterministic). Rerankers keep only these (the reference's callers run
 * `scores.topk(k)` on the full matrix: examples/demo.py:126-134,
 * benchmarks/bench.py:36; the reference library has no top-k entry point).
 *
 * fm_topk_workspace_size: bytes of the candidate workspace for Nq queries
 *   and k (depends on the current device's SM count); 16-byte aligned.
 * fm_maxsim_topk: fm_maxsim_fwd (shared documents) whose kernel also keeps
 *   each query's k best documents per CTA, then one merge kernel. scores
 *   [Nq, B] is still written in full; top_scores fp32 [Nq, k], top_idx
 *   int64 [Nq, k]. 1 <= k <= min(B, 1024).
 * fm_topk_select: the same selection over any score matrix [Nq, B] (e.g. of
 *   fm_maxsim_int8_fwd); id_offset is added to every document id (the first
 *   document of a shard).
 * fm_topk_merge: final merge of candidates cand_scores / cand_ids
 *   [Nq, parts, k] (ids < 0 = none), e.g. the per-rank top-k lists of a
 *   document-sharded corpus after an all-gather.
 * No counterpart in the reference.
 */
int64_t fm_topk_workspace_size(int Nq, int k);
int fm_maxsim_topk(const uint16_t* Q, const uint16_t* D, const int32_t* doc_lengths, float* scores, int k,
                   float* top_scores, int64_t* top_idx, int Nq, int B, int Lq, int Ld, int d,
                   void* workspace, int64_t workspace_bytes, int32_t* status, void* stream);
int fm_topk_select(const float* scores, int Nq, int B, int k, int64_t id_offset, float* top_scores,
                   int64_t* top_idx, void* workspace, int64_t workspace_bytes, void* stream);
int fm_topk_merge(const float* cand_scores, const int32_t* cand_ids, int Nq, int parts, int k,
                  float* top_scores, int64_t* top_idx, void* stream);

/*
 * Training backward from the forward's argmax (shared docs).
 *   grad_Q[n,q,:] = sum_b g[n,b] * D[b, argmax[n,b,q], :]
 *   grad_D[b,t,:] = sum_{(n,q): argmax[n,b,q]==t} g[n,b] * Q[n,q,:]
 * grad_scores: fp32 [Nq, B]. grad_Q: fp16 [Nq, Lq, d], grad_D: fp16
 * [B, Ld, d]; both fully written (no pre-zeroing needed). Deterministic:
 * grad_Q is summed over document ranges in fp32 partials (workspace) that are
 * added in a fixed order. workspace: caller-owned device memory of at least
 * fm_maxsim_bwd_workspace_size(...) bytes, 16-byte aligned (NULL allowed when
 * that size is 0). Requires Nq * Lq <= 32768.
 * Replaces `_maxsim_bwd_dQ_kernel` and `_maxsim_bwd_dD_kernel` launched by
 *   _FlashMaxSimFn.backward (flash_maxsim/flash_maxsim.py:266-286,
 *   kernels :153-188).
 */
int64_t fm_maxsim_bwd_workspace_size(int Nq, int B, int Lq, int Ld, int d);
int fm_maxsim_bwd(const uint16_t* Q, const uint16_t* D, const int32_t* argmax,
                  const float* grad_scores, uint16_t* grad_Q, uint16_t* grad_D, int Nq, int B,
                  int Lq, int Ld, int d, void* workspace, int64_t workspace_bytes, void* stream);

/*
 * Same backward as fm_maxsim_bwd for callers that cannot allocate device
 * memory -- for example a host program that hands this library only the
 * tensors it already owns, inside an engine whose device memory is fully
 * reserved by its own allocator, or that must not allocate once serving has
 * started. Nothing is allocated: the dQ partial sums go to a 16 MiB scratch
 * array compiled into the library (every device that loads the library keeps
 * it until the process exits). When fm_maxsim_bwd's usual number of document
 * ranges would need more than 16 MiB, fewer ranges are used (still added in a
 * fixed order, so dQ may differ from fm_maxsim_bwd's in the last bits);
 * shapes where two ranges of Nq * Lq * d fp32 partial sums exceed 16 MiB are
 * rejected with FM_ERR_SCRATCH_TOO_SMALL. The first call on a device looks up
 * the scratch address for that device (and again in a new CUDA context, e.g.
 * after cudaDeviceReset); make that first call before any stream capture.
 * All calls share the one scratch array, so calls that overlap on the GPU
 * (different streams, or different host threads) race; serialise them. Every
 * partial sum is written before it is read, so nothing needs clearing between
 * calls. No counterpart in the reference.
 */
int fm_maxsim_bwd_noalloc(const uint16_t* Q, const uint16_t* D, const int32_t* argmax,
                          const float* grad_scores, uint16_t* grad_Q, uint16_t* grad_D, int Nq,
                          int B, int Lq, int Ld, int d, void* stream);

/* element types accepted by fm_quantize_int8 */
#define FM_DTYPE_F16 0
#define FM_DTYPE_F32 1
#define FM_DTYPE_BF16 2

/*
 * Per-token affine uint8 quantisation of `rows` rows of d elements
 * (d % 8 == 0) of type `dtype` (FM_DTYPE_*), bit-exact with quantize_int8
 * (flash_maxsim/flash_maxsim_quant.py:11-28): min/max in fp32,
 * scale = max((max - min) / 255, 1e-8), u = clamp(round_half_even((x - min) / scale), 0, 255).
 * Outputs: D_u8 [rows, d]; scales and mins fp16 [rows].
 */
int fm_quantize_int8(const void* D, int dtype, uint8_t* D_u8, uint16_t* scales, uint16_t* mins,
                     int64_t rows, int d, void* stream);

/*
 * Index-time quantisation of freshly encoded embeddings, fused with their
 * L2 normalisation: every row is divided by max(||x||_2, 1e-12) (the rule of
 * torch.nn.functional.normalize, the norm summed in a fixed order so that the
 * result is reproducible on the host) and then quantised exactly as
 * fm_quantize_int8 / fm_quantize_fp8 quantise their input. One pass over the
 * embeddings instead of a normalise pass, a cast and a quantise pass. No
 * counterpart in the reference (its quantize_int8 takes normalised input,
 * flash_maxsim/flash_maxsim_quant.py:11-28).
 */
int fm_normalize_quantize_int8(const void* D, int dtype, uint8_t* D_u8, uint16_t* scales, uint16_t* mins,
                               int64_t rows, int d, void* stream);
int fm_normalize_quantize_fp8(const void* D, int dtype, uint8_t* D_fp8, float* scales, int64_t rows, int d,
                              void* stream);

/*
 * Failure-detection self test: launches one CTA that waits on a barrier that
 * nothing arrives at. The bounded wait gives up after timeout_ns and writes
 * FM_ERR_TIMEOUT_SELFTEST into *status; the context stays usable.
 * No counterpart in the reference (which has no device-side waits).
 */
int fm_wait_selftest(int32_t* status, int64_t timeout_ns, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* FLASH_MAXSIM_SM100_H */
