/*
 * greyhound_b200 — C-ABI of the B200 (sm_100a) replacement for greyhound's
 * chunked linear cross-entropy hot path and the two row kernels that share
 * its reduction core.
 *
 * Conventions for every entry point:
 *   - pointers are DEVICE pointers unless stated otherwise; tensors are dense
 *     and row-major (C-contiguous), exactly the layouts the reference demands
 *     (src/greyhound/kernels/cross_entropy.py:183, kernels/logprobs.py:152);
 *   - `stream` is a cudaStream_t passed as void* (0 = legacy default stream);
 *     every call only enqueues work on it and never synchronises the host;
 *   - the return value is GH_OK or an error code; gh_last_error_string()
 *     gives a human-readable message for the last failure on this host thread;
 *   - the library never allocates device memory: scratch space is passed in
 *     by the caller (`workspace`, sized by the matching *_workspace_bytes);
 *   - device-side problems (e.g. a label outside [0, V)) never trap: they are
 *     recorded in the workspace status word, see gh_workspace_status_offset(),
 *     and every entry point with a workspace ends by OR-ing that word into a
 *     per-device sticky slot in pinned host memory (gh_take_device_errors).
 */
#ifndef GREYHOUND_B200_H
#define GREYHOUND_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define GH_API __attribute__((visibility("default")))
#else
#define GH_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* dtype codes (logits / hidden / weight / index / output element types) */
enum {
  GH_F16 = 0,
  GH_BF16 = 1,
  GH_F32 = 2,
  GH_I32 = 3,
  GH_I64 = 4
};

/* status codes; the Python layer maps EINVAL->ValueError, ETYPE->TypeError,
 * everything else -> RuntimeError (mirrors kernels/cross_entropy.py:173-184) */
enum {
  GH_OK = 0,
  GH_EINVAL = 1,
  GH_ETYPE = 2,
  GH_ECUDA = 3,
  GH_EWORKSPACE = 4,
  GH_EUNSUPPORTED = 5
};

/* device-side status bits written into the workspace status word */
enum {
  GH_DEV_BAD_LABEL = 1   /* a non-ignored label/index outside [0, V) */
};

GH_API int gh_abi_version(void);
GH_API const char* gh_last_error_string(void);
/* Number of kernels this library has launched in this process (all devices). */
GH_API long long gh_launch_count(void);
/* Byte offset of the int32 device status word inside any workspace. */
GH_API size_t gh_workspace_status_offset(void);
/* Returns and clears the GH_DEV_* bits that calls on `device` have recorded
 * since the last call of this function (no counterpart in the reference,
 * whose kernels raise ValueError for bad labels on the host before launch,
 * src/greyhound/kernels/cross_entropy.py:173-184; here labels are checked on
 * the device, so the check costs no host sync). Never synchronises: bits of
 * a call that the GPU has not run yet are not visible. The first entry point
 * called in a process allocates the small pinned host array behind these
 * slots (cudaHostAlloc); make that call before any stream capture. */
GH_API int gh_take_device_errors(int device);

/* ------------------------------------------------------------------------ *
 * Standalone cross-entropy with logits gradient.
 * Replaces cross_entropy_with_grad_kernel(logits, labels, z_loss_multiplier,
 * ignore_index) -> (ce_sum, z_sum, n_valid)       kernels/cross_entropy.py:166
 * and the op around it                           ops/cross_entropy.py:11-26.
 *
 *   logits  [rows, vocab] dtype in {F16, BF16, F32}
 *   dlogits [rows, vocab] same dtype; may equal `logits` (in place, as the
 *           reference kernel does) or be NULL (loss only, no gradient)
 *   labels  [rows] int64; `ignore_index` rows contribute nothing and get a
 *           zero gradient row
 *   ce_sum, z_sum, n_valid: float scalars, overwritten (not added to)
 *   lse_out optional float[rows] <- natural-log logsumexp of each row
 *   mean_reduction: 0 -> gradient of the SUM (reference op semantics);
 *                   1 -> gradient already divided by max(n_valid, 1), i.e. the
 *                   mean scaling of ops/cross_entropy.py:63-66 fused in.
 *   grad_scale      optional device float; when given the gradient is also
 *                   multiplied by *grad_scale (e.g. 1/global_n_valid computed
 *                   on the device by a data-parallel caller)
 * Gradient: softmax * (1 + 2 z lse) - onehot(label)   kernels/cross_entropy.py:94-108
 * Loss sums are reduced deterministically (fixed order, no float atomics).
 * ------------------------------------------------------------------------ */
GH_API size_t gh_ce_workspace_bytes(int64_t rows, int64_t vocab, int dtype);
GH_API int gh_ce_fwd_grad(const void* logits, void* dlogits, const int64_t* labels,
                   int64_t rows, int64_t vocab, int dtype,
                   float z_loss_multiplier, int64_t ignore_index,
                   int mean_reduction, const float* grad_scale,
                   float* ce_sum, float* z_sum, float* n_valid, float* lse_out,
                   void* workspace, size_t workspace_bytes, void* stream);

/* Allocation-free form of gh_ce_fwd_grad (no counterpart in the reference).
 * For callers that cannot allocate device memory where they need the loss
 * (a forbidding allocator, a runtime whose pool offers no scratch, a binding
 * without a device allocator): the scratch is a fixed library-owned device
 * array of gh_ce_noalloc_scratch_bytes() (4 MiB) that every GPU loading the
 * library holds until exit. Shapes whose scratch would exceed it are rejected
 * (about 349,000 rows at any vocab size). The first call on a
 * device looks up the array's device address (make it before any stream
 * capture). All calls share the array, so calls that overlap on the GPU
 * (concurrent streams) race; serialise them. Arguments and results as
 * gh_ce_fwd_grad, except: a shape too large for the array returns
 * GH_EWORKSPACE (the code gh_ce_fwd_grad gives a too-small workspace), and
 * the device status word is not published to gh_take_device_errors (that
 * would allocate); read it with gh_ce_noalloc_status. */
GH_API size_t gh_ce_noalloc_scratch_bytes(void);
GH_API int gh_ce_fwd_grad_noalloc(const void* logits, void* dlogits, const int64_t* labels,
                                  int64_t rows, int64_t vocab, int dtype,
                                  float z_loss_multiplier, int64_t ignore_index,
                                  int mean_reduction, const float* grad_scale,
                                  float* ce_sum, float* z_sum, float* n_valid, float* lse_out,
                                  void* stream);
/* The GH_DEV_* status bits of the last gh_ce_fwd_grad_noalloc call on this
 * device, copied to *host_out (a host int). Synchronises `stream`. */
GH_API int gh_ce_noalloc_status(int* host_out, void* stream);

/* ------------------------------------------------------------------------ *
 * Selective log-softmax: out[r] = logits[r, index[r]] - logsumexp(logits[r]).
 * Replaces selective_log_softmax_kernel(logits, index)  kernels/logprobs.py:131
 *   index dtype in {I32, I64}; out dtype in {F16, BF16, F32} (the reference
 *   writes the logits dtype, kernels/logprobs.py:158); lse_out optional.
 * ------------------------------------------------------------------------ */
GH_API size_t gh_sls_workspace_bytes(int64_t rows, int64_t vocab, int dtype);
GH_API int gh_sls_fwd(const void* logits, const void* index, int index_dtype,
               int64_t rows, int64_t vocab, int dtype,
               void* out, int out_dtype, float* lse_out,
               void* workspace, size_t workspace_bytes, void* stream);

/* Backward of selective log-softmax (the reference raises NotImplementedError,
 * ops/logprobs.py:30; this is the autograd derivative of
 * gather(log_softmax(logits), index)):
 *   grad_logits[r, v] = grad_out[r] * ([v == index[r]] - exp(logits[r, v] - lse[r]))
 * lse comes from gh_sls_fwd's lse_out. grad_out dtype in {F16, BF16, F32}. */
GH_API int gh_sls_bwd(const void* logits, const void* index, int index_dtype,
               const float* lse, const void* grad_out, int grad_dtype,
               int64_t rows, int64_t vocab, int dtype, void* grad_logits,
               void* stream);

/* ------------------------------------------------------------------------ *
 * Logits gradient from a known per-row logsumexp (no reduction):
 *   dlogits[r, v] = exp(logits[r, v] - lse[r]) * (1 + 2 z lse[r]) * s
 *                   - s * [v == labels[r] - label_offset]
 * with s = *grad_scale (1 if NULL); rows with labels[r] == ignore_index get 0.
 * A label outside [label_offset, label_offset + vocab) only contributes the
 * softmax term (vocab-sharded use). dlogits may equal logits.
 * This is the second half of the reference kernel (kernels/cross_entropy.py:94-108)
 * split out so the statistics can come from a fused GEMM epilogue or from
 * other vocab shards.
 * ------------------------------------------------------------------------ */
GH_API int gh_logits_grad(const void* logits, void* dlogits, const int64_t* labels,
                          const float* lse, int64_t rows, int64_t vocab, int dtype,
                          float z_loss_multiplier, int64_t ignore_index,
                          int64_t label_offset, const float* grad_scale, void* stream);

/* ------------------------------------------------------------------------ *
 * Chunked linear cross-entropy, forward + backward, on tcgen05 GEMMs.
 * Replaces the op greyhound::chunked_linear_cross_entropy_fwd
 * (src/greyhound/ops/chunked_linear_cross_entropy.py:19-67) and the chunk
 * loop it drives (src/greyhound/ops/chunked_linear_loss.py:56-103).
 *
 *   H      [N, D] activations, dtype BF16 or F16 (row-major)
 *   W      [V, D] weight, same dtype (row-major; the reference passes the
 *          [D, V] view W.T, which is this same memory)
 *   target [N] int64 class ids or ignore_index
 *   chunk_rows: rows per chunk (<= 0: all rows in one chunk); the logits of
 *          one chunk ([chunk, V] in the activation dtype) live in the workspace
 *   grad_input  [N, D] (same dtype) or NULL
 *   grad_weight [V, D] row-major (same dtype) or NULL; both NULL -> loss
 *          only. This is the reference op's [D, V] grad_weight stored
 *          transposed, so the autograd layer can return it as the [D, V]
 *          view and W.grad ([V, D]) needs no re-layout copy
 *   fp32_grad_weight_accum: 1 -> weight gradient accumulated across chunks in
 *          fp32 and cast once; 0 -> accumulated in the weight dtype
 *   mean_reduction / grad_scale: as for gh_ce_fwd_grad; the scale is folded
 *          into the logits gradient, so both gradients come out scaled
 *   flags: GH_LCE_DEFER_LAST_DH -> the last chunk's grad_input rows are not
 *          computed; call gh_lce_dh_last_chunk later (lets a data-parallel
 *          caller start the grad_weight all-reduce first);
 *          GH_LCE_KEEP_DW_OPERAND with grad_weight == NULL -> leave the weight
 *          gradient's operands in the workspace for gh_lce_dw_peers;
 *          GH_LCE_GRADS_LATER with both gradient pointers NULL and all rows
 *          in one chunk -> loss plus everything both gradient GEMMs need, kept
 *          in the workspace; the gradients come later from gh_lce_dw_peers
 *          and gh_lce_dh_last_chunk, scaled by the autograd grad_output (so
 *          the backward needs no separate scaling pass)
 *   ce_sum, z_sum, n_valid: float scalars (overwritten)
 * ------------------------------------------------------------------------ */
enum { GH_LCE_DEFER_LAST_DH = 1, GH_LCE_KEEP_DW_OPERAND = 2, GH_LCE_GRADS_LATER = 4 };

GH_API size_t gh_lce_workspace_bytes(int64_t N, int64_t D, int64_t V, int64_t chunk_rows,
                                     int dtype, int fp32_grad_weight_accum);
/* Workspace for the loss-only form (grad_input == grad_weight == NULL): the
 * forward-only path (src/greyhound/ops/chunked_linear_cross_entropy.py:91-132)
 * keeps only per-row statistics, the logits are never written to memory. */
GH_API size_t gh_lce_loss_workspace_bytes(int64_t N, int64_t D, int64_t V, int64_t chunk_rows,
                                          int dtype);
GH_API int gh_lce_fwd_bwd(const void* H, const void* W, const int64_t* target,
                          int64_t N, int64_t D, int64_t V, int dtype,
                          float z_loss_multiplier, int64_t ignore_index,
                          int mean_reduction, const float* grad_scale,
                          int64_t chunk_rows, int fp32_grad_weight_accum, int flags,
                          void* grad_input, void* grad_weight,
                          float* ce_sum, float* z_sum, float* n_valid,
                          void* workspace, size_t workspace_bytes, void* stream);
/* grad_input rows [row_begin, row_end) of the last chunk (offsets inside the
 * chunk; row_end < 0: to the end), from what gh_lce_fwd_bwd(...,
 * GH_LCE_DEFER_LAST_DH or GH_LCE_GRADS_LATER) left in the workspace, times
 * *scale when scale != NULL (a device float). max_ctas <= 0: all SMs; fewer
 * leave SMs to a concurrently running collective. */
GH_API int gh_lce_dh_last_chunk(const void* W, int64_t N, int64_t D, int64_t V, int dtype,
                                int64_t chunk_rows, int fp32_grad_weight_accum,
                                int64_t row_begin, int64_t row_end, const float* scale,
                                void* grad_input, void* workspace, size_t workspace_bytes,
                                int max_ctas, void* stream);

/* Weight gradient (times *scale when scale != NULL, a device float) of a
 * single-chunk call (N <= chunk rows) whose gh_lce_fwd_bwd ran with
 * grad_weight == NULL and GH_LCE_KEEP_DW_OPERAND or GH_LCE_GRADS_LATER,
 * stored in row bands: rows [b * band_rows, (b + 1) * band_rows) of the
 * [V, D] gradient go to band_out[b] (row-major, pitch D), b < nbands <= 8,
 * band_rows a multiple of 256. band_out[b] may point into another GPU's
 * memory (a CUDA IPC mapping): the data-parallel caller gives each rank's
 * receive slot, so the GEMM's epilogue performs the scatter of a
 * reduce-scatter of the weight gradient (no counterpart in the reference,
 * which is single-device). The GEMM computes band first_band's tiles first
 * and wraps around (each rank passes its own index, so the ranks' stores
 * go to different owners at any moment). The kernel ends with a
 * system-scope fence, so
 * once it has completed the stores are visible to the owners. */
GH_API int gh_lce_dw_peers(const void* H, int64_t N, int64_t D, int64_t V, int dtype,
                           int64_t chunk_rows, int fp32_grad_weight_accum, const float* scale,
                           void* const* band_out, int nbands, int64_t band_rows, int first_band,
                           void* workspace, size_t workspace_bytes, void* stream);

/* out0[r, c] (and out1[r, c] when out1 != NULL) = sum over s < nslots of
 * slots[s * slot_stride + r * ld + c], summed in fp32 in slot order and
 * rounded once (deterministic): the reduction step of that reduce-scatter.
 * dtype F16 or BF16; all pointers and ld 16-byte aligned. */
GH_API int gh_sum_slots(const void* slots, int nslots, int64_t slot_stride, int64_t rows, int64_t cols,
                        int64_t ld, int dtype, void* out0, void* out1, void* stream);

/* CUDA IPC of a device buffer that need not start its allocation:
 * gh_ipc_get_handle writes the 64-byte handle of the allocation holding ptr
 * and ptr's byte offset in it; gh_ipc_open maps a handle from another
 * process on this node into the current device (peer access enabled) and
 * returns the mapped base + offset; gh_ipc_close unmaps (give the pointer
 * and offset gh_ipc_open used). */
GH_API int gh_ipc_get_handle(const void* ptr, void* handle_out, size_t* offset_out);
GH_API int gh_ipc_open(const void* handle, size_t offset, void** ptr_out);
GH_API int gh_ipc_close(void* ptr, size_t offset);
/* Device-to-device copy on `stream` (the copy engines; src or dst may be
 * an IPC mapping of another GPU's memory, then the copy crosses NVLink). */
GH_API int gh_memcpy_async(void* dst, const void* src, size_t bytes, void* stream);

/* ------------------------------------------------------------------------ *
 * Vocab-parallel linear cross-entropy (no counterpart in the reference, which
 * is single-device): this rank holds rows [vocab_start, vocab_start + V_shard)
 * of W and all N rows of H. Phase 1 computes the shard's logits (kept in the
 * workspace) with the fused statistics and writes stats3 [N, 3] =
 * (logsumexp over the shard, 1, target logit or -inf when the target is not
 * in the shard). The caller all-gathers stats3 over ranks and merges them
 * into the global per-row logsumexp (exact: lse = M + log sum_p exp(lse_p - M)).
 * Phase 2 (same workspace) writes the shard's logits gradient with that
 * global lse, grad_weight_shard [V_shard, D] (row-major) and this shard's
 * partial grad_input [N, D], which the caller sums over ranks.
 * ------------------------------------------------------------------------ */
GH_API size_t gh_lce_shard_workspace_bytes(int64_t N, int64_t D, int64_t V_shard, int dtype);
GH_API int gh_lce_shard_stats(const void* H, const void* W_shard, const int64_t* target,
                              int64_t N, int64_t D, int64_t V_shard, int64_t vocab_start,
                              int dtype, float* stats3, void* workspace, size_t workspace_bytes,
                              void* stream);
GH_API int gh_lce_shard_grads(const void* H, const void* W_shard, const int64_t* target,
                              const float* lse, int64_t N, int64_t D, int64_t V_shard,
                              int64_t vocab_start, int dtype, float z_loss_multiplier,
                              int64_t ignore_index, const float* grad_scale,
                              void* grad_input_partial, void* grad_weight_shard,
                              void* workspace, size_t workspace_bytes, void* stream);

/* The shard's grad_weight alone, from the logits gradient that a previous
 * gh_lce_shard_grads(..., grad_weight_shard = NULL) left in the workspace:
 * lets the caller start the grad_input all-reduce before this GEMM.
 * max_ctas <= 0: all SMs. */
GH_API int gh_lce_shard_dw(const void* H, int64_t N, int64_t D, int64_t V_shard, int dtype,
                           void* grad_weight_shard, void* workspace, size_t workspace_bytes,
                           int max_ctas, void* stream);

/* ------------------------------------------------------------------------ *
 * Plain tcgen05 GEMM (the GEMMs of the generic chunked_linear_loss path,
 * src/greyhound/ops/chunked_linear_loss.py:82,94,95-101):
 *   out[M, N] = scale * sum_k A[m, k] B[n, k]  (+ addend[M, N])
 * A is [M, K] with pitch lda (a_mn_major = 0) or [K, M] (a_mn_major = 1);
 * B likewise [N, K] / [K, N]. Operands BF16 or F16, 16-byte aligned with
 * 16-byte row pitches. out_dtype F32 or the operand dtype; the addend has
 * the output dtype and pitch ld_add (may alias out for accumulation).
 * status: optional device int receiving error bits.
 * ------------------------------------------------------------------------ */
GH_API int gh_gemm(const void* A, int64_t lda, int a_mn_major,
                   const void* B, int64_t ldb, int b_mn_major,
                   int64_t M, int64_t N, int64_t K, int dtype,
                   void* out, int64_t ldo, int out_dtype,
                   const void* addend, int64_t ld_add, const float* scale,
                   int* status, void* stream);

/* ------------------------------------------------------------------------ *
 * out[i] = in[i] * (*g) for n elements (F16 / BF16 / F32), g a device float.
 * The backward of the ops whose gradients are computed in the forward
 * (src/greyhound/ops/chunked_linear_cross_entropy.py:175-185,
 * ops/cross_entropy.py:79-85: saved_grad * grad_output) without a host sync
 * and without torch's mixed-dtype broadcast path. 16-byte aligned buffers.
 * ------------------------------------------------------------------------ */
GH_API int gh_scale(const void* in, void* out, int64_t n, int dtype, const float* g, void* stream);

/* Optional event timing of the library's launches, by kernel class:
 * 0 logits GEMM + fused CE epilogue, 1 dW GEMM, 2 dH GEMM, 3 dlogits pass,
 * 4 standalone row kernels, 5 other GEMMs. gh_profile_read synchronises on
 * the recorded events and returns total ms and launch count per class. */
GH_API void gh_profile_enable(int on);
GH_API int gh_profile_read(double* ms_out, long long* count_out, int n_classes, int reset);

/* Failure-detection self-test of the GEMM pipeline (no counterpart in the
 * reference): launches one small GEMM whose load stage deliberately issues
 * nothing, with all pipeline waits limited to wait_ms. The kernel must give
 * up, free its tensor memory, set bit 4 (GH_DEV_PIPELINE_TIMEOUT) in *status
 * (device int, caller-zeroed) and return, leaving the context usable.
 * scratch: >= 112 KB of device memory used only to describe the operands. */
enum { GH_DEV_PIPELINE_TIMEOUT = 4 };
GH_API int gh_gemm_selftest_stall(void* scratch, size_t scratch_bytes, int* status, int wait_ms,
                                  void* stream);

#ifdef __cplusplus
}
#endif

#endif /* GREYHOUND_B200_H */
