/*
 * lmce — C ABI of the B200 (sm_100a) fused lm_head cross-entropy head.
 *
 * Plain pointers, sizes and a CUDA stream handle; no framework types. Every
 * call is stream-ordered on `stream` (a cudaStream_t passed as void*), never
 * synchronises, never aborts, and never allocates device memory: the caller
 * owns every buffer, including workspaces sized by the *_bytes queries.
 * Every function returns LMCE_OK or an LMCE_ERR_* code; lmce_last_error()
 * gives a thread-local message for the last failing call on this thread.
 * Conditions detected by kernels (a bounded wait that gave up, a label
 * outside [0, V)) are recorded in a per-device error word read by
 * lmce_device_error().
 *
 * Reference interface replaced (fokyso82002-rgb/rus):
 *   FusedChunkedLMHeadFn.forward  solution/ops.py:179-330
 *   FusedChunkedLMHeadFn.backward solution/ops.py:332-339
 *   lm_head_piece_kernel          solution/kernels.py:453-531
 *   lm_head_finish_kernel         solution/kernels.py:534-565
 * The Python autograd wrapper rus_b200.ops.chunked_lm_head binds these with
 * ctypes and keeps the reference's signature (solution/ops.py:342-349).
 */
#ifndef LMCE_H_
#define LMCE_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define LMCE_ABI_VERSION 1

#if defined(__GNUC__)
#define LMCE_API __attribute__((visibility("default")))
#else
#define LMCE_API
#endif

enum {
  LMCE_OK = 0,
  LMCE_ERR_INVALID_ARGUMENT = 1, /* null pointer, bad size, misaligned buffer */
  LMCE_ERR_UNSUPPORTED = 2,      /* device is not sm_100, dtype or shape not supported */
  LMCE_ERR_CUDA = 3,             /* a CUDA runtime/driver call failed */
  LMCE_ERR_TIMEOUT = 4,          /* a bounded on-device wait gave up (device error word) */
  LMCE_ERR_LABEL_RANGE = 5,      /* a label was neither -100 nor in [0, V) (device error word) */
  LMCE_ERR_WORKSPACE = 6         /* workspace too small */
};

enum { LMCE_DTYPE_F16 = 0, LMCE_DTYPE_BF16 = 1 };

/* Per-token partial softmax statistics, 24 bytes:
 *   m    running max of the logits (logits rounded to the input dtype)
 *   s    sum_v exp(z_v - m)
 *   w    sum_v exp(z_v - m) * (z_v - m)
 *   best max logit, idx its lowest global vocab id
 *   zy   target logit, -inf if the target is outside the covered vocab range
 * The same record is produced by a vocab slab, a vocab shard, or their merge. */
typedef struct lmce_part {
  float m, s, w, best;
  int32_t idx;
  float zy;
} lmce_part;

LMCE_API int lmce_abi_version(void);
LMCE_API const char* lmce_last_error(void);

/* Reads the device error word of the current device (synchronous: waits for
 * the device). reset != 0 clears it afterwards. Returns LMCE_OK, or the first
 * LMCE_ERR_* code a kernel recorded. */
LMCE_API int lmce_device_error(int reset);

/* ---------------------------------------------------------------- forward */

/* Number of per-token partial records lmce_fwd_stats writes for this shape on
 * the current device (vocab slabs processed by different CTAs). */
LMCE_API int64_t lmce_fwd_num_parts(int64_t n_tokens, int64_t vocab_local);

/* Fused logits GEMM + online statistics over one vocab shard
 * (replaces ops.py:216-251 pass 1 and kernels.py:480-516 MODE 0).
 *   hidden  [n_tokens, hidden_dim]     dtype, row-major, 16-byte aligned rows
 *   weight  [vocab_local, hidden_dim]  dtype, rows vocab_offset.. of the full head
 *   labels  [n_tokens] int64, global vocab ids, -100 = ignored
 *   parts   [n_tokens, n_parts] lmce_part, n_parts = lmce_fwd_num_parts(...)
 * hidden_dim must be a multiple of 64. No [n_tokens, vocab] buffer is used. */
LMCE_API int lmce_fwd_stats(const void* hidden, const void* weight, const int64_t* labels, int64_t n_tokens,
                   int64_t hidden_dim, int64_t vocab_local, int64_t vocab_offset, int dtype, lmce_part* parts,
                   int64_t n_parts, void* stream);

/* Merges n_parts records per token into one record per token (used before a
 * cross-GPU gather). Record (token t, part p) is parts[t*tok_stride + p*part_stride]. */
LMCE_API int lmce_stats_reduce(const lmce_part* parts, int64_t n_parts, int64_t tok_stride, int64_t part_stride,
                      int64_t n_tokens, lmce_part* record_out, void* stream);

/* Merges the records and finishes the forward (replaces kernels.py:534-565 and
 * the loss reduction at ops.py:268-277):
 *   lse = m + ln s;  entropy = ln s - w / s;  nll = lse - z_y (0 when label == -100)
 *   argmax = lowest vocab id of the max logit
 *   denom = *num_items_dev if non-null, else num_items unless it is NaN, else #(label != -100);
 *           clamped to >= 1 (like the reference's max(float(num_items_in_batch), 1.0), a zero or
 *           negative count gives 1). Pass NaN for "not given".
 *   loss = sum(nll) / denom  (fixed-order reduction, deterministic)
 * Outputs: lse, nll, entropy [n_tokens] fp32; argmax [n_tokens] int64; loss, denom fp32 scalars. */
LMCE_API int lmce_stats_finish(const lmce_part* parts, int64_t n_parts, int64_t tok_stride, int64_t part_stride,
                      const int64_t* labels, int64_t n_tokens, const float* num_items_dev, double num_items,
                      float* lse, float* nll, float* entropy, int64_t* argmax, float* loss, float* denom,
                      void* stream);

/* --------------------------------------------------------------- backward */

/* Workspace bytes for lmce_backward (vocab-chunk gradient tiles, compacted
 * rows, fp32 dX accumulator). v_chunk is rounded up to a multiple of 256;
 * v_chunk <= 0 selects the default: gradient buffers of about 90 MiB within
 * 4096..20480 vocab rows for the CTA-pair kernel (hidden_dim >= 256), about
 * 64 MiB within 8192..32768 rows for the one-CTA kernel; either way at most
 * half the bytes of an [n_tokens, vocab_local] logits buffer. */
LMCE_API size_t lmce_bwd_workspace_bytes(int64_t n_tokens, int64_t hidden_dim, int64_t vocab_local, int64_t v_chunk);

/* Recomputes the logits per vocab chunk, forms G = (softmax - onehot) in
 * registers and contracts it into dX and dW (replaces ops.py:280-322 and
 * ops.py:333-339; dW is new). Only tokens with label != -100 are processed.
 * One persistent launch: on CTA pairs (tcgen05 cta_group::2) when hidden_dim
 * >= 256, else on single CTAs; LMCE_BWD_KERNEL=single forces the latter.
 *   lse        [n_tokens] fp32 from lmce_stats_finish (global over all shards)
 *   grad_loss  device fp32 scalar d(loss) (nullable: 1.0)
 *   denom      device fp32 scalar from lmce_stats_finish
 *   d_hidden     [n_tokens, hidden_dim] dtype  (nullable) receives dX
 *   d_hidden_f32 [n_tokens, hidden_dim] fp32   (nullable) receives this shard's
 *                fp32 dX contribution, zero rows for ignored tokens; it must be
 *                zero-filled by the caller and is meant for a cross-GPU sum
 *   d_weight   [vocab_local, hidden_dim] dtype (nullable) receives dW */
LMCE_API int lmce_backward(const void* hidden, const void* weight, const int64_t* labels, const float* lse,
                  int64_t n_tokens, int64_t hidden_dim, int64_t vocab_local, int64_t vocab_offset, int dtype,
                  const float* grad_loss, const float* denom, void* d_hidden, float* d_hidden_f32,
                  void* d_weight, int64_t v_chunk, void* workspace, size_t workspace_bytes, void* stream);

/* Buffers of the cross-GPU dX sum that lmce_backward_nvls fuses into the
 * backward of a vocab-sharded head. All three are allocations that every rank of
 * the group has mapped into one NVLink multicast object (NVLink SHARP; e.g. torch
 * symmetric memory): the *_mc fields are multicast addresses, the others this
 * rank's own view. */
typedef struct lmce_dx_exchange {
  /* The buffers may be sized for any capacity >= n_tokens (rows of hidden_dim elements) and
     reused by calls with fewer tokens: a call uses the leading rows and flag words only. */
  float* partial;          /* fp32 [n_tokens, hidden_dim]: this rank's dX contribution (scratch) */
  const float* partial_mc; /* multicast address of `partial` */
  void* out_mc;            /* dtype [n_tokens, hidden_dim]: on return every rank's copy holds the
                              summed dX rows of the labelled tokens (other rows are not written) */
  const uint32_t* flags;   /* uint32 [world + 2 * ceil(n_tokens / 256) * world * ceil(hidden_dim / 256)],
                              zeroed on every rank (and a group barrier passed) before the first call;
                              the word of (row block m, rank, column tile) does not depend on n_tokens */
  uint32_t* flags_mc;      /* multicast address of `flags` */
  uint32_t epoch;          /* 1 on the first call with these flags, then +1 per call; equal on all ranks */
  int32_t rank, world;     /* this rank and the group size */
} lmce_dx_exchange;

/* lmce_backward for a vocab-sharded head with the cross-GPU dX sum fused into
 * the kernel. When a row block's last-chunk dX tiles are written (into
 * xch->partial), the rank stamps their flags on every GPU (multimem.st of the
 * epoch); rank r then sums its slice of the block's columns over all GPUs
 * through the switch (multimem.ld_reduce) and stores the result to every GPU's
 * output copy (multimem.st), while the last two vocab chunks' dW tiles still
 * compute. Each GPU's NVLink traffic is about one fp32 read and one dtype write
 * of dX, spread over the end of the kernel, instead of a separate all-reduce
 * after it. Before the kernel ends it waits until every rank has finished its
 * part, so when the call's stream work completes, the local copy of out_mc holds
 * the sums (read it out with lmce_dx_copy_labelled) and the buffers may be reused
 * by the next call, with epoch + 1. Every rank of the group makes every call with
 * the same epoch. The waits for other ranks are bounded (LMCE_ERR_TIMEOUT through
 * lmce_device_error). The reference is single-GPU (ops.py:320-338); this is the
 * vocab-sharded form of its dX accumulation. */
LMCE_API int lmce_backward_nvls(const void* hidden, const void* weight, const int64_t* labels, const float* lse,
                                int64_t n_tokens, int64_t hidden_dim, int64_t vocab_local, int64_t vocab_offset,
                                int dtype, const float* grad_loss, const float* denom, const lmce_dx_exchange* xch,
                                void* d_weight, int64_t v_chunk, void* workspace, size_t workspace_bytes,
                                void* stream);

/* d_hidden[t] = src[t] for tokens whose label is not -100, zero rows otherwise
 * ([n_tokens, hidden_dim] in dtype; the read-out of lmce_backward_nvls). No
 * counterpart in the reference, which is single-GPU. */
LMCE_API int lmce_dx_copy_labelled(const void* src, const int64_t* labels, int64_t n_tokens, int64_t hidden_dim,
                                   int dtype, void* d_hidden, void* stream);

/* d_hidden = dtype(d_hidden_f32), elementwise over n_tokens x hidden_dim: the final
 * cast of an fp32 dX summed across GPUs (the reference's single-GPU dX leaves its
 * fp16 accumulator through the rescale at ops.py:337-338). */
LMCE_API int lmce_dx_finalize(const float* d_hidden_f32, int64_t n_tokens, int64_t hidden_dim, int dtype,
                     void* d_hidden, void* stream);

/* ------------------------------------------------ packing around the head */

/* Packing before the head (replaces the label shift, keep mask and compaction of
 * the patched Qwen2ForCausalLM.forward, ops.py:1107-1127). For labels [batch, seq]
 * and an optional attention mask [batch, seq] (nonzero = attended; NULL = all),
 * position t = b * seq + s has the shifted label labels[b, s + 1] (-100 for the
 * last position) and is kept when it is attended or its shifted label is not
 * -100; when no position is kept, position 0 of every row is. Kept positions are
 * compacted in order into shift_labels[0, n) and valid_idx[0, n) (= t); *count
 * (device int32) receives n and row_lengths[b] the kept positions of row b. With
 * hidden ([batch * seq, hidden_dim], dtype) and hidden_packed (same size), the
 * kept rows are gathered into hidden_packed[0, n). shift_labels and valid_idx
 * need batch * seq entries. 1 <= batch * seq <= 2^22. */
LMCE_API int lmce_pack_tokens(const int64_t* labels, const int64_t* attention_mask, int64_t batch, int64_t seq,
                              int64_t* shift_labels, int64_t* valid_idx, int32_t* row_lengths, int32_t* count,
                              const void* hidden, int64_t hidden_dim, int dtype, void* hidden_packed,
                              void* stream);

/* Scatter of the head's per-token outputs back to all `total` positions (replaces
 * ops.py:1151-1164): position valid_idx[i] gets nll[i], entropy[i], argmax[i] for
 * i < *count; every other position gets nll 0, argmax 0 and the mean entropy of
 * the kept tokens (0 when none), computed on the device. */
LMCE_API int lmce_scatter_token_outputs(const float* nll, const float* entropy, const int64_t* argmax,
                                        const int64_t* valid_idx, const int32_t* count, int64_t total,
                                        float* full_nll, float* full_entropy, int64_t* full_argmax, void* stream);

/* ------------------------------------------------ final RMSNorm + packing */

/* Final RMSNorm fused with the packing gather (the reference normalises every row
 * with rms_norm_fwd, ops.py:824 / kernels.py:124-164, before packing): for i < n,
 * n = *count when count is given (device, from lmce_pack_tokens; n_rows is then an
 * upper bound) else n_rows, with r = row_idx[i] (NULL: r = i):
 *   rstd_out[i] = rsqrt(mean(hidden[r, :]^2) + eps)            (fp32)
 *   x_out[i, :] = dtype(dtype(hidden[r, :] * rstd_out[i]) * weight)
 * hidden [rows, hidden_dim] and weight [hidden_dim] in dtype; x_out [n_rows, hidden_dim]. */
LMCE_API int lmce_rmsnorm_pack(const void* hidden, const void* weight, float eps, const int64_t* row_idx,
                               const int32_t* count, int64_t n_rows, int64_t hidden_dim, int dtype, void* x_out,
                               float* rstd_out, void* stream);

/* Its backward fused with the scatter (ops.py:850 / kernels.py:167-190): for the same
 * rows, with x_hat = hidden[r] * rstd[i], wdy = weight * d_x[i]:
 *   d_hidden[r, :] = (wdy - x_hat * mean(x_hat * wdy)) * rstd[i]
 * Rows of d_hidden that no i maps to are left unchanged (zero them first). The
 * weight's gradient is not computed (the reference keeps the norm weight frozen). */
LMCE_API int lmce_rmsnorm_backward(const void* d_x, const void* hidden, const void* weight, const float* rstd,
                                   const int64_t* row_idx, const int32_t* count, int64_t n_rows, int64_t hidden_dim,
                                   int dtype, void* d_hidden, void* stream);

/* ------------------------------------------------ tied input embedding */

/* Bytes of the workspace lmce_embedding_grad_add needs. */
LMCE_API size_t lmce_embedding_grad_workspace_bytes(int64_t n_tokens, int64_t vocab_local);

/* Gradient of a tied input embedding added into the head's dW, so the weight's two
 * contributions share one buffer instead of two [V, H] tensors that autograd adds
 * (the reference's forward lookup is HostHead.embed, hostload.py:381-386; it has no
 * weight gradient). For every position i whose token id lies in
 * [vocab_offset, vocab_offset + vocab_local):
 *   d_weight[id - vocab_offset, :] += d_embed[i, :]
 * summed per id in fp64 with the existing value and rounded once to dtype. fp16
 * values are multiples of 2^-24 below 2^16, so up to 8192 positions per id add
 * exactly and the result does not depend on their order; bf16 sums are exact
 * while one id's values in a column span less than about 2^32.
 *   d_embed    [n_tokens, hidden_dim] dtype, gradient of the lookup's output
 *   token_ids  [n_tokens] int64
 *   d_weight   [vocab_local, hidden_dim] dtype, updated in place */
LMCE_API int lmce_embedding_grad_add(const void* d_embed, const int64_t* token_ids, int64_t n_tokens,
                                     int64_t hidden_dim, int64_t vocab_local, int64_t vocab_offset, int dtype,
                                     void* d_weight, void* workspace, size_t workspace_bytes, void* stream);

/* out[i, :] = weight[token_ids[i] - vocab_offset, :] (zero rows for ids outside the
 * shard); [n_tokens, hidden_dim] of a 16-bit dtype. */
LMCE_API int lmce_embedding_lookup(const void* weight, const int64_t* token_ids, int64_t n_tokens,
                                   int64_t hidden_dim, int64_t vocab_local, int64_t vocab_offset, void* out,
                                   void* stream);

/* ----------------------------------------------- no-allocation forward */

/* Bytes of the library's fixed device scratch used by lmce_forward_noalloc. */
#define LMCE_NOALLOC_SCRATCH_BYTES (8u << 20)

/* Forward (statistics + finish) that allocates nothing. No counterpart in the
 * reference: it exists for callers that cannot allocate device memory
 * themselves — plugins inside a runtime that owns every device allocation,
 * foreign-language bindings that can only pass tensor pointers, and serving
 * loops that forbid allocation after warm-up because an allocation can stall
 * the device. Such callers pass only the inputs and outputs of
 * lmce_fwd_stats + lmce_stats_finish; the per-token partial records live in
 * a file-scope device array of LMCE_NOALLOC_SCRATCH_BYTES (8 MiB) inside this
 * library, held by every GPU that loads the library until the process exits.
 *   limit: n_tokens <= LMCE_NOALLOC_SCRATCH_BYTES / sizeof(lmce_part)
 *          (349525 tokens); larger n_tokens returns LMCE_ERR_INVALID_ARGUMENT.
 * The first call on a device looks up the array's device address (once per
 * device, with that device current); make that first call before any stream
 * capture. All calls share the one array and it keeps the last call's
 * contents: calls that overlap on the GPU (other streams, other host threads)
 * race on it and must be serialised by the caller. Nothing in it needs to
 * start at zero: every record the finish step reads is written earlier in the
 * same call. Outputs and semantics are those of lmce_stats_finish. */
LMCE_API int lmce_forward_noalloc(const void* hidden, const void* weight, const int64_t* labels, int64_t n_tokens,
                                  int64_t hidden_dim, int64_t vocab, int dtype, const float* num_items_dev,
                                  double num_items, float* lse, float* nll, float* entropy, int64_t* argmax,
                                  float* loss, float* denom, void* stream);

/* ------------------------------------------------------------ diagnostics */

/* Number of kernels this library has launched in this process (all devices). */
LMCE_API uint64_t lmce_launch_count(void);

/* Timing hook for benchmarks: process-wide, record the CUDA events
 * `begin` and `end` (cudaEvent_t passed as void*) on the call's stream right
 * before and after the main tensor-core kernel of later calls:
 *   which = 0: the statistics kernel of lmce_fwd_stats
 *   which = 1: the persistent kernel of lmce_backward
 * NULL events switch recording off. The events must already exist. */
LMCE_API int lmce_set_timing_events(int which, void* begin, void* end);

/* Role counters of the CTA-pair backward kernel; no counterpart in the reference.
 * Only a library compiled with -DLMCE_ROLE_PROFILE=1 collects them; the normal
 * build returns LMCE_ERR_UNSUPPORTED. Copies (synchronously) up to counter_bytes of
 * the per-CTA cycle counters (32 uint64 per CTA, slots in csrc/lmce_prof.cuh) and
 * up to timeline_bytes of the per-tile timeline (1024 entries of 8 uint64 per CTA),
 * then zeroes both when `reset` is non-zero. */
LMCE_API int lmce_profile_read(void* counters, size_t counter_bytes, void* timeline, size_t timeline_bytes,
                               int reset);

/* Measures how fast TMA loads reach the SMs through a ring of stages; no counterpart in the
 * reference. One CTA per SM streams `iters` stages of `stage_bytes` from `tensor` (a
 * caller-owned 16-bit [rows, cols] array, both multiples of 128, 16-byte aligned; a few tens
 * of MB stays in L2, a few hundred MB comes from DRAM) through a ring of `stages` stages
 * (2..8, stages x stage_bytes + 2 KB within 226 KB): one thread loads each stage as soon as
 * it is free, another holds each landed stage for `hold_cycles` SM cycles (a stand-in for the
 * UMMAs that read it; 0 frees it at once) and frees it. load_kind 0: 2-D {64, 128} boxes (128
 * bytes of each of 128 rows, 16 KB each); 1: 3-D {64, 128, 2} boxes (256 contiguous bytes of
 * each of 128 rows, 32 KB each), the boxes the kernels load; 2: plain bulk copies of 32
 * contiguous KB. stage_bytes must be a multiple of the piece size (16 KB for kind 0, 32 KB
 * otherwise). cycles[sm] receives the SM clock cycles of the last iters - 9 stages, so bytes
 * per clock per SM = (iters - 9) * stage_bytes / cycles[sm], and the share of time the
 * holder was busy = (iters - 9) * hold_cycles / cycles[sm]. Allocates nothing; n_cycles must
 * be at least the number of SMs. */
LMCE_API int lmce_probe_tma_pipeline(const void* tensor, int64_t rows, int64_t cols, int load_kind,
                                     int stage_bytes, int stages, int hold_cycles, int iters,
                                     unsigned long long* cycles, int64_t n_cycles, void* stream);

/* lmce_probe_tma_pipeline with three 32 KB stages freed at once; box_kind 0 or 1 as its
 * load_kind. */
LMCE_API int lmce_probe_tma_rate(const void* tensor, int64_t rows, int64_t cols, int box_kind, int iters,
                                 unsigned long long* cycles, int64_t n_cycles, void* stream);

/* Launches a kernel whose bounded wait is never satisfied; after timeout_ns it
 * records LMCE_ERR_TIMEOUT in the device error word and returns normally.
 * Exercises the failure path without hanging or faulting the GPU. */
LMCE_API int lmce_selftest_wait_timeout(uint64_t timeout_ns, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* LMCE_H_ */
