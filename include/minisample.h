/*
 * libminisample — B200 token sampler behind a plain C ABI.
 *
 * This library replaces the token-sampling step of mini.js, `pickToken`
 * (src/generation.js:71-81), for a [B, V] block of fp32 logits.  Each row gets
 * exactly what `pickToken` does to one row:
 *
 *   1. repetition penalty over the row's id history   (src/generation.js:19-25, :73-75)
 *   2. greedy argmax when do_sample is false or T<=1e-4 (src/generation.js:51-55, :76)
 *   3. temperature divide                              (src/generation.js:77-79)
 *   4. softmax                                         (src/generation.js:9-17)
 *   5. top-k, top-p and the inverse-CDF draw           (src/generation.js:27-49)
 *
 * The reference binds none of this natively: it calls the JS functions above.
 * The N-API shim (omni.js_b200/csrc/napi_minisample.c) turns
 * `addon.sample(...)` into `ms_sample` calls.
 *
 * Conventions
 *   - Every entry point returns 0 on success or a negative MS_ERR_* code and
 *     leaves a message for ms_last_error().  Nothing traps, nothing falls back
 *     to a CPU implementation.
 *   - The caller owns every buffer.  The logits are never modified (the
 *     reference copies them first, src/generation.js:72).
 *   - A context is used by one host thread at a time.  Its scratch memory is
 *     shared by every call made on it: two ms_sample calls whose kernels can
 *     run at the same time (MS_DEVICE_PTRS calls on two streams with nothing
 *     ordering them) race on that scratch.  Order such calls on one stream, or
 *     give each stream its own context.
 *   - Every bounded kernel wait that runs out marks its call as failed: the
 *     rows of that call get id -1 (and MS_ROW_TIMEOUT in diag->row_flags).
 *     Top-k calls of at most 16 rows finalize each row as soon as its chunks
 *     are done, so there only the rows finalized after the wait ran out get
 *     -1 (always the row whose wait it was); the others keep correct ids.  A
 *     synchronous call (MS_HOST_PTRS, or MS_DEVICE_PTRS | MS_SYNC) then returns
 *     MS_ERR_TIMEOUT; an asynchronous device call reports it only through
 *     those -1 ids.  A later call is not affected.
 */
#ifndef MINISAMPLE_H
#define MINISAMPLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define MS_ABI_VERSION 2

/* Error codes. */
#define MS_OK            0
#define MS_ERR_ARG      -1   /* invalid argument (shape, pointer, flag)          */
#define MS_ERR_CUDA     -2   /* a CUDA runtime call failed                       */
#define MS_ERR_NCCL     -3   /* an NCCL call failed                              */
#define MS_ERR_TIMEOUT  -4   /* a bounded wait ran out                           */
#define MS_ERR_OOM      -5   /* device or pinned allocation failed               */
#define MS_ERR_STATE    -6   /* context in the wrong state / no device           */

/* ms_sample flags. */
#define MS_HOST_PTRS      0x1  /* every pointer argument is host memory                */
#define MS_DEVICE_PTRS    0x2  /* every pointer argument is device memory (ctx device 0) */
#define MS_ROW_SHARDED    0x4  /* host pointers: split the rows over all ctx devices  */
#define MS_SYNC           0x8  /* device pointers: synchronize the stream before return */
#define MS_PROFILE       0x10  /* record CUDA events around each kernel (ms_profile_read) */

/*
 * Sampling options, one set for the whole batch (the reference applies one
 * `opts` object to every step, src/generation.js:57-68).  Doubles because the
 * JS compares doubles: `T <= 0.0001`, `T !== 1.0`, `p !== 1.0`, `acc >= topP`.
 *   do_sample           0 = greedy                       (src/generation.js:60,76)
 *   temperature         divide when != 1.0               (src/generation.js:61,77-79)
 *   top_k               used when 0 < top_k < V          (src/generation.js:62,32)
 *   top_p               used when top_p != 0 and < 1     (src/generation.js:63,33)
 *   repetition_penalty  used when != 0, != 1.0 and the row history is non-empty
 *                       (src/generation.js:64,73).  The caller passes an empty
 *                       history while `generated.length == 0`.
 */
typedef struct ms_params {
    int32_t do_sample;
    double  temperature;
    int32_t top_k;
    double  top_p;
    double  repetition_penalty;
} ms_params;

/*
 * Optional per-row diagnostics.  Every pointer may be NULL; the non-NULL ones
 * are host or device memory exactly like the data pointers of the call.
 *   cand_ids/cand_probs  [B, cand_cap]: the candidates that survive top-k and
 *                        top-p, in the reference's order (prob desc, id asc),
 *                        with their fp32 softmax probabilities
 *   n_cand    [B]  number of surviving candidates (may exceed cand_cap)
 *   row_max   [B]  max of the tempered logits
 *   row_sum   [B]  softmax denominator sum(fp32(exp(x - max)))
 *   total     [B]  fp64 sum of the surviving candidates' probabilities
 *   row_flags [B]  MS_ROW_* bits below
 *   pen_logits [B, pen_ld] fp32: every row after the repetition penalty and
 *             before the temperature divide, i.e. the reference's `work` array
 *             after src/generation.js:72-75 (pen_ld >= V; for MS_HOST_PTRS
 *             calls, pen_ld is the stride of the host array)
 */
typedef struct ms_diag {
    int32_t  cand_cap;
    int32_t* cand_ids;
    float*   cand_probs;
    int32_t* n_cand;
    double*  row_max;
    double*  row_sum;
    double*  total;
    int32_t* row_flags;
    float*   pen_logits;
    int64_t  pen_ld;
} ms_diag;

#define MS_ROW_GREEDY    0x1   /* greedy argmax row                                  */
#define MS_ROW_NAN       0x2   /* softmax produced NaN (NaN/+Inf logit, all -Inf row) */
#define MS_ROW_FULLVOCAB 0x4   /* candidates ranked over the whole vocabulary        */
#define MS_ROW_SLOWPATH  0x8   /* candidate set resolved by the exact row rescan     */
#define MS_ROW_UNSETTLED 0x10  /* vocab-sharded merge: the shard lists cannot settle
                                  the row (see ms_merge_records); out_ids gets -1    */
#define MS_ROW_TIMEOUT   0x20  /* a bounded wait of this call ran out; out_ids gets -1 */

typedef struct ms_ctx ms_ctx;

/* ABI version of the loaded library (MS_ABI_VERSION). */
int ms_version(void);

/*
 * Create a context on `n_devices` CUDA devices (devices == NULL: the current
 * device only).  Replaces the reference's backend selection,
 * setBackend('cpu'|'webgl') (src/tensor.js:15-20): the 'cuda' sampler backend
 * is one context.
 */
int ms_create(ms_ctx** out, const int* devices, int n_devices);

/* Free the context, its scratch memory, streams and pinned staging buffers. */
int ms_destroy(ms_ctx* ctx);

/* Message of the last failed call on this context (never NULL). */
const char* ms_last_error(ms_ctx* ctx);

/*
 * Sample one token id per row.  Replaces `pickToken(lastLogits, generated,
 * inputIds, opts)` (src/generation.js:71-81), applied to each of B rows.
 *   logits    [B, ld] fp32, ld >= V (row stride in elements);
 *             1 <= V <= 65535 * 16384 (1,073,725,440)
 *   hist      concatenated per-row id histories (int32), may be NULL when
 *             every row is empty; ids outside [0, V) are ignored, repeated ids
 *             count once (the reference builds a Set, src/generation.js:20)
 *   hist_off  [B+1] int64 offsets into hist (NULL = no history)
 *   params    sampling options (host memory always)
 *   u         [B] fp64 uniforms in [0,1), one per row, standing in for the
 *             reference's `Math.random()` (src/generation.js:43); read only
 *             by sampled rows (may be NULL for greedy calls)
 *   out_ids   [B] int32 sampled ids
 *   diag      optional diagnostics (NULL = none)
 *   flags     MS_HOST_PTRS or MS_DEVICE_PTRS, optionally | MS_ROW_SHARDED / MS_SYNC
 *   stream    cudaStream_t for MS_DEVICE_PTRS calls (NULL = the ctx stream)
 * With MS_HOST_PTRS the call is synchronous (copies in, sample, copy out),
 * like the reference's synchronous `generateTokens` (src/generation.js:97-114).
 */
int ms_sample(ms_ctx* ctx, const float* logits, int64_t B, int64_t V, int64_t ld,
              const int32_t* hist, const int64_t* hist_off, const ms_params* params,
              const double* u, int32_t* out_ids, ms_diag* diag, int flags,
              void* stream);

/*
 * Kernel time of the calls made with MS_PROFILE since the last read, summed
 * over calls (milliseconds, CUDA events on the launch stream):
 *   stream_ms    the chunk kernel, which reads every logit once
 *   finalize_ms  the kernels after it: the per-row finalize (top-k rows), or
 *                the plan, extract and resolve kernels (whole-vocabulary
 *                rows); 0 for greedy rows and top-k calls of at most 16 rows,
 *                whose chunk kernel's last CTA of each row finalizes it (its
 *                time is then part of stream_ms)
 * In a profiled call an event sits between the two kernels, so the finalize
 * cannot start early; profile a sample of the calls, not all of them.
 * Waits for those calls' events.  No reference counterpart: the reference
 * has no profiling hooks (its demo times with performance.now(),
 * demo.template.html:230,295).
 */
int ms_profile_read(ms_ctx* ctx, double* stream_ms, double* finalize_ms, int64_t* calls);

/*
 * Kernels this context has launched (all its devices, since ms_create): per
 * ms_sample call and slice of rows (a slice holds about 2^31 / ceil(V/16384)
 * rows), one when greedy or for top-k calls of at most 16 rows, two for
 * larger top-k calls (the chunk kernel and the row finalize), four for
 * whole-vocabulary rows (chunk kernel, plan, extract,
 * resolve); one per ms_history_append.  No reference counterpart.
 */
int ms_launch_count(ms_ctx* ctx, int64_t* kernels);

/*
 * Keeps a generation loop's penalty history on the device.  Replaces the
 * reference's per-step history `inputIds.concat(generated)` (src/generation.js:
 * 73-74, grown by `generated.push(nextId)` at :105): instead of uploading it
 * every step, the caller keeps a [B, cap] int32 device buffer `hist` whose row r
 * holds the row's ids in hist[r*cap .. r*cap + len[r]) and -1 in the rest, and
 * passes it to ms_sample with hist_off[r] = r*cap (ids outside [0, V) are
 * ignored by the penalty, so the -1 slots change nothing).  This call appends
 * ids[r] to row r (ids < 0 are skipped; a full row, len[r] == cap, drops the id:
 * size cap for the prompt plus every generated id).  Device pointers, on
 * `stream` (NULL = the ctx stream), on the context's first device; asynchronous.
 * As in the reference, the penalty starts once something was generated: pass
 * no history to the first ms_sample call of a generation.
 */
int ms_history_append(ms_ctx* ctx, int32_t* hist, int32_t* len, int64_t B, int64_t cap, const int32_t* ids,
                      void* stream);

/*
 * Bytes of device scratch that ms_sample needs for a [B, V] call with these
 * params (the context allocates it on first use and keeps it).
 */
int ms_scratch_bytes(int64_t B, int64_t V, const ms_params* params, int64_t* out_bytes);

/*
 * Failure injection for testing the error paths; no reference counterpart.
 * One-shot: the setting applies to the next ms_sample call on this context.
 *   MS_INJECT_WAIT   the first chunk CTA of the next call waits `arg` (> 0)
 *                    clock cycles on an mbarrier that nothing completes, so its
 *                    bounded wait runs out: the call fails with MS_ERR_TIMEOUT
 *                    (synchronous calls) and its ids are -1; nothing is in
 *                    flight when the kernel returns
 *   MS_INJECT_ALLOC  the next device allocation of the context fails as if
 *                    cudaMalloc had, so the call returns MS_ERR_OOM
 * arg 0 clears the setting.
 */
#define MS_INJECT_WAIT  1
#define MS_INJECT_ALLOC 2
int ms_debug_inject(ms_ctx* ctx, int what, int64_t arg);

/*
 * The double exp the sampler uses for exact softmax terms, fp32(exp(x' - mx))
 * (src/generation.js:14), over n device doubles: y[i] = exp(x[i]) computed by
 * fdlibm's published method, as V8's Math.exp does.  For testing that
 * function against a host restatement; no reference counterpart.  Device
 * pointers, on `stream` (NULL = default stream); asynchronous.
 */
int ms_debug_exp(const double* x, double* y, int64_t n, void* stream);

/*
 * ms_sample without a context and without allocating.  No counterpart in the
 * reference: it exists for callers that cannot call cudaMalloc.  Examples are a
 * host program whose own allocator already reserved the device memory, or a
 * latency-critical decode loop where a cudaMalloc (which may synchronize the
 * device) is not acceptable.
 *
 * Device pointers only, on the caller's `stream` (NULL = default stream).  The
 * arguments mean what they mean for ms_sample; there are no diagnostics.
 *
 * Scratch.  The call does not allocate.  It uses a fixed device array of
 * MS_NOALLOC_SCRATCH_BYTES inside this library, which every GPU that loads the
 * library holds until the process exits.  A call whose scratch would exceed it
 * returns MS_ERR_SCRATCH; ms_scratch_bytes plus about 4*B + 512 bytes is what a
 * call needs.  Each call clears the parts that must start at zero.  Calls whose
 * work overlaps on the GPU (on different streams, or different host threads)
 * share the array and race: order them on one stream.
 *
 * Set-up.  The first call on each device looks up the array's device address
 * there (cudaGetSymbolAddress), with that device current.  Make that first call
 * before any stream capture.
 *
 * Returns MS_OK, MS_ERR_ARG, MS_ERR_SCRATCH, MS_ERR_STATE or MS_ERR_CUDA.  No
 * message is kept (there is no context).  The call returns before its kernels
 * run, so a kernel wait that runs out is not in its return code: the rows of
 * such a call come back as id -1.
 */
#define MS_NOALLOC_SCRATCH_BYTES (8u << 20)
#define MS_ERR_SCRATCH  -7   /* ms_sample_noalloc: the call needs more than MS_NOALLOC_SCRATCH_BYTES */
int ms_sample_noalloc(const float* logits, int64_t B, int64_t V, int64_t ld,
                      const int32_t* hist, const int64_t* hist_off, const ms_params* params,
                      const double* u, int32_t* out_ids, void* stream);

/*
 * Vocabulary sharding (one process and GPU per shard, the shards exchanging
 * over NCCL).  No reference counterpart: the reference samples one whole row
 * at a time.  GPU g holds columns [col0, col0 + cols) of every row.  A step is
 *   1. ms_shard_records on every GPU: its shard of each row reduced to one
 *      fixed-size record (rec_bytes from ms_shard_record_bytes): the shard's
 *      penalised max, its fast softmax partial sum, and its candidates, which
 *      are all its elements >= its k-th largest penalised logit (ties included);
 *   2. the caller exchanges records so that the GPU merging a row holds that
 *      row's record from every shard, in shard order (an all-to-all over rows);
 *   3. ms_merge_records: per row, the global max and softmax sum, the exact
 *      fp32 probabilities of the union of the candidates, top-k by
 *      (prob desc, id asc), top-p and the draw - the same id as ms_sample on the
 *      whole row, because the global top-k lies inside that union.
 * Supported: greedy rows and 0 < top_k <= 256.  A row whose candidates cannot
 * be proven sufficient (a shard's tie group at its k-th value too large, or a
 * probability outside the union tying with the k-th) gets out_ids -1 and
 * MS_ROW_UNSETTLED in diag->row_flags; the caller samples it from the whole row.
 *
 *   ms_shard_record_bytes  record size per row for these params
 *   ms_shard_records       logits: [B, ld] fp32 device pointer to the shard's
 *                          first column; hist/hist_off as for ms_sample (global
 *                          ids); records: [B, rec_bytes] device buffer
 *   ms_merge_records       records: [B, G, rec_bytes] device buffer (row-major,
 *                          then shard); u, out_ids [B] device pointers
 * Both run on `stream` (NULL = the ctx stream) on the context's first device.
 */
int ms_shard_record_bytes(int64_t V, const ms_params* params, int64_t* rec_bytes);
int ms_shard_records(ms_ctx* ctx, const float* logits, int64_t B, int64_t V, int64_t col0, int64_t cols,
                     int64_t ld, const int32_t* hist, const int64_t* hist_off, const ms_params* params,
                     void* records, int64_t rec_bytes, void* stream);
int ms_merge_records(ms_ctx* ctx, const void* records, int64_t B, int64_t G, int64_t V,
                     const ms_params* params, const double* u, int32_t* out_ids, ms_diag* diag,
                     int64_t rec_bytes, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* MINISAMPLE_H */
