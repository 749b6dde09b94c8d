/*
 * ffa_b200.h -- C ABI of the B200-native CTC forced aligner (libffa_b200.so).
 *
 * The library aligns known CTC transcripts to fp32 emission matrices that are
 * already resident on one CUDA device.  It is the native boundary under the
 * Python package fast_forced_aligner_b200, whose align()/emission_validity()
 * mirror the reference's public API (brthor/fast-forced-aligner,
 * src/fast_forced_aligner/alignment.py:312-502).
 *
 * The reference binds its path through two TORCH_LIBRARY ops
 * (src/fast_forced_aligner/csrc/alignment.cu:1064-1070):
 *   align(Tensor[] emissions, Tensor[] targets, int[] blanks, ...)
 *       -> (Tensor[] outputs, int[] lengths)                 alignment.cu:919
 *   emission_validity(Tensor[] emissions) -> Tensor           alignment.cu:893
 * Each entry point below replaces one of them with plain pointers and sizes:
 * no torch types cross this boundary.  The caller owns every buffer: inputs
 * are borrowed, outputs and scratch are caller-allocated, and all work is
 * enqueued on the caller's stream without any host synchronisation.
 *
 * Conventions
 *   - Functions return FFA_OK (0) or a negative ffa_status.  The message of
 *     the most recent failure on the calling thread is ffa_last_error().
 *   - Per-record alignment outcomes are NOT return codes: they are written to
 *     the device `status` array (0 ok, 1 no finite path, 2 masked by the
 *     emission-validity mask, 3 invalid target IDs, 4 too few frames),
 *     exactly as the reference's status contract (alignment.py:88-94).
 *   - Thread safety: every function except ffa_align_noalloc is reentrant;
 *     concurrent calls on different streams or devices share no mutable
 *     state.  ffa_align_noalloc uses one process-wide device scratch array
 *     and one host staging array: see its own comment.  A call of optimized
 *     mode with work for both of its routes runs one route on a side stream
 *     of the calling thread and device (see ffa_outputs), so two such calls
 *     from one thread on different streams order their side-stream work one
 *     after the other; their results are unaffected.
 */
#ifndef FFA_B200_H
#define FFA_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define FFA_ABI_VERSION 2 /* 2: input formats (ffa_record.format), ffa_row_logsumexp */

#if defined(__GNUC__)
#define FFA_API __attribute__((visibility("default")))
#else
#define FFA_API
#endif

typedef struct CUstream_st* ffa_stream_t; /* == cudaStream_t; NULL = legacy default stream */

typedef enum ffa_status {
  FFA_OK = 0,
  FFA_ERR_INVALID_ARGUMENT = -1, /* malformed batch metadata (ValueError upstream) */
  FFA_ERR_UNSUPPORTED = -2,      /* sizes outside the supported limits (ValueError) */
  FFA_ERR_BUFFER_TOO_SMALL = -3, /* workspace/staging smaller than the plan needs */
  FFA_ERR_CUDA = -4,             /* a CUDA runtime call failed (RuntimeError) */
  FFA_ERR_INTERNAL = -5
} ffa_status;

typedef enum ffa_mode {
  FFA_MODE_CONVENTIONAL = 0, /* full-record max-plus Viterbi DP */
  FFA_MODE_OPTIMIZED = 1     /* greedy-bounded window DP / chunked route, exact DP fallback */
} ffa_mode;

/* Optimized mode has two routes.
 *   Window route: a greedy pass over the emission rows (per frame, the
 *     largest emission over the transcript alphabet -- the maximum the
 *     reference's greedy_shortcuts finds, alignment.cu:29-153 -- and its
 *     greedy chunk statistics), then the conventional DP restricted to a
 *     64-state window that slides up the trellis, one warp per record,
 *     certified on the device against those bounds: its outputs are then the
 *     conventional DP's, bit for bit, ties included.  Where the certificate
 *     fails, a 128-state window, then the full conventional DP.  For records
 *     whose rows can be TMA-staged (vocab <= 64, 16-byte aligned rows), with
 *     at most 4096 states and 8192 frames.
 *   Chunked route (the reference's optimized design, alignment.cu:163-228,
 *     525-592): relaxed 32-frame pieces joined at legal seams, repairs of
 *     merged regions, the full DP as fallback.
 * By default the window route takes the records of at most 2048 frames of a
 * batch with more than 4 such records per SM (where one warp per record keeps
 * the GPU busy), the chunked route the rest; the flags choose one route for
 * every record it can take. */
enum {
  FFA_FLAG_CHECK_INPUTS = 1, /* validate target IDs and frame feasibility on the device */
  FFA_FLAG_PIECE_ROUTE = 2,  /* optimized mode: the chunked route for every record */
  FFA_FLAG_WINDOW_ROUTE = 4  /* optimized mode: the window route for every record it can take */
};

/* Limits (alignment.py:237, 249-250).  The reference stops at 2047 tokens
 * (4095 states); this build also aligns longer transcripts, up to 65536 states,
 * on thread-block clusters. */
#define FFA_MAX_RECORDS 65535
#define FFA_MAX_VOCAB 8192
#define FFA_MAX_FRAMES 2147483647LL
#define FFA_MAX_TOKENS 32767

/* What a record's [frames, vocab] matrix holds.  The reference aligns fp32
 * log-probabilities (format 0); its example pipelines get them from a
 * model's logits with torch.log_softmax (examples/transformers_ctc/
 * align.py:55-56).  Formats 1 and 2 take the logits themselves and align
 * their log_softmax without writing it out: the emission of (t, v) is
 * x[t, v] - z[t], one fp32 round-to-nearest subtraction, where z[t] is row
 * t's log-sum-exp as ffa_row_logsumexp computes it.  Every record of one
 * call has the same format. */
typedef enum ffa_input_format {
  FFA_INPUT_LOG_PROBS = 0,   /* fp32 log-probabilities, used as stored */
  FFA_INPUT_LOGITS_F32 = 1,  /* fp32 logits */
  FFA_INPUT_LOGITS_BF16 = 2  /* bf16 logits (uint16 bit patterns) */
} ffa_input_format;

/* One record: a device-resident [frames, vocab] row-major emission (or
 * logits) matrix and an int64 [tokens] transcript (reference: one entry of
 * the `emissions` / `targets` tensor lists, alignment.cu:961-988). */
typedef struct ffa_record {
  const void* emissions;   /* device pointer: fp32 (formats 0, 1; 4-byte aligned) or bf16 (2-byte aligned) */
  const int64_t* targets;  /* device pointer; may be NULL when tokens == 0 */
  int64_t frames;          /* T, 1 .. FFA_MAX_FRAMES */
  int32_t vocab;           /* V, 1 .. FFA_MAX_VOCAB */
  int32_t tokens;          /* U >= 0; states S = 2U + 1 */
  int32_t blank;           /* 0 .. V-1 */
  int32_t format;          /* ffa_input_format (version 1 named it `reserved`, always 0) */
} ffa_record;

/* Caller-allocated device outputs, packed in record order without padding
 * (reference AlignmentBatch fields, alignment.py:138-148).  Diagnostics in
 * optimized mode: shortcut_stats holds the reference's greedy chunk counts
 * (accepted 128-frame chunks, their frames, chunks with several placements)
 * for every record with at most 4096 states, on either route, and 0 for the
 * others and for records of status >= 2; stitched, repair_passes, repaired_frames and reuse_stats count
 * the chunked route's joins and repairs (0 on the window route); the routing
 * state routing_stats[i, 0] is 2 when a window-route record ran the full DP as
 * fallback (the reference's completed early fallback), else 0.  When a call
 * has work for both routes, one of them runs on a per-thread side stream
 * forked from `stream` and joined back into it before ffa_align returns. */
typedef struct ffa_outputs {
  int64_t* labels;          /* [sum T] vocabulary id per frame; -1 for failed records */
  float* scores;            /* [sum T] selected emission per frame; -inf for failed */
  int32_t* status;          /* [B] */
  float* objective;         /* [B] native accumulated path score */
  int32_t* stitched;        /* [B] 1 = the chunked route joined piece paths */
  int32_t* repair_passes;   /* [B] */
  int64_t* repaired_frames; /* [B] */
  int64_t* shortcut_stats;  /* [B, 3] */
  int32_t* routing_stats;   /* [B, 3] */
  int64_t* reuse_stats;     /* [B, 4] or NULL */
} ffa_outputs;

/* Sizes a call needs, computed on the host from the batch metadata alone. */
typedef struct ffa_sizes {
  size_t staging_bytes;   /* host staging (pinned for a truly async upload) */
  size_t workspace_bytes; /* device scratch, 256-byte aligned */
  int64_t total_frames;   /* sum of T: length of labels/scores */
} ffa_sizes;

FFA_API int ffa_abi_version(void);
FFA_API const char* ffa_last_error(void);

/* ---- align (replaces torch.ops.fast_forced_aligner_cuda.align,
 *      alignment.cu:919-1061 and alignment.py:346-502) ---------------------- */

/* Host only.  Validates the batch (the reference's metadata checks,
 * alignment.py:233-252 and alignment.cu:961-971) and reports the buffer
 * sizes ffa_align needs.  Touches no device memory. */
FFA_API int ffa_align_query(const ffa_record* records, int64_t count, int mode, int flags,
                    ffa_sizes* sizes);

/* Enqueue one alignment on `stream`.
 *   emission_validity: optional device bool[count] mask (NULL = none); a
 *       false entry gives status 2 unless target validation fails
 *       (alignment.cu:836, 870-874).
 *   staging: host memory of sizes.staging_bytes.  The call writes the device
 *       descriptor table into it and enqueues its upload: from pinned (mapped)
 *       memory, a small kernel that reads the table through the buffer's
 *       device mapping in 16-byte loads -- so the buffer must be readable up
 *       to sizes.staging_bytes rounded up to a multiple of 16; from any other
 *       memory, one cudaMemcpyAsync.  Keep it unchanged until the stream has
 *       passed this call.
 *   workspace: device scratch of sizes.workspace_bytes, 256-byte aligned,
 *       not shared with concurrent work on another stream.
 * No host synchronisation, no allocation, no device-to-host transfer. */
FFA_API int ffa_align(const ffa_record* records, int64_t count, int mode, int flags,
              const uint8_t* emission_validity, const ffa_outputs* outputs,
              void* staging, size_t staging_bytes,
              void* workspace, size_t workspace_bytes, ffa_stream_t stream);

/* ---- emission_validity (replaces torch.ops.fast_forced_aligner_cuda.
 *      emission_validity, alignment.cu:879-917 and alignment.py:312-343) ---- */

/* Host only: sizes for ffa_emission_validity (targets/tokens/blank ignored). */
FFA_API int ffa_emission_validity_query(const ffa_record* records, int64_t count, ffa_sizes* sizes);

/* valid[i] = 1 unless record i holds a NaN or +inf (-inf is allowed).
 * Scans the stored fp32 values (formats 0 and 1; bf16 records are
 * rejected with FFA_ERR_UNSUPPORTED).  Same staging/workspace contract as
 * ffa_align. */
FFA_API int ffa_emission_validity(const ffa_record* records, int64_t count, uint8_t* valid,
                          void* staging, size_t staging_bytes,
                          void* workspace, size_t workspace_bytes, ffa_stream_t stream);

/* ---- allocation-free align (no counterpart in the reference, whose
 *      align always allocates its scratch with at::empty).  NOT reentrant:
 *      the reentrancy convention at the top of this header excludes it. ---- */

/* For callers that cannot allocate device memory when they align -- code
 * running inside a framework that owns every device allocation, pipelines
 * whose memory is fixed at start-up -- this runs exactly what ffa_align runs,
 * but its scratch comes from buffers built into the library instead of from
 * the caller: a 64 MiB device array (held on each GPU that loads it until
 * the process exits) and a 2 MiB static host staging array.  Inputs and
 * outputs are the caller's, as for ffa_align.  No cudaMalloc, cudaFree or
 * other allocating routine is called.
 *   - A batch whose ffa_align_query sizes exceed those limits is rejected
 *     with FFA_ERR_UNSUPPORTED and a message in ffa_last_error().
 *   - The first call on a device looks up the array's device address
 *     (cudaGetSymbolAddress) with that device current; make that first call
 *     before any stream capture.
 *   - All calls share the two buffers, and the host staging array serves
 *     every device: calls must be serialised across the whole process -- one
 *     call in flight at a time, on any GPU, from any host thread -- not only
 *     per GPU.  Calls that overlap race.  Nothing in them needs clearing
 *     between calls. */
FFA_API int ffa_align_noalloc(const ffa_record* records, int64_t count, int mode, int flags,
                              const uint8_t* emission_validity, const ffa_outputs* outputs,
                              ffa_stream_t stream);

/* ---- profiling hook (no reference counterpart: the reference exposes no
 *      per-kernel timing) --------------------------------------------------- */

/* While set, ffa_align calls made on the calling thread record `before` and
 * `after` (two cudaEvent_t created by the caller) immediately around the
 * launch that streams every emission row once, on the stream it runs on --
 * the greedy pass (after its preparation) when the call has records of the
 * window route, else the first forward pass (every piece of the chunked
 * route, every record of the conventional mode) -- so the caller can read its
 * device time with cudaEventElapsedTime.  Pass NULL, NULL to clear. */
FFA_API int ffa_profile_forward_events(void* before, void* after);

/* Number of CUDA kernels the ffa_* calls of the calling thread have launched
 * so far (monotonic).  No reference counterpart: lets a benchmark report how
 * many of this library's kernels ran in its timed region. */
FFA_API int64_t ffa_launch_count(void);

/* Phase boundaries of one ffa_align call, in launch order.  A conventional
 * call has no finishing launch; its point is recorded where it would be, so
 * that phase measures zero. */
enum {
  FFA_PROFILE_START = 0,   /* after the descriptor upload (and a logits call's row log-sum-exps) */
  FFA_PROFILE_FIRST,       /* after the first forward pass (every piece / record) */
  FFA_PROFILE_FINISH,      /* after the optimized route's seam plans, repairs and fallback */
  FFA_PROFILE_FILL,        /* after the traceback fill (and objective fold) */
  FFA_PROFILE_POINTS
};

/* While set, ffa_align calls made on the calling thread record events[k] (a
 * cudaEvent_t created by the caller) at phase boundary k, for all
 * FFA_PROFILE_POINTS boundaries.  No reference counterpart: a timing hook for
 * benchmarks.  Pass NULL, 0 to clear; any other count is an error. */
FFA_API int ffa_profile_phase_events(void* const* events, int count);

/* ---- target validation (replaces the per-record checks of the reference's
 *      validate_inputs, alignment.py:255-309) ------------------------------- */

/* Host only: sizes for ffa_check_targets. */
FFA_API int ffa_check_targets_query(const ffa_record* records, int64_t count, ffa_sizes* sizes);

/* status[i] (device int32[count]) = 3 if a target ID is outside [0, V) or
 * equals the blank, else 4 if U + adjacent repeats > T, else 0 -- the same
 * codes and precedence ffa_align writes with FFA_FLAG_CHECK_INPUTS
 * (alignment.cu:852-874).  Same staging/workspace contract as ffa_align. */
FFA_API int ffa_check_targets(const ffa_record* records, int64_t count, int32_t* status,
                              void* staging, size_t staging_bytes,
                              void* workspace, size_t workspace_bytes, ffa_stream_t stream);

/* ---- row log-sum-exp of logits (no op in the reference, whose examples
 *      apply torch.log_softmax before aligning) ---------------------------- */

/* Host only: sizes for ffa_row_logsumexp (records of format 1 or 2; targets,
 * tokens and blank are ignored). */
FFA_API int ffa_row_logsumexp_query(const ffa_record* records, int64_t count, ffa_sizes* sizes);

/* z (device float [sum frames], record i's frames in record order) = each
 * row's log-sum-exp, m + logf(sum_v __expf(x - m)) with m the row's maximum,
 * exactly the values ffa_align subtracts from logits: x - z[t] in fp32 is
 * the emission matrix it aligns.  A row holding NaN or +inf, or only -inf,
 * gets NaN.  Same staging/workspace contract as ffa_align. */
FFA_API int ffa_row_logsumexp(const ffa_record* records, int64_t count, float* z,
                              void* staging, size_t staging_bytes,
                              void* workspace, size_t workspace_bytes, ffa_stream_t stream);

/* ---- token spans (no op in the reference: its README describes the
 *      conversion, README.md:509-517) ------------------------------------- */

/* Host only: sizes for ffa_token_spans (total_frames = sum of frames). */
FFA_API int ffa_token_spans_query(const int64_t* frames, const int32_t* tokens, int64_t count,
                                  ffa_sizes* sizes);

/* From the labels ffa_align wrote (device int64 [sum frames], record i's
 * frames[i] rows in record order), each record's token spans: the frame
 * range [start, end) of its k-th run of equal non-blank labels, the frames
 * its k-th target token occupies.  spans: device int64 [sum tokens, 2], record
 * i's tokens[i] rows in record order.  A record whose non-blank run count is
 * not tokens[i] (a failed record: labels -1) gets -1 in all of its rows.
 * frames, tokens, blanks: host arrays of count entries.  Same staging /
 * workspace contract as ffa_align. */
FFA_API int ffa_token_spans(const int64_t* labels, const int64_t* frames, const int32_t* tokens,
                            const int32_t* blanks, int64_t count, int64_t* spans,
                            void* staging, size_t staging_bytes,
                            void* workspace, size_t workspace_bytes, ffa_stream_t stream);

#ifdef __cplusplus
}
#endif
#endif /* FFA_B200_H */
