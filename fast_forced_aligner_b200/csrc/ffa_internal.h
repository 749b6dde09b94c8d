// ffa_internal.h -- layouts shared by the host planner (ffa_host.cpp) and the
// sm_100a kernels (ffa_kernels.cu).  Not part of the public C ABI.
#pragma once

#include <cstddef>
#include <cstdint>

#include <cuda_runtime.h>

namespace ffa {

// DP geometry.  A record's CTC states s = 0..S-1 are owned in contiguous
// runs of K per thread (thread i owns K*i..K*i+K-1; K in {4, 8}), 32
// threads per warp, up to kMaxWarps warps per record.  With an even run length
// the first state of every run is a blank, so a thread needs only the last
// state of its left neighbour.  S <= 4096, the reference's own limit
// (alignment.cu:970).
constexpr int kMaxWarps = 16;
constexpr int kCtaThreads = 32 * kMaxWarps;  // 512
constexpr int kMaxStates = 4096;
// Frame loop unroll / emission staging granularity (frames per group).
constexpr int kGroup = 8;
// Row staging: a record's emission rows arrive by TMA bulk copy, one
// kChunkFrames-row chunk per copy, in a ring of kRowRing chunks.
constexpr int kChunkGroups = 4;
constexpr int kChunkFrames = kChunkGroups * kGroup;  // 32
constexpr int kRowRing = 3;
constexpr int kRowModeMaxVocab = 64;
// Time limit of a bounded mbarrier wait before the record is flagged as
// failed (status kStatusDeviceFault), and of the drain after such a failure.
constexpr unsigned long long kWaitNs = 500000000ull;   // 0.5 s
constexpr unsigned long long kDrainNs = 50000000ull;   // 50 ms
// Per-record status written when a bounded device wait gave up.
constexpr int kStatusDeviceFault = 5;
constexpr size_t kSmemBudget = 227 * 1024;
// Backpointers: a 2-bit jump code per state and frame (0 stay, 1 step from
// s-1, 2 skip from s-2), in one row per frame of bp_row_words(S) 32-bit
// words, state s at bits 2*(s % 16) of word s / 16.  The layout does not
// depend on how states are spread over threads, so different DPs of one
// record (wide threads for throughput, narrow ones for latency) share it.
__host__ __device__ constexpr int bp_row_words(int S) { return (S + 63) / 64 * 4; }
// Per-state arrays (frontiers, segment maps) of a record: one stride for all
// thread layouts (K <= 16, 32 threads per warp).
__host__ __device__ constexpr int state_stride(int S) { return (S + 511) / 512 * 512; }
// Long records (kMaxStates < S <= kMaxLongStates, beyond the reference's own
// limit): one thread-block cluster per record, CTA c of the cluster owning
// the kCtaThreads * K consecutive states from c * kCtaThreads * K, K = 8 or
// 16 per thread.  Each frame, the last state of CTA c reaches CTA c + 1
// through a kLinkRing-frame ring in CTA c + 1's shared memory.
constexpr int kMaxClusterCtas = 16;
constexpr int kMaxLongStates = kMaxClusterCtas * kCtaThreads * 8;  // 65536
constexpr int kLinkRing = 64;
// Traceback segment length bounds (power of two).
constexpr int kMinSegLog2 = 5;
constexpr int kMaxSegLog2 = 10;
constexpr int kFillWarps = 8;

// Device-side descriptor of one record (80 bytes).
struct RecordDev {
  const float* emissions;   // [T, V], caller memory: fp32 (formats 0, 1) or bf16 bits (format 2)
  const int64_t* targets;   // [U] int64, caller memory (may be null if U == 0)
  int64_t out_off;          // first frame of this record in labels/scores
  int64_t bp_off;           // first uint32 word of the record's backpointer rows
  int64_t map_off;          // first uint16 entry in the segment-map arena
  int32_t T, V, U, blank;
  int32_t seg_off;          // first anchor (one per traceback segment)
  uint8_t nw;               // warps running this record's DP
  uint8_t kst;              // states per thread K
  uint8_t seg_log2;         // traceback segment length H = 1 << seg_log2
  uint8_t row_mode;         // 1: TMA row staging, 0: per-thread column gather
  int64_t frontier_off;     // first float of the per-piece frontier arena
  int32_t first_piece;      // this record's pieces are first_piece ..
  int32_t num_pieces;       //   first_piece + num_pieces - 1
};
static_assert(sizeof(RecordDev) == 80, "RecordDev layout");

// Optimized route.  A record of at least kPieceMinFrames frames is cut into
// pieces of kPieceFrames frames (the last one also takes a remainder shorter
// than half a piece).  Each piece runs a relaxed DP -- free start state
// (unless it is the record's first piece), best end state (unless it is the
// last) -- and the pieces' paths are joined when every seam between them is a
// legal CTC move.  A joined path then scores the sum of the per-piece maxima,
// an upper bound on every legal path, so it is optimal.  Seams that fail
// merge their two regions, and the merged region resumes from the left
// region's end frontier (kRepairRounds rounds); records that still fail, or
// whose pieces saw NaN, run the conventional DP.
constexpr int kPieceFrames = 32;
constexpr int kPieceMinFrames = 2 * kPieceFrames + 1;
constexpr int kPieceSegLog2 = 5;
constexpr int kRepairRounds = 2;
// The first pass runs up to kMaxRunPieces consecutive pieces of a record in
// one slot, back to back (each still a separate relaxed DP), so that its
// set-up is paid once and the pass fits the GPU in about one wave.
constexpr int kMaxRunPieces = 8;
// States per thread of the DPs of a record of the optimized route (pieces,
// repairs, fallback share the record's backpointer layout): 8 or 16, chosen
// per record for the fewest instructions (wider threads amortise the
// per-frame overhead; narrower ones pad fewer states).

// One first-pass slot: piece `piece` of record `record` (frames
// [32 piece, ...) of a record of the optimized route; piece 0 = the whole
// record otherwise).  Its piece id -- the index of its PieceState -- is the
// record's first_piece + piece.
struct SlotRef {
  int32_t record;
  int32_t piece;
};
static_assert(sizeof(SlotRef) == 8, "SlotRef layout");

// Device-written state of one piece.  `start` is valid on the first piece of
// a region, `end` and `flags` on its last.
struct PieceState {
  int32_t start;
  int32_t end;
  int32_t flags;            // kPieceOk | kPieceFault
  int32_t start_skip;       // 1 if a skip into `start` is a legal CTC move
  // 1 if this piece begins a region, as planned by round k (region_start[0]:
  // after the first pass).  Round k reads entry k and writes entry k + 1, so
  // CTAs that plan the same round concurrently only write equal values into
  // an entry that nobody reads during that round.
  int32_t region_start[4];
};
static_assert(sizeof(PieceState) == 32, "PieceState layout");
enum : int32_t { kPieceOk = 1, kPieceFault = 2 };
// Per-record route of the optimized mode (device-written).
enum : int32_t { kRouteNone = 0, kRoutePending = 1, kRouteStitched = 2, kRouteFallback = 3 };

// One forward CTA ("bundle"): `count` slots of `nw` warps, each running one
// piece; all with the same states per thread, listed at
// order[first .. first+count).
struct Bundle {
  int32_t first;
  uint8_t nw;
  uint8_t count;
  uint8_t kst;
  uint8_t reserved;
};
static_assert(sizeof(Bundle) == 8, "Bundle layout");

// One traceback-fill CTA: kFillWarps consecutive segments of one record.
struct FillItem {
  int32_t record;
  int32_t first_seg;
};

// Emission-validity scan: one CTA per 64 KiB chunk (16-byte aligned) of one
// record, kScanBatch float4 loads in flight per thread.
constexpr int kScanThreads = 256;
constexpr int kScanChunkBytes = 65536;
constexpr int kScanBatch = 8;
struct ScanRecord {
  const float* data;
  int64_t count;  // elements
};
struct ScanItem {
  int32_t record;
  int32_t chunk;
};

struct OutputsDev {
  int64_t* labels;
  float* scores;
  int32_t* status;
  float* objective;
  int32_t* stitched;
  int32_t* repair_passes;
  int64_t* repaired_frames;
  int64_t* shortcut_stats;
  int32_t* routing_stats;
  int64_t* reuse_stats;  // may be null
};

// Kernel launchers (ffa_kernels.cu).  Return cudaSuccess or the launch error.
// Dynamic shared memory of a forward launch: a fixed header, then either one
// row ring per record slot (row staging) or one per-thread gather ring.
constexpr unsigned gather_ring_bytes(int K) { return kGroup * (K / 2 + 1) * kCtaThreads * 4; }
size_t forward_header_bytes();

// Finisher launch groups: (row-staged, gathered) x (128, 256, 512 threads).
constexpr int kFinishGroups = 6;

// Arguments of one forward launch.
struct ForwardParams {
  const RecordDev* recs;
  const Bundle* bundles;
  const SlotRef* order;      // first-pass slots, grouped by bundle
  const uint8_t* mask;       // emission-validity mask or null
  int32_t check_inputs;
  uint32_t* bp;
  uint16_t* maps;
  int32_t* anchors;
  // The chunked route's path: the state at each frame, as the piece and
  // repair traces found it (record r's frame t at path_states[recs[r].out_off + t]).
  int16_t* path_states;
  float* frontiers;
  PieceState* pstates;
  int32_t* route;            // per record: kRoute* (the finisher writes it)
  OutputsDev out;
  uint32_t row_slot_bytes;
  // First pass: consecutive pieces per slot of the chunked route, by
  // [row-staged][16 states per thread][warps] (run_pieces_of).
  uint8_t run_by[2][2][kMaxWarps + 1];
  int32_t* fill_done;        // per record: fill CTAs finished (zeroed by the first pass)
  int32_t* finish_done;      // per record: finisher CTAs through round 0 (zeroed by the first pass)
  // Round 0's plan in the first pass (set when the optimized route's records
  // outnumber the SMs): the record's last slot to finish plans it; a record
  // it joins is done, the others go to the finisher's list of their group
  // (finish_list + finish_base[g], finish_count[g] entries).  slot_done and
  // finish_count arrive zeroed with the descriptor upload.
  int32_t plan_first;
  int32_t finish_narrow;     // the finisher's 128/256-thread CTA groups are in use
  // The finisher also fills the traceback and folds the objective of each of
  // its records (set when every record of the route has its own 512-thread
  // finisher CTA and nothing else queues behind it: the fill launch then
  // skips them).
  int32_t fill_in_finisher;
  int32_t* slot_done;        // per record: first-pass slots finished
  int32_t* finish_list;
  int32_t* finish_count;     // [kFinishGroups]
  int32_t finish_base[kFinishGroups];
  // Logits input (formats 1, 2): row log-sum-exps, z of record r's frame t
  // at lse[recs[r].out_off + t]; null for log-probabilities.
  const float* lse;
  // Per record: its first greedy verdict, or -1 for a record the greedy pass
  // does not cover.  The greedy pass owns a covered record's shortcut
  // statistics (it may run concurrently on another stream).
  const int32_t* greedy_first;
};

// row_vocab: the vocabulary shared by every row-staged record of the
// launch, or 0 when they differ.  fmt: the call's input format
// (ffa_input_format; the same for every record).
cudaError_t launch_forward(const ForwardParams& params, int num_bundles, bool row_mode,
                           int row_vocab, int fmt, unsigned smem_bytes, cudaStream_t stream);
// Everything after the first pass of the optimized route -- seam plans,
// repair rounds, conventional fallback -- in one launch: round 0's repairs on
// ctas_per_record CTAs per listed record, the rest on the last of them.
// `threads`: 512, or 256 / 128 (records of at most 8 / 4 warps at 8 states
// per thread) when many records share the GPU and two / four CTAs per SM pay.
// `device_count` (or null): the number of listed records, written by the
// first pass; CTAs past it exit at once (`count` is then the list's room).
cudaError_t launch_finish(const ForwardParams& params, const int32_t* records, int count,
                          const int32_t* device_count, int ctas_per_record, int threads, bool row_mode,
                          int row_vocab, int fmt, unsigned smem_bytes, cudaStream_t stream);
// Traceback fill of every segment; for records of the optimized route the
// last fill CTA of the record also folds the objective of a joined path.
cudaError_t launch_fill(const RecordDev* recs, const FillItem* items, int num_items,
                        const uint32_t* bp, const int32_t* anchors, const OutputsDev& out,
                        const int32_t* route, int32_t* fill_done, const int16_t* path_states, const float* lse,
                        int fmt, cudaStream_t stream);
// Row log-sum-exps of a logits batch (fmt 1 or 2): z[i] for each of the
// `rows` frames in packed record order (records' out_off, T, V, emissions);
// max_vocab: the largest V among the records.
constexpr int kLseThreads = 256;
constexpr int kLseRowsPerWarp = 8;
cudaError_t launch_lse(const RecordDev* recs, int count, int64_t rows, int max_vocab, int fmt, float* z,
                       cudaStream_t stream);
cudaError_t launch_validity(const ScanRecord* recs, int64_t count, const ScanItem* items,
                            int64_t num_items, uint8_t* valid, cudaStream_t stream);

// Arguments of one long-record launch: `count` records, one cluster of
// `cluster` CTAs each.
struct LongParams {
  const RecordDev* recs;
  const int32_t* records;    // indices of the launch's records
  const uint8_t* mask;       // emission-validity mask or null
  int32_t check_inputs;
  uint32_t* bp;
  uint16_t* maps;
  int32_t* anchors;
  OutputsDev out;
  const float* lse;          // as ForwardParams::lse
};
// Conventional DP of long records (ffa_long.cu), K states per thread (8 or
// 16).  Returns cudaErrorInvalidClusterSize when the device cannot run one
// cluster of that many CTAs.
cudaError_t launch_long(const LongParams& params, int count, int cluster, int k, bool row_mode,
                        int row_vocab, int fmt, unsigned smem_bytes, cudaStream_t stream);
// How many such clusters the current device runs at once (0: none fit).
int long_capacity(int k, int cluster, bool row_mode, int row_vocab, int fmt, unsigned smem_bytes);
// Dynamic shared memory a long-record CTA needs besides its emission ring.
size_t long_header_bytes();

// The descriptor upload by a kernel that reads pinned host memory through
// its device mapping (no copy-engine queue); `bytes` rounded up to 16.
cudaError_t launch_upload(const void* mapped_src, void* dst, size_t bytes, cudaStream_t stream);

// ---- Window route of the optimized mode (ffa_window.cu) -------------------
// First the greedy pass: one warp per kGreedyChunk-frame chunk of a record
// finds each frame's greedy bound m[t] -- the largest emission over the
// record's transcript alphabet, the maximum the reference's greedy_shortcuts
// finds (alignment.cu:60-91) -- and, as that kernel does, whether the chunk's
// greedy labels have exactly one legal placement (the shortcut statistics).
// Then one warp per record runs the conventional DP restricted to a window of
// kWinStates consecutive states that slides up the trellis, 2 states per
// lane.  No path gains more than m[t] at frame t, so a state that leaves the
// window with prefix loss lambda = m[0] + ... + m[t] - alpha larger than the
// final path's loss plus the fp32 rounding bound cannot lie on the
// conventional DP's path; when every state that left is that far behind, the
// window DP made every decision of the full DP along its path and returned
// its exact outputs (certified).  Otherwise the record runs the full
// conventional DP (ffa_window_fallback).
constexpr int kWinWarps = 12;         // records (warps) per CTA at most (two CTAs share an SM)
constexpr int kWinStates = 64;        // window width: 32 lanes x 2 states
constexpr int kWinSlide = 16;         // states a slide moves the window by
constexpr int kWinHigh = 32;          // slide when the best state sits this far up (4 frames before)
constexpr int kWinChunk = 32;         // frames per TMA row copy = traceback segment
constexpr int kWinRing = 2;           // row copies in flight per record (a chunk takes microseconds)
constexpr int kWinMaxFrames = 8192;   // longer records take the chunked route
constexpr int kWinWideMaxFrames = 4096;  // the 128-state tier's limit (longer: the full DP)
constexpr int kGreedyChunk = 128;     // the reference's greedy chunk (alignment.py:498: chunk_frames)
constexpr int kGreedyWarps = 8;       // greedy chunks per CTA
// Greedy chunk verdict byte: bits 0-1 the reference's outcome (0 rejected, 1
// accepted, 2 several placements); bit 2 an alphabet column holds NaN or
// +inf; bit 3 a frame's bound is positive.
enum : uint8_t { kGreedyAccepted = 1, kGreedyMultiple = 2, kGreedyPoison = 4, kGreedyPositive = 8 };

struct GreedyItem {
  int32_t record;
  int32_t chunk;  // frames [kGreedyChunk chunk, ...)
};
// Per record of a greedy launch, from the greedy preparation: the
// transcript alphabet (label columns, blank included) as a 64-bit mask, and
// its token positions grouped by label: lpos[tok_off[r] + lstart[kGreedyLabels
// r + c] ..] are the positions u with label c, for the placement search.
// The greedy pass covers every record of the optimized mode with at most 64
// row-staged columns and kMaxStates states: the window route's records need
// its bounds; for the others (chunked route, short records) it computes the
// reference's shortcut statistics only, on a side stream.
constexpr int kGreedyLabels = 66;  // V + 1 <= 65 list starts, rounded up
struct GreedyParams {
  const RecordDev* recs;
  const int32_t* records;       // preparation: the launch's records, a warp each
  int64_t num_records;
  const GreedyItem* items;      // the pass: a warp per chunk
  int64_t count;
  const int32_t* greedy_first;  // per record: its first chunk's verdict
  const int32_t* tok_off;       // per record: its first token in lpos
  uint64_t* alphabet;           // per record; 0 for a record of status >= 2
  uint16_t* lpos;
  uint16_t* lstart;             // kGreedyLabels per record
  const float* lse;             // as ForwardParams::lse
  float* bound;                 // m[t] of record r's frame t at recs[r].out_off + t
  uint8_t* verdicts;            // one per chunk
  const uint8_t* mask;          // emission-validity mask or null (status 2)
  int32_t check_inputs;         // statuses 3 and 4 are checked
  int64_t* shortcut_stats;      // [count, 3]: zeroed by the preparation, counted by the pass
};
// The preparation (a warp per record) and the pass (a warp per chunk);
// `between` (or null) is recorded on the stream between the two.
cudaError_t launch_greedy(const GreedyParams& params, int row_vocab, int fmt, cudaStream_t stream,
                          cudaEvent_t between = nullptr);
// The statistics-only greedy pass of the other records of the optimized mode
// (more than 64 columns, or gathered rows): a CTA per chunk of `items`
// (count of them); it reads recs, mask, check_inputs, lse and
// shortcut_stats, which the first pass has zeroed before it runs.
// max_tokens, max_vocab: the largest transcript and row among them.
cudaError_t launch_greedy_wide(const GreedyParams& params, int max_tokens, int max_vocab, int fmt,
                               cudaStream_t stream);

// One record's slice of a window CTA's dynamic shared memory for K states
// per lane (a window of 32 K states); offsets in bytes from the slice start
// (the host sizes CTAs with the same function).  The window's backpointer
// codes are in the slice when smem_codes is set (a batch whose window
// records all fit the SMs at once: the traceback then walks shared memory),
// else in global memory (win_codes_offset), which keeps the slice small
// enough for more records per SM.
struct WinLayout {
  uint32_t ring, tok, bp, gb, map, anc, stash, path, bytes;
};
__host__ __device__ inline WinLayout win_layout(int T, int U, int V, int esize, int K, bool smem_codes) {
  auto up = [](uint32_t x, uint32_t a) { return (x + a - 1) / a * a; };
  const uint32_t groups = static_cast<uint32_t>((T + 7) / 8), segs = static_cast<uint32_t>((T + 31) / 32);
  WinLayout w{};
  uint32_t off = 0;
  w.ring = off;   off = up(off + static_cast<uint32_t>(kWinRing * kWinChunk * V * esize), 128);
  w.tok = off;    off = up(off + static_cast<uint32_t>(U) + 1, 16);  // label column of each token
  w.bp = off;     off = up(off + (smem_codes ? groups * 32 * 4 * static_cast<uint32_t>(K / 2) : 0), 16);  // per 8 frames: K/2 words a lane
  w.gb = off;     off = up(off + groups * 2, 16);        // window base per 8 frames
  w.map = off;    off = up(off + segs * 32 * static_cast<uint32_t>(K) * 2, 16);  // per segment: each state's ancestor
  w.anc = off;    off = up(off + segs * 2, 16);          // path state at each segment end
  w.stash = off;  off = up(off + kWinChunk * 4, 16);     // the top window state's score per frame of a chunk
  w.path = off;   off = up(off + static_cast<uint32_t>(T) * 2, 128);  // path state per frame
  w.bytes = off;
  return w;
}
// First word of record r's window codes in WindowParams::codes: each
// 8-frame group of the window holds K/2 words a lane (32 lanes), at most 64
// words (K = 4, the 128-state tier), so a record takes at most
// 8 (T + 7) words; 8 words per frame of the call plus 64 per record cover
// every record (out_off: the record's first frame).
__host__ __device__ inline int64_t win_codes_offset(int64_t out_off, int r) {
  return 8 * (out_off + 8 * static_cast<int64_t>(r));
}
struct WinSlot {
  int32_t record;
  uint32_t smem_off;  // the record's slice in its CTA's dynamic shared memory
};
struct WinCta {
  int32_t first;  // slots[first .. first + count)
  int32_t count;
};
struct WindowParams {
  const RecordDev* recs;
  const WinSlot* slots;
  const WinCta* ctas;
  const uint8_t* mask;
  int32_t check_inputs;
  OutputsDev out;
  const float* lse;           // as ForwardParams::lse
  const float* bound;         // the greedy pass's m[t] (GreedyParams::bound)
  uint32_t* codes;            // the windows' backpointer codes (win_codes_offset), unless smem_codes
  int32_t smem_codes;         // codes in each record's shared-memory slice (win_layout)
  const uint8_t* verdicts;    // the greedy pass's chunk verdicts
  const int32_t* greedy_first;  // per record: its first greedy item
  int32_t* fallback_list;     // records handed to the next tier
  int32_t* fallback_count;    // zeroed with the descriptor upload
  const int32_t* in_list;     // the 128-state tier: the records it takes
  const int32_t* in_count;
};
cudaError_t launch_window(const WindowParams& params, int num_ctas, int row_vocab, int fmt, unsigned smem_bytes,
                          cudaStream_t stream);
// The 128-state window over the device-written list of records the 64-state
// window did not certify (in_list, in_count); one warp per CTA, smem_bytes
// the largest record's slice.
cudaError_t launch_window_wide(const WindowParams& params, int max_count, int row_vocab, int fmt,
                               unsigned smem_bytes, cudaStream_t stream);
// The full conventional DP, traceback and outputs of each listed record
// (one CTA per record, grid-stride over the device-written list).
cudaError_t launch_window_fallback(const ForwardParams& params, const int32_t* list, const int32_t* count,
                                   int max_count, int row_vocab, int fmt, unsigned smem_bytes, cudaStream_t stream);

// Token spans: one warp per record.
struct SpanRecord {
  const int64_t* labels;  // the record's frames of an ffa_align labels output
  int64_t* spans;         // its [U, 2] rows of the spans output
  int32_t T, U, blank, reserved;
};
cudaError_t launch_spans(const SpanRecord* recs, int64_t count, cudaStream_t stream);

// Kernels launched so far by the calling thread (ffa_kernels.cu), and the
// hook every launcher calls.
int64_t launches_so_far();
void count_launch();

// Sets the message ffa_last_error() returns on this thread (ffa_host.cpp).
void set_last_error(const char* message);

cudaError_t launch_check_targets(const RecordDev* recs, int64_t count, int32_t* status,
                                 cudaStream_t stream);


}  // namespace ffa
