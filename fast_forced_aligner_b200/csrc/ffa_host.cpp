// ffa_host.cpp -- C ABI host layer of the B200-native CTC forced aligner.
//
// Replaces the reference's C++ host layer (alignment.cu:893-1061): metadata
// validation, launch planning and the single descriptor upload.  Differences
// by design:
//   - no allocation: outputs, workspace and host staging belong to the caller
//     (the torch shim hands in caching-allocator memory), so the call is
//     stream-ordered and never synchronises the host;
//   - records (or, in the optimized route, their pieces) are planned on the
//     host into packed CTAs ("bundles") of equal slot size, longest first, so
//     one launch covers a ragged batch;
//   - the planner builds every table in the caller's staging buffer in place
//     (no heap allocation), then enqueues one upload of it: a small kernel
//     reading pinned staging through its device mapping, or a cudaMemcpyAsync
//     from any other memory.
#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <string>
#include <utility>
#include <vector>

#include <cuda_runtime.h>

#include "ffa_b200.h"
#include "ffa_internal.h"

namespace {

thread_local std::string g_error;
thread_local cudaEvent_t g_profile_before = nullptr;
thread_local cudaEvent_t g_profile_after = nullptr;
thread_local cudaEvent_t g_phase_events[FFA_PROFILE_POINTS] = {};
thread_local bool g_phase_profiling = false;

// Records the phase-boundary event `point` when phase profiling is on.
cudaError_t mark_phase(int point, cudaStream_t stream) {
  if (!g_phase_profiling) return cudaSuccess;
  return cudaEventRecord(g_phase_events[point], stream);
}

int fail(int code, const std::string& message) {
  g_error = message;
  return code;
}

constexpr size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

constexpr int kKnownFlags = FFA_FLAG_CHECK_INPUTS | FFA_FLAG_PIECE_ROUTE | FFA_FLAG_WINDOW_ROUTE;

struct Geometry {
  bool window;   // optimized mode: the window DP (ffa_window.cu), full DP as fallback
  bool chunked;  // optimized mode: solved in pieces
  int cluster;   // > 0: a long record, solved by a cluster of this many CTAs
  int K;         // states per thread
  int nw;        // warps for the DP
  int seg_log2;  // traceback segment length
  int64_t segments;
  int64_t greedy_items;  // greedy pass chunks (greedy_record)
  int64_t wide_items;    // chunks of the statistics-only pass of the other records (wide_greedy_record)
  int64_t bp_words;
  int64_t map_elems;
  int64_t pieces;
  int64_t frontier_elems;
};

// States per thread.  A record that has an SM to itself (at most one record
// per SM in the batch) is latency-bound: its frame time is the per-frame
// dependency chain, shortest with 4 states per thread and up to 16 warps
// (measured: ~260 cycles per frame at 8 warps against ~280 for K = 8 at 4
// warps).  Packed records and pieces share SMs, where fewer instructions per
// state win: K = 8.
int choose_k(int64_t S, bool latency_bound) {
  if (latency_bound && S <= 32 * 4 * 16) return 4;
  return 8;
}

// States per thread for a record of the optimized route: whichever of 8 and
// 16 runs fewer instructions per frame, modelled as warps x (fixed per-frame
// cost + per-state cost x K), with warps = ceil(S / (32 K)).
int piece_k(int64_t S) {
  const int64_t cost16 = ((S + 511) >> 9) * (24 + 6 * 16), cost8 = ((S + 255) >> 8) * (24 + 6 * 8);
  return cost16 <= cost8 ? 16 : 8;
}

// Bytes per stored element of an input format (ffa_input_format).
size_t element_bytes(int format) { return format == FFA_INPUT_LOGITS_BF16 ? 2 : 4; }

// TMA row staging needs 16-byte aligned rows and a small row.
bool row_staged(const ffa_record& r) {
  return r.vocab * element_bytes(r.format) % 16 == 0 && r.vocab <= ffa::kRowModeMaxVocab &&
         (reinterpret_cast<uintptr_t>(r.emissions) & 15) == 0;
}

// Which records of the optimized mode the window DP takes: row-staged, at
// most kMaxStates states, and at most max_frames frames (0: none).  By
// default the window route runs only where it is faster: a batch with many
// records (more than kWinAutoRecordsPerSm per SM: one warp per record is a
// latency chain, so it pays where records keep every SM busy) and records of
// at most kWinAutoMaxFrames frames; FFA_FLAG_WINDOW_ROUTE gives it every
// record it can hold, FFA_FLAG_PIECE_ROUTE none.
struct WindowPolicy {
  int64_t max_frames;
};
constexpr int64_t kWinAutoRecordsPerSm = 4;
constexpr int64_t kWinAutoMaxFrames = 2048;
// Window records per SM up to which their codes stay in shared memory.
constexpr int64_t kWinSmemCodesSpread = 8;

bool window_shape(const ffa_record& r, int64_t max_frames) {
  return 2 * static_cast<int64_t>(r.tokens) + 1 <= ffa::kMaxStates && r.frames <= max_frames && row_staged(r);
}

int device_sms();
// Whether a call's window records keep their codes in global memory: they
// spread more than kWinSmemCodesSpread to an SM (the workspace planner and
// the CTA packing decide it with this one function).
bool window_codes_global(int64_t window_records) {
  const int64_t sms = device_sms();
  return window_records > 0 && (window_records + sms - 1) / sms > kWinSmemCodesSpread;
}
WindowPolicy window_policy(const ffa_record* records, int64_t count, int mode, int flags) {
  if (mode != FFA_MODE_OPTIMIZED || (flags & FFA_FLAG_PIECE_ROUTE)) return WindowPolicy{0};
  if (flags & FFA_FLAG_WINDOW_ROUTE) return WindowPolicy{ffa::kWinMaxFrames};
  int64_t n = 0;
  for (int64_t i = 0; i < count; ++i) n += window_shape(records[i], kWinAutoMaxFrames) ? 1 : 0;
  return WindowPolicy{n > kWinAutoRecordsPerSm * device_sms() ? kWinAutoMaxFrames : 0};
}

bool window_record(const ffa_record& r, const WindowPolicy& w) {
  return w.max_frames > 0 && window_shape(r, w.max_frames);
}

// Records of the optimized mode the greedy pass covers: row-staged (at most
// 64 columns: the alphabet is a 64-bit mask) with at most kMaxStates states
// (the reference's own limit).  The window route needs its bounds; for the
// other records it computes the reference's shortcut statistics.
bool greedy_record(const ffa_record& r, bool optimized) {
  return optimized && r.frames > 0 && 2 * static_cast<int64_t>(r.tokens) + 1 <= ffa::kMaxStates && row_staged(r);
}

// The other records of the optimized mode within the reference's limit (more
// than 64 columns, or rows that are not staged): the reference counts their
// greedy chunks too, so a statistics-only pass takes them.
bool wide_greedy_record(const ffa_record& r, bool optimized) {
  return optimized && r.frames > 0 && 2 * static_cast<int64_t>(r.tokens) + 1 <= ffa::kMaxStates && !row_staged(r);
}

// Records of the optimized mode solved in pieces: the rest, when long enough.
bool chunked_record(const ffa_record& r, bool optimized, const WindowPolicy& w) {
  return optimized && !window_record(r, w) && r.frames >= ffa::kPieceMinFrames;
}

// Pieces of kPieceFrames frames; the last one also takes a remainder shorter
// than half a piece.
int64_t piece_count(int64_t T) {
  int64_t C = T / ffa::kPieceFrames;
  if (T % ffa::kPieceFrames >= ffa::kPieceFrames / 2) ++C;
  return std::max<int64_t>(C, 1);
}

Geometry geometry(const ffa_record& r, bool optimized, const WindowPolicy& windows, bool latency_bound) {
  Geometry g{};
  const int64_t S = 2 * static_cast<int64_t>(r.tokens) + 1;
  if (S > ffa::kMaxStates) {
    // Long record: the conventional DP on a cluster of 4096-state CTAs.
    // (8 states per thread here; ffa_align may choose 16 for a batch whose
    // records would not all fit the GPU at once.)
    g.cluster = static_cast<int>((S + 8 * ffa::kCtaThreads - 1) / (8 * ffa::kCtaThreads));
    g.K = 8;
    g.nw = ffa::kMaxWarps;
  } else {
    g.window = window_record(r, windows);
    g.chunked = chunked_record(r, optimized, windows);
    // A window record's fallback is a whole-record DP at 8 states per thread.
    g.K = g.chunked ? piece_k(S) : (g.window ? 8 : choose_k(S, latency_bound));
    const int slot_log2 = g.K == 4 ? 7 : g.K == 8 ? 8 : 9;  // log2(32 K): states per warp
    g.nw = static_cast<int>((S + (int64_t{1} << slot_log2) - 1) >> slot_log2);
  }
  if (g.chunked) {
    g.seg_log2 = ffa::kPieceSegLog2;
  } else {
    // Segment length ~2*sqrt(T) balances the serial map walk (T/H steps)
    // against the per-segment backpointer walk (H steps): the power of two
    // nearest 2*sqrt(T) is 2^k for 2^(2k-3) <= T < 2^(2k-1).
    g.seg_log2 = ffa::kMinSegLog2;
    while (g.seg_log2 < ffa::kMaxSegLog2 && r.frames >= (int64_t{1} << (2 * (g.seg_log2 + 1) - 3)))
      ++g.seg_log2;
  }
  g.segments = (r.frames + (int64_t{1} << g.seg_log2) - 1) >> g.seg_log2;
  g.greedy_items = greedy_record(r, optimized) ? (r.frames + ffa::kGreedyChunk - 1) / ffa::kGreedyChunk : 0;
  g.wide_items = wide_greedy_record(r, optimized) ? (r.frames + ffa::kGreedyChunk - 1) / ffa::kGreedyChunk : 0;
  // Backpointer rows, frontiers and maps do not depend on the thread layout.
  const int S32 = static_cast<int>(S);
  g.bp_words = r.frames * ffa::bp_row_words(S32);
  g.map_elems = g.segments * ffa::state_stride(S32);
  g.pieces = g.chunked ? piece_count(r.frames) : 1;
  g.frontier_elems = g.chunked ? g.pieces * ffa::state_stride(S32) : 0;
  return g;
}

int check_record(const ffa_record& r, int64_t i, bool need_targets) {
  if (r.format < FFA_INPUT_LOG_PROBS || r.format > FFA_INPUT_LOGITS_BF16)
    return fail(FFA_ERR_INVALID_ARGUMENT, "record " + std::to_string(i) + ": unknown input format");
  if (r.emissions == nullptr ||
      (reinterpret_cast<uintptr_t>(r.emissions) & (element_bytes(r.format) - 1)) != 0)
    return fail(FFA_ERR_INVALID_ARGUMENT,
                "record " + std::to_string(i) + ": emissions must be a " +
                    std::to_string(element_bytes(r.format)) + "-byte aligned device pointer");
  if (r.frames < 1 || r.frames > FFA_MAX_FRAMES || r.vocab < 1 || r.vocab > FFA_MAX_VOCAB)
    return fail(FFA_ERR_UNSUPPORTED, "record " + std::to_string(i) +
                                         ": unsupported frame count or vocabulary");
  if (!need_targets) return FFA_OK;
  if (r.tokens < 0 || (r.tokens > 0 && r.targets == nullptr))
    return fail(FFA_ERR_INVALID_ARGUMENT, "record " + std::to_string(i) + ": missing targets");
  if (2 * static_cast<int64_t>(r.tokens) + 1 > ffa::kMaxLongStates || r.blank < 0 || r.blank >= r.vocab)
    return fail(FFA_ERR_UNSUPPORTED, "record " + std::to_string(i) +
                                         ": unsupported target length or blank ID");
  return FFA_OK;
}

int device_sms() {
  static std::atomic<int> cache[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  if (dev >= 0 && dev < 64) {
    int v = cache[dev].load(std::memory_order_relaxed);
    if (v > 0) return v;
  }
  int sms = 0;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms <= 0)
    sms = 148;
  if (dev >= 0 && dev < 64) cache[dev].store(sms, std::memory_order_relaxed);
  return sms;
}

// Byte layout of the staging buffer / the copy of it at the workspace start,
// followed by the device-only arenas.  The slot region holds the first-pass
// slot list and its bundles, packed back to back once their counts are known
// (it reserves room for one slot and one bundle per piece); the upload stops
// at their end.
struct AlignLayout {
  size_t recs, chunked, longs, fill, counters, win_slots, win_ctas, greedy_items, greedy_first, tok_off, greedy_recs,
      wide_items, slots, keys,
      classes,
      staging_bytes;
  size_t bp, maps, anchors, path_states, frontiers, pstates, route, fill_done, finish_done, fallback, bound, verdicts, alphabet,
      lpos, lstart, lse, win_codes, workspace_bytes;
  int64_t total_frames, num_pieces, num_chunked, num_long, fill_items, num_greedy, num_greedy_window, num_wide;
  int wide_max_tokens, wide_max_vocab;  // the largest transcript and row among the wide_greedy_record records
  int format;  // the call's input format
};

// Every record of a call has one input format (the kernels are specialised
// on it).
int common_format(const ffa_record* records, int64_t count, int* format) {
  for (int64_t i = 1; i < count; ++i)
    if (records[i].format != records[0].format)
      return fail(FFA_ERR_INVALID_ARGUMENT, "every record of a call must have the same input format");
  *format = records[0].format;
  return FFA_OK;
}

bool latency_bound(int64_t slots) { return slots <= device_sms(); }

// Sizes of one call.  Everything here is independent of the thread layout
// (states per thread), so one pass over the records suffices.
int plan_align(const ffa_record* records, int64_t count, bool optimized, const WindowPolicy& windows,
               AlignLayout* L) {
  if (records == nullptr || count < 1 || count > FFA_MAX_RECORDS)
    return fail(FFA_ERR_INVALID_ARGUMENT, "provide 1..65535 records");
  int64_t frames = 0, bp_words = 0, map_elems = 0, segments = 0, fill = 0, frontier = 0, chunked = 0,
          pieces = 0, longs = 0, greedy = 0, greedy_window = 0, tokens = 0, wide = 0, windows_n = 0;
  int wide_tokens = 0, wide_vocab = 0;
  for (int64_t i = 0; i < count; ++i) {
    const int rc = check_record(records[i], i, true);
    if (rc) return rc;
    const Geometry g = geometry(records[i], optimized, windows, false);
    frames += records[i].frames;
    bp_words += g.bp_words;
    map_elems += align_up(static_cast<size_t>(g.map_elems), 8);
    segments += g.segments;
    if (!g.window) fill += (g.segments + ffa::kFillWarps - 1) / ffa::kFillWarps;
    frontier += g.frontier_elems;
    chunked += g.chunked ? 1 : 0;
    longs += g.cluster > 0 ? 1 : 0;
    pieces += g.pieces;
    greedy += g.greedy_items;
    greedy_window += g.window ? g.greedy_items : 0;
    windows_n += g.window ? 1 : 0;
    tokens += records[i].tokens;
    wide += g.wide_items;
    if (g.wide_items > 0) {
      wide_tokens = std::max(wide_tokens, records[i].tokens);
      wide_vocab = std::max(wide_vocab, records[i].vocab);
    }
  }
  if (segments > INT32_MAX || fill > INT32_MAX || pieces > INT32_MAX)
    return fail(FFA_ERR_UNSUPPORTED, "batch exceeds the traceback segment index range");
  const int rc = common_format(records, count, &L->format);
  if (rc) return rc;
  L->total_frames = frames;
  L->num_pieces = pieces;
  L->num_chunked = chunked;
  L->num_long = longs;
  L->fill_items = fill;
  size_t off = 0;
  L->recs = off; off = align_up(off + sizeof(ffa::RecordDev) * count, 16);
  L->chunked = off; off = align_up(off + sizeof(int32_t) * chunked, 16);
  L->longs = off; off = align_up(off + sizeof(int32_t) * longs, 16);
  L->fill = off; off = align_up(off + sizeof(ffa::FillItem) * fill, 16);
  // Zeroed counters of round 0's plan in the first pass (per record, then
  // per finisher group), uploaded with the descriptors.
  // (and the window tiers' list lengths).
  L->counters = off; off = align_up(off + sizeof(int32_t) * (count + ffa::kFinishGroups + 2), 16);
  // Window route: one slot per record, at most one CTA per record.
  L->win_slots = off; off = align_up(off + sizeof(ffa::WinSlot) * count, 16);
  L->win_ctas = off; off = align_up(off + sizeof(ffa::WinCta) * count, 16);
  // Greedy pass: its chunks (the window records' first), each record's first
  // chunk verdict (-1: none) and first token, and its records (window first).
  L->greedy_items = off; off = align_up(off + sizeof(ffa::GreedyItem) * greedy, 16);
  L->greedy_first = off; off = align_up(off + sizeof(int32_t) * count, 16);
  L->tok_off = off; off = align_up(off + sizeof(int32_t) * count, 16);
  L->greedy_recs = off; off = align_up(off + sizeof(int32_t) * count, 16);
  L->num_greedy = greedy;
  L->num_greedy_window = greedy_window;
  // The statistics-only pass of the other records: its chunks.
  L->wide_items = off; off = align_up(off + sizeof(ffa::GreedyItem) * wide, 16);
  L->num_wide = wide;
  L->wide_max_tokens = wide_tokens;
  L->wide_max_vocab = wide_vocab;
  L->slots = off; off = align_up(off + (sizeof(ffa::SlotRef) + sizeof(ffa::Bundle)) * pieces + 32, 256);
  const size_t device_part = off;  // the most that is uploaded
  L->keys = off; off = align_up(off + sizeof(int32_t) * count, 16);
  L->classes = off; off = align_up(off + count, 256);
  L->staging_bytes = off;
  off = device_part;
  L->bp = off; off = align_up(off + sizeof(uint32_t) * bp_words, 256);
  L->maps = off; off = align_up(off + sizeof(uint16_t) * map_elems, 256);
  L->anchors = off; off = align_up(off + sizeof(int32_t) * segments, 256);
  L->path_states = off; off = align_up(off + (chunked ? sizeof(int16_t) * frames : 0), 256);
  L->frontiers = off; off = align_up(off + sizeof(float) * frontier, 256);
  L->pstates = off; off = align_up(off + sizeof(ffa::PieceState) * pieces, 256);
  L->route = off; off = align_up(off + sizeof(int32_t) * count, 256);
  L->fill_done = off; off = align_up(off + sizeof(int32_t) * count, 256);
  L->finish_done = off; off = align_up(off + sizeof(int32_t) * count, 256);
  L->fallback = off; off = align_up(off + sizeof(int32_t) * 2 * count, 256);  // the two tiers' lists
  L->bound = off; off = align_up(off + (greedy ? sizeof(float) * frames : 0), 256);
  L->verdicts = off; off = align_up(off + greedy, 256);
  L->alphabet = off; off = align_up(off + (greedy ? sizeof(uint64_t) * count : 0), 256);
  L->lpos = off; off = align_up(off + (greedy ? sizeof(uint16_t) * tokens : 0), 256);
  L->lstart = off; off = align_up(off + (greedy ? sizeof(uint16_t) * ffa::kGreedyLabels * count : 0), 256);
  // Logits: each frame's row log-sum-exp.
  L->lse = off; off = align_up(off + (L->format != FFA_INPUT_LOG_PROBS ? sizeof(float) * frames : 0), 256);
  // The window route's backpointer codes (ffa::win_codes_offset): 32 B per
  // frame plus 256 B per record, when they go to global memory.
  L->win_codes = off;
  off = align_up(off + (window_codes_global(windows_n) ? sizeof(uint32_t) * static_cast<size_t>(8 * (frames + 8 * count))
                                                      : 0),
                 256);
  L->workspace_bytes = off;
  return FFA_OK;
}

// Slot class of a record: row staging, route, states per thread and warps,
// packed so that ascending order puts row-staged before gathered, pieces of
// the optimized route before whole records, K = 4 before K = 8 and wider
// slots (longer transcripts, usually longer records) first.
uint8_t slot_class(const ffa::RecordDev& d) {
  return static_cast<uint8_t>((d.row_mode ? 0u : 1u) << 7 | (d.num_pieces > 1 ? 0u : 1u) << 6 |
                              (d.kst == 4 ? 0u : 1u) << 5 | static_cast<uint32_t>(ffa::kMaxWarps - d.nw));
}
bool class_row(uint8_t cls) { return (cls >> 7) == 0; }
int class_warps(uint8_t cls) { return ffa::kMaxWarps - (cls & 31); }

// Length bucket of a record: 16 buckets per power of two (about 6% wide),
// exact below 16 frames; always below kLengthBuckets.
constexpr int kLengthBuckets = 512;
inline int length_bucket(uint32_t T) {
  if (T < 16) return static_cast<int>(T);
  const int msb = 31 - __builtin_clz(T);
  return (msb - 3) << 4 | static_cast<int>((T >> (msb - 4)) & 15);
}

// Record order for packing: by slot class, then longest first (by length
// bucket; ties keep index order), written to `sorted`.  A counting sort over
// the (class, bucket) cells of the classes present: the cells of consecutive
// records differ, so no pass is serialised on one counter the way a radix
// pass over a few classes is.
void sort_records(const ffa::RecordDev* recs, const uint8_t* classes, int64_t count, int32_t* sorted) {
  int16_t index[256];
  std::fill_n(index, 256, static_cast<int16_t>(-1));
  for (int64_t i = 0; i < count; ++i) index[classes[i]] = 0;
  int used = 0;
  for (int c = 0; c < 256; ++c)
    if (index[c] == 0) index[c] = static_cast<int16_t>(used++);
  thread_local std::vector<int32_t> cells;
  cells.assign(static_cast<size_t>(used) * kLengthBuckets, 0);
  auto cell = [&](int64_t i) {
    return static_cast<size_t>(index[classes[i]]) * kLengthBuckets +
           (kLengthBuckets - 1 - length_bucket(static_cast<uint32_t>(recs[i].T)));
  };
  for (int64_t i = 0; i < count; ++i) ++cells[cell(i)];
  int32_t sum = 0;
  for (int32_t& c : cells) { const int32_t h = c; c = sum; sum += h; }
  for (int64_t i = 0; i < count; ++i) sorted[cells[cell(i)]++] = static_cast<int32_t>(i);
}

// Slots of the optimized route's records per slot class, as a function of
// the run length M (pieces per slot): a record of P pieces takes ceil(P / M)
// slots.  Piece counts below kBins are histogrammed per class, so evaluating
// one M costs O(classes x largest count) rather than O(records).
class RunLengthModel {
 public:
  static constexpr int kBins = 256;
  RunLengthModel() { std::fill_n(index_, 256, static_cast<int16_t>(-1)); }
  void reset() {
    for (int c = 0; c < nused_; ++c) index_[used_[c]] = -1;
    nused_ = 0;
    big_.clear();
  }
  void add(uint8_t cls, int64_t pieces) {
    const int k = slot(cls);
    if (pieces < kBins) {
      ++hist_[static_cast<size_t>(k) * kBins + pieces];
      maxp_[k] = std::max<int>(maxp_[k], static_cast<int>(pieces));
    } else {
      big_.push_back({k, pieces});
    }
  }
  void add_whole(uint8_t cls) { ++whole_[slot(cls)]; }
  // CTAs of the first pass at run length m when a CTA holds at most
  // capacity(cls) slots of its class.
  template <typename Capacity>
  int64_t ctas(int m, Capacity capacity) const {
    int64_t slots[256];
    for (int c = 0; c < nused_; ++c) {
      int64_t n = whole_[c];
      const int32_t* h = hist_.data() + static_cast<size_t>(c) * kBins;
      for (int p = 1; p <= maxp_[c]; ++p) n += h[p] * ((p + m - 1) / m);
      slots[c] = n;
    }
    for (const auto& b : big_) slots[b.first] += (b.second + m - 1) / m;
    int64_t total = 0;
    for (int c = 0; c < nused_; ++c) {
      const int64_t cap = capacity(used_[c]);
      total += (slots[c] + cap - 1) / cap;
    }
    return total;
  }

 private:
  int slot(uint8_t cls) {
    if (index_[cls] < 0) {
      index_[cls] = static_cast<int16_t>(nused_);
      used_[nused_] = cls;
      whole_[nused_] = 0;
      maxp_[nused_] = 0;
      if (hist_.size() < static_cast<size_t>(nused_ + 1) * kBins)
        hist_.resize(static_cast<size_t>(nused_ + 1) * kBins);
      std::fill_n(hist_.begin() + static_cast<size_t>(nused_) * kBins, kBins, 0);
      ++nused_;
    }
    return index_[cls];
  }
  int16_t index_[256];
  uint8_t used_[256] = {};
  int64_t whole_[256] = {};
  int maxp_[256] = {};
  int nused_ = 0;
  std::vector<int32_t> hist_;
  std::vector<std::pair<int, int64_t>> big_;
};

struct ScanLayout {
  size_t recs, items, staging_bytes, workspace_bytes;
  int64_t num_items;
};

int64_t scan_chunks(const ffa_record& r) {
  const uintptr_t base = reinterpret_cast<uintptr_t>(r.emissions);  // fp32 (checked by plan_scan)
  const uintptr_t end = base + static_cast<uintptr_t>(r.frames) * r.vocab * 4;
  const uintptr_t aligned = base & ~static_cast<uintptr_t>(15);
  return static_cast<int64_t>((end - aligned + ffa::kScanChunkBytes - 1) / ffa::kScanChunkBytes);
}

int plan_scan(const ffa_record* records, int64_t count, ScanLayout* L) {
  if (records == nullptr || count < 1 || count > FFA_MAX_RECORDS)
    return fail(FFA_ERR_INVALID_ARGUMENT, "provide 1..65535 emission records");
  int64_t items = 0;
  for (int64_t i = 0; i < count; ++i) {
    const int rc = check_record(records[i], i, false);
    if (rc) return rc;
    if (records[i].format == FFA_INPUT_LOGITS_BF16)
      return fail(FFA_ERR_UNSUPPORTED, "the emission-validity scan reads fp32 records only");
    const int64_t chunks = scan_chunks(records[i]);
    if (chunks > INT32_MAX) return fail(FFA_ERR_UNSUPPORTED, "record too large to scan");
    items += chunks;
  }
  if (items > INT32_MAX) return fail(FFA_ERR_UNSUPPORTED, "batch too large to scan");
  L->num_items = items;
  size_t off = 0;
  L->recs = off; off = align_up(off + sizeof(ffa::ScanRecord) * count, 16);
  L->items = off; off = align_up(off + sizeof(ffa::ScanItem) * items, 256);
  L->staging_bytes = off;
  L->workspace_bytes = off;
  return FFA_OK;
}

// The descriptor upload.  From pinned staging a small kernel reads the bytes
// through the buffer's device mapping, so the upload never waits in a copy
// engine's queue behind a large copy another stream has submitted (the next
// batch's emissions, say); from any other staging it is a plain
// cudaMemcpyAsync.  The workspace has room for the upload rounded up to 16
// bytes, and so has the staging buffer.
cudaError_t upload_descriptors(void* dst, const void* staging, size_t bytes, cudaStream_t s) {
  cudaPointerAttributes attr{};
  if (cudaPointerGetAttributes(&attr, staging) == cudaSuccess && attr.type == cudaMemoryTypeHost &&
      attr.devicePointer != nullptr && (reinterpret_cast<uintptr_t>(attr.devicePointer) & 15) == 0)
    return ffa::launch_upload(attr.devicePointer, dst, bytes, s);
  (void)cudaGetLastError();  // a failed attribute query leaves no error behind
  return cudaMemcpyAsync(dst, staging, bytes, cudaMemcpyHostToDevice, s);
}

// A side stream and two events per host thread and device: a call whose
// records take both optimized routes runs the window route there, forked
// from and joined back into the caller's stream, so the two routes' kernels
// share the GPU instead of queueing behind each other.
struct SideStream {
  cudaStream_t stream = nullptr;
  cudaEvent_t fork = nullptr, join = nullptr;
  cudaEvent_t first_pass = nullptr;  // the first pass is done (the statistics-only wide pass waits for it)
};
cudaError_t side_stream(SideStream** out) {
  thread_local SideStream sides[64];
  int dev = 0;
  cudaError_t err = cudaGetDevice(&dev);
  if (err != cudaSuccess) return err;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  SideStream& side = sides[dev];
  if (side.stream == nullptr) {
    if ((err = cudaStreamCreateWithFlags(&side.stream, cudaStreamNonBlocking)) != cudaSuccess) return err;
    if ((err = cudaEventCreateWithFlags(&side.fork, cudaEventDisableTiming)) != cudaSuccess) return err;
    if ((err = cudaEventCreateWithFlags(&side.join, cudaEventDisableTiming)) != cudaSuccess) return err;
    if ((err = cudaEventCreateWithFlags(&side.first_pass, cudaEventDisableTiming)) != cudaSuccess) return err;
  }
  *out = &side;
  return cudaSuccess;
}

int cuda_fail(cudaError_t err, const char* what) {
  return fail(FFA_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(err));
}

}  // namespace

void ffa::set_last_error(const char* message) { g_error = message; }

namespace {
int check_spans(const int64_t* frames, const int32_t* tokens, int64_t count, int64_t* total) {
  if (frames == nullptr || tokens == nullptr || count < 1 || count > FFA_MAX_RECORDS)
    return fail(FFA_ERR_INVALID_ARGUMENT, "provide 1..65535 frame and token counts");
  int64_t n = 0;
  for (int64_t i = 0; i < count; ++i) {
    if (frames[i] < 1 || frames[i] > INT32_MAX || tokens[i] < 0 || tokens[i] > FFA_MAX_TOKENS)
      return fail(FFA_ERR_UNSUPPORTED, "record " + std::to_string(i) + ": unsupported frame or token count");
    n += frames[i];
  }
  *total = n;
  return FFA_OK;
}
size_t spans_bytes(int64_t count) { return align_up(sizeof(ffa::SpanRecord) * static_cast<size_t>(count), 256); }
}  // namespace

extern "C" {

int ffa_abi_version(void) { return FFA_ABI_VERSION; }

const char* ffa_last_error(void) { return g_error.c_str(); }

int ffa_profile_forward_events(void* before, void* after) {
  if ((before == nullptr) != (after == nullptr))
    return fail(FFA_ERR_INVALID_ARGUMENT, "pass two events or none");
  g_profile_before = static_cast<cudaEvent_t>(before);
  g_profile_after = static_cast<cudaEvent_t>(after);
  return FFA_OK;
}

int64_t ffa_launch_count(void) { return ffa::launches_so_far(); }

int ffa_profile_phase_events(void* const* events, int count) {
  if (events == nullptr && count == 0) {
    g_phase_profiling = false;
    return FFA_OK;
  }
  if (events == nullptr || count != FFA_PROFILE_POINTS)
    return fail(FFA_ERR_INVALID_ARGUMENT, "pass FFA_PROFILE_POINTS events, or NULL and 0");
  for (int k = 0; k < count; ++k) {
    if (events[k] == nullptr) return fail(FFA_ERR_INVALID_ARGUMENT, "profile events must not be NULL");
    g_phase_events[k] = static_cast<cudaEvent_t>(events[k]);
  }
  g_phase_profiling = true;
  return FFA_OK;
}

int ffa_align_query(const ffa_record* records, int64_t count, int mode, int flags,
                    ffa_sizes* sizes) {
  if (sizes == nullptr) return fail(FFA_ERR_INVALID_ARGUMENT, "sizes must not be NULL");
  if (mode != FFA_MODE_CONVENTIONAL && mode != FFA_MODE_OPTIMIZED)
    return fail(FFA_ERR_INVALID_ARGUMENT, "mode must be conventional or optimized");
  if (flags & ~kKnownFlags) return fail(FFA_ERR_INVALID_ARGUMENT, "unknown flags");
  AlignLayout L{};
  const bool optimized = mode == FFA_MODE_OPTIMIZED;
  if (records == nullptr || count < 1 || count > FFA_MAX_RECORDS)
    return fail(FFA_ERR_INVALID_ARGUMENT, "provide 1..65535 records");
  const int rc = plan_align(records, count, optimized, window_policy(records, count, mode, flags), &L);
  if (rc) return rc;
  sizes->staging_bytes = L.staging_bytes;
  sizes->workspace_bytes = L.workspace_bytes;
  sizes->total_frames = L.total_frames;
  return FFA_OK;
}

int ffa_align(const ffa_record* records, int64_t count, int mode, int flags,
              const uint8_t* emission_validity, const ffa_outputs* outputs,
              void* staging, size_t staging_bytes,
              void* workspace, size_t workspace_bytes, ffa_stream_t stream) {
  if (outputs == nullptr || outputs->labels == nullptr || outputs->scores == nullptr ||
      outputs->status == nullptr || outputs->objective == nullptr || outputs->stitched == nullptr ||
      outputs->repair_passes == nullptr || outputs->repaired_frames == nullptr ||
      outputs->shortcut_stats == nullptr || outputs->routing_stats == nullptr)
    return fail(FFA_ERR_INVALID_ARGUMENT, "every output buffer except reuse_stats is required");
  if (mode != FFA_MODE_CONVENTIONAL && mode != FFA_MODE_OPTIMIZED)
    return fail(FFA_ERR_INVALID_ARGUMENT, "mode must be conventional or optimized");
  if (flags & ~kKnownFlags) return fail(FFA_ERR_INVALID_ARGUMENT, "unknown flags");
  if ((flags & FFA_FLAG_PIECE_ROUTE) && (flags & FFA_FLAG_WINDOW_ROUTE))
    return fail(FFA_ERR_INVALID_ARGUMENT, "choose one of the piece and window routes");
  const bool optimized = mode == FFA_MODE_OPTIMIZED;
  if (records == nullptr || count < 1 || count > FFA_MAX_RECORDS)
    return fail(FFA_ERR_INVALID_ARGUMENT, "provide 1..65535 records");
  const WindowPolicy windows = window_policy(records, count, mode, flags);
  AlignLayout L{};
  int rc = plan_align(records, count, optimized, windows, &L);
  if (rc) return rc;
  if (staging == nullptr || staging_bytes < L.staging_bytes)
    return fail(FFA_ERR_BUFFER_TOO_SMALL, "staging buffer smaller than ffa_align_query reports");
  if (workspace == nullptr || workspace_bytes < L.workspace_bytes ||
      (reinterpret_cast<uintptr_t>(workspace) & 255) != 0)
    return fail(FFA_ERR_BUFFER_TOO_SMALL, "workspace missing, too small or not 256-byte aligned");

  auto* host = static_cast<unsigned char*>(staging);
  auto* recs = reinterpret_cast<ffa::RecordDev*>(host + L.recs);
  auto* chunked = reinterpret_cast<int32_t*>(host + L.chunked);
  auto* longs = reinterpret_cast<int32_t*>(host + L.longs);
  auto* fill = reinterpret_cast<ffa::FillItem*>(host + L.fill);
  auto* classes = reinterpret_cast<uint8_t*>(host + L.classes);
  const int64_t P = L.num_pieces;

  // Per-record descriptors, fill items and arena offsets.
  int64_t out_off = 0, bp_off = 0, map_off = 0, seg_off = 0, nfill = 0, frontier_off = 0;
  int64_t np = 0, nchunked = 0;
  const bool lat = latency_bound(P);
  const int fmt = L.format;
  const size_t esize = element_bytes(fmt);  // bytes per stored element
  unsigned max_row_vocab = 0;
  int row_vocab = -1;  // common vocabulary of the row-staged records, 0 if mixed
  thread_local RunLengthModel runs_model;
  runs_model.reset();
  // Long records, keyed for their launches: (gathered, K = 16, cluster size,
  // index).
  thread_local std::vector<uint64_t> long_keys;
  long_keys.clear();
  thread_local std::vector<int32_t> win_records;
  win_records.clear();
  auto* gitems = reinterpret_cast<ffa::GreedyItem*>(host + L.greedy_items);
  auto* gfirst = reinterpret_cast<int32_t*>(host + L.greedy_first);
  auto* tokoff = reinterpret_cast<int32_t*>(host + L.tok_off);
  auto* grecs = reinterpret_cast<int32_t*>(host + L.greedy_recs);
  auto* witems = reinterpret_cast<ffa::GreedyItem*>(host + L.wide_items);
  int64_t nwide = 0;
  // Greedy chunks: the window records' from 0, the others' after them.
  int64_t ngreedy = 0, nstats_items = 0, ntok = 0;
  int64_t unchunked_fill = 0;  // records off both optimized routes (the fill launch's own)
  thread_local std::vector<int32_t> stats_records;  // greedy records off the window route
  stats_records.clear();
  int stats_vocab = -1;  // their common vocabulary, 0 if mixed
  for (int64_t i = 0; i < count; ++i) {
    const ffa_record& r = records[i];
    const Geometry g = geometry(r, optimized, windows, lat);
    ffa::RecordDev d{};
    d.emissions = static_cast<const float*>(r.emissions);  // bf16 bits for format 2
    d.targets = r.targets;
    d.out_off = out_off;
    d.bp_off = bp_off;
    d.map_off = map_off;
    d.T = static_cast<int32_t>(r.frames);
    d.V = r.vocab;
    d.U = r.tokens;
    d.blank = r.blank;
    d.seg_off = static_cast<int32_t>(seg_off);
    d.nw = static_cast<uint8_t>(g.nw);
    d.kst = static_cast<uint8_t>(g.K);
    d.seg_log2 = static_cast<uint8_t>(g.seg_log2);
    d.row_mode = row_staged(r) ? 1 : 0;
    d.frontier_off = frontier_off;
    d.first_piece = static_cast<int32_t>(np);
    d.num_pieces = static_cast<int32_t>(g.pieces);
    recs[i] = d;
    const uint8_t cls = slot_class(d);
    classes[i] = cls;
    if (d.row_mode) {
      max_row_vocab = std::max<unsigned>(max_row_vocab, r.vocab);
      row_vocab = (row_vocab < 0 || row_vocab == r.vocab) ? r.vocab : 0;
    }
    if (g.cluster > 0) {
      long_keys.push_back(static_cast<uint64_t>(i));  // keyed below, once the batch is known
    } else if (g.window) {
      win_records.push_back(static_cast<int32_t>(i));
    } else if (g.chunked) {
      ++nchunked;
      runs_model.add(cls, g.pieces);
    } else {
      runs_model.add_whole(cls);
    }
    gfirst[i] = -1;
    if (g.greedy_items > 0) {
      int64_t first = ngreedy;
      if (!g.window) {
        first = L.num_greedy_window + nstats_items;
        nstats_items += g.greedy_items;
        stats_records.push_back(static_cast<int32_t>(i));
        stats_vocab = (stats_vocab < 0 || stats_vocab == r.vocab) ? r.vocab : 0;
      } else {
        ngreedy += g.greedy_items;
      }
      gfirst[i] = static_cast<int32_t>(first);
      tokoff[i] = static_cast<int32_t>(ntok);
      ntok += r.tokens;
      for (int64_t k = 0; k < g.greedy_items; ++k)
        gitems[first + k] = ffa::GreedyItem{static_cast<int32_t>(i), static_cast<int32_t>(k)};
    }
    for (int64_t k = 0; k < g.wide_items; ++k)
      witems[nwide++] = ffa::GreedyItem{static_cast<int32_t>(i), static_cast<int32_t>(k)};
    np += g.pieces;
    if (!g.window && !g.chunked) ++unchunked_fill;
    if (!g.window)
      for (int64_t s = 0; s < g.segments; s += ffa::kFillWarps)
        fill[nfill++] = ffa::FillItem{static_cast<int32_t>(i), static_cast<int32_t>(s)};
    out_off += r.frames;
    bp_off += g.bp_words;
    map_off += static_cast<int64_t>(align_up(static_cast<size_t>(g.map_elems), 8));
    seg_off += g.segments;
    frontier_off += g.frontier_elems;
  }

  std::copy(win_records.begin(), win_records.end(), grecs);
  std::copy(stats_records.begin(), stats_records.end(), grecs + win_records.size());
  std::memset(host + L.counters, 0, sizeof(int32_t) * (count + ffa::kFinishGroups + 2));
  const size_t header = ffa::forward_header_bytes();  // 128-byte aligned ring offset
  const unsigned row_slot_bytes = static_cast<unsigned>(
      align_up(static_cast<size_t>(ffa::kRowRing) * ffa::kChunkFrames * max_row_vocab * esize, 128));
  const int64_t row_slots =
      row_slot_bytes ? std::max<int64_t>(1, static_cast<int64_t>((ffa::kSmemBudget - header) / row_slot_bytes))
                     : ffa::kMaxWarps;
  // Pieces per first-pass slot: the fewest that let the pass fit the GPU in
  // one wave of CTAs (each slot still restarts a relaxed DP every piece).
  // A CTA holds slots of one class only, up to kMaxWarps warps (and, when
  // row-staged, up to row_slots rings); one CTA runs per SM.
  const int64_t sms = device_sms();
  auto slots_per_cta = [&](uint8_t cls) {
    int64_t c = ffa::kMaxWarps / class_warps(cls);
    if (class_row(cls)) c = std::min(c, row_slots);
    return c;
  };
  (void)slots_per_cta;
  (void)runs_model;
  // A slot's work per frame, fitted to per-CTA times measured on a B200
  // (cfg1, CTAs of 4 to 16 slots sharing an SM): about 22.6 + 1.06 K ns per
  // warp at K states per thread, plus 10.6 ns per slot (its barrier and
  // boundary exchange) -- in units of about 1.06 ns, nw (21 + K) + 10.
  auto frame_cost = [](const ffa::RecordDev& d) {
    return static_cast<int64_t>(d.nw) * (21 + static_cast<int64_t>(d.kst)) + 10;
  };
  // Pieces per slot of the chunked route, per (staging, states per thread,
  // warps) class: as many as make a CTA full of the class's slots (kMaxWarps
  // warps, or row_slots rings) about one SM's share of the pass's work, so
  // that the classes' CTAs take about the same time; each piece of a slot
  // still restarts its relaxed DP.
  uint8_t run_by[2][2][ffa::kMaxWarps + 1];
  std::fill_n(&run_by[0][0][0], sizeof(run_by), static_cast<uint8_t>(1));
  auto run_of = [&](const ffa::RecordDev& d) -> int32_t {
    return d.num_pieces > 1 ? run_by[d.row_mode ? 1 : 0][d.kst == 16 ? 1 : 0][d.nw] : 1;
  };
  auto first_pass = [&](int32_t i) {
    return 2 * recs[i].U + 1 <= ffa::kMaxStates && !window_record(records[i], windows);
  };
  if (nchunked > 0) {
    int64_t total = 0;
    for (int64_t i = 0; i < count; ++i)
      if (first_pass(static_cast<int32_t>(i))) total += recs[i].T * frame_cost(recs[i]);
    const double share = static_cast<double>(total) / static_cast<double>(sms);
    for (int row = 0; row < 2; ++row)
      for (int k16 = 0; k16 < 2; ++k16)
        for (int nw = 1; nw <= ffa::kMaxWarps; ++nw) {
          int64_t cap = ffa::kMaxWarps / nw;
          if (row) cap = std::min(cap, row_slots);
          const double per_piece = static_cast<double>(cap) * ffa::kPieceFrames *
                                   static_cast<double>(nw * (21 + (k16 ? 16 : 8)) + 10);
          run_by[row][k16][nw] = static_cast<uint8_t>(
              std::clamp<int64_t>(std::llround(share / per_piece), 1, ffa::kMaxRunPieces));
        }
  }

  // Packing order: records by slot class, longest first; a record's pieces
  // stay together.  Slots of one class form one contiguous run.
  auto* sorted = reinterpret_cast<int32_t*>(host + L.keys);
  sort_records(recs, classes, count, sorted);
  struct ClassRun {
    int64_t first, slots;
    uint8_t cls, kst;
  };
  thread_local std::vector<ClassRun> runs;
  auto* order = reinterpret_cast<ffa::SlotRef*>(host + L.slots);
  int64_t n_first = 0;
  auto build_order = [&]() {
    runs.clear();
    n_first = 0;
    for (int64_t k = 0; k < count; ++k) {
      const int32_t i = sorted[k];
      const ffa::RecordDev& d = recs[i];
      if (!first_pass(i)) continue;  // long records run on clusters; window records on their route
      const int64_t before = n_first;
      const int32_t step = run_of(d);
      for (int32_t j = 0; j < d.num_pieces; j += step) order[n_first++] = ffa::SlotRef{i, j};
      if (runs.empty() || runs.back().cls != classes[i])
        runs.push_back(ClassRun{before, 0, classes[i], d.kst});
      runs.back().slots += n_first - before;
    }
  };
  build_order();
  // Records of the optimized route for the finisher, one launch per group:
  // row-staged before gathered, then by CTA size.  A record's CTA runs its
  // repair jobs in slots side by side, so every record gets a 512-thread CTA
  // unless the records outnumber the SMs more than 32 times (throughput-
  // bound): then smaller CTAs share an SM, 128 threads for records whose
  // repairs need at most 4 warps (8 states per thread), 256 for at most 8.
  // (Finisher on B200, cfg4 records on one GPU, 512-thread CTAs against the
  // smaller ones: 1031 records 221 vs 306 us, 2063: 296 vs 354, 4128: 440
  // vs 450, 8256: 737 vs 540.)
  const bool many_chunked = nchunked > 32 * sms;
  auto finish_threads = [&](const ffa::RecordDev& d) {
    const int nw8 = (2 * d.U + 1 + 255) / 256;
    if (!many_chunked) return ffa::kCtaThreads;
    if (nw8 <= ffa::kMaxWarps / 4) return ffa::kCtaThreads / 4;
    return nw8 <= ffa::kMaxWarps / 2 ? ffa::kCtaThreads / 2 : ffa::kCtaThreads;
  };
  auto group_threads = [](int grp) { return ffa::kCtaThreads >> (2 - grp % 3); };
  int64_t finish_end[ffa::kFinishGroups] = {}, nc = 0;
  for (int grp = 0; grp < ffa::kFinishGroups; ++grp) {
    const bool row = grp < 3;
    for (int64_t i = 0; i < count; ++i)
      if (recs[i].num_pieces > 1 && (recs[i].row_mode != 0) == row && finish_threads(recs[i]) == group_threads(grp))
        chunked[nc++] = static_cast<int32_t>(i);
    finish_end[grp] = nc;
  }
  // CTAs of the first pass: each class run cut into consecutive slots whose
  // work stays within one budget, the smallest that still fits one wave (one
  // CTA per SM), so that the SMs finish together.  A slot's work per frame,
  // fitted to per-CTA times measured on a B200 (cfg1, CTAs of 4 to 16 slots
  // sharing an SM): about 22.6 + 1.06 K ns per warp at K states per thread,
  // plus 10.6 ns per slot (its barrier and boundary exchange) -- in units of
  // about 1.06 ns, nw (21 + K) + 10 -- times its frames.
  auto slot_cost = [&](int64_t s) -> int64_t {
    const ffa::RecordDev& d = recs[order[s].record];
    const int32_t m = run_of(d);
    const int64_t first = static_cast<int64_t>(order[s].piece) * ffa::kPieceFrames;
    const int64_t frames = d.num_pieces > 1 && order[s].piece + m < d.num_pieces
                               ? static_cast<int64_t>(m) * ffa::kPieceFrames
                               : d.T - first;
    return frame_cost(d) * frames;
  };
  // Cuts one class run at `budget` (and at kMaxWarps warps and, row-staged,
  // row_slots rings per CTA); emit(first slot, slots) for each CTA.
  auto cut = [&](const ClassRun& run, int64_t budget, auto&& emit) {
    const int nw = class_warps(run.cls);
    int64_t cap = ffa::kMaxWarps / nw;
    if (class_row(run.cls)) cap = std::min(cap, row_slots);
    int64_t first = run.first, m = 0, work = 0;
    for (int64_t k = run.first; k < run.first + run.slots; ++k) {
      const int64_t c = slot_cost(k);
      if (m > 0 && (m == cap || work + c > budget)) {
        emit(first, m);
        first = k;
        m = 0;
        work = 0;
      }
      ++m;
      work += c;
    }
    if (m > 0) emit(first, m);
  };
  auto ctas_for = [&](int64_t budget) {
    int64_t n = 0;
    for (const ClassRun& run : runs) cut(run, budget, [&](int64_t, int64_t) { ++n; });
    return n;
  };
  // Longer runs while even full CTAs would take more than one wave.
  for (int grow = 0; grow < ffa::kMaxRunPieces && ctas_for(INT64_MAX) > sms; ++grow) {
    uint8_t* m = &run_by[0][0][0];
    for (size_t k = 0; k < sizeof(run_by); ++k) m[k] = static_cast<uint8_t>(std::min<int>(m[k] + 1, ffa::kMaxRunPieces));
    build_order();
  }
  int64_t budget = INT64_MAX;  // (when even full CTAs take more than one wave)
  if (ctas_for(budget) <= sms) {
    int64_t total = 0;
    for (const ClassRun& run : runs)
      for (int64_t k = run.first; k < run.first + run.slots; ++k) total += slot_cost(k);
    budget = std::max<int64_t>(1, (total + sms - 1) / sms);
    while (ctas_for(budget) > sms) budget += std::max<int64_t>(1, budget / 32);
  }
  // Bundles; the row-staged runs come first (one launch each kind).
  const size_t bundles_off = align_up(L.slots + sizeof(ffa::SlotRef) * n_first, 16);
  auto* bundles = reinterpret_cast<ffa::Bundle*>(host + bundles_off);
  int64_t nb = 0, nb_row = 0, max_row_slots = 1;
  int max_gather_k = 8;
  for (const ClassRun& run : runs) {
    const int nw = class_warps(run.cls);
    cut(run, budget, [&](int64_t first, int64_t m) {
      bundles[nb++] = ffa::Bundle{static_cast<int32_t>(first), static_cast<uint8_t>(nw), static_cast<uint8_t>(m),
                                  run.kst, 0};
      if (class_row(run.cls)) max_row_slots = std::max(max_row_slots, m);
    });
    if (class_row(run.cls)) nb_row = nb;
  }
  for (int64_t i = 0; i < count; ++i)
    if (!recs[i].row_mode) max_gather_k = std::max<int>(max_gather_k, recs[i].kst);
  // Long records: 8 states per thread, unless the device cannot run the
  // clusters of all of the batch's long records of one staging kind at once
  // and 16 states per thread (half the cluster size) fits more of them.
  const size_t long_header = ffa::long_header_bytes();
  auto long_smem = [&](int k, bool row) {
    return static_cast<unsigned>(
        long_header + (row ? static_cast<size_t>(ffa::kRowRing) * ffa::kChunkFrames * max_row_vocab * esize
                           : ffa::gather_ring_bytes(k)));
  };
  const int rv_long = row_vocab > 0 ? row_vocab : 0;
  int64_t n_long_row = 0;
  for (uint64_t key : long_keys) n_long_row += recs[key].row_mode ? 1 : 0;
  for (uint64_t& key : long_keys) {
    ffa::RecordDev& d = recs[key];
    const bool row = d.row_mode != 0;
    const int64_t n = row ? n_long_row : static_cast<int64_t>(long_keys.size()) - n_long_row;
    const int64_t S = 2 * static_cast<int64_t>(d.U) + 1;
    const int c8 = static_cast<int>((S + 8 * ffa::kCtaThreads - 1) / (8 * ffa::kCtaThreads));
    const int c16 = static_cast<int>((S + 16 * ffa::kCtaThreads - 1) / (16 * ffa::kCtaThreads));
    int k = 8, c = c8;
    const int cap8 = ffa::long_capacity(8, c8, row, rv_long, fmt, long_smem(8, row));
    if (cap8 < n && ffa::long_capacity(16, c16, row, rv_long, fmt, long_smem(16, row)) > cap8) {
      k = 16;
      c = c16;
    }
    d.kst = static_cast<uint8_t>(k);
    key = static_cast<uint64_t>(row ? 0 : 1) << 44 | static_cast<uint64_t>(k == 16 ? 1 : 0) << 40 |
          static_cast<uint64_t>(c) << 32 | key;
  }
  // By launch: row-staged first, then by states per thread and cluster size.
  std::sort(long_keys.begin(), long_keys.end());
  for (size_t k = 0; k < long_keys.size(); ++k) longs[k] = static_cast<int32_t>(long_keys[k] & 0xffffffffu);
  // Window route: records longest first (by length bucket), packed into CTAs
  // of at most kWinWarps records -- one record per CTA while the records do
  // not outnumber the SMs (each then has an SM to itself), else as many as
  // spread them evenly over the SMs -- with each record's shared-memory slice
  // (win_layout) side by side, and the launch sized for the largest CTA.
  auto* wslots = reinterpret_cast<ffa::WinSlot*>(host + L.win_slots);
  auto* wctas = reinterpret_cast<ffa::WinCta*>(host + L.win_ctas);
  int64_t n_wcta = 0;
  uint32_t win_smem = 0, wide_smem = 0;
  int win_vocab = -1;
  bool win_smem_codes = false;
  if (!win_records.empty()) {
    const int64_t nwin = static_cast<int64_t>(win_records.size());
    thread_local std::vector<int32_t> bucket_start;
    bucket_start.assign(kLengthBuckets + 1, 0);
    auto bucket = [&](int32_t i) { return kLengthBuckets - 1 - length_bucket(static_cast<uint32_t>(recs[i].T)); };
    for (int32_t i : win_records) ++bucket_start[bucket(i) + 1];
    for (int b = 0; b < kLengthBuckets; ++b) bucket_start[b + 1] += bucket_start[b];
    auto* sorted_win = reinterpret_cast<int32_t*>(host + L.keys);  // the first pass is done with the keys
    for (int32_t i : win_records) sorted_win[bucket_start[bucket(i)]++] = i;
    // Spread over the SMs, at most kWinSmemCodesSpread records each: the
    // batch is latency-bound and fits the SMs at once with the codes in the
    // slices, where the traceback walks them fastest.  More records per SM:
    // the codes go to global memory and the smaller slices let up to
    // kWinWarps records share a CTA.
    const int64_t spread = (nwin + sms - 1) / sms;
    win_smem_codes = !window_codes_global(nwin);
    const int64_t per_cta = std::clamp<int64_t>(spread, 1, win_smem_codes ? kWinSmemCodesSpread : ffa::kWinWarps);
    // Two CTAs share an SM when each stays under half the budget: twice the
    // warps to cover each warp's per-frame dependency chain.  A record larger
    // than that gets a CTA of its own.
    const uint32_t budget = static_cast<uint32_t>((ffa::kSmemBudget - 2048) / 2);
    uint32_t cur = 0;
    for (int64_t k = 0; k < nwin; ++k) {
      const int32_t i = sorted_win[k];
      const ffa::RecordDev& d = recs[i];
      win_vocab = (win_vocab < 0 || win_vocab == d.V) ? d.V : 0;
      const uint32_t need = ffa::win_layout(d.T, d.U, d.V, static_cast<int>(esize), 2, win_smem_codes).bytes;
      wide_smem = std::max(wide_smem, ffa::win_layout(std::min(d.T, ffa::kWinWideMaxFrames), d.U, d.V,
                                                      static_cast<int>(esize), 4, win_smem_codes).bytes);
      if (n_wcta == 0 || wctas[n_wcta - 1].count == per_cta || cur + need > budget) {
        wctas[n_wcta++] = ffa::WinCta{static_cast<int32_t>(k), 0};
        cur = 0;
      }
      wslots[k] = ffa::WinSlot{i, cur};
      cur += need;
      ++wctas[n_wcta - 1].count;
      win_smem = std::max(win_smem, cur);
    }
  }
  const size_t upload_bytes = bundles_off + sizeof(ffa::Bundle) * nb;
  const unsigned row_smem = static_cast<unsigned>(header + max_row_slots * row_slot_bytes);
  const unsigned gather_smem = static_cast<unsigned>(header + ffa::gather_ring_bytes(max_gather_k));

  auto* dev = static_cast<unsigned char*>(workspace);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  cudaError_t err = upload_descriptors(dev, host, upload_bytes, s);
  if (err != cudaSuccess) return cuda_fail(err, "descriptor upload");

  ffa::ForwardParams fp{};
  fp.recs = reinterpret_cast<const ffa::RecordDev*>(dev + L.recs);
  fp.order = reinterpret_cast<const ffa::SlotRef*>(dev + L.slots);
  fp.mask = emission_validity;
  fp.check_inputs = (flags & FFA_FLAG_CHECK_INPUTS) ? 1 : 0;
  fp.bp = reinterpret_cast<uint32_t*>(dev + L.bp);
  fp.maps = reinterpret_cast<uint16_t*>(dev + L.maps);
  fp.anchors = reinterpret_cast<int32_t*>(dev + L.anchors);
  fp.path_states = reinterpret_cast<int16_t*>(dev + L.path_states);
  fp.frontiers = reinterpret_cast<float*>(dev + L.frontiers);
  fp.pstates = reinterpret_cast<ffa::PieceState*>(dev + L.pstates);
  fp.route = reinterpret_cast<int32_t*>(dev + L.route);
  fp.fill_done = reinterpret_cast<int32_t*>(dev + L.fill_done);
  fp.finish_done = reinterpret_cast<int32_t*>(dev + L.finish_done);
  // Round 0 is planned in the first pass when the records outnumber the SMs
  // but the finisher still gives each its own 512-thread CTA: records joined
  // there never occupy one.  (cfg4 shards on one B200, first pass + finisher
  // with and without: 1031 records 565 vs 606 us, 2063: 914 vs 1016, 4128:
  // 1747 vs 1842; 8256 records, on the finisher's small CTAs: 3274 vs 3240.)
  fp.plan_first = nchunked > sms && !many_chunked ? 1 : 0;
  fp.finish_narrow = many_chunked ? 1 : 0;
  // Records that do not outnumber the SMs each have a finisher CTA to
  // themselves, which then also fills and folds the record: one launch and
  // its tail less on the latency-bound path.
  fp.fill_in_finisher = nchunked > 0 && nchunked <= sms ? 1 : 0;
  fp.slot_done = reinterpret_cast<int32_t*>(dev + L.counters);
  fp.finish_count = fp.slot_done + count;
  fp.finish_list = reinterpret_cast<int32_t*>(dev + L.chunked);
  for (int grp = 0; grp < ffa::kFinishGroups; ++grp)
    fp.finish_base[grp] = static_cast<int32_t>(grp == 0 ? 0 : finish_end[grp - 1]);
  fp.out = ffa::OutputsDev{outputs->labels, outputs->scores, outputs->status, outputs->objective,
                           outputs->stitched, outputs->repair_passes, outputs->repaired_frames,
                           outputs->shortcut_stats, outputs->routing_stats, outputs->reuse_stats};
  fp.row_slot_bytes = row_slot_bytes;
  std::memcpy(fp.run_by, run_by, sizeof(run_by));
  fp.lse = fmt != FFA_INPUT_LOG_PROBS ? reinterpret_cast<const float*>(dev + L.lse) : nullptr;
  fp.greedy_first = reinterpret_cast<const int32_t*>(dev + L.greedy_first);
  const auto* dbundles = reinterpret_cast<const ffa::Bundle*>(dev + bundles_off);
  const int rv = row_vocab > 0 ? row_vocab : 0;

  // Logits: every row's log-sum-exp, which each kernel below subtracts from
  // the logits it reads.
  if (fmt != FFA_INPUT_LOG_PROBS) {
    int max_vocab = 1;
    for (int64_t i = 0; i < count; ++i) max_vocab = std::max(max_vocab, records[i].vocab);
    err = ffa::launch_lse(fp.recs, static_cast<int>(count), L.total_frames, max_vocab, fmt,
                          reinterpret_cast<float*>(dev + L.lse), s);
    if (err != cudaSuccess) return cuda_fail(err, "log-sum-exp launch");
  }
  if (g_profile_before != nullptr) {
    err = cudaEventRecord(g_profile_before, s);
    if (err != cudaSuccess) return cuda_fail(err, "profiling event");
  }
  auto mark = [&](int point) {
    const cudaError_t e = mark_phase(point, s);
    return e == cudaSuccess ? FFA_OK : cuda_fail(e, "profiling event");
  };
  if ((rc = mark(FFA_PROFILE_START))) return rc;
  // Window route: the greedy pass, the window DP of every such record, then
  // the wider window and the full DP of those a tier did not certify
  // (device-written lists) -- on a side stream when the chunked route or the
  // long records have work too.  The greedy pass of the other records
  // (statistics only) follows on the side stream, once the first pass has
  // taken its SMs; that of the records with wider rows runs there after the
  // first pass, beside the finisher.
  cudaStream_t ws = s;
  SideStream* side = nullptr;
  const bool stats_greedy = !stats_records.empty();
  const bool wide_greedy = L.num_wide > 0;
  const bool forked = (n_wcta > 0 && (nb > 0 || !long_keys.empty())) || stats_greedy || (wide_greedy && n_wcta == 0);
  ffa::GreedyParams gp{};
  gp.recs = fp.recs;
  gp.greedy_first = reinterpret_cast<const int32_t*>(dev + L.greedy_first);
  gp.tok_off = reinterpret_cast<const int32_t*>(dev + L.tok_off);
  gp.alphabet = reinterpret_cast<uint64_t*>(dev + L.alphabet);
  gp.lpos = reinterpret_cast<uint16_t*>(dev + L.lpos);
  gp.lstart = reinterpret_cast<uint16_t*>(dev + L.lstart);
  gp.lse = fp.lse;
  gp.bound = reinterpret_cast<float*>(dev + L.bound);
  gp.verdicts = reinterpret_cast<uint8_t*>(dev + L.verdicts);
  gp.mask = fp.mask;
  gp.check_inputs = fp.check_inputs;
  gp.shortcut_stats = outputs->shortcut_stats;
  if (forked) {
    if ((err = side_stream(&side)) != cudaSuccess) return cuda_fail(err, "side stream");
    if ((err = cudaEventRecord(side->fork, s)) != cudaSuccess) return cuda_fail(err, "stream fork");
    if ((err = cudaStreamWaitEvent(side->stream, side->fork, 0)) != cudaSuccess) return cuda_fail(err, "stream fork");
    ws = side->stream;
  }
  if (n_wcta > 0) {
    const int wv = win_vocab > 0 ? win_vocab : 0;
    // The greedy pass streams every row of the window records once: it is
    // the launch the forward profiling events bracket (after the preparation).
    gp.records = reinterpret_cast<const int32_t*>(dev + L.greedy_recs);
    gp.num_records = static_cast<int64_t>(win_records.size());
    gp.items = reinterpret_cast<const ffa::GreedyItem*>(dev + L.greedy_items);
    gp.count = ngreedy;
    err = ffa::launch_greedy(gp, wv, fmt, ws, g_profile_before);
    if (err != cudaSuccess) return cuda_fail(err, "greedy pass launch");
    if (g_profile_after != nullptr && (err = cudaEventRecord(g_profile_after, ws)) != cudaSuccess)
      return cuda_fail(err, "profiling event");
    ffa::WindowParams wp{};
    wp.recs = fp.recs;
    wp.slots = reinterpret_cast<const ffa::WinSlot*>(dev + L.win_slots);
    wp.ctas = reinterpret_cast<const ffa::WinCta*>(dev + L.win_ctas);
    wp.mask = fp.mask;
    wp.check_inputs = fp.check_inputs;
    wp.out = fp.out;
    wp.lse = fp.lse;
    wp.bound = gp.bound;
    wp.codes = reinterpret_cast<uint32_t*>(dev + L.win_codes);
    wp.smem_codes = win_smem_codes ? 1 : 0;
    wp.verdicts = gp.verdicts;
    wp.greedy_first = reinterpret_cast<const int32_t*>(dev + L.greedy_first);
    // Tier lists: the 64-state window hands records to the 128-state one
    // (list 1), which hands them to the full DP (list 2).
    int32_t* list1 = reinterpret_cast<int32_t*>(dev + L.fallback);
    int32_t* list2 = list1 + count;
    int32_t* count1 = fp.slot_done + count + ffa::kFinishGroups;
    int32_t* count2 = count1 + 1;
    wp.fallback_list = list1;
    wp.fallback_count = count1;
    err = ffa::launch_window(wp, static_cast<int>(n_wcta), wv, fmt, win_smem, ws);
    if (err != cudaSuccess) return cuda_fail(err, "window launch");
    ffa::WindowParams wide = wp;
    wide.in_list = list1;
    wide.in_count = count1;
    wide.fallback_list = list2;
    wide.fallback_count = count2;
    err = ffa::launch_window_wide(wide, static_cast<int>(win_records.size()), wv, fmt, wide_smem, ws);
    if (err != cudaSuccess) return cuda_fail(err, "wide window launch");
    err = ffa::launch_window_fallback(fp, list2, count2, static_cast<int>(win_records.size()), wv, fmt,
                                      static_cast<unsigned>(header + row_slot_bytes), ws);
    if (err != cudaSuccess) return cuda_fail(err, "window fallback launch");
  }
  // Long records: the conventional DP on one cluster each, one launch per
  // (staging kind, states per thread, cluster size).
  if (!long_keys.empty()) {
    ffa::LongParams lp{};
    lp.recs = fp.recs;
    lp.mask = fp.mask;
    lp.check_inputs = fp.check_inputs;
    lp.bp = fp.bp;
    lp.maps = fp.maps;
    lp.anchors = fp.anchors;
    lp.out = fp.out;
    lp.lse = fp.lse;
    const auto* dlongs = reinterpret_cast<const int32_t*>(dev + L.longs);
    for (size_t k = 0; k < long_keys.size();) {
      const uint64_t group = long_keys[k] >> 32;
      size_t m = 1;
      while (k + m < long_keys.size() && (long_keys[k + m] >> 32) == group) ++m;
      const bool row = ((group >> 12) & 1) == 0;
      const int kst = ((group >> 8) & 1) ? 16 : 8;
      const int cluster = static_cast<int>(group & 0xff);
      lp.records = dlongs + k;
      err = ffa::launch_long(lp, static_cast<int>(m), cluster, kst, row, rv, fmt, long_smem(kst, row), s);
      if (err == cudaErrorInvalidClusterSize)
        return fail(FFA_ERR_UNSUPPORTED, "this GPU cannot co-schedule a cluster of " + std::to_string(cluster) +
                                             " CTAs, which records of up to " +
                                             std::to_string(cluster * kst * ffa::kCtaThreads) + " states need");
      if (err != cudaSuccess) return cuda_fail(err, "long-record launch");
      k += m;
    }
  }
  // First pass: every piece of every record (a one-piece record is the
  // conventional DP).
  fp.bundles = dbundles;
  err = ffa::launch_forward(fp, static_cast<int>(nb_row), true, rv, fmt, row_smem, s);
  if (err != cudaSuccess) return cuda_fail(err, "forward launch");
  fp.bundles = dbundles + nb_row;
  err = ffa::launch_forward(fp, static_cast<int>(nb - nb_row), false, 0, fmt, gather_smem, s);
  if (err != cudaSuccess) return cuda_fail(err, "forward launch");
  if (g_profile_after != nullptr && n_wcta == 0) {  // (with window records: around the greedy pass)
    err = cudaEventRecord(g_profile_after, s);
    if (err != cudaSuccess) return cuda_fail(err, "profiling event");
  }
  // The greedy pass of the records off the window route (their statistics
  // only): beside the first pass on the side stream when the window route has
  // nothing there, else after the fill on this stream, which then ends before
  // the window route's chain.
  auto stats_pass = [&](cudaStream_t stream) {
    ffa::GreedyParams sp = gp;
    sp.records = reinterpret_cast<const int32_t*>(dev + L.greedy_recs) + win_records.size();
    sp.num_records = static_cast<int64_t>(stats_records.size());
    sp.items = reinterpret_cast<const ffa::GreedyItem*>(dev + L.greedy_items) + L.num_greedy_window;
    sp.count = nstats_items;
    const cudaError_t e = ffa::launch_greedy(sp, stats_vocab > 0 ? stats_vocab : 0, fmt, stream);
    return e == cudaSuccess ? FFA_OK : cuda_fail(e, "greedy pass launch");
  };
  if (stats_greedy && n_wcta == 0 && (rc = stats_pass(ws))) return rc;
  // The statistics of the records with wider rows: after the first pass,
  // which zeroes them (on the side stream beside the finisher when the window
  // route leaves it free, else after the fill).
  auto wide_pass = [&](cudaStream_t stream) -> int {
    ffa::GreedyParams wp = gp;
    wp.items = reinterpret_cast<const ffa::GreedyItem*>(dev + L.wide_items);
    wp.count = L.num_wide;
    const cudaError_t e = ffa::launch_greedy_wide(wp, L.wide_max_tokens, L.wide_max_vocab, fmt, stream);
    return e == cudaSuccess ? FFA_OK : cuda_fail(e, "greedy statistics launch");
  };
  if (wide_greedy && n_wcta == 0) {
    if ((err = cudaEventRecord(side->first_pass, s)) != cudaSuccess) return cuda_fail(err, "stream fork");
    if ((err = cudaStreamWaitEvent(ws, side->first_pass, 0)) != cudaSuccess) return cuda_fail(err, "stream fork");
    if ((rc = wide_pass(ws))) return rc;
  }
  if ((rc = mark(FFA_PROFILE_FIRST))) return rc;
  // The optimized route's seam plans, repairs and fallback: a CTA per record
  // (the first round spread over up to four while the records leave SMs
  // free), the groups planned above.  Repairs run 8 states per thread, so a
  // gathered CTA needs that ring only; a 256-thread CTA keeps under half the
  // shared memory so that two share an SM.
  const auto* dchunked = reinterpret_cast<const int32_t*>(dev + L.chunked);
  const int spread = static_cast<int>(std::clamp<int64_t>(sms / std::max<int64_t>(nchunked, 1), 1, 4));
  const unsigned finish_gather_smem = static_cast<unsigned>(header + ffa::gather_ring_bytes(8));
  for (int grp = 0; grp < ffa::kFinishGroups; ++grp) {
    const int64_t first = grp == 0 ? 0 : finish_end[grp - 1];
    const int64_t n = finish_end[grp] - first;
    if (n == 0) continue;
    const bool row = grp < 3;
    const int threads = group_threads(grp);
    const int per_sm = ffa::kCtaThreads / threads;  // CTAs that share an SM
    unsigned smem = finish_gather_smem;
    if (row) {
      const size_t budget = (ffa::kSmemBudget - 2048) / per_sm - (per_sm > 1 ? 2048 : 0);
      const int64_t slots = std::max<int64_t>(1, std::min<int64_t>(std::max(1, threads / 32 - 1),
                                                                   static_cast<int64_t>((budget - header) / row_slot_bytes)));
      smem = static_cast<unsigned>(header + slots * row_slot_bytes);
    }
    err = ffa::launch_finish(fp, dchunked + first, static_cast<int>(n), fp.plan_first ? fp.finish_count + grp : nullptr,
                             spread, threads, row, row ? rv : 0, fmt, smem, s);
    if (err != cudaSuccess) return cuda_fail(err, "finish launch");
  }
  if ((rc = mark(FFA_PROFILE_FINISH))) return rc;
  if (!fp.fill_in_finisher || unchunked_fill > 0) {
    err = ffa::launch_fill(fp.recs, reinterpret_cast<const ffa::FillItem*>(dev + L.fill),
                           static_cast<int>(nfill), fp.bp, fp.anchors, fp.out, fp.route, fp.fill_done,
                           fp.path_states, fp.lse, fmt, s);
    if (err != cudaSuccess) return cuda_fail(err, "traceback launch");
  }
  if (stats_greedy && n_wcta > 0 && (rc = stats_pass(s))) return rc;
  if (wide_greedy && n_wcta > 0 && (rc = wide_pass(s))) return rc;
  if (forked) {
    if ((err = cudaEventRecord(side->join, ws)) != cudaSuccess) return cuda_fail(err, "stream join");
    if ((err = cudaStreamWaitEvent(s, side->join, 0)) != cudaSuccess) return cuda_fail(err, "stream join");
  }
  if ((rc = mark(FFA_PROFILE_FILL))) return rc;
  return FFA_OK;
}

int ffa_emission_validity_query(const ffa_record* records, int64_t count, ffa_sizes* sizes) {
  if (sizes == nullptr) return fail(FFA_ERR_INVALID_ARGUMENT, "sizes must not be NULL");
  ScanLayout L{};
  const int rc = plan_scan(records, count, &L);
  if (rc) return rc;
  sizes->staging_bytes = L.staging_bytes;
  sizes->workspace_bytes = L.workspace_bytes;
  sizes->total_frames = 0;
  for (int64_t i = 0; i < count; ++i) sizes->total_frames += records[i].frames;
  return FFA_OK;
}

int ffa_emission_validity(const ffa_record* records, int64_t count, uint8_t* valid,
                          void* staging, size_t staging_bytes,
                          void* workspace, size_t workspace_bytes, ffa_stream_t stream) {
  if (valid == nullptr) return fail(FFA_ERR_INVALID_ARGUMENT, "valid must not be NULL");
  ScanLayout L{};
  int rc = plan_scan(records, count, &L);
  if (rc) return rc;
  if (staging == nullptr || staging_bytes < L.staging_bytes)
    return fail(FFA_ERR_BUFFER_TOO_SMALL, "staging buffer smaller than the query reports");
  if (workspace == nullptr || workspace_bytes < L.workspace_bytes ||
      (reinterpret_cast<uintptr_t>(workspace) & 255) != 0)
    return fail(FFA_ERR_BUFFER_TOO_SMALL, "workspace missing, too small or not 256-byte aligned");
  auto* host = static_cast<unsigned char*>(staging);
  auto* recs = reinterpret_cast<ffa::ScanRecord*>(host + L.recs);
  auto* items = reinterpret_cast<ffa::ScanItem*>(host + L.items);
  int64_t n = 0;
  for (int64_t i = 0; i < count; ++i) {
    recs[i] = ffa::ScanRecord{static_cast<const float*>(records[i].emissions), records[i].frames * records[i].vocab};
    const int64_t chunks = scan_chunks(records[i]);
    for (int64_t c = 0; c < chunks; ++c)
      items[n++] = ffa::ScanItem{static_cast<int32_t>(i), static_cast<int32_t>(c)};
  }
  auto* dev = static_cast<unsigned char*>(workspace);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  cudaError_t err = upload_descriptors(dev, host, L.staging_bytes, s);
  if (err != cudaSuccess) return cuda_fail(err, "descriptor upload");
  err = ffa::launch_validity(reinterpret_cast<const ffa::ScanRecord*>(dev + L.recs), count,
                             reinterpret_cast<const ffa::ScanItem*>(dev + L.items), n, valid, s);
  if (err != cudaSuccess) return cuda_fail(err, "validity launch");
  return FFA_OK;
}

int ffa_check_targets_query(const ffa_record* records, int64_t count, ffa_sizes* sizes) {
  if (sizes == nullptr) return fail(FFA_ERR_INVALID_ARGUMENT, "sizes must not be NULL");
  if (records == nullptr || count < 1 || count > FFA_MAX_RECORDS)
    return fail(FFA_ERR_INVALID_ARGUMENT, "provide 1..65535 records");
  sizes->total_frames = 0;
  for (int64_t i = 0; i < count; ++i) {
    const int rc = check_record(records[i], i, true);
    if (rc) return rc;
    sizes->total_frames += records[i].frames;
  }
  sizes->staging_bytes = align_up(sizeof(ffa::RecordDev) * count, 256);
  sizes->workspace_bytes = sizes->staging_bytes;
  return FFA_OK;
}

int ffa_check_targets(const ffa_record* records, int64_t count, int32_t* status,
                      void* staging, size_t staging_bytes,
                      void* workspace, size_t workspace_bytes, ffa_stream_t stream) {
  if (status == nullptr) return fail(FFA_ERR_INVALID_ARGUMENT, "status must not be NULL");
  ffa_sizes sizes{};
  int rc = ffa_check_targets_query(records, count, &sizes);
  if (rc) return rc;
  if (staging == nullptr || staging_bytes < sizes.staging_bytes)
    return fail(FFA_ERR_BUFFER_TOO_SMALL, "staging buffer smaller than the query reports");
  if (workspace == nullptr || workspace_bytes < sizes.workspace_bytes ||
      (reinterpret_cast<uintptr_t>(workspace) & 255) != 0)
    return fail(FFA_ERR_BUFFER_TOO_SMALL, "workspace missing, too small or not 256-byte aligned");
  auto* recs = static_cast<ffa::RecordDev*>(staging);
  for (int64_t i = 0; i < count; ++i) {
    ffa::RecordDev d{};
    d.emissions = static_cast<const float*>(records[i].emissions);
    d.targets = records[i].targets;
    d.T = static_cast<int32_t>(records[i].frames);
    d.V = records[i].vocab;
    d.U = records[i].tokens;
    d.blank = records[i].blank;
    recs[i] = d;
  }
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  cudaError_t err = upload_descriptors(workspace, staging, sizes.staging_bytes, s);
  if (err != cudaSuccess) return cuda_fail(err, "descriptor upload");
  err = ffa::launch_check_targets(static_cast<const ffa::RecordDev*>(workspace), count, status, s);
  if (err != cudaSuccess) return cuda_fail(err, "target check launch");
  return FFA_OK;
}

int ffa_row_logsumexp_query(const ffa_record* records, int64_t count, ffa_sizes* sizes) {
  if (sizes == nullptr) return fail(FFA_ERR_INVALID_ARGUMENT, "sizes must not be NULL");
  if (records == nullptr || count < 1 || count > FFA_MAX_RECORDS)
    return fail(FFA_ERR_INVALID_ARGUMENT, "provide 1..65535 records");
  int format = 0;
  int rc = common_format(records, count, &format);
  if (rc) return rc;
  if (format == FFA_INPUT_LOG_PROBS)
    return fail(FFA_ERR_INVALID_ARGUMENT, "the row log-sum-exp takes logits (input format 1 or 2)");
  sizes->total_frames = 0;
  for (int64_t i = 0; i < count; ++i) {
    if ((rc = check_record(records[i], i, false))) return rc;
    sizes->total_frames += records[i].frames;
  }
  sizes->staging_bytes = align_up(sizeof(ffa::RecordDev) * count, 256);
  sizes->workspace_bytes = sizes->staging_bytes;
  return FFA_OK;
}

int ffa_row_logsumexp(const ffa_record* records, int64_t count, float* z,
                      void* staging, size_t staging_bytes,
                      void* workspace, size_t workspace_bytes, ffa_stream_t stream) {
  if (z == nullptr) return fail(FFA_ERR_INVALID_ARGUMENT, "z must not be NULL");
  ffa_sizes sizes{};
  int rc = ffa_row_logsumexp_query(records, count, &sizes);
  if (rc) return rc;
  if (staging == nullptr || staging_bytes < sizes.staging_bytes)
    return fail(FFA_ERR_BUFFER_TOO_SMALL, "staging buffer smaller than the query reports");
  if (workspace == nullptr || workspace_bytes < sizes.workspace_bytes ||
      (reinterpret_cast<uintptr_t>(workspace) & 255) != 0)
    return fail(FFA_ERR_BUFFER_TOO_SMALL, "workspace missing, too small or not 256-byte aligned");
  // The kernel reads a record's emissions, out_off, T and V.
  auto* recs = static_cast<ffa::RecordDev*>(staging);
  int64_t off = 0;
  int max_vocab = 1;
  for (int64_t i = 0; i < count; ++i) {
    max_vocab = std::max(max_vocab, records[i].vocab);
    ffa::RecordDev d{};
    d.emissions = static_cast<const float*>(records[i].emissions);
    d.out_off = off;
    d.T = static_cast<int32_t>(records[i].frames);
    d.V = records[i].vocab;
    recs[i] = d;
    off += records[i].frames;
  }
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  cudaError_t err = upload_descriptors(workspace, staging, sizes.staging_bytes, s);
  if (err != cudaSuccess) return cuda_fail(err, "descriptor upload");
  err = ffa::launch_lse(static_cast<const ffa::RecordDev*>(workspace), static_cast<int>(count), off, max_vocab,
                        records[0].format, z, s);
  if (err != cudaSuccess) return cuda_fail(err, "log-sum-exp launch");
  return FFA_OK;
}

int ffa_token_spans_query(const int64_t* frames, const int32_t* tokens, int64_t count, ffa_sizes* sizes) {
  if (sizes == nullptr) return fail(FFA_ERR_INVALID_ARGUMENT, "sizes must not be null");
  int64_t total = 0;
  const int rc = check_spans(frames, tokens, count, &total);
  if (rc) return rc;
  sizes->staging_bytes = spans_bytes(count);
  sizes->workspace_bytes = spans_bytes(count);
  sizes->total_frames = total;
  return FFA_OK;
}

int ffa_token_spans(const int64_t* labels, const int64_t* frames, const int32_t* tokens,
                    const int32_t* blanks, int64_t count, int64_t* spans,
                    void* staging, size_t staging_bytes,
                    void* workspace, size_t workspace_bytes, ffa_stream_t stream) {
  int64_t total = 0;
  int rc = check_spans(frames, tokens, count, &total);
  if (rc) return rc;
  if (labels == nullptr || blanks == nullptr)
    return fail(FFA_ERR_INVALID_ARGUMENT, "labels and blanks are required");
  const size_t need = spans_bytes(count);
  if (staging == nullptr || staging_bytes < need)
    return fail(FFA_ERR_BUFFER_TOO_SMALL, "staging buffer smaller than ffa_token_spans_query reports");
  if (workspace == nullptr || workspace_bytes < need || (reinterpret_cast<uintptr_t>(workspace) & 255) != 0)
    return fail(FFA_ERR_BUFFER_TOO_SMALL, "workspace missing, too small or not 256-byte aligned");
  auto* recs = static_cast<ffa::SpanRecord*>(staging);
  int64_t frame_off = 0, token_off = 0, total_tokens = 0;
  for (int64_t i = 0; i < count; ++i) total_tokens += tokens[i];
  if (total_tokens > 0 && spans == nullptr) return fail(FFA_ERR_INVALID_ARGUMENT, "spans output is required");
  for (int64_t i = 0; i < count; ++i) {
    if (blanks[i] < 0) return fail(FFA_ERR_UNSUPPORTED, "record " + std::to_string(i) + ": negative blank ID");
    recs[i] = ffa::SpanRecord{labels + frame_off, spans + 2 * token_off, static_cast<int32_t>(frames[i]),
                              tokens[i], blanks[i], 0};
    frame_off += frames[i];
    token_off += tokens[i];
  }
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  cudaError_t err = upload_descriptors(workspace, staging, sizeof(ffa::SpanRecord) * count, s);
  if (err != cudaSuccess) return cuda_fail(err, "span descriptor upload");
  err = ffa::launch_spans(static_cast<const ffa::SpanRecord*>(workspace), count, s);
  if (err != cudaSuccess) return cuda_fail(err, "span launch");
  return FFA_OK;
}

}  // extern "C"
