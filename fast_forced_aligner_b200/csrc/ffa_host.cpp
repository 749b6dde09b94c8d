// ffa_host.cpp -- C ABI host layer of the B200-native CTC forced aligner.
//
// Replaces the reference's C++ host layer (alignment.cu:893-1061): metadata
// validation, launch planning and the single descriptor upload.  Differences
// by design:
//   - no allocation: outputs, workspace and host staging belong to the caller
//     (the torch shim hands in caching-allocator memory), so the call is
//     stream-ordered and never synchronises the host;
//   - records are planned on the host into packed CTAs ("bundles") of equal
//     slot size, longest first, so one launch covers a ragged batch;
//   - the planner builds every table in the caller's staging buffer in place
//     (no heap allocation), then enqueues one cudaMemcpyAsync.
#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <string>

#include <cuda_runtime.h>

#include "ffa_b200.h"
#include "ffa_internal.h"

namespace {

thread_local std::string g_error;
thread_local cudaEvent_t g_profile_before = nullptr;
thread_local cudaEvent_t g_profile_after = nullptr;

int fail(int code, const std::string& message) {
  g_error = message;
  return code;
}

constexpr size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

int ceil_log2(int64_t x) {
  int k = 0;
  while ((int64_t{1} << k) < x) ++k;
  return k;
}

struct Geometry {
  int K;         // states per thread
  int nw;        // warps for the DP
  int slot_log2; // packing slot: 1 << slot_log2 warps
  int seg_log2;  // traceback segment length
  int64_t segments;
  int64_t bp_words;
  int64_t map_elems;
};

// States per thread.  A record that has an SM to itself (at most one record
// per SM in the batch) is latency-bound: its frame time is the per-frame
// dependency chain, shortest with 4 states per thread and up to 16 warps
// (measured: ~260 cycles per frame at 8 warps against ~280 for K = 8 at 4
// warps).  Packed records share SMs, where fewer instructions per state win:
// K = 8.
int choose_k(int64_t S, bool latency_bound) {
  if (latency_bound && S <= 32 * 4 * 16) return 4;
  return 8;
}

Geometry geometry(const ffa_record& r, bool latency_bound) {
  Geometry g{};
  const int64_t S = 2 * static_cast<int64_t>(r.tokens) + 1;
  g.K = choose_k(S, latency_bound);
  g.nw = static_cast<int>((S + 32 * g.K - 1) / (32 * g.K));
  g.slot_log2 = ceil_log2(g.nw);
  // Segment length ~2*sqrt(T) balances the serial map walk (T/H steps) against
  // the per-segment backpointer walk (H steps).
  const double ideal = 2.0 * std::sqrt(static_cast<double>(r.frames));
  g.seg_log2 = std::clamp(static_cast<int>(std::lround(std::log2(std::max(ideal, 1.0)))),
                          ffa::kMinSegLog2, ffa::kMaxSegLog2);
  const int64_t H = int64_t{1} << g.seg_log2;
  g.segments = (r.frames + H - 1) / H;
  const int64_t nt = 32 * static_cast<int64_t>(g.nw);
  const int fpw = ffa::frames_per_word_host(g.K);
  g.bp_words = (r.frames + fpw - 1) / fpw * nt;
  g.map_elems = (g.segments - 1) * nt * g.K;
  return g;
}

int check_record(const ffa_record& r, int64_t i, bool need_targets) {
  if (r.emissions == nullptr || (reinterpret_cast<uintptr_t>(r.emissions) & 3) != 0 ||
      r.reserved != 0)
    return fail(FFA_ERR_INVALID_ARGUMENT,
                "record " + std::to_string(i) + ": emissions must be a 4-byte aligned device pointer");
  if (r.frames < 1 || r.frames > FFA_MAX_FRAMES || r.vocab < 1 || r.vocab > FFA_MAX_VOCAB)
    return fail(FFA_ERR_UNSUPPORTED, "record " + std::to_string(i) +
                                         ": unsupported frame count or vocabulary");
  if (!need_targets) return FFA_OK;
  if (r.tokens < 0 || (r.tokens > 0 && r.targets == nullptr))
    return fail(FFA_ERR_INVALID_ARGUMENT, "record " + std::to_string(i) + ": missing targets");
  if (2 * static_cast<int64_t>(r.tokens) + 1 > ffa::kMaxStates || r.blank < 0 || r.blank >= r.vocab)
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
// followed by the device-only arenas.
struct AlignLayout {
  size_t recs, bundles, order, fill, staging_bytes;
  size_t bp, maps, anchors, workspace_bytes;
  int64_t total_frames, bp_words, map_elems, segments, fill_items;
};

// One record per SM or fewer: every record's DP is latency-bound.
bool latency_bound(int64_t count) { return count <= device_sms(); }

int plan_align(const ffa_record* records, int64_t count, AlignLayout* L) {
  if (records == nullptr || count < 1 || count > FFA_MAX_RECORDS)
    return fail(FFA_ERR_INVALID_ARGUMENT, "provide 1..65535 records");
  int64_t frames = 0, bp_words = 0, map_elems = 0, segments = 0, fill = 0;
  const bool lat = latency_bound(count);
  for (int64_t i = 0; i < count; ++i) {
    const int rc = check_record(records[i], i, true);
    if (rc) return rc;
    const Geometry g = geometry(records[i], lat);
    frames += records[i].frames;
    bp_words += g.bp_words;
    map_elems += align_up(static_cast<size_t>(g.map_elems), 8);
    segments += g.segments;
    fill += (g.segments + ffa::kFillWarps - 1) / ffa::kFillWarps;
  }
  if (segments > INT32_MAX || fill > INT32_MAX)
    return fail(FFA_ERR_UNSUPPORTED, "batch exceeds the traceback segment index range");
  L->total_frames = frames;
  L->bp_words = bp_words;
  L->map_elems = map_elems;
  L->segments = segments;
  L->fill_items = fill;
  size_t off = 0;
  L->recs = off; off = align_up(off + sizeof(ffa::RecordDev) * count, 16);
  L->bundles = off; off = align_up(off + sizeof(ffa::Bundle) * count, 16);
  L->order = off; off = align_up(off + sizeof(int32_t) * count, 16);
  L->fill = off; off = align_up(off + sizeof(ffa::FillItem) * fill, 256);
  L->staging_bytes = off;
  L->bp = off; off = align_up(off + sizeof(uint32_t) * bp_words, 256);
  L->maps = off; off = align_up(off + sizeof(uint16_t) * map_elems, 256);
  L->anchors = off; off = align_up(off + sizeof(int32_t) * segments, 256);
  L->workspace_bytes = off;
  return FFA_OK;
}

struct ScanLayout {
  size_t recs, items, staging_bytes, workspace_bytes;
  int64_t num_items;
};

int64_t scan_chunks(const ffa_record& r) {
  const uintptr_t base = reinterpret_cast<uintptr_t>(r.emissions);
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

int cuda_fail(cudaError_t err, const char* what) {
  return fail(FFA_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(err));
}

}  // namespace

void ffa::set_last_error(const char* message) { g_error = message; }

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

int ffa_align_query(const ffa_record* records, int64_t count, int mode, int flags,
                    ffa_sizes* sizes) {
  if (sizes == nullptr) return fail(FFA_ERR_INVALID_ARGUMENT, "sizes must not be NULL");
  if (mode != FFA_MODE_CONVENTIONAL && mode != FFA_MODE_OPTIMIZED)
    return fail(FFA_ERR_INVALID_ARGUMENT, "mode must be conventional or optimized");
  if (flags & ~FFA_FLAG_CHECK_INPUTS) return fail(FFA_ERR_INVALID_ARGUMENT, "unknown flags");
  AlignLayout L{};
  const int rc = plan_align(records, count, &L);
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
  if (flags & ~FFA_FLAG_CHECK_INPUTS) return fail(FFA_ERR_INVALID_ARGUMENT, "unknown flags");
  AlignLayout L{};
  int rc = plan_align(records, count, &L);
  if (rc) return rc;
  if (staging == nullptr || staging_bytes < L.staging_bytes)
    return fail(FFA_ERR_BUFFER_TOO_SMALL, "staging buffer smaller than ffa_align_query reports");
  if (workspace == nullptr || workspace_bytes < L.workspace_bytes ||
      (reinterpret_cast<uintptr_t>(workspace) & 255) != 0)
    return fail(FFA_ERR_BUFFER_TOO_SMALL, "workspace missing, too small or not 256-byte aligned");

  auto* host = static_cast<unsigned char*>(staging);
  auto* recs = reinterpret_cast<ffa::RecordDev*>(host + L.recs);
  auto* bundles = reinterpret_cast<ffa::Bundle*>(host + L.bundles);
  auto* order = reinterpret_cast<int32_t*>(host + L.order);
  auto* fill = reinterpret_cast<ffa::FillItem*>(host + L.fill);

  // Per-record descriptors and arena offsets.
  int64_t out_off = 0, bp_off = 0, map_off = 0, seg_off = 0, nfill = 0;
  const bool lat = latency_bound(count);
  for (int64_t i = 0; i < count; ++i) {
    const ffa_record& r = records[i];
    const Geometry g = geometry(r, lat);
    ffa::RecordDev d{};
    d.emissions = r.emissions;
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
    // TMA row staging needs 16-byte aligned rows and a small row.
    d.row_mode = (r.vocab % 4 == 0 && r.vocab <= ffa::kRowModeMaxVocab &&
                  (reinterpret_cast<uintptr_t>(r.emissions) & 15) == 0)
                     ? 1
                     : 0;
    recs[i] = d;
    for (int64_t s = 0; s < g.segments; s += ffa::kFillWarps)
      fill[nfill++] = ffa::FillItem{static_cast<int32_t>(i), static_cast<int32_t>(s)};
    out_off += r.frames;
    bp_off += g.bp_words;
    map_off += static_cast<int64_t>(align_up(static_cast<size_t>(g.map_elems), 8));
    seg_off += g.segments;
    order[i] = static_cast<int32_t>(i);
  }

  // Records are grouped by emission staging (TMA row rings vs per-thread
  // column gather: one launch each), then by slot size, longest first.
  unsigned max_row_vocab = 0;
  int row_vocab = -1;  // common vocabulary of the row-staged records, 0 if mixed
  for (int64_t i = 0; i < count; ++i)
    if (recs[i].row_mode) {
      max_row_vocab = std::max<unsigned>(max_row_vocab, records[i].vocab);
      row_vocab = (row_vocab < 0 || row_vocab == records[i].vocab) ? records[i].vocab : 0;
    }
  const size_t header = ffa::forward_header_bytes();  // 128-byte aligned ring offset
  const unsigned row_slot_bytes = static_cast<unsigned>(
      align_up(static_cast<size_t>(ffa::kRowRing) * ffa::kChunkFrames * max_row_vocab * 4, 128));
  const int64_t row_slots =
      row_slot_bytes ? std::max<int64_t>(1, static_cast<int64_t>((ffa::kSmemBudget - header) / row_slot_bytes))
                     : ffa::kMaxWarps;

  auto slot_of = [&](int32_t i) { return ceil_log2(recs[i].nw); };
  std::sort(order, order + count, [&](int32_t a, int32_t b) {
    if (recs[a].row_mode != recs[b].row_mode) return recs[a].row_mode > recs[b].row_mode;
    if (recs[a].kst != recs[b].kst) return recs[a].kst < recs[b].kst;
    const int sa = slot_of(a), sb = slot_of(b);
    if (sa != sb) return sa < sb;
    if (records[a].frames != records[b].frames) return records[a].frames > records[b].frames;
    return a < b;
  });
  // Records per CTA grow only when the batch would otherwise need more than
  // one wave; a row-staged slot also needs its ring to fit in shared memory.
  const int64_t sms = device_sms();
  const int64_t per_cta_target = std::max<int64_t>(1, (count + sms - 1) / sms);
  int64_t nb = 0, n_row_bundles = 0, max_row_slots = 1;
  for (int64_t k = 0; k < count;) {
    const int cls = slot_of(order[k]);
    const bool row = recs[order[k]].row_mode != 0;
    const int kst = recs[order[k]].kst;
    int64_t capacity = std::min(static_cast<int64_t>(ffa::kMaxWarps >> cls), per_cta_target);
    if (row) capacity = std::min(capacity, row_slots);
    int64_t n = 0;
    while (k + n < count && n < capacity && slot_of(order[k + n]) == cls &&
           (recs[order[k + n]].row_mode != 0) == row && recs[order[k + n]].kst == kst)
      ++n;
    bundles[nb++] = ffa::Bundle{static_cast<int32_t>(k), static_cast<uint8_t>(cls),
                                static_cast<uint8_t>(n), static_cast<uint8_t>(kst), 0};
    if (row) { ++n_row_bundles; max_row_slots = std::max(max_row_slots, n); }
    k += n;
  }
  auto longest_first = [&](const ffa::Bundle& a, const ffa::Bundle& b) {
    return records[order[a.first]].frames > records[order[b.first]].frames;
  };
  std::stable_sort(bundles, bundles + n_row_bundles, longest_first);
  std::stable_sort(bundles + n_row_bundles, bundles + nb, longest_first);
  const unsigned row_smem = static_cast<unsigned>(header + max_row_slots * row_slot_bytes);
  int max_gather_k = 8;
  for (int64_t i = 0; i < count; ++i)
    if (!recs[i].row_mode) max_gather_k = std::max<int>(max_gather_k, recs[i].kst);
  const unsigned gather_smem = static_cast<unsigned>(header + ffa::gather_ring_bytes(max_gather_k));

  auto* dev = static_cast<unsigned char*>(workspace);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  cudaError_t err = cudaMemcpyAsync(dev, host, L.staging_bytes, cudaMemcpyHostToDevice, s);
  if (err != cudaSuccess) return cuda_fail(err, "descriptor upload");

  ffa::OutputsDev out{outputs->labels, outputs->scores, outputs->status, outputs->objective,
                      outputs->stitched, outputs->repair_passes, outputs->repaired_frames,
                      outputs->shortcut_stats, outputs->routing_stats, outputs->reuse_stats};
  const auto* drecs = reinterpret_cast<const ffa::RecordDev*>(dev + L.recs);
  auto* bp = reinterpret_cast<uint32_t*>(dev + L.bp);
  auto* anchors = reinterpret_cast<int32_t*>(dev + L.anchors);
  // The optimized route currently resolves every record with the exact
  // conventional DP, which satisfies its contract (stitched = 0 denotes the
  // conventional route, alignment.py:101-104).
  if (g_profile_before != nullptr) {
    err = cudaEventRecord(g_profile_before, s);
    if (err != cudaSuccess) return cuda_fail(err, "profiling event");
  }
  const auto* dbundles = reinterpret_cast<const ffa::Bundle*>(dev + L.bundles);
  const auto* dorder = reinterpret_cast<const int32_t*>(dev + L.order);
  auto* maps = reinterpret_cast<uint16_t*>(dev + L.maps);
  const int check = (flags & FFA_FLAG_CHECK_INPUTS) ? 1 : 0;
  err = ffa::launch_forward(drecs, dbundles, dorder, static_cast<int>(n_row_bundles), true,
                            row_vocab > 0 ? row_vocab : 0, emission_validity, check, bp, maps,
                            anchors, out, row_smem, row_slot_bytes, s);
  if (err != cudaSuccess) return cuda_fail(err, "forward launch");
  err = ffa::launch_forward(drecs, dbundles + n_row_bundles, dorder,
                            static_cast<int>(nb - n_row_bundles), false, 0, emission_validity,
                            check, bp, maps, anchors, out, gather_smem, 0, s);
  if (err != cudaSuccess) return cuda_fail(err, "forward launch");
  if (g_profile_after != nullptr) {
    err = cudaEventRecord(g_profile_after, s);
    if (err != cudaSuccess) return cuda_fail(err, "profiling event");
  }
  err = ffa::launch_fill(drecs, reinterpret_cast<const ffa::FillItem*>(dev + L.fill),
                         static_cast<int>(nfill), bp, anchors, out, s);
  if (err != cudaSuccess) return cuda_fail(err, "traceback launch");
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
    recs[i] = ffa::ScanRecord{records[i].emissions, records[i].frames * records[i].vocab};
    const int64_t chunks = scan_chunks(records[i]);
    for (int64_t c = 0; c < chunks; ++c)
      items[n++] = ffa::ScanItem{static_cast<int32_t>(i), static_cast<int32_t>(c)};
  }
  auto* dev = static_cast<unsigned char*>(workspace);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  cudaError_t err = cudaMemcpyAsync(dev, host, L.staging_bytes, cudaMemcpyHostToDevice, s);
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
    d.emissions = records[i].emissions;
    d.targets = records[i].targets;
    d.T = static_cast<int32_t>(records[i].frames);
    d.V = records[i].vocab;
    d.U = records[i].tokens;
    d.blank = records[i].blank;
    recs[i] = d;
  }
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  cudaError_t err = cudaMemcpyAsync(workspace, staging, sizes.staging_bytes,
                                    cudaMemcpyHostToDevice, s);
  if (err != cudaSuccess) return cuda_fail(err, "descriptor upload");
  err = ffa::launch_check_targets(static_cast<const ffa::RecordDev*>(workspace), count, status, s);
  if (err != cudaSuccess) return cuda_fail(err, "target check launch");
  return FFA_OK;
}

}  // extern "C"
