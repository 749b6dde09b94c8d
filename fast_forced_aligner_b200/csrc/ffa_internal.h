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
// Backpointers: 1.5*K bits per frame and thread (a "moved" bit per state and
// a "skipped" bit per token), two frames per 32-bit word when they fit.
constexpr int frames_per_word_host(int K) { return 3 * K / 2 <= 16 ? 2 : 1; }
// Traceback segment length bounds (power of two, multiple of kFramesPerWord).
constexpr int kMinSegLog2 = 5;
constexpr int kMaxSegLog2 = 10;
constexpr int kFillWarps = 8;

// Device-side descriptor of one record (64 bytes).
struct RecordDev {
  const float* emissions;   // [T, V] fp32, caller memory
  const int64_t* targets;   // [U] int64, caller memory (may be null if U == 0)
  int64_t out_off;          // first frame of this record in labels/scores
  int64_t bp_off;           // first uint32 word in the backpointer arena
  int64_t map_off;          // first uint16 entry in the checkpoint-map arena
  int32_t T, V, U, blank;
  int32_t seg_off;          // first anchor (one per traceback segment)
  uint8_t nw;               // warps running this record's DP
  uint8_t kst;              // states per thread K
  uint8_t seg_log2;         // traceback segment length H = 1 << seg_log2
  uint8_t row_mode;         // 1: TMA row staging, 0: per-thread column gather
};
static_assert(sizeof(RecordDev) == 64, "RecordDev layout");

// One forward CTA ("bundle"): `count` records of the same slot size
// (1 << slot_log2 warps each) and states per thread, listed at
// order[first .. first+count).
struct Bundle {
  int32_t first;
  uint8_t slot_log2;
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

// Emission-validity scan: one CTA per 16 KiB-aligned chunk of one record.
constexpr int kScanThreads = 256;
constexpr int kScanChunkBytes = 16384;
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

// row_vocab: the vocabulary shared by every row-staged record of the
// launch, or 0 when they differ.
cudaError_t launch_forward(const RecordDev* recs, const Bundle* bundles, const int32_t* order,
                           int num_bundles, bool row_mode, int row_vocab, const uint8_t* mask,
                           int check_inputs,
                           uint32_t* bp, uint16_t* maps, int32_t* anchors,
                           const OutputsDev& out, unsigned smem_bytes, unsigned row_slot_bytes,
                           cudaStream_t stream);
cudaError_t launch_fill(const RecordDev* recs, const FillItem* items, int num_items,
                        const uint32_t* bp, const int32_t* anchors, const OutputsDev& out,
                        cudaStream_t stream);
cudaError_t launch_validity(const ScanRecord* recs, int64_t count, const ScanItem* items,
                            int64_t num_items, uint8_t* valid, cudaStream_t stream);

// Sets the message ffa_last_error() returns on this thread (ffa_host.cpp).
void set_last_error(const char* message);

cudaError_t launch_check_targets(const RecordDev* recs, int64_t count, int32_t* status,
                                 cudaStream_t stream);


}  // namespace ffa
