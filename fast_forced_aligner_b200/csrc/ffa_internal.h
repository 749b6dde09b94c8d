// ffa_internal.h -- layouts shared by the host planner (ffa_host.cpp) and the
// sm_100a kernels (ffa_kernels.cu).  Not part of the public C ABI.
#pragma once

#include <cstddef>
#include <cstdint>

#include <cuda_runtime.h>

namespace ffa {

// DP geometry.  A record's CTC states s = 0..S-1 are owned in contiguous
// runs of kStates per thread (thread i owns 4i..4i+3), 32 threads per warp,
// up to kMaxWarps warps per record: S <= 4096, the reference's own limit
// (alignment.cu:970).  With an even run length the first state of every run
// is a blank, so a thread needs only the last state of its left neighbour.
constexpr int kStates = 4;
constexpr int kMaxWarps = 32;
constexpr int kCtaThreads = 1024;
constexpr int kMaxStates = kStates * 32 * kMaxWarps;  // 4096
// Emission prefetch ring: frames in flight per thread (cp.async groups).
constexpr int kRing = 8;
// Backpointers: 2 bits per state, 4 states per thread -> one byte per frame
// per thread; 4 frames share one 32-bit word.
constexpr int kFramesPerWord = 4;
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
  uint16_t nw;              // warps running this record's DP
  uint8_t seg_log2;         // traceback segment length H = 1 << seg_log2
  uint8_t reserved;
};
static_assert(sizeof(RecordDev) == 64, "RecordDev layout");

// One forward CTA ("bundle"): `count` records of the same slot size
// (1 << slot_log2 warps each), listed at order[first .. first+count).
struct Bundle {
  int32_t first;
  uint8_t slot_log2;
  uint8_t count;
  uint16_t reserved;
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
cudaError_t launch_forward(const RecordDev* recs, const Bundle* bundles, const int32_t* order,
                           int num_bundles, const uint8_t* mask, int check_inputs,
                           uint32_t* bp, uint16_t* maps, int32_t* anchors,
                           const OutputsDev& out, cudaStream_t stream);
cudaError_t launch_fill(const RecordDev* recs, const FillItem* items, int num_items,
                        const uint32_t* bp, const int32_t* anchors, const OutputsDev& out,
                        cudaStream_t stream);
cudaError_t launch_validity(const ScanRecord* recs, int64_t count, const ScanItem* items,
                            int64_t num_items, uint8_t* valid, cudaStream_t stream);

cudaError_t launch_check_targets(const RecordDev* recs, int64_t count, int32_t* status,
                                 cudaStream_t stream);

size_t forward_smem_bytes();

}  // namespace ffa
