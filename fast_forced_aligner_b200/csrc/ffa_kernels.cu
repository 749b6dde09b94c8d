// ffa_kernels.cu -- sm_100a kernels of the B200-native CTC forced aligner.
//
//   ffa_viterbi_forward   conventional max-plus Viterbi forward pass, one
//                         record per warp group, packed into 1024-thread CTAs;
//                         writes 2-bit backpointers and per-segment ancestor
//                         maps, then walks the maps from the terminal state
//                         (semantics: reference alignment.cu:354-523)
//   ffa_trace_fill        parallel traceback of every segment of every
//                         record + label/score gather (alignment.cu:597-667)
//   ffa_validity_scan     NaN/+inf scan of the emissions (alignment.cu:879-891)
//
// Arithmetic contract: each DP cell is ONE fp32 round-to-nearest addition of
// the selected predecessor score and the cell's emission, with the selection
// stay > step > skip decided by strict '>' comparisons, exactly as
// alignment.cu:418-424.  Max-plus with a single rounded add per cell is
// independent of how states are spread over threads, so every thread layout
// reproduces the reference bit for bit.
#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>

#include "ffa_internal.h"

namespace ffa {
namespace {

__device__ __forceinline__ void named_barrier(int id, int count) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

__device__ __forceinline__ void cp_async4(float* smem_dst, const float* gmem_src) {
  const unsigned dst = static_cast<unsigned>(__cvta_generic_to_shared(smem_dst));
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(dst), "l"(gmem_src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ int clamp_label(int64_t token, int V) {
  // Only out-of-range IDs (rejected with status 3 when checks are on) are
  // changed; clamping keeps unchecked calls from reading outside the row.
  return token < 0 ? 0 : (token >= V ? V - 1 : static_cast<int>(token));
}

struct Boundary {
  float alpha;  // score of the warp's last state
  int delta;    // its ancestor delta
};

// Dynamic shared memory of one forward CTA.
struct ForwardSmem {
  float ring[kRing][3][kCtaThreads];   // per-thread emission prefetch ring
  Boundary bnd[2][kMaxWarps];          // last-state hand-off between warps
  int red_bad[kMaxWarps];
  int red_rep[kMaxWarps];
  float term_last[kMaxWarps];          // per slot: alpha[S-1], alpha[S-2]
  float term_prev[kMaxWarps];
  int slot_status[kMaxWarps];
};

}  // namespace

// One CTA = one Bundle of records of the same slot size.  Warps of a slot run
// the record's DP in lock step with one named barrier per frame; a one-warp
// slot needs only __syncwarp.  Thread i of a record owns states 4i..4i+3.
__global__ void __launch_bounds__(kCtaThreads, 1)
ffa_viterbi_forward(const RecordDev* __restrict__ recs, const Bundle* __restrict__ bundles,
                    const int32_t* __restrict__ order, const uint8_t* __restrict__ mask,
                    int check_inputs, uint32_t* __restrict__ bp_arena,
                    uint16_t* __restrict__ map_arena, int32_t* __restrict__ anchors,
                    OutputsDev out) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  ForwardSmem& sm = *reinterpret_cast<ForwardSmem*>(smem_raw);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const Bundle bd = bundles[blockIdx.x];
  const int slot = warp >> bd.slot_log2;
  if (slot >= bd.count) return;
  const int r = order[bd.first + slot];
  const RecordDev rec = recs[r];
  const int lw = warp & ((1 << bd.slot_log2) - 1);  // warp within the record
  if (lw >= rec.nw) return;
  const int NT = rec.nw * 32;
  const int tl = lw * 32 + lane;  // thread within the record
  const bool single = rec.nw == 1;
  auto slot_sync = [&]() {
    if (single) __syncwarp();
    else named_barrier(slot, NT);
  };

  const int T = rec.T, V = rec.V, U = rec.U, blank = rec.blank;
  const int S = 2 * U + 1;
  const int64_t* tgt = rec.targets;

  // ---- status: mask, then target validation (alignment.cu:836, 852-874) ----
  int status = (mask != nullptr && !mask[r]) ? 2 : 0;
  if (check_inputs) {
    int bad = 0, rep = 0;
    for (int k = tl; k < U; k += NT) {
      const int64_t token = tgt[k];
      bad |= (token < 0 || token >= V || token == blank) ? 1 : 0;
      if (k > 0) rep += token == tgt[k - 1] ? 1 : 0;
    }
    bad = __reduce_or_sync(0xffffffffu, bad);
    rep = __reduce_add_sync(0xffffffffu, rep);
    if (lane == 0) { sm.red_bad[warp] = bad; sm.red_rep[warp] = rep; }
    slot_sync();
    if (tl == 0) {
      int b = 0, p = 0;
      for (int w = 0; w < rec.nw; ++w) { b |= sm.red_bad[warp + w]; p += sm.red_rep[warp + w]; }
      if (b) status = 3;
      else if (static_cast<int64_t>(U) + p > T) status = 4;
      sm.slot_status[slot] = status;
    }
    slot_sync();
    status = sm.slot_status[slot];
  }
  if (tl == 0) {
    // Diagnostics of the conventional route are all zero (alignment.py:101-129).
    out.stitched[r] = 0;
    out.repair_passes[r] = 0;
    out.repaired_frames[r] = 0;
    for (int j = 0; j < 3; ++j) { out.shortcut_stats[3 * r + j] = 0; out.routing_stats[3 * r + j] = 0; }
    if (out.reuse_stats) for (int j = 0; j < 4; ++j) out.reuse_stats[4 * r + j] = 0;
    if (status >= 2) { out.status[r] = status; out.objective[r] = -INFINITY; }
  }
  if (status >= 2) return;

  // ---- states owned by this thread: s = 4*tl + k; odd k carry tokens ----
  const int tok1 = 2 * tl, tok3 = 2 * tl + 1;
  const int col1 = tok1 < U ? clamp_label(tgt[tok1], V) : blank;
  const int col3 = tok3 < U ? clamp_label(tgt[tok3], V) : blank;
  const int colm = (tok1 >= 1 && tok1 - 1 < U) ? clamp_label(tgt[tok1 - 1], V) : -1;
  // Skip s-2 -> s is legal for a token state that differs from the token two
  // states back (alignment.cu:407).
  const bool sk1 = tok1 < U && tok1 >= 1 && col1 != blank && col1 != colm;
  const bool sk3 = tok3 < U && col3 != blank && col3 != col1;

  const float* e = rec.emissions;
  float* ring0 = &sm.ring[0][0][tid];
  auto issue = [&](int64_t f) {
    if (f < T) {
      const float* row = e + static_cast<int64_t>(f) * V;
      float* dst = ring0 + (f % kRing) * 3 * kCtaThreads;
      cp_async4(dst, row + blank);
      cp_async4(dst + kCtaThreads, row + col1);
      cp_async4(dst + 2 * kCtaThreads, row + col3);
    }
    cp_async_commit();
  };
#pragma unroll
  for (int f = 0; f < kRing - 1; ++f) issue(f);

  // ---- frame 0: alpha[s] = e[0, l[s]] for s < 2 (alignment.cu:409) ----
  issue(kRing - 1);
  cp_async_wait<kRing - 1>();
  float a0, a1, a2, a3;
  {
    const float* cur = ring0;
    a0 = (tl == 0) ? cur[0] : -INFINITY;
    a1 = (tl == 0 && S > 1) ? cur[kCtaThreads] : -INFINITY;
    a2 = -INFINITY;
    a3 = -INFINITY;
  }
  int d0 = 0, d1 = 0, d2 = 0, d3 = 0;
  if (lane == 31) sm.bnd[1][warp] = Boundary{a3, d3};
  slot_sync();

  const int hmask = (1 << rec.seg_log2) - 1;
  const int H = 1 << rec.seg_log2;
  uint32_t* bp = bp_arena + rec.bp_off + tl;
  uint16_t* maps = map_arena + rec.map_off + 4 * tl;
  const int64_t map_stride = static_cast<int64_t>(NT) * kStates;
  uint32_t word = 0;

  for (int t = 1; t < T; ++t) {
    issue(static_cast<int64_t>(t) + kRing - 1);
    cp_async_wait<kRing - 1>();
    const float* cur = ring0 + (t % kRing) * 3 * kCtaThreads;
    const float eb = cur[0], e1 = cur[kCtaThreads], e3 = cur[2 * kCtaThreads];

    // Left neighbour's last state (s-1 for k=0, s-2 for k=1).
    float p1 = __shfl_up_sync(0xffffffffu, a3, 1);
    int pd = __shfl_up_sync(0xffffffffu, d3, 1);
    if (lane == 0) {
      if (lw > 0) {
        const Boundary b = sm.bnd[t & 1][warp - 1];
        p1 = b.alpha;
        pd = b.delta;
      } else {
        p1 = -INFINITY;
        pd = 0;
      }
    }
    if ((t & hmask) == 0) { d0 = d1 = d2 = d3 = 0; pd = 0; }  // new traceback segment

    // k = 0 (blank): stay, step.
    const bool c0 = p1 > a0;
    const float b0 = c0 ? p1 : a0;
    const int n0 = c0 ? pd + 1 : d0;
    // k = 1 (token): stay, step, skip.
    const bool c1 = a0 > a1;
    float b1 = c1 ? a0 : a1;
    unsigned j1 = c1 ? 1u : 0u;
    int s1 = c1 ? d0 : d1;
    if (sk1 && p1 > b1) { b1 = p1; j1 = 2u; s1 = pd; }
    // k = 2 (blank): stay, step.
    const bool c2 = a1 > a2;
    const float b2 = c2 ? a1 : a2;
    const int n2 = c2 ? d1 + 1 : d2;
    // k = 3 (token): stay, step, skip.
    const bool c3 = a2 > a3;
    float b3 = c3 ? a2 : a3;
    unsigned j3 = c3 ? 1u : 0u;
    int s3 = c3 ? d2 : d3;
    if (sk3 && a1 > b3) { b3 = a1; j3 = 2u; s3 = d1; }

    a0 = __fadd_rn(b0, eb);
    a1 = __fadd_rn(b1, e1);
    a2 = __fadd_rn(b2, eb);
    a3 = __fadd_rn(b3, e3);
    d0 = n0;
    d1 = s1 + static_cast<int>(j1);
    d2 = n2;
    d3 = s3 + static_cast<int>(j3);

    const unsigned bits = (c0 ? 1u : 0u) | (j1 << 2) | ((c2 ? 1u : 0u) << 4) | (j3 << 6);
    word |= bits << (8 * (t & 3));
    if ((t & 3) == 3 || t == T - 1) {
      bp[static_cast<int64_t>(t >> 2) * NT] = word;
      word = 0;
    }
    if (t >= H && ((t & hmask) == hmask || t == T - 1)) {
      // Ancestor map of segment c = t/H: state at its last frame -> state at
      // the last frame of segment c-1, stored as a delta.
      const int64_t c = t >> rec.seg_log2;
      uint2 packed;
      packed.x = static_cast<uint32_t>(d0) | (static_cast<uint32_t>(d1) << 16);
      packed.y = static_cast<uint32_t>(d2) | (static_cast<uint32_t>(d3) << 16);
      *reinterpret_cast<uint2*>(maps + (c - 1) * map_stride) = packed;
    }
    if (lane == 31) sm.bnd[(t + 1) & 1][warp] = Boundary{a3, d3};
    slot_sync();
  }
  cp_async_wait<0>();

  // ---- terminal state (alignment.cu:497-510) ----
  const int last = S - 1;  // even
  if ((last >> 2) == tl) sm.term_last[slot] = (last & 3) == 0 ? a0 : a2;
  if (S > 1 && ((last - 1) >> 2) == tl) sm.term_prev[slot] = ((last - 1) & 3) == 1 ? a1 : a3;
  slot_sync();
  if (tl == 0) {
    const float vlast = sm.term_last[slot];
    int terminal = last;
    float objective = vlast;
    if (S > 1) {
      const float vprev = sm.term_prev[slot];
      if (vprev >= vlast) { terminal = last - 1; objective = vprev; }
    }
    const bool ok = isfinite(objective);
    out.objective[r] = objective;
    out.status[r] = ok ? 0 : 1;
    if (ok) {
      // Walk the segment maps back from the terminal: one anchor per segment.
      const int C = static_cast<int>((static_cast<int64_t>(T) + hmask) >> rec.seg_log2);
      int32_t* anc = anchors + rec.seg_off;
      const uint16_t* mp = map_arena + rec.map_off;
      int s = terminal;
      anc[C - 1] = s;
      for (int c = C - 1; c >= 1; --c) {
        s -= mp[static_cast<int64_t>(c - 1) * map_stride + s];
        anc[c - 1] = s;
      }
    }
  }
}

// One warp per traceback segment: lane 0 walks the 2-bit backpointers from the
// segment's anchor (path[t-1] = path[t] - bp[t, path[t]], alignment.cu:656-659),
// then the warp maps states to labels and gathers the selected scores
// (alignment.cu:662-666).  Failed records get -1 / -inf (alignment.cu:650-652).
__global__ void __launch_bounds__(32 * kFillWarps)
ffa_trace_fill(const RecordDev* __restrict__ recs, const FillItem* __restrict__ items,
               const uint32_t* __restrict__ bp_arena, const int32_t* __restrict__ anchors,
               OutputsDev out) {
  __shared__ int32_t path[kFillWarps][1 << kMaxSegLog2];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const FillItem item = items[blockIdx.x];
  const RecordDev rec = recs[item.record];
  const int c = item.first_seg + warp;
  const int T = rec.T;
  const int H = 1 << rec.seg_log2;
  const int C = static_cast<int>((static_cast<int64_t>(T) + H - 1) >> rec.seg_log2);
  if (c >= C) return;
  const int a = c * H;
  const int b = static_cast<int>(min(static_cast<int64_t>(T), static_cast<int64_t>(a) + H));
  int64_t* labels = out.labels + rec.out_off;
  float* scores = out.scores + rec.out_off;
  if (out.status[item.record] != 0) {
    for (int t = a + lane; t < b; t += 32) { labels[t] = -1; scores[t] = -INFINITY; }
    return;
  }
  int32_t* p = path[warp];
  if (lane == 0) {
    const int NT = rec.nw * 32;
    const uint32_t* bp = bp_arena + rec.bp_off;
    int s = anchors[rec.seg_off + c];
    int64_t cached = -1;
    uint32_t word = 0;
    p[b - 1 - a] = s;
    for (int t = b - 1; t > a; --t) {
      const int64_t key = static_cast<int64_t>(t >> 2) * NT + (s >> 2);
      if (key != cached) { word = bp[key]; cached = key; }
      s -= (word >> (8 * (t & 3) + 2 * (s & 3))) & 3u;
      p[t - 1 - a] = s;
    }
  }
  __syncwarp();
  const float* e = rec.emissions;
  for (int t = a + lane; t < b; t += 32) {
    const int s = p[t - a];
    const int label = (s & 1) ? clamp_label(rec.targets[s >> 1], rec.V) : rec.blank;
    labels[t] = label;
    scores[t] = e[static_cast<int64_t>(t) * rec.V + label];
  }
}

// valid[r] was set to 1; any CTA finding NaN or +inf in its chunk clears it.
// Chunks are 16 KiB windows aligned to 16 bytes, so interior loads are float4.
__global__ void __launch_bounds__(kScanThreads)
ffa_validity_scan(const ScanRecord* __restrict__ recs, const ScanItem* __restrict__ items,
                  uint8_t* __restrict__ valid) {
  const ScanItem item = items[blockIdx.x];
  const ScanRecord rec = recs[item.record];
  const uintptr_t base = reinterpret_cast<uintptr_t>(rec.data);
  const uintptr_t aligned = base & ~static_cast<uintptr_t>(15);
  const uintptr_t end = base + static_cast<uintptr_t>(rec.count) * 4;
  const uintptr_t lo = aligned + static_cast<uintptr_t>(item.chunk) * kScanChunkBytes;
  const uintptr_t hi = lo + kScanChunkBytes < end ? lo + kScanChunkBytes : end;
  bool bad = false;
  for (uintptr_t p = lo + 16 * threadIdx.x; p < hi; p += 16 * kScanThreads) {
    // Whole 16-byte blocks are read; lanes outside [base, end) are ignored.
    const float4 v = __ldcs(reinterpret_cast<const float4*>(p));
    const float x[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const uintptr_t q = p + 4 * k;
      if (q >= base && q < end) bad |= isnan(x[k]) || x[k] == INFINITY;
    }
  }
  if (__syncthreads_or(bad) && threadIdx.x == 0) valid[item.record] = 0;
}

// One warp per record: the target checks of the forward kernel without the DP.
__global__ void __launch_bounds__(256)
ffa_check_targets_kernel(const RecordDev* __restrict__ recs, int64_t count,
                         int32_t* __restrict__ status) {
  const int64_t r = blockIdx.x * 8LL + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (r >= count) return;
  const RecordDev rec = recs[r];
  int bad = 0, rep = 0;
  for (int k = lane; k < rec.U; k += 32) {
    const int64_t token = rec.targets[k];
    bad |= (token < 0 || token >= rec.V || token == rec.blank) ? 1 : 0;
    if (k > 0) rep += token == rec.targets[k - 1] ? 1 : 0;
  }
  bad = __reduce_or_sync(0xffffffffu, bad);
  rep = __reduce_add_sync(0xffffffffu, rep);
  if (lane == 0)
    status[r] = bad ? 3 : (static_cast<int64_t>(rec.U) + rep > rec.T ? 4 : 0);
}

__global__ void ffa_fill_u8(uint8_t* p, int64_t n, uint8_t value) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    p[i] = value;
}

size_t forward_smem_bytes() { return sizeof(ForwardSmem); }

cudaError_t launch_forward(const RecordDev* recs, const Bundle* bundles, const int32_t* order,
                           int num_bundles, const uint8_t* mask, int check_inputs,
                           uint32_t* bp, uint16_t* maps, int32_t* anchors,
                           const OutputsDev& out, cudaStream_t stream) {
  if (num_bundles <= 0) return cudaSuccess;
  const size_t smem = sizeof(ForwardSmem);
  // Opting in to >48 KiB of dynamic shared memory is per device; the call is
  // cheap and idempotent, so it is repeated rather than cached.
  cudaError_t err = cudaFuncSetAttribute(ffa_viterbi_forward,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
  if (err != cudaSuccess) return err;
  ffa_viterbi_forward<<<num_bundles, kCtaThreads, smem, stream>>>(
      recs, bundles, order, mask, check_inputs, bp, maps, anchors, out);
  return cudaGetLastError();
}

cudaError_t launch_fill(const RecordDev* recs, const FillItem* items, int num_items,
                        const uint32_t* bp, const int32_t* anchors, const OutputsDev& out,
                        cudaStream_t stream) {
  if (num_items <= 0) return cudaSuccess;
  ffa_trace_fill<<<num_items, 32 * kFillWarps, 0, stream>>>(recs, items, bp, anchors, out);
  return cudaGetLastError();
}

cudaError_t launch_check_targets(const RecordDev* recs, int64_t count, int32_t* status,
                                 cudaStream_t stream) {
  ffa_check_targets_kernel<<<static_cast<unsigned>((count + 7) / 8), 256, 0, stream>>>(recs, count, status);
  return cudaGetLastError();
}

cudaError_t launch_validity(const ScanRecord* recs, int64_t count, const ScanItem* items,
                            int64_t num_items, uint8_t* valid, cudaStream_t stream) {
  const int fill_blocks = static_cast<int>((count + 255) / 256);
  ffa_fill_u8<<<fill_blocks, 256, 0, stream>>>(valid, count, 1);
  cudaError_t err = cudaGetLastError();
  if (err != cudaSuccess || num_items <= 0) return err;
  ffa_validity_scan<<<static_cast<unsigned>(num_items), kScanThreads, 0, stream>>>(recs, items, valid);
  return cudaGetLastError();
}

}  // namespace ffa
