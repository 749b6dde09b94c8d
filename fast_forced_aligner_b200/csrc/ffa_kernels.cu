// ffa_kernels.cu -- sm_100a kernels of the B200-native CTC forced aligner.
//
//   ffa_viterbi_forward   conventional max-plus Viterbi forward pass, one
//                         record per warp group, packed into 512-thread CTAs;
//                         writes 2-bit backpointers and per-segment ancestor
//                         maps, then walks the maps from the terminal state
//                         (semantics: reference alignment.cu:354-523)
//   ffa_trace_fill        parallel traceback of every segment of every
//                         record + label/score gather (alignment.cu:597-667)
//   ffa_validity_scan     NaN/+inf scan of the emissions (alignment.cu:879-891)
//   ffa_check_targets     target-ID and frame-feasibility checks alone
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
__device__ __forceinline__ unsigned smem_u32(const void* p) {
  return static_cast<unsigned>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void cp_async4(float* smem_dst, const float* gmem_src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(smem_dst)), "l"(gmem_src)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ void mbar_init(unsigned long long* bar, unsigned count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(unsigned long long* bar, unsigned bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(unsigned long long* bar, unsigned parity) {
  unsigned ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
// Bounded wait: gives up after kWaitNs nanoseconds and reports the failure
// instead of hanging.  A caller that saw one failure makes no further waits.
__device__ __forceinline__ bool mbar_wait(unsigned long long* bar, unsigned parity,
                                          unsigned long long limit_ns = kWaitNs) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long start = global_ns();
  while (!mbar_try_wait(bar, parity))
    if (global_ns() - start > limit_ns) return false;
  return true;
}
// One TMA bulk copy global -> shared (no tensor map, no multicast), completed
// on `bar` with a transaction-byte count.
__device__ __forceinline__ void tma_bulk_load(void* smem_dst, const void* gmem_src, unsigned bytes,
                                              unsigned long long* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(smem_dst)),
      "l"(gmem_src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}
__device__ __forceinline__ void fence_proxy_async() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ int clamp_label(int64_t token, int V) {
  // Only out-of-range IDs (rejected with status 3 when checks are on) are
  // changed; clamping keeps unchecked calls from reading outside the row.
  return token < 0 ? 0 : (token >= V ? V - 1 : static_cast<int>(token));
}

struct Boundary {
  float alpha;  // score of a warp's last state
  int delta;    // its ancestor delta
};

// Shared-memory header of one forward CTA; emission rings follow it.
struct ForwardShared {
  Boundary bnd[2][kMaxWarps];  // last-state hand-off between warps of a slot
  Boundary edge;               // {-inf, 0}: the "left neighbour" of a record's first warp
  int red_bad[kMaxWarps];
  int red_rep[kMaxWarps];
  float term_last[kMaxWarps];  // per slot: alpha[S-1], alpha[S-2]
  float term_prev[kMaxWarps];
  int slot_status[kMaxWarps];
  int slot_fault[kMaxWarps];   // a bounded wait ran out (reported as status 5)
  unsigned long long full[kMaxWarps][kRowRing];  // per slot: row group landed
};

// Emission rings start at this 128-byte aligned offset (TMA destinations
// must be 16-byte aligned); the host planner uses the same value.
constexpr size_t kForwardHeader = (sizeof(ForwardShared) + 127) / 128 * 128;
static_assert(kForwardHeader % 128 == 0, "ring offset alignment");

// One DP frame for this thread's K states (s = K*tl + k; odd k are tokens).
// Selection: stay, then step if strictly greater, then skip if strictly
// greater and legal (alignment.cu:418-424); one fp32 add per cell.  Also
// advances the ancestor deltas d (distance back to the state at the end of the
// previous traceback segment).  Returns the frame's backpointers as two bit
// planes: bit k = "moved" (jump >= 1) of state k, bit K+q = "skipped"
// (jump == 2) of token q = k/2, so jump = moved + skipped.
template <int K>
__device__ __forceinline__ unsigned dp_frame(float (&a)[K], int (&d)[K], float p1, int pd, float eb,
                                             const float (&et)[K / 2], unsigned skip) {
  float na[K];
  int nd[K];
  unsigned bits = 0;
#pragma unroll
  for (int k = 0; k < K; ++k) {
    const float x1 = k >= 1 ? a[k - 1] : p1;
    const int d1 = k >= 1 ? d[k - 1] : pd;
    const bool c = x1 > a[k];
    float b = c ? x1 : a[k];
    int n = c ? d1 + 1 : d[k];
    if (k & 1) {
      const float x2 = k >= 2 ? a[k - 2] : p1;
      const int d2 = k >= 2 ? d[k - 2] : pd;
      const bool j2 = ((skip >> (k >> 1)) & 1u) && x2 > b;
      b = j2 ? x2 : b;
      n = j2 ? d2 + 2 : n;
      bits |= (static_cast<unsigned>(c || j2) << k) | (static_cast<unsigned>(j2) << (K + (k >> 1)));
      na[k] = __fadd_rn(b, et[k >> 1]);
    } else {
      bits |= static_cast<unsigned>(c) << k;
      na[k] = __fadd_rn(b, eb);
    }
    nd[k] = n;
  }
#pragma unroll
  for (int k = 0; k < K; ++k) { a[k] = na[k]; d[k] = nd[k]; }
  return bits;
}

// Backpointer word geometry: 1.5*K bits per frame and thread, packed in
// 16-bit lanes of 32-bit words when they fit (two frames per word).
__host__ __device__ constexpr int frames_per_word(int K) { return 3 * K / 2 <= 16 ? 2 : 1; }

// Jump of state s (owned by a thread with K states) from one frame's bits.
__device__ __forceinline__ int jump_of(unsigned bits, int s, int K) {
  const int k = s % K;
  const unsigned moved = (bits >> k) & 1u;
  const unsigned skipped = (k & 1) ? (bits >> (K + (k >> 1))) & 1u : 0u;
  return static_cast<int>(moved + skipped);
}

// Per-record geometry shared by the DP body.
struct SlotCtx {
  int tid, warp, lane, slot, lw, NT, tl, r;
  bool single;
  __device__ __forceinline__ void sync() const {
    // Unconditional (a one-warp record uses a 32-thread barrier): a branch
    // here costs more than the barrier.
    named_barrier(slot, NT);
  }
};

// The DP of one record after its status checks: frame loop unrolled by
// kGroup, terminal state, segment-map walk.  Thread tl owns states
// K*tl .. K*tl+K-1 (odd offsets are tokens K/2*tl + k/2).
template <int K, bool kRow, int kV>
__device__ __forceinline__ void record_dp(const SlotCtx& x, const RecordDev& rec,
                                          ForwardShared& sh, unsigned char* smem_raw,
                                          uint32_t* __restrict__ bp_arena,
                                          uint16_t* __restrict__ map_arena,
                                          int32_t* __restrict__ anchors, const OutputsDev& out,
                                          unsigned row_slot_bytes) {
  constexpr int KT = K / 2;
  constexpr int FPW = frames_per_word(K);
  const int tl = x.tl, lane = x.lane, warp = x.warp, NT = x.NT, slot = x.slot;
  const int T = rec.T, U = rec.U, blank = rec.blank;
  const int V = kV > 0 ? kV : rec.V;
  const int S = 2 * U + 1;
  const int64_t* tgt = rec.targets;

  int col[KT];
  unsigned skip = 0;
  {
    const int first = KT * tl;
    int prev = (first >= 1 && first - 1 < U) ? clamp_label(tgt[first - 1], V) : -1;
#pragma unroll
    for (int q = 0; q < KT; ++q) {
      const int u = first + q;
      col[q] = u < U ? clamp_label(tgt[u], V) : blank;
      // Skip s-2 -> s is legal for a token that differs from the previous
      // token and from the blank (alignment.cu:407).
      if (u < U && u >= 1 && col[q] != blank && col[q] != prev) skip |= 1u << q;
      prev = col[q];
    }
  }

  const float* e = rec.emissions;
  const int ngroups = (T + kGroup - 1) / kGroup;
  float* ring = reinterpret_cast<float*>(smem_raw + kForwardHeader) +
                static_cast<size_t>(slot) * (row_slot_bytes / 4);
  float* gring = reinterpret_cast<float*>(smem_raw + kForwardHeader) + x.tid;
  unsigned long long* full = sh.full[slot];
  bool fault = false;

  const int nchunks = (T + kChunkFrames - 1) / kChunkFrames;
  auto issue_chunk = [&](int c) {  // kRow: by the record's thread 0
    const int first = c * kChunkFrames;
    const int rows = min(kChunkFrames, T - first);
    const unsigned bytes = static_cast<unsigned>(rows) * V * 4u;
    unsigned long long* bar = &full[c % kRowRing];
    mbar_expect_tx(bar, bytes);
    tma_bulk_load(ring + (c % kRowRing) * kChunkFrames * V, e + static_cast<int64_t>(first) * V, bytes, bar);
  };
  auto gather = [&](int64_t f) {  // !kRow: KT + 1 private 4-byte copies
    if (f < T) {
      const float* row = e + f * V;
      float* dst = gring + (f % kGroup) * (KT + 1) * kCtaThreads;
      cp_async4(dst, row + blank);
#pragma unroll
      for (int q = 0; q < KT; ++q) cp_async4(dst + (q + 1) * kCtaThreads, row + col[q]);
    }
    cp_async_commit();
  };
  if constexpr (kRow) {
    if (tl == 0) {
      for (int k = 0; k < kRowRing; ++k) mbar_init(&full[k], 1);
      fence_mbar_init();
      for (int c = 0; c < kRowRing && c < nchunks; ++c) issue_chunk(c);
    }
  } else {
#pragma unroll
    for (int f = 0; f < kGroup - 1; ++f) gather(f);
  }
  x.sync();

  float a[K];
  int d[K];
#pragma unroll
  for (int k = 0; k < K; ++k) { a[k] = -INFINITY; d[k] = 0; }
  const int hmask = (1 << rec.seg_log2) - 1;
  uint32_t* bp = bp_arena + rec.bp_off + tl;
  uint16_t* maps = map_arena + rec.map_off + K * tl;
  const int64_t map_stride = static_cast<int64_t>(NT) * K;
  const Boundary* left = x.lw > 0 ? &sh.bnd[0][warp - 1] : &sh.edge;
  const int left_stride = x.lw > 0 ? kMaxWarps : 0;
  // Skip frames in which none of this warp's states lies in the reachable
  // band [S - 2(T - t), 2t + 1]: states above it are still unreachable (-inf)
  // and states below it can no longer reach the end, and in-band states read
  // only in-band states, so skipping is exact.  Active iff
  // band_lo <= 2t <= band_hi.
  const int w_lo = x.lw * 32 * K;
  const int w_hi = w_lo + 32 * K - 1;
  const unsigned band_lo = static_cast<unsigned>(max(w_lo - 1, 0));
  const int64_t hi64 = static_cast<int64_t>(w_hi) - S + 2 * static_cast<int64_t>(T);
  const bool never = hi64 < 0;
  const unsigned band_hi = never ? 0u : (hi64 > 0xffffffffLL ? 0xffffffffu : static_cast<unsigned>(hi64));
  uint32_t word = 0;

  auto load = [&](int t, int j, const float* rows, float& eb, float (&et)[KT]) {
    if constexpr (kRow) {
      const float* row = rows + j * V;
      eb = row[blank];
#pragma unroll
      for (int q = 0; q < KT; ++q) et[q] = row[col[q]];
    } else {
      gather(static_cast<int64_t>(t) + kGroup - 1);
      cp_async_wait<kGroup - 1>();
      const float* cur = gring + (t & (kGroup - 1)) * (KT + 1) * kCtaThreads;
      eb = cur[0];
#pragma unroll
      for (int q = 0; q < KT; ++q) et[q] = cur[(q + 1) * kCtaThreads];
    }
  };
  auto store_map = [&](int t) {
    // Ancestor map of segment t/H: state at its last frame -> state at the
    // last frame of the previous segment, as a delta.
    uint32_t* dst = reinterpret_cast<uint32_t*>(maps + ((t >> rec.seg_log2) - 1) * map_stride);
#pragma unroll
    for (int q = 0; q < KT; ++q)
      dst[q] = static_cast<uint32_t>(d[2 * q]) | (static_cast<uint32_t>(d[2 * q + 1]) << 16);
  };
  auto store_word = [&](int t) {
    bp[static_cast<int64_t>(t / FPW) * NT] = word;
    word = 0;
  };
  auto frame = [&](int t, int j, const float* rows) {
    float eb, et[KT];
    load(t, j, rows, eb, et);
    // Left neighbour's last state at t-1 (s-1 for k=0, s-2 for k=1): from
    // lane-1, or for lane 0 from the warp on the left (branch-free).
    float p1 = __shfl_up_sync(0xffffffffu, a[K - 1], 1);
    int pd = __shfl_up_sync(0xffffffffu, d[K - 1], 1);
    const Boundary nb = left[(t & 1) * left_stride];
    if (lane == 0) { p1 = nb.alpha; pd = nb.delta; }
    if (j == 0 && (t & hmask) == 0) {  // a new traceback segment starts at t
#pragma unroll
      for (int k = 0; k < K; ++k) d[k] = 0;
      pd = 0;
    }
    const unsigned bits = dp_frame<K>(a, d, p1, pd, eb, et, skip);
    if constexpr (FPW == 2) {
      word |= bits << (16 * (t & 1));
      if (t & 1) store_word(t);
    } else {
      word = bits;
      store_word(t);
    }
    if (j == kGroup - 1 && (t & hmask) == hmask && t > hmask) store_map(t);
    if (lane == 31) sh.bnd[(t + 1) & 1][warp] = Boundary{a[K - 1], d[K - 1]};
    x.sync();
  };

  for (int g = 0; g < ngroups; ++g) {
    const float* rows = nullptr;
    if constexpr (kRow) {
      const int c = g / kChunkGroups;
      if (g % kChunkGroups == 0 && !fault && !mbar_wait(&full[c % kRowRing], (c / kRowRing) & 1))
        fault = true;
      rows = ring + ((c % kRowRing) * kChunkFrames + (g % kChunkGroups) * kGroup) * V;
    }
    const int t0 = g * kGroup;
    // The band test is made once per group: a group with at least one frame
    // in which this warp has in-band states runs every frame (the plain DP is
    // exact everywhere); a group with none only keeps the barriers (and the
    // gather ring) in step.  Its backpointers and maps are never read.
    const unsigned g2 = 2u * static_cast<unsigned>(t0);
    const bool group_active = g == 0 || (!never && g2 + 2u * (kGroup - 1) >= band_lo && g2 <= band_hi);
    if (!group_active) {
#pragma unroll 1
      for (int j = 0; j < kGroup && t0 + j < T; ++j) {
        if constexpr (!kRow) {
          float eb, et[KT];
          load(t0 + j, j, rows, eb, et);
        }
        x.sync();
      }
      if constexpr (FPW == 2) word = 0;
    } else if (g == 0) {
      // Frame 0: alpha[s] = e[0, l[s]] for s < 2, else -inf (alignment.cu:409).
      float eb, et[KT];
      load(0, 0, rows, eb, et);
#pragma unroll
      for (int k = 0; k < K; ++k) { a[k] = -INFINITY; d[k] = 0; }
      if (tl == 0) {
        a[0] = eb;
        if (S > 1) a[1] = et[0];
      }
      if (lane == 31) sh.bnd[1][warp] = Boundary{a[K - 1], 0};
      x.sync();
#pragma unroll 1
      for (int j = 1; j < kGroup && j < T; ++j) frame(j, j, rows);
    } else {
#pragma unroll
      for (int j = 0; j < kGroup; ++j)
        if (t0 + j < T) frame(t0 + j, j, rows);
    }
    if constexpr (kRow) {
      // Every thread has read this chunk's rows (the last barrier above), so
      // its ring slot can take the chunk kRowRing ahead.
      const int c = g / kChunkGroups;
      if (tl == 0 && (g % kChunkGroups == kChunkGroups - 1 || g == ngroups - 1) &&
          c + kRowRing < nchunks) {
        fence_proxy_async();
        issue_chunk(c + kRowRing);
      }
    }
  }
  if constexpr (!kRow) cp_async_wait<0>();
  if constexpr (kRow) {
    // After a failed wait, give the issuing thread's copies still in flight a
    // short, bounded chance to land before the CTA's shared memory goes away.
    if (fault && tl == 0)
      for (int c = max(0, nchunks - kRowRing); c < nchunks; ++c)
        mbar_wait(&full[c % kRowRing], (c / kRowRing) & 1, kDrainNs);
  }
  {  // a word or a map the last frame left open
    const int tl_ = T - 1;
    if (FPW == 2 && tl_ > 0 && (tl_ & 1) == 0) store_word(tl_);
    if (tl_ > hmask && (tl_ & hmask) != hmask) store_map(tl_);
  }
  if (fault) sh.slot_fault[slot] = 1;

  // ---- terminal state (alignment.cu:497-510) ----
  const int last = S - 1;  // even
  // One predicated store per state keeps a[] in registers (a runtime index
  // into it would move the array to local memory).
#pragma unroll
  for (int k = 0; k < K; ++k) {
    const int s = K * tl + k;
    if (s == last) sh.term_last[slot] = a[k];
    if (s == last - 1) sh.term_prev[slot] = a[k];
  }
  x.sync();
  if (tl == 0) {
    const float vlast = sh.term_last[slot];
    int terminal = last;
    float objective = vlast;
    if (S > 1) {
      const float vprev = sh.term_prev[slot];
      if (vprev >= vlast) { terminal = last - 1; objective = vprev; }
    }
    const bool ok = isfinite(objective);
    out.objective[x.r] = objective;
    out.status[x.r] = sh.slot_fault[slot] ? kStatusDeviceFault : (ok ? 0 : 1);
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

}  // namespace

// One CTA = one Bundle of records with the same slot size and the same states
// per thread.  Warps of a slot run the record's DP in lock step with one named
// barrier per frame (a one-warp slot needs only __syncwarp).  kRow: emission
// rows arrive kGroup frames at a time by one TMA bulk copy into a
// kRowRing-deep ring per record; otherwise each thread gathers its columns
// with cp.async into a private ring (large vocabularies).
template <bool kRow, int kV>
__global__ void __launch_bounds__(kCtaThreads, 1)
ffa_viterbi_forward(const RecordDev* __restrict__ recs, const Bundle* __restrict__ bundles,
                    const int32_t* __restrict__ order, const uint8_t* __restrict__ mask,
                    int check_inputs, uint32_t* __restrict__ bp_arena,
                    uint16_t* __restrict__ map_arena, int32_t* __restrict__ anchors,
                    OutputsDev out, unsigned row_slot_bytes) {
  extern __shared__ __align__(128) unsigned char smem_raw[];
  ForwardShared& sh = *reinterpret_cast<ForwardShared*>(smem_raw);

  SlotCtx x;
  x.tid = threadIdx.x;
  x.warp = x.tid >> 5;
  x.lane = x.tid & 31;
  const Bundle bd = bundles[blockIdx.x];
  x.slot = x.warp >> bd.slot_log2;
  if (x.tid == 0) sh.edge = Boundary{-INFINITY, 0};
  __syncthreads();
  if (x.slot >= bd.count) return;
  x.r = order[bd.first + x.slot];
  const RecordDev rec = recs[x.r];
  x.lw = x.warp & ((1 << bd.slot_log2) - 1);  // warp within the record
  if (x.lw >= rec.nw) return;
  x.NT = rec.nw * 32;
  x.tl = x.lw * 32 + x.lane;  // thread within the record
  x.single = rec.nw == 1;
  const int tl = x.tl, lane = x.lane, warp = x.warp, r = x.r;
  const int T = rec.T, V = rec.V, U = rec.U, blank = rec.blank;
  const int64_t* tgt = rec.targets;

  // ---- status: mask, then target validation (alignment.cu:836, 852-874) ----
  int status = (mask != nullptr && !mask[r]) ? 2 : 0;
  if (tl == 0) sh.slot_fault[x.slot] = 0;
  if (check_inputs) {
    int bad = 0, rep = 0;
    for (int k = tl; k < U; k += x.NT) {
      const int64_t token = tgt[k];
      bad |= (token < 0 || token >= V || token == blank) ? 1 : 0;
      if (k > 0) rep += token == tgt[k - 1] ? 1 : 0;
    }
    bad = __reduce_or_sync(0xffffffffu, bad);
    rep = __reduce_add_sync(0xffffffffu, rep);
    if (lane == 0) { sh.red_bad[warp] = bad; sh.red_rep[warp] = rep; }
    x.sync();
    if (tl == 0) {
      int b = 0, p = 0;
      for (int w = 0; w < rec.nw; ++w) { b |= sh.red_bad[warp + w]; p += sh.red_rep[warp + w]; }
      if (b) status = 3;
      else if (static_cast<int64_t>(U) + p > T) status = 4;
      sh.slot_status[x.slot] = status;
    }
    x.sync();
    status = sh.slot_status[x.slot];
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

  switch (rec.kst) {
    default:
      record_dp<8, kRow, kV>(x, rec, sh, smem_raw, bp_arena, map_arena, anchors, out, row_slot_bytes);
      break;
    case 4:
      record_dp<4, kRow, kV>(x, rec, sh, smem_raw, bp_arena, map_arena, anchors, out, row_slot_bytes);
      break;


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
  {
    // The path moves at most 2 states per frame, so over FB frames it stays
    // within 2*FB/K + 2 threads' words: the warp loads those FB x NTH words
    // in one round trip, then steps through them with shuffles.  Every lane
    // tracks the same state.
    const int NT = rec.nw * 32;
    const int K = rec.kst;
    const int fpw = frames_per_word(K);
    const int FB = K >= 8 ? 8 : 6;
    const int NTH = 2 * FB / K + 2;
    const uint32_t* bp = bp_arena + rec.bp_off;
    int s = anchors[rec.seg_off + c];
    if (lane == 0) p[b - 1 - a] = s;
    for (int t = b - 1; t > a;) {
      const int f = lane / NTH, dd = lane % NTH;
      const int tt = t - f;
      const int th = s / K - dd;
      uint32_t w = 0;
      if (f < FB && tt > a && th >= 0) w = bp[static_cast<int64_t>(tt / fpw) * NT + th];
      const int steps = min(FB, t - a);
      const int th0 = s / K;
      for (int i = 0; i < steps; ++i) {
        const int ct = t - i;
        const uint32_t word = __shfl_sync(0xffffffffu, w, i * NTH + (th0 - s / K));
        s -= jump_of(fpw == 2 ? word >> (16 * (ct & 1)) : word, s, K);
        if (lane == 0) p[ct - 1 - a] = s;
      }
      t -= steps;
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

size_t forward_header_bytes() { return kForwardHeader; }

cudaError_t launch_forward(const RecordDev* recs, const Bundle* bundles, const int32_t* order,
                           int num_bundles, bool row_mode, int row_vocab, const uint8_t* mask,
                           int check_inputs,
                           uint32_t* bp, uint16_t* maps, int32_t* anchors,
                           const OutputsDev& out, unsigned smem_bytes, unsigned row_slot_bytes,
                           cudaStream_t stream) {
  if (num_bundles <= 0) return cudaSuccess;
  auto kernel = !row_mode ? ffa_viterbi_forward<false, 0>
                         : (row_vocab == 32 ? ffa_viterbi_forward<true, 32> : ffa_viterbi_forward<true, 0>);
  // Opting in to >48 KiB of dynamic shared memory is per device; the call is
  // cheap and idempotent, so it is repeated rather than cached.
  cudaError_t err = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem_bytes));
  if (err != cudaSuccess) return err;
  kernel<<<num_bundles, kCtaThreads, smem_bytes, stream>>>(
      recs, bundles, order, mask, check_inputs, bp, maps, anchors, out, row_slot_bytes);
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
