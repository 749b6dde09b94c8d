// ffa_kernels.cu -- sm_100a kernels of the B200-native CTC forced aligner.
//
//   ffa_viterbi_forward   the first pass: max-plus Viterbi forward over every
//                         whole record (conventional DP, semantics of the
//                         reference's alignment.cu:354-523) and over every
//                         32-frame piece of a record of the optimized route
//                         (relaxed DPs, free start, best end); slots of warps
//                         packed into 512-thread CTAs, emission rows staged by
//                         TMA bulk copies; writes 2-bit backpointer rows,
//                         segment anchors and, for pieces, end frontiers
//   ffa_finish_route      the optimized route after the first pass: seam
//                         plans, repairs of merged regions resumed from saved
//                         frontiers, the conventional DP as fallback, routes
//                         and diagnostics (alignment.cu:157-228, 525-592)
//   ffa_trace_fill        parallel traceback of every segment of every
//                         record + label/score gather (alignment.cu:597-667),
//                         and the objective of joined records
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

#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdint>

#include "ffa_device.cuh"
#include "ffa_internal.h"

namespace ffa {
using namespace dev;
namespace {

// Per-slot geometry shared by the DP body.
struct SlotCtx {
  int tid, warp, lane, slot, lw, NT, tl, r, first_warp, bar;
  __device__ __forceinline__ void sync() const {
    // Unconditional (a one-warp slot uses a 32-thread barrier): a branch
    // here costs more than the barrier.
    named_barrier(bar, NT);
  }
};

// How a run's first frame is seeded.
enum : int {
  kInitRecord = 0,    // frame 0 of the record: alpha[s] = e[0, l[s]] for s < 2
  kInitFree = 1,      // free start: alpha[s] = e[t0, l[s]] on the reachable band
  kInitFrontier = 2,  // alpha at t0-1 from a saved frontier
};

// One DP run over frames [t0, t1) of a record, made of `pieces` consecutive
// pieces: piece k starts at t0 + k * kPieceFrames (the last one runs to t1),
// and every piece after the first restarts with a free start.  A piece ends
// at its best reachable state, or by the terminal rule at the record's last
// frame.  a0 is the first frame of the region whose segment chain the single
// piece of a one-piece run walks (a0 < t0 when a repair resumes a region).
//   end_piece < 0   the whole record, with the conventional outputs;
//   otherwise       piece k writes PieceState end_piece + k (its end state
//                   and flags) and start_piece + k (its region's start).
struct PieceRun {
  int a0, t0, t1, init, pieces;
  const float* frontier_in;
  float* frontier_out;  // piece k's end frontier at frontier_out + k * NT*K
  int end_piece, start_piece;
  bool new_region;
  // Row staging: emission chunks the slot's ring has already carried in
  // earlier runs of this launch.  The ring's mbarriers are initialised once,
  // by a slot's first run (chunk_base 0); later runs continue their phases.
  int chunk_base;
};

// The DP of one run: frame loop unrolled by kGroup, emission staging, end
// states, and the path's state at every segment end (anchors) and at the
// region's first frame.  kMaps: ancestor deltas ride along with the DP and
// segment maps are stored, so the anchors come from a walk over the maps
// (whole records, where the fill traces segments in parallel); otherwise the
// anchors come from warp traces over the backpointers after the DP (pieces,
// one or two segments each, and repaired regions).  Thread tl owns states
// K*tl .. K*tl+K-1 (odd offsets are tokens K/2*tl + k/2).
// kFmt: the input format (Input<kFmt>); logits rows are staged and gathered
// as stored and normalised as they are read.
// Returns the number of emission chunks the run staged (row staging).
template <int K, bool kRow, int kV, bool kMaps, int kFmt>
__device__ __forceinline__ int piece_dp(const SlotCtx& x, const RecordDev& rec, const PieceRun& run,
                                        ForwardShared& sh, unsigned char* smem_raw,
                                        const ForwardParams& P) {
  using In = Input<kFmt>;
  using Elem = typename In::Elem;
  constexpr int KT = K / 2;
  constexpr int kGroupsPerPiece = kPieceFrames / kGroup;
  const int tl = x.tl, lane = x.lane, warp = x.warp, NT = x.NT, slot = x.slot;
  const int T = rec.T, U = rec.U, blank = rec.blank;
  const int V = kV > 0 ? kV : rec.V;
  const int S = 2 * U + 1;
  const int t0 = run.t0, t1 = run.t1, nfr = t1 - t0;
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

  // Emission rows of this run, frame t0 first.
  const Elem* e = reinterpret_cast<const Elem*>(rec.emissions) + static_cast<int64_t>(t0) * V;
  const int ngroups = (nfr + kGroup - 1) / kGroup;
  Elem* ring = reinterpret_cast<Elem*>(smem_raw + kForwardHeader) +
               static_cast<size_t>(slot) * (P.row_slot_bytes / sizeof(Elem));
  float* gring = reinterpret_cast<float*>(smem_raw + kForwardHeader) + x.tid;
  unsigned long long* full = sh.full[slot];
  bool fault = false;
  HalfWords hw{};
  if constexpr (In::kHalf && !kRow) hw.set(rec.emissions);
  // z of the run's frames, a 32-frame block at a time (blocks follow the
  // emission chunks).
  static_assert(kChunkGroups * kGroup == 32, "log-sum-exp blocks");
  LseStream lse{};
  if constexpr (In::kLogits) lse.start(P.lse + rec.out_off, T, t0, lane);

  const int nchunks = (nfr + kChunkFrames - 1) / kChunkFrames;
  const int cb = run.chunk_base;
  // Chunk c of this run is the slot's chunk cb + c: ring entry and mbarrier
  // (cb + c) % kRowRing, phase parity ((cb + c) / kRowRing) & 1.
  auto issue_chunk = [&](int c) {  // kRow: by the slot's thread 0
    const int first = c * kChunkFrames;
    const int rows = min(kChunkFrames, nfr - first);
    const unsigned bytes = static_cast<unsigned>(rows) * V * static_cast<unsigned>(sizeof(Elem));
    unsigned long long* bar = &full[(cb + c) % kRowRing];
    mbar_expect_tx(bar, bytes);
    tma_bulk_load(ring + ((cb + c) % kRowRing) * kChunkFrames * V, e + static_cast<int64_t>(first) * V,
                  bytes, bar);
  };
  auto gather = [&](int f) {  // !kRow: KT + 1 private 4-byte copies of run frame f
    if (f < nfr) {
      float* dst = gring + (f % kGroup) * (KT + 1) * kCtaThreads;
      if constexpr (In::kHalf) {
        const int64_t i = static_cast<int64_t>(t0 + f) * V;
        cp_async4(dst, hw.word(i + blank));
#pragma unroll
        for (int q = 0; q < KT; ++q) cp_async4(dst + (q + 1) * kCtaThreads, hw.word(i + col[q]));
      } else {
        const float* row = e + static_cast<int64_t>(f) * V;
        cp_async4(dst, row + blank);
#pragma unroll
        for (int q = 0; q < KT; ++q) cp_async4(dst + (q + 1) * kCtaThreads, row + col[q]);
      }
    }
    cp_async_commit();
  };
  if constexpr (kRow) {
    if (tl == 0) {
      if (cb == 0) {
        for (int k = 0; k < kRowRing; ++k) mbar_init(&full[k], 1);
        fence_mbar_init();
      } else {
        // The ring's entries were read by the previous run (generic proxy)
        // before this run's copies (async proxy) overwrite them.
        fence_proxy_async();
      }
      for (int c = 0; c < kRowRing && c < nchunks; ++c) issue_chunk(c);
    }
  } else {
#pragma unroll
    for (int f = 0; f < kGroup - 1; ++f) gather(f);
  }

  float a[K];
  int d[K];  // ancestor deltas (kMaps only)
#pragma unroll
  for (int k = 0; k < K; ++k) { a[k] = -INFINITY; d[k] = 0; }
  if (run.init == kInitFrontier) {
    // Resume: alpha at frame t0-1 as the previous run left it.
    const float4* src = reinterpret_cast<const float4*>(run.frontier_in + K * tl);
#pragma unroll
    for (int k = 0; k < K; k += 4) {
      const float4 v = __ldcg(src + k / 4);  // through L2: another CTA may have written it
      a[k] = v.x; a[k + 1] = v.y; a[k + 2] = v.z; a[k + 3] = v.w;
    }
    if (lane == 31) sh.bnd[t0 & 1][warp] = Boundary{a[K - 1], 0};
  }
  x.sync();

  const int hmask = (1 << rec.seg_log2) - 1;
  // Backpointer rows (a 2-bit code per state, bp_row_words(S) words per
  // frame); a thread whose states start past the row has none to store.
  const int row_words = bp_row_words(S);
  uint8_t* bp_rows = reinterpret_cast<uint8_t*>(P.bp + rec.bp_off);
  const bool stores_codes = K * tl < row_words * 16;
  uint16_t* maps = P.maps + rec.map_off + K * tl;
  const int64_t map_stride = state_stride(S);
  const Boundary* left = x.lw > 0 ? &sh.bnd[0][warp - 1] : &sh.edge;
  const int left_stride = x.lw > 0 ? kMaxWarps : 0;
  // Skip frames in which none of this warp's states lies in the reachable
  // band [S - 2(T - t), 2t + 1]: states below it can no longer reach the end,
  // and in-band states read only in-band states, so skipping is exact.  States
  // above the band are still unreachable: the reference holds -inf there,
  // or NaN once an emission of NaN or +inf has landed on them (NaN then stays:
  // no predecessor compares greater).  A skipped frame above the band keeps
  // exactly that.  Active iff band_lo <= 2t <= band_hi.
  const int w_lo = x.lw * 32 * K;
  const int w_hi = w_lo + 32 * K - 1;
  const unsigned band_lo = static_cast<unsigned>(max(w_lo - 1, 0));
  const int64_t hi64 = static_cast<int64_t>(w_hi) - S + 2 * static_cast<int64_t>(T);
  const bool never = hi64 < 0;
  const unsigned band_hi = never ? 0u : (hi64 > 0xffffffffLL ? 0xffffffffu : static_cast<unsigned>(hi64));
  // Frame t0 + f's emissions of this thread's states (row j of the staged
  // group `rows`); logits become x - z.  Called by whole warps.
  auto load = [&](int f, int j, const Elem* rows, float& eb, float (&et)[KT]) {
    if constexpr (kRow) {
      const Elem* row = rows + j * V;
      eb = elem_to_float(row[blank]);
#pragma unroll
      for (int q = 0; q < KT; ++q) et[q] = elem_to_float(row[col[q]]);
    } else {
      gather(f + kGroup - 1);
      cp_async_wait<kGroup - 1>();
      const float* cur = gring + (f & (kGroup - 1)) * (KT + 1) * kCtaThreads;
      if constexpr (In::kHalf) {
        const bool odd = hw.row_odd(t0 + f, V);
        eb = bf16_of_word(__float_as_uint(cur[0]), odd ^ (blank & 1));
#pragma unroll
        for (int q = 0; q < KT; ++q)
          et[q] = bf16_of_word(__float_as_uint(cur[(q + 1) * kCtaThreads]), odd ^ (col[q] & 1));
      } else {
        eb = cur[0];
#pragma unroll
        for (int q = 0; q < KT; ++q) et[q] = cur[(q + 1) * kCtaThreads];
      }
    }
    if constexpr (In::kLogits) {
      const float z = lse.at(f);
      eb = __fsub_rn(eb, z);
#pragma unroll
      for (int q = 0; q < KT; ++q) et[q] = __fsub_rn(et[q], z);
    }
  };
  auto store_map = [&](int t) {
    // Map of segment t/H: state at its last frame -> state at the last frame
    // of the previous segment (or at the region's first frame), as a delta.
    uint32_t* dst = reinterpret_cast<uint32_t*>(maps + (t >> rec.seg_log2) * map_stride);
#pragma unroll
    for (int q = 0; q < KT; ++q)
      dst[q] = static_cast<uint32_t>(d[2 * q]) | (static_cast<uint32_t>(d[2 * q + 1]) << 16);
  };
  auto store_codes_at = [&](int t, unsigned bits) {
    if (stores_codes) store_codes<K>(bp_rows + static_cast<int64_t>(t) * row_words * 4, tl, bits);
  };
  auto frame = [&](int t, int j, const Elem* rows) {
    float eb, et[KT];
    load(t - t0, j, rows, eb, et);
    // Left neighbour's last state at t-1 (s-1 for k=0, s-2 for k=1): from
    // lane-1, or for lane 0 from the warp on the left (branch-free).
    float p1 = __shfl_up_sync(0xffffffffu, a[K - 1], 1);
    const Boundary nb = left[(t & 1) * left_stride];
    unsigned bits;
    if constexpr (kMaps) {
      int pd = __shfl_up_sync(0xffffffffu, d[K - 1], 1);
      if (lane == 0) { p1 = nb.alpha; pd = nb.delta; }
      if (j == 0 && (t & hmask) == 0) {  // a new traceback segment starts at t
#pragma unroll
        for (int k = 0; k < K; ++k) d[k] = 0;
        pd = 0;
      }
      bits = dp_frame<K>(a, d, p1, pd, eb, et, skip);
    } else {
      if (lane == 0) p1 = nb.alpha;
      bits = dp_frame_plain<K>(a, p1, eb, et, skip);
    }
    store_codes_at(t, bits);
    if (kMaps && j == kGroup - 1 && (t & hmask) == hmask) store_map(t);
    if (lane == 31) sh.bnd[(t + 1) & 1][warp] = Boundary{a[K - 1], kMaps ? d[K - 1] : 0};
    x.sync();
  };
  // End of piece k at frame te (all threads, after te's barrier): the
  // terminal states at the record's last frame, else this warp's best state
  // on the band (lowest index among equals) and whether it holds NaN at or
  // above the band; plus the frontier a later repair may resume from.
  const int last = S - 1;  // even
  auto piece_end = [&](int k, int te) {
    if (te == T - 1) {
      // One predicated store per state keeps a[] in registers (a runtime
      // index would move it to local memory).
#pragma unroll
      for (int q = 0; q < K; ++q) {
        const int s = K * tl + q;
        if (s == last) sh.term_last[slot] = a[q];
        if (s == last - 1) sh.term_prev[slot] = a[q];
      }
      return;
    }
    const int lo = max(0, S - 2 * (T - te));
    const int hi = min(S - 1, 2 * te + 1);
    float bv = -INFINITY;
    int bi = 0x7fffffff;
    bool nan = false;
#pragma unroll
    for (int q = 0; q < K; ++q) {
      const int s = K * tl + q;
      if (s >= lo && s <= hi && a[q] > bv) { bv = a[q]; bi = s; }
      nan |= s >= lo && s < S && a[q] != a[q];
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, off);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, off);
      if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
    }
    nan = __any_sync(0xffffffffu, nan);
    if (lane == 0) { sh.red_val[k][warp] = bv; sh.red_idx[k][warp] = bi; sh.red_nan[k][warp] = nan; }
    if (run.frontier_out != nullptr) {
      float4* dst = reinterpret_cast<float4*>(run.frontier_out + static_cast<int64_t>(k) * map_stride + K * tl);
#pragma unroll
      for (int q = 0; q < K; q += 4) dst[q / 4] = make_float4(a[q], a[q + 1], a[q + 2], a[q + 3]);
    }
  };

  int piece = 0;  // current piece of the run
  for (int g = 0; g < ngroups; ++g) {
    const Elem* rows = nullptr;
    if constexpr (In::kLogits)
      if (g > 0 && g % kChunkGroups == 0) lse.advance(t0 + g * kGroup, lane);
    if constexpr (kRow) {
      const int c = cb + g / kChunkGroups;
      if (g % kChunkGroups == 0 && !fault && !mbar_wait(&full[c % kRowRing], (c / kRowRing) & 1))
        fault = true;
      rows = ring + ((c % kRowRing) * kChunkFrames + (g % kChunkGroups) * kGroup) * V;
    }
    const int tg = t0 + g * kGroup;
    // A new piece of the run starts here: close the previous one, then seed
    // this one with a free start.
    const bool boundary = g > 0 && g % kGroupsPerPiece == 0 && piece + 1 < run.pieces;
    if (boundary) piece_end(piece++, tg - 1);
    const int init = g == 0 ? run.init : kInitFree;
    const bool seeded = (g == 0 && run.init != kInitFrontier) || boundary;
    // The band test is made once per group: a group with at least one frame
    // in which this warp has in-band states runs every frame (the plain DP is
    // exact everywhere); a group with none keeps the barriers (and the gather
    // ring) in step.  Its backpointers and maps are never read.
    const unsigned g2 = 2u * static_cast<unsigned>(tg);
    const bool group_active = seeded || (!never && g2 + 2u * (kGroup - 1) >= band_lo && g2 <= band_hi);
    if (!group_active) {
      const bool above = g2 + 2u * (kGroup - 1) < band_lo;
#pragma unroll 1
      for (int j = 0; j < kGroup && tg + j < t1; ++j) {
        if (above || !kRow) {
          float eb, et[KT];
          load(tg + j - t0, j, rows, eb, et);
          if (above) {
#pragma unroll
            for (int k = 0; k < K; ++k)
              if (poisons((k & 1) ? et[k >> 1] : eb)) a[k] = NAN;
          }
        }
        x.sync();
      }
    } else if (seeded) {
      float eb, et[KT];
      load(tg - t0, 0, rows, eb, et);
#pragma unroll
      for (int k = 0; k < K; ++k) { a[k] = -INFINITY; d[k] = 0; }
      if (init == kInitRecord) {
        // Frame 0: alpha[s] = e[0, l[s]] for s < 2, else -inf (alignment.cu:409).
        if (tl == 0) {
          a[0] = eb;
          if (S > 1) a[1] = et[0];
        }
      } else {
        // Free start on the band of frame tg; above it, -inf (or NaN from a
        // poisoning emission) as the full DP holds there.
        const int lo0 = max(0, S - 2 * (T - tg));
        const int hi0 = min(S - 1, 2 * tg + 1);
#pragma unroll
        for (int k = 0; k < K; ++k) {
          const int s = K * tl + k;
          const float ek = (k & 1) ? et[k >> 1] : eb;
          a[k] = s < lo0 ? -INFINITY : (s <= hi0 ? ek : (poisons(ek) ? NAN : -INFINITY));
        }
      }
      if (lane == 31) sh.bnd[(tg + 1) & 1][warp] = Boundary{a[K - 1], 0};
      x.sync();
#pragma unroll 1
      for (int j = 1; j < kGroup && tg + j < t1; ++j) frame(tg + j, j, rows);
    } else {
#pragma unroll
      for (int j = 0; j < kGroup; ++j)
        if (tg + j < t1) frame(tg + j, j, rows);
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
      for (int c = cb + max(0, nchunks - kRowRing); c < cb + nchunks; ++c)
        mbar_wait(&full[c % kRowRing], (c / kRowRing) & 1, kDrainNs);
  }
  {  // a map the last frame left open
    const int tl_ = t1 - 1;
    if (kMaps && (tl_ & hmask) != hmask) store_map(tl_);
  }
  if (fault) sh.slot_fault[slot] = 1;
  piece_end(piece, t1 - 1);
  x.sync();

  // Lane k of the slot's first warp finishes piece k: its end state and
  // flags; then the path's anchors and region start come from the segment
  // maps (kMaps) or from warp traces over the backpointers.
  int32_t* anc = P.anchors + rec.seg_off;
  if (x.lw == 0 && lane < run.pieces) {
    const int k = lane;
    const int first = t0 + k * kPieceFrames;
    const int end = k + 1 < run.pieces ? first + kPieceFrames : t1;
    int end_state;
    float best;
    bool nan = false;
    if (end == T) {
      const float vlast = sh.term_last[slot];
      end_state = last;
      best = vlast;
      if (S > 1) {
        const float vprev = sh.term_prev[slot];
        if (vprev >= vlast) { end_state = last - 1; best = vprev; }
      }
    } else {
      best = -INFINITY;
      end_state = 0x7fffffff;
      for (int w = x.first_warp; w < x.first_warp + NT / 32; ++w) {
        const float v = sh.red_val[k][w];
        const int i = sh.red_idx[k][w];
        if (v > best || (v == best && i < end_state)) { best = v; end_state = i; }
        nan |= sh.red_nan[k][w] != 0;
      }
    }
    const bool slot_fault = sh.slot_fault[slot] != 0;
    const bool finite = isfinite(best);
    if (run.end_piece < 0) {
      P.out.objective[x.r] = best;
      P.out.status[x.r] = slot_fault ? kStatusDeviceFault : (finite ? 0 : 1);
    } else {
      PieceState& pe = P.pstates[run.end_piece + k];
      pe.end = end_state;
      pe.flags = (finite && !nan && !slot_fault ? kPieceOk : 0) | (slot_fault ? kPieceFault : 0);
      if (run.new_region) pe.region_start[0] = 1;
    }
    const bool trace = finite && !slot_fault && !(run.end_piece >= 0 && nan);
    if constexpr (kMaps) {
      if (trace) {
        // (The clamp never acts on maps a completed DP wrote; it keeps every
        // read inside the arena.)
        const int a0 = run.pieces > 1 ? first : run.a0;
        const uint16_t* mp = P.maps + rec.map_off;
        int s = end_state;
        for (int g = (end - 1) >> rec.seg_log2; g >= (a0 >> rec.seg_log2); --g) {
          anc[g] = s;
          s = min(max(s - mp[static_cast<int64_t>(g) * map_stride + s], 0), S - 1);
        }
        if (run.end_piece >= 0) P.pstates[run.start_piece + k].start = s;
      }
    } else {
      sh.red_idx[k][x.first_warp] = trace ? end_state : -1;
    }
  }
  if constexpr (!kMaps) {
    x.sync();
    // Warp lw traces pieces lw, lw + nw, ...: from the end state back to the
    // piece's (or the repaired region's) first frame.
    const uint32_t* bpr = P.bp + rec.bp_off;
    for (int k = x.lw; k < run.pieces; k += NT / 32) {
      const int s_end = sh.red_idx[k][x.first_warp];
      if (s_end < 0) continue;
      const int first = t0 + k * kPieceFrames;
      const int end = k + 1 < run.pieces ? first + kPieceFrames : t1;
      const int a0 = run.pieces > 1 ? first : run.a0;
      // The path's state at every frame of the region as well (the fill of
      // a joined record gathers its outputs from them without a walk).
      int16_t* states = P.path_states + rec.out_off;
      if (lane == 0) {
        anc[(end - 1) >> rec.seg_log2] = s_end;
        states[end - 1] = static_cast<int16_t>(s_end);
      }
      const int s0 = warp_trace(bpr, row_words, s_end, end - 1, a0, lane, [&](int t, int s) {
        if (lane == 0) {
          if ((t & hmask) == hmask) anc[t >> rec.seg_log2] = s;
          states[t] = static_cast<int16_t>(s);
        }
      });
      if (lane == 0 && run.end_piece >= 0) {
        // Whether a skip into the region's first state is legal: it is a
        // token that differs from the previous token and from the blank.
        bool skip_in = false;
        if ((s0 & 1) && s0 >= 3) {
          const int u = s0 >> 1;
          const int cu = clamp_label(tgt[u], V);
          skip_in = cu != blank && cu != clamp_label(tgt[u - 1], V);
        }
        PieceState& ps = P.pstates[run.start_piece + k];
        ps.start = s0;
        ps.start_skip = skip_in ? 1 : 0;
      }
    }
  }
  return nchunks;
}

}  // namespace

// Repair jobs of one round of one record (shared memory of the finisher).
constexpr int kMaxJobs = 128;
struct JobList {
  int count;
  int piece[kMaxJobs];  // first piece re-solved (resumes from the frontier of piece - 1)
  int first[kMaxJobs];  // first piece of the merged region
  int last[kMaxJobs];   // last piece of the merged region
};

// What one round's plan adds to a record's diagnostics.
struct PlanStats {
  int64_t merged = 0;   // frames of the merged regions
  int64_t skipped = 0;  // frames the saved frontiers spared
  int jobs = 0;
};

// A piece's state as other CTAs of the running launch may have left it:
// loaded through L2 (ld.global.cg), never from a stale L1 line.
__device__ __forceinline__ PieceState load_piece_state(const PieceState* p) {
  const int4 a = __ldcg(reinterpret_cast<const int4*>(p));
  const int4 b = __ldcg(reinterpret_cast<const int4*>(p) + 1);
  PieceState s;
  s.start = a.x; s.end = a.y; s.flags = a.z; s.start_skip = a.w;
  s.region_start[0] = b.x; s.region_start[1] = b.y; s.region_start[2] = b.z; s.region_start[3] = b.w;
  return s;
}

// Seam check and repair planning of one round of one record, by one warp.  A
// region is a run of pieces solved as one DP; a seam is legal when the right
// region's start state follows the left region's end state by a CTC move
// (stay, step, or a skip into a token that differs from the previous token
// and from the blank -- precomputed for each region's start).  Every run of
// consecutive failing seams becomes one repair job: the merged region
// resumes from the end frontier of its first region and re-solves the
// regions after it.  Returns the record's route:
//   all seams legal, every region finite and NaN-free  -> joined (stitched)
//   a region non-finite or with NaN                     -> conventional DP
//   seams still failing after the last round            -> conventional DP
//   a bounded wait gave up                               -> none (status 5)
// Status >= 2 (rejected inputs) -> none.
// write_regions: this warp records the next round's region starts (one
// planner per record does; others that plan the same round only read).
__device__ int plan_record(const RecordDev& rec, int r, PieceState* __restrict__ ps,
                           const OutputsDev& out, int round, bool final_round, bool write_regions,
                           JobList* jobs, int lane, PlanStats& stats) {
  const int C = rec.num_pieces, P0 = rec.first_piece;
  const int status = out.status[r];
  bool bad = false, fault = false, any_fail = false, run_open = false, overflow = false;
  int run_job = 0, run_first = 0, cur_first = 0, njobs = 0;
  // Piece j covers frames [j * kPieceFrames, end_of(j)); the last one ends at T.
  auto end_of = [&](int j) { return j == C - 1 ? rec.T : (j + 1) * kPieceFrames; };
  auto emit = [&](int job, int last) {
    // All lanes take the same decisions; lane 0 writes them.
    stats.merged += end_of(last) - run_first * kPieceFrames;
    stats.skipped += (job - run_first) * kPieceFrames;
    if (njobs == kMaxJobs) overflow = true;
    if (lane == 0 && jobs != nullptr && !final_round && njobs < kMaxJobs) {
      jobs->piece[njobs] = P0 + job;
      jobs->first[njobs] = P0 + run_first;
      jobs->last[njobs] = P0 + last;
    }
    ++njobs;
  };
  for (int base = 0; base < C; base += 32) {
    // Each lane checks the seam in front of its piece (if it starts a region)
    // and whether its piece ends a region that failed.
    const int j = base + lane;
    bool seam = false, fail = false, region_bad = false, region_fault = false;
    if (j < C) {
      const PieceState mine = load_piece_state(ps + P0 + j);
      const bool next_rs = j + 1 >= C || __ldcg(&ps[P0 + j + 1].region_start[round]) != 0;
      const int prev_end = j > 0 ? __ldcg(&ps[P0 + j - 1].end) : 0;
      seam = mine.region_start[round] != 0 && j > 0;
      // The next round's regions start as this round's; merges clear below.
      if (!final_round && write_regions) ps[P0 + j].region_start[round + 1] = mine.region_start[round];
      if (seam) {
        const int jump = mine.start - prev_end;
        fail = !(jump == 0 || jump == 1 || (jump == 2 && mine.start_skip));
      }
      region_bad = next_rs && (mine.flags & kPieceOk) == 0;
      region_fault = next_rs && (mine.flags & kPieceFault) != 0;
    }
    if (status != 0) break;  // rejected inputs: nothing to plan
    unsigned seams = __ballot_sync(0xffffffffu, seam);
    const unsigned fails = __ballot_sync(0xffffffffu, fail);
    bad |= __any_sync(0xffffffffu, region_bad) != 0;
    fault |= __any_sync(0xffffffffu, region_fault) != 0;
    // Runs of consecutive failing seams, in piece order (uniform over lanes).
    while (seams) {
      const int q = __ffs(seams) - 1;
      seams &= seams - 1;
      const int jj = base + q;
      if ((fails >> q) & 1u) {
        any_fail = true;
        if (!run_open) { run_open = true; run_job = jj; run_first = cur_first; }
      } else {
        if (run_open) { emit(run_job, jj - 1); run_open = false; }
        cur_first = jj;
      }
    }
  }
  if (status != 0) {
    if (lane == 0 && jobs != nullptr) jobs->count = 0;
    __syncwarp();
    return kRouteNone;
  }
  if (run_open) emit(run_job, C - 1);
  int decision;
  if (fault) decision = kRouteNone;
  else if (bad || (any_fail && (final_round || overflow))) decision = kRouteFallback;
  else if (!any_fail) decision = kRouteStitched;
  else decision = kRoutePending;
  stats.jobs = njobs;
  // Merge the failing runs into the next round's regions only when there is
  // a next round for this record: a record already routed keeps its regions,
  // so a later planner of it sees the same bad or joined regions again.
  __syncwarp();  // the lanes' copies above land before lane 0 clears
  if (lane == 0 && jobs != nullptr && decision == kRoutePending && write_regions) {
    for (int q = 0; q < njobs && q < kMaxJobs; ++q)
      for (int k = jobs->piece[q]; k <= jobs->last[q]; ++k) ps[k].region_start[round + 1] = 0;
  }
  if (lane == 0 && jobs != nullptr) jobs->count = decision == kRoutePending ? njobs : 0;
  __syncwarp();
  return decision;
}

// The finisher group of a record of the optimized route (the host planner's
// rule, ffa_host.cpp): row-staged before gathered, then the CTA size its
// repairs get: 128 / 256 threads for at most 4 / 8 warps at 8 states per
// thread when the narrow groups are in use, else 512.
__device__ __forceinline__ int finish_group(const RecordDev& rec, bool narrow) {
  const int nw8 = (2 * rec.U + 1 + 255) / 256;
  const int size = !narrow ? 2 : (nw8 <= kMaxWarps / 4 ? 0 : (nw8 <= kMaxWarps / 2 ? 1 : 2));
  return (rec.row_mode ? 0 : 3) + size;
}

// Pieces per first-pass slot of a record of the chunked route.
__device__ __forceinline__ int run_pieces_of(const ForwardParams& P, const RecordDev& rec) {
  return P.run_by[rec.row_mode ? 1 : 0][rec.kst == 16 ? 1 : 0][rec.nw];
}

// Round 0's plan in the first pass: every slot of a record counts itself out
// once its pieces' states are written; the last one plans round 0 with its
// first warp.  A joined record is done here (route and diagnostics; the fill
// folds its objective); any other goes to the finisher's list.  Called by
// every thread of the slot.
__device__ void plan_round0(const SlotCtx& x, const RecordDev& rec, ForwardShared& sh,
                            const ForwardParams& P) {
  x.sync();  // the slot's traces have written its pieces' states
  if (x.tl == 0) {
    __threadfence();
    const int rp = run_pieces_of(P, rec);
    const int slots = (rec.num_pieces + rp - 1) / rp;
    sh.slot_status[x.slot] = atomicAdd(&P.slot_done[x.r], 1) == slots - 1 ? 1 : 0;
    __threadfence();
  }
  x.sync();
  if (!sh.slot_status[x.slot] || x.lw != 0) return;
  PlanStats stats;
  const int decision = plan_record(rec, x.r, P.pstates, P.out, 0, false, false, nullptr, x.lane, stats);
  if (x.lane != 0) return;
  if (decision == kRouteStitched) {
    // Diagnostics of a record joined without repairs (the rest stay zero).
    P.route[x.r] = kRouteStitched;
    P.out.stitched[x.r] = 1;
    if (P.out.reuse_stats)
      P.out.reuse_stats[4 * x.r + 2] = static_cast<int64_t>(rec.num_pieces - 1) * (2 * rec.U + 1);
  } else {
    const int g = finish_group(rec, P.finish_narrow != 0);
    P.finish_list[P.finish_base[g] + atomicAdd(&P.finish_count[g], 1)] = x.r;
  }
}

// The first pass.  One CTA = one Bundle of slots of `nw` warps with the same
// states per thread; a slot runs one whole record (conventional DP with its
// outputs) or a run of consecutive pieces of one record of the optimized
// route, and the first slot of each record also checks its inputs.  Warps of
// a slot run the DP in lock step with one named barrier per frame.  kRow:
// emission rows arrive kChunkFrames frames at a time by one TMA bulk copy
// into a kRowRing-deep ring per slot; otherwise each thread gathers its
// columns with cp.async into a private ring (large vocabularies).
template <bool kRow, int kV, int kFmt>
__global__ void __launch_bounds__(kCtaThreads, 1)
ffa_viterbi_forward(const __grid_constant__ ForwardParams P) {
  extern __shared__ __align__(128) unsigned char smem_raw[];
  ForwardShared& sh = *reinterpret_cast<ForwardShared*>(smem_raw);

  SlotCtx x;
  x.tid = threadIdx.x;
  x.warp = x.tid >> 5;
  x.lane = x.tid & 31;
  const Bundle bd = P.bundles[blockIdx.x];
  x.slot = x.warp / bd.nw;
  if (x.tid == 0) sh.edge = Boundary{-INFINITY, 0};
  __syncthreads();
  if (x.slot >= bd.count) return;
  const SlotRef ref = P.order[bd.first + x.slot];
  x.r = ref.record;
  const RecordDev rec = P.recs[x.r];
  const int pidx = ref.piece;                // rank of the slot's first piece in the record
  const int p = rec.first_piece + pidx;      // its piece id
  const int pfirst = pidx * kPieceFrames;    // its first frame (0 for a whole record)
  x.first_warp = x.slot * bd.nw;
  x.bar = x.slot;
  x.lw = x.warp - x.first_warp;  // warp within the slot
  if (x.lw >= rec.nw) return;
  x.NT = rec.nw * 32;
  x.tl = x.lw * 32 + x.lane;  // thread within the slot
  const int tl = x.tl, lane = x.lane, warp = x.warp, r = x.r;
  const int T = rec.T, V = rec.V, U = rec.U, blank = rec.blank;
  const int64_t* tgt = rec.targets;
  const bool chunked = rec.num_pieces > 1;

  PieceRun run{0, 0, T, kInitRecord, 1, nullptr, nullptr, -1, -1, false, 0};
  {
    const bool masked = P.mask != nullptr && !P.mask[r];
    if (pidx == 0) {
      // ---- status: mask, then target validation (alignment.cu:836, 852-874) ----
      int status = masked ? 2 : 0;
      if (tl == 0) sh.slot_fault[x.slot] = 0;
      if (P.check_inputs) {
        // Four strides of loads in flight at a time: a one-warp slot walks a
        // long transcript in few round trips.
        int bad = 0, rep = 0;
        for (int k0 = tl; k0 < U; k0 += 4 * x.NT) {
          int64_t cur[4], prv[4];
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const int k = k0 + q * x.NT;
            cur[q] = k < U ? tgt[k] : 0;
            prv[q] = k < U && k > 0 ? tgt[k - 1] : 0;
          }
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const int k = k0 + q * x.NT;
            if (k < U) {
              bad |= (cur[q] < 0 || cur[q] >= V || cur[q] == blank) ? 1 : 0;
              if (k > 0) rep += cur[q] == prv[q] ? 1 : 0;
            }
          }
        }
        bad = __reduce_or_sync(0xffffffffu, bad);
        rep = __reduce_add_sync(0xffffffffu, rep);
        if (lane == 0) { sh.chk_bad[warp] = bad; sh.chk_rep[warp] = rep; }
        x.sync();
        if (tl == 0) {
          int b = 0, q = 0;
          for (int w = 0; w < rec.nw; ++w) { b |= sh.chk_bad[warp + w]; q += sh.chk_rep[warp + w]; }
          if (b) status = 3;
          else if (static_cast<int64_t>(U) + q > T) status = 4;
          sh.slot_status[x.slot] = status;
        }
        x.sync();
        status = sh.slot_status[x.slot];
      }
      if (tl == 0) {
        // Diagnostics start at zero (alignment.py:101-129); the optimized
        // route's plan counts repairs and joins into them.
        P.fill_done[r] = 0;
        P.finish_done[r] = 0;
        P.out.stitched[r] = 0;
        P.out.repair_passes[r] = 0;
        P.out.repaired_frames[r] = 0;
        for (int j = 0; j < 3; ++j) P.out.routing_stats[3 * r + j] = 0;
        // A record the greedy pass covers gets its shortcut statistics there.
        if (P.greedy_first == nullptr || P.greedy_first[r] < 0)
          for (int j = 0; j < 3; ++j) P.out.shortcut_stats[3 * r + j] = 0;
        if (P.out.reuse_stats) for (int j = 0; j < 4; ++j) P.out.reuse_stats[4 * r + j] = 0;
        if (status >= 2) P.out.objective[r] = -INFINITY;
        if (status >= 2 || chunked) P.out.status[r] = status;
      }
      if (status >= 2) {
        if (chunked && P.plan_first) plan_round0(x, rec, sh, P);
        return;
      }
    } else {
      if (masked) {
        if (chunked && P.plan_first) plan_round0(x, rec, sh, P);
        return;
      }
      if (tl == 0) sh.slot_fault[x.slot] = 0;
    }
    if (chunked) {
      // Pieces index .. index+m-1 of the record, back to back.
      const int m = min(run_pieces_of(P, rec), rec.num_pieces - pidx);
      run.a0 = run.t0 = pfirst;
      run.t1 = pidx + m == rec.num_pieces ? T : pfirst + m * kPieceFrames;
      run.pieces = m;
      run.init = pfirst == 0 ? kInitRecord : kInitFree;
      run.frontier_out = P.frontiers + rec.frontier_off + static_cast<int64_t>(pidx) * state_stride(2 * U + 1);
      run.end_piece = run.start_piece = p;
      run.new_region = true;
    }
  }

  // Pieces of the optimized route (K = 8 or 16) find their anchors by
  // tracing; whole records walk segment maps.
  if (chunked && rec.kst == 16)
    piece_dp<16, kRow, kV, false, kFmt>(x, rec, run, sh, smem_raw, P);
  else if (chunked)
    piece_dp<8, kRow, kV, false, kFmt>(x, rec, run, sh, smem_raw, P);
  else if (rec.kst == 4)
    piece_dp<4, kRow, kV, true, kFmt>(x, rec, run, sh, smem_raw, P);
  else
    piece_dp<8, kRow, kV, true, kFmt>(x, rec, run, sh, smem_raw, P);
  if (chunked && P.plan_first) plan_round0(x, rec, sh, P);
}

// Traceback segment c of a record by one warp: the warp walks the
// backpointers from the segment's anchor (path[t-1] = path[t] - bp[t, path[t]],
// alignment.cu:656-659), then maps states to labels and gathers the selected
// scores (alignment.cu:662-666); a logits input's score is the same x - z the
// DPs used (fmt, lse: as in ForwardParams).  A failed record gets -1 / -inf
// (alignment.cu:650-652).  p: this warp's path scratch (1 << kMaxSegLog2).
__device__ __forceinline__ void fill_segment(const RecordDev& rec, int record, int c, const uint32_t* bp_arena,
                                             const int32_t* anchors, const OutputsDev& out, const float* lse,
                                             int fmt, int32_t* p, int lane) {
  const int T = rec.T;
  const int H = 1 << rec.seg_log2;
  const int C = static_cast<int>((static_cast<int64_t>(T) + H - 1) >> rec.seg_log2);
  if (c >= C) return;
  int64_t* labels = out.labels + rec.out_off;
  float* scores = out.scores + rec.out_off;
  const int a = c * H;
  const int b = static_cast<int>(min(static_cast<int64_t>(T), static_cast<int64_t>(a) + H));
  if (out.status[record] != 0) {
    for (int t = a + lane; t < b; t += 32) { labels[t] = -1; scores[t] = -INFINITY; }
    return;
  }
  const int s_end = __ldcg(anchors + rec.seg_off + c);  // another CTA may have written it
  if (lane == 0) p[b - 1 - a] = s_end;
  warp_trace_lean(bp_arena + rec.bp_off, bp_row_words(2 * rec.U + 1), s_end, b - 1, a, lane,
                  [&](int t, int s) { if (lane == 0) p[t - a] = s; });
  __syncwarp();
  for (int t = a + lane; t < b; t += 32) {
    const int s = p[t - a];
    const int label = (s & 1) ? clamp_label(rec.targets[s >> 1], rec.V) : rec.blank;
    const int64_t i = static_cast<int64_t>(t) * rec.V + label;
    float score = fmt == 2 ? bf16_to_float(reinterpret_cast<const uint16_t*>(rec.emissions)[i])
                           : rec.emissions[i];
    if (fmt != 0) score = __fsub_rn(score, lse[rec.out_off + t]);
    labels[t] = label;
    scores[t] = score;
  }
  __syncwarp();
}

// Outputs of frames [a, b) of a joined record of the chunked route from the
// path's state at each frame (the traces' path_states), by `nthreads`
// threads: labels and the selected scores as fill_segment writes them, with
// no backpointer walk.
// stash (or null): shared memory that also takes frame t's score at t - a.
__device__ __forceinline__ void gather_joined(const RecordDev& rec, int record, int a, int b,
                                              const int16_t* path_states, const OutputsDev& out, const float* lse,
                                              int fmt, int tid, int nthreads, float* stash = nullptr) {
  int64_t* labels = out.labels + rec.out_off;
  float* scores = out.scores + rec.out_off;
  if (out.status[record] != 0) {
    for (int t = a + tid; t < b; t += nthreads) { labels[t] = -1; scores[t] = -INFINITY; }
    return;
  }
  const int16_t* states = path_states + rec.out_off;
#pragma unroll 4
  for (int t = a + tid; t < b; t += nthreads) {
    const int s = __ldcg(states + t);  // written by other CTAs of the traces' launches
    const int label = (s & 1) ? clamp_label(rec.targets[s >> 1], rec.V) : rec.blank;
    const int64_t i = static_cast<int64_t>(t) * rec.V + label;
    float score = fmt == 2 ? bf16_to_float(reinterpret_cast<const uint16_t*>(rec.emissions)[i])
                           : rec.emissions[i];
    if (fmt != 0) score = __fsub_rn(score, lse[rec.out_off + t]);
    labels[t] = label;
    scores[t] = score;
    if (stash != nullptr) stash[t - a] = score;
  }
}

// n values of shared memory added in order to obj with one fp32 add each
// (by one thread): the next 8 load while the current 8 are added.
__device__ __forceinline__ float fold_span(const float* window, int n, float obj) {
  int k = 0;
  float cur[8], nxt[8];
  if (n >= 8) {
#pragma unroll
    for (int q = 0; q < 8; ++q) cur[q] = window[q];
    for (k = 8; k + 8 <= n; k += 8) {
#pragma unroll
      for (int q = 0; q < 8; ++q) nxt[q] = window[k + q];
#pragma unroll
      for (int q = 0; q < 8; ++q) obj = __fadd_rn(obj, cur[q]);
#pragma unroll
      for (int q = 0; q < 8; ++q) cur[q] = nxt[q];
    }
#pragma unroll
    for (int q = 0; q < 8; ++q) obj = __fadd_rn(obj, cur[q]);
  }
  for (; k < n; ++k) obj = __fadd_rn(obj, window[k]);
  return obj;
}

// Objective of a joined record: the path's selected emissions summed in
// frame order with one fp32 add each -- the conventional DP's accumulation
// along the same path (alignment.cu:423), so equal paths give equal
// objectives.  By every thread of the CTA: the scores pass through `window`
// (shared, room floats) and thread 0 adds them (its result; the others
// return -0).
__device__ float fold_path_scores(const float* scores, int T, float* window, int room, int tid, int nthreads) {
  float obj = -0.0f;  // -0 + x == x exactly for every x
  for (int base = 0; base < T; base += room) {
    const int n = min(room, T - base);
    __syncthreads();
#pragma unroll 4
    for (int k = tid; k < n; k += nthreads) window[k] = __ldcg(scores + base + k);
    __syncthreads();
    if (tid == 0) obj = fold_span(window, n, obj);
  }
  return obj;
}

// fill_done of a record the finisher filled and folded (ffa_trace_fill skips it).
constexpr int32_t kFilledByFinisher = INT32_MIN;

// The finisher's static shared memory (its job list) stays under 2 KiB; the
// rest of the budget is dynamic.
constexpr size_t kFinishDynamicSmem = kSmemBudget - 2048;
static_assert(sizeof(JobList) + 64 <= 2048, "finisher static shared memory");

// Everything after the first pass of the optimized route, in one launch
// (records need nothing from one another).  R CTAs per record each plan
// round 0 (the same plan) and run the round's repair jobs j with j % R == its
// index, so a record's first jobs spread over R SMs; the record's last CTA to
// finish them (a counter per record) then continues alone: rounds 1 ..
// kRepairRounds of planning (warp 0) and repairs (slots of nw warps, in
// parallel), the final plan, the conventional DP when the route cannot join
// the record, and the record's route and diagnostics.  A record that round 0
// already routes is finished by its CTA 0.  Data other CTAs of this launch
// wrote (piece states, frontiers, backpointer rows) is read through L2.
template <bool kRow, int kV, int kFmt>
__global__ void __launch_bounds__(kCtaThreads, 1)
ffa_finish_route(const __grid_constant__ ForwardParams P, const int32_t* __restrict__ records,
                 const int32_t* __restrict__ device_count, int ctas_per_record, unsigned dynamic_smem) {
  if (device_count != nullptr && static_cast<int>(blockIdx.x) / ctas_per_record >= *device_count) return;
  extern __shared__ __align__(128) unsigned char smem_raw[];
  ForwardShared& sh = *reinterpret_cast<ForwardShared*>(smem_raw);
  __shared__ JobList jobs;
  __shared__ int route_s;
  __shared__ int last_s;
  int part = static_cast<int>(blockIdx.x % ctas_per_record);
  int parts = ctas_per_record;
  const int r = records[blockIdx.x / ctas_per_record];
  const RecordDev rec = P.recs[r];
  SlotCtx x;
  x.tid = threadIdx.x;
  x.warp = x.tid >> 5;
  x.lane = x.tid & 31;
  x.r = r;
  // Repairs and the fallback run 8 states per thread (shorter per-frame
  // chains than the first pass's 16): the backpointer rows do not depend on
  // the thread layout.
  const int nw = (2 * rec.U + 1 + 255) / 256;
  // Slot barriers use ids 1.. (id 0 is __syncthreads); row-staged slots also
  // need a ring each.  The CTA has 4, 8 or 16 warps (fewer when many records
  // share the GPU: four or two such CTAs fit an SM).
  const int nwarps = static_cast<int>(blockDim.x >> 5);
  int nslots = min(kMaxWarps - 1, nwarps / nw);
  if (kRow) nslots = min(nslots, static_cast<int>((dynamic_smem - kForwardHeader) / P.row_slot_bytes));
  x.slot = x.warp / nw;
  x.lw = x.warp - x.slot * nw;
  x.NT = nw * 32;
  x.tl = x.lw * 32 + x.lane;
  x.first_warp = x.slot * nw;
  x.bar = x.slot + 1;
  const bool in_slot = x.slot < nslots;
  if (x.tid == 0) sh.edge = Boundary{-INFINITY, 0};
  int chunk_base = 0;  // this slot's emission chunks so far (row staging)
  // Warp 0 keeps the record's diagnostics and writes them once at the end.
  int passes = 0;
  int64_t repaired = 0, spared = 0, frontier_reads = 0;
  for (int round = 0; round <= kRepairRounds; ++round) {
    __syncthreads();
    if (x.warp == 0) {
      PlanStats stats;
      const int decision = plan_record(rec, r, P.pstates, P.out, round, round == kRepairRounds, part == 0,
                                       &jobs, x.lane, stats);
      if (decision == kRoutePending) {
        ++passes;
        repaired += stats.merged;
        spared += stats.skipped;
        frontier_reads += static_cast<int64_t>(stats.jobs) * (2 * rec.U + 1);
      }
      if (x.lane == 0) route_s = decision;
    }
    __syncthreads();
    if (route_s != kRoutePending) break;
    const int n = jobs.count;
    const int64_t fstride = state_stride(2 * rec.U + 1);
    if (in_slot) {
      for (int j = part + x.slot * parts; j < n; j += nslots * parts) {
        const int p = jobs.piece[j];
        const int idx = p - rec.first_piece;
        const int last = jobs.last[j] - rec.first_piece;
        PieceRun run{};
        run.a0 = (jobs.first[j] - rec.first_piece) * kPieceFrames;
        run.t0 = idx * kPieceFrames;
        run.t1 = last == rec.num_pieces - 1 ? rec.T : (last + 1) * kPieceFrames;
        run.init = kInitFrontier;
        run.pieces = 1;
        run.frontier_in = P.frontiers + rec.frontier_off + (idx - 1) * fstride;
        run.frontier_out = run.t1 < rec.T ? P.frontiers + rec.frontier_off + last * fstride : nullptr;
        run.end_piece = jobs.last[j];
        run.start_piece = jobs.first[j];
        run.new_region = false;
        run.chunk_base = chunk_base;
        if (x.tl == 0) sh.slot_fault[x.slot] = 0;
        chunk_base += piece_dp<8, kRow, kV, false, kFmt>(x, rec, run, sh, smem_raw, P);
      }
    }
    if (parts > 1) {
      // The record's CTAs ran round 0's jobs between them; the last one to
      // finish continues alone (release: every CTA's results before its
      // count; acquire: the counts before the continuing CTA's reads).
      __syncthreads();
      if (x.tid == 0) {
        __threadfence();
        last_s = atomicAdd(&P.finish_done[r], 1) == parts - 1;
        __threadfence();
      }
      __syncthreads();
      if (!last_s) return;
      part = 0;
      parts = 1;
    }
  }
  // Round 0 routed the record: every CTA planned it, CTA 0 finishes it.
  if (part != 0) return;
  if (x.tid == 0) {
    // Route and diagnostics (alignment.py:101-129).
    const int route = route_s;
    P.route[r] = route;
    if (route == kRouteNone && P.out.status[r] == 0) {
      P.out.status[r] = kStatusDeviceFault;
      P.out.objective[r] = -INFINITY;
    }
    if (route == kRouteStitched) P.out.stitched[r] = 1;
    P.out.repair_passes[r] = passes;
    P.out.repaired_frames[r] = repaired;
    if (P.out.reuse_stats) {
      P.out.reuse_stats[4 * r + 0] = spared;
      P.out.reuse_stats[4 * r + 2] = static_cast<int64_t>(rec.num_pieces - 1) * (2 * rec.U + 1);
      P.out.reuse_stats[4 * r + 3] = frontier_reads;
    }
  }
  if (route_s == kRouteFallback && x.slot == 0) {
    PieceRun run{0, 0, rec.T, kInitRecord, 1, nullptr, nullptr, -1, -1, false, chunk_base};
    if (x.tl == 0) sh.slot_fault[0] = 0;
    piece_dp<8, kRow, kV, true, kFmt>(x, rec, run, sh, smem_raw, P);
  }
  if (!P.fill_in_finisher) return;
  // The record's traceback fill and, for a joined path, its objective
  // (as ffa_trace_fill does, which then skips the record): every warp of the
  // CTA takes segments, their path scratch and then the fold's window in the
  // dynamic shared memory the DPs' rings are done with.
  __syncthreads();  // route, status, anchors and backpointers are written
  const int T = rec.T;
  const int C = static_cast<int>((static_cast<int64_t>(T) + (1 << rec.seg_log2) - 1) >> rec.seg_log2);
  int32_t* scratch = reinterpret_cast<int32_t*>(smem_raw + kForwardHeader);
  const int room = static_cast<int>((dynamic_smem - kForwardHeader) / sizeof(int32_t));
  // A joined record that fits the scratch keeps its scores there for the fold.
  float* window = reinterpret_cast<float*>(scratch);
  const bool stashed = route_s == kRouteStitched && T <= room;
  if (route_s == kRouteStitched) {
    gather_joined(rec, r, 0, T, P.path_states, P.out, P.lse, kFmt, x.tid, static_cast<int>(blockDim.x),
                  stashed ? window : nullptr);
  } else {
    // The conventional DP's path (segment maps and anchors), or -1 / -inf.
    const int fill_warps = min(nwarps, room >> rec.seg_log2);
    if (x.warp < fill_warps)
      for (int c = x.warp; c < C; c += fill_warps)
        fill_segment(rec, r, c, P.bp, P.anchors, P.out, P.lse, kFmt, scratch + (x.warp << rec.seg_log2), x.lane);
  }
  if (route_s == kRouteStitched) {
    // (fold_path_scores begins with a barrier: the fill's scores are written.)
    float obj;
    if (stashed) {
      __syncthreads();
      obj = x.tid == 0 ? fold_span(window, T, -0.0f) : 0.0f;
    } else {
      obj = fold_path_scores(P.out.scores + rec.out_off, T, window, room, x.tid, static_cast<int>(blockDim.x));
    }
    if (x.tid == 0) {
      P.out.objective[r] = obj;
      last_s = isfinite(obj) ? 1 : 0;
      if (!isfinite(obj)) P.out.status[r] = 1;
    }
    __syncthreads();
    if (!last_s)
      for (int t = x.tid; t < T; t += static_cast<int>(blockDim.x)) {
        P.out.labels[rec.out_off + t] = -1;
        P.out.scores[rec.out_off + t] = -INFINITY;
      }
  }
  if (x.tid == 0) P.fill_done[r] = kFilledByFinisher;
}

// One warp per traceback segment (fill_segment); a joined record of the
// chunked route gathers its CTA's frames from the path states instead, and
// the record's last fill CTA to finish (a counter per record) then folds its
// objective.
__global__ void __launch_bounds__(32 * kFillWarps)
ffa_trace_fill(const RecordDev* __restrict__ recs, const FillItem* __restrict__ items,
               const uint32_t* __restrict__ bp_arena, const int32_t* __restrict__ anchors,
               OutputsDev out, const int32_t* __restrict__ route, int32_t* __restrict__ fill_done,
               const int16_t* __restrict__ path_states, const float* __restrict__ lse, int fmt) {
  __shared__ int32_t path[kFillWarps][1 << kMaxSegLog2];
  __shared__ int fold_flag;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const FillItem item = items[blockIdx.x];
  const RecordDev rec = recs[item.record];
  // A record of the chunked route the finisher filled and folded (its
  // counter is zeroed by the first pass; other records' is not used).
  // Uniform over the CTA.
  if (rec.num_pieces > 1 && fill_done[item.record] < 0) return;
  const int T = rec.T;
  const int H = 1 << rec.seg_log2;
  const int C = static_cast<int>((static_cast<int64_t>(T) + H - 1) >> rec.seg_log2);
  int64_t* labels = out.labels + rec.out_off;
  float* scores = out.scores + rec.out_off;
  if (rec.num_pieces <= 1) {
    fill_segment(rec, item.record, item.first_seg + warp, bp_arena, anchors, out, lse, fmt, path[warp], lane);
    return;  // uniform over the CTA
  }
  if (route[item.record] == kRouteStitched) {
    const int a = item.first_seg << rec.seg_log2;
    const int b = static_cast<int>(min(static_cast<int64_t>(T), static_cast<int64_t>(a) + (kFillWarps << rec.seg_log2)));
    gather_joined(rec, item.record, a, b, path_states, out, lse, fmt, threadIdx.x, 32 * kFillWarps);
  } else {
    fill_segment(rec, item.record, item.first_seg + warp, bp_arena, anchors, out, lse, fmt, path[warp], lane);
  }

  // The objective of a joined path (fold_path_scores); a non-finite sum
  // marks the record failed (alignment.cu:507-510, 650-652).
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const int ctas = (C + kFillWarps - 1) / kFillWarps;
    fold_flag = atomicAdd(&fill_done[item.record], 1) == ctas - 1 &&
                route[item.record] == kRouteStitched;
  }
  __syncthreads();
  if (!fold_flag) return;
  __threadfence();
  const float obj = fold_path_scores(scores, T, reinterpret_cast<float*>(&path[0][0]), kFillWarps << kMaxSegLog2,
                                     threadIdx.x, 32 * kFillWarps);
  if (threadIdx.x == 0) {
    out.objective[item.record] = obj;
    fold_flag = isfinite(obj) ? 1 : 0;
    if (!isfinite(obj)) out.status[item.record] = 1;
  }
  __syncthreads();
  if (fold_flag) return;
  for (int t = threadIdx.x; t < T; t += 32 * kFillWarps) { labels[t] = -1; scores[t] = -INFINITY; }
}

// Records of the window route (ffa_window.cu) whose window was not
// certified: the full conventional DP (alignment.cu:354-523), 4 or 8 states
// per thread with segment maps, then the traceback and outputs of its
// segments by the CTA's first kFillWarps warps.  The list and its count are
// written by the window kernel; CTAs stride over it.
template <bool kRow, int kV, int kFmt>
__global__ void __launch_bounds__(kCtaThreads, 1)
ffa_window_fallback(const __grid_constant__ ForwardParams P, const int32_t* __restrict__ list,
                    const int32_t* __restrict__ count) {
  extern __shared__ __align__(128) unsigned char smem_raw[];
  ForwardShared& sh = *reinterpret_cast<ForwardShared*>(smem_raw);
  __shared__ int32_t path[kFillWarps][1 << kMaxSegLog2];
  const int n = *count;
  int chunk_base = 0;  // emission chunks the slot's ring has carried (row staging)
  for (int i = static_cast<int>(blockIdx.x); i < n; i += static_cast<int>(gridDim.x)) {
    const int r = list[i];
    const RecordDev rec = P.recs[r];
    SlotCtx x;
    x.tid = threadIdx.x;
    x.warp = x.tid >> 5;
    x.lane = x.tid & 31;
    x.r = r;
    x.slot = 0;
    x.first_warp = 0;
    x.bar = 1;
    x.lw = x.warp;
    x.NT = rec.nw * 32;
    x.tl = x.tid;
    __syncthreads();  // the previous record's fill is done with the shared state
    if (x.tid == 0) {
      sh.edge = Boundary{-INFINITY, 0};
      sh.slot_fault[0] = 0;
    }
    __syncthreads();
    if (x.warp < rec.nw) {
      PieceRun run{0, 0, rec.T, kInitRecord, 1, nullptr, nullptr, -1, -1, false, chunk_base};
      if (rec.kst == 4) piece_dp<4, kRow, kV, true, kFmt>(x, rec, run, sh, smem_raw, P);
      else piece_dp<8, kRow, kV, true, kFmt>(x, rec, run, sh, smem_raw, P);
    }
    chunk_base += (rec.T + kChunkFrames - 1) / kChunkFrames;
    __syncthreads();  // objective, status, anchors and backpointers are written
    if (x.warp < kFillWarps) {
      const int C = static_cast<int>((static_cast<int64_t>(rec.T) + (1 << rec.seg_log2) - 1) >> rec.seg_log2);
      for (int c = x.warp; c < C; c += kFillWarps)
        fill_segment(rec, r, c, P.bp, P.anchors, P.out, P.lse, kFmt, path[x.warp], x.lane);
    }
  }
}

// valid[r] was set to 1; any CTA finding NaN or +inf in its chunk clears it.
// Chunks are kScanChunkBytes windows aligned to 16 bytes.  Each thread keeps
// kScanBatch float4 loads in flight (streaming, evict-first) before it tests
// any, so the read stream has the memory parallelism HBM needs; only the two
// edge chunks of a record test every element against the record's bounds.
__global__ void __launch_bounds__(kScanThreads)
ffa_validity_scan(const ScanRecord* __restrict__ recs, const ScanItem* __restrict__ items,
                  uint8_t* __restrict__ valid) {
  constexpr int kPerThread = kScanChunkBytes / (16 * kScanThreads);
  static_assert(kPerThread % kScanBatch == 0, "scan batches");
  const ScanItem item = items[blockIdx.x];
  const ScanRecord rec = recs[item.record];
  const uintptr_t base = reinterpret_cast<uintptr_t>(rec.data);
  const uintptr_t aligned = base & ~static_cast<uintptr_t>(15);
  const uintptr_t end = base + static_cast<uintptr_t>(rec.count) * 4;
  const uintptr_t lo = aligned + static_cast<uintptr_t>(item.chunk) * kScanChunkBytes;
  const uintptr_t hi = lo + kScanChunkBytes < end ? lo + kScanChunkBytes : end;
  const bool interior = lo >= base && hi == lo + kScanChunkBytes;
  auto poisoned = [](float x) { return isnan(x) || x == INFINITY; };
  bool bad = false;
#pragma unroll
  for (int b = 0; b < kPerThread; b += kScanBatch) {
    float4 v[kScanBatch];
#pragma unroll
    for (int u = 0; u < kScanBatch; ++u) {
      // Whole 16-byte blocks are read; lanes outside [base, end) are ignored.
      const uintptr_t p = lo + 16 * (threadIdx.x + static_cast<uintptr_t>(b + u) * kScanThreads);
      v[u] = p < hi ? __ldcs(reinterpret_cast<const float4*>(p)) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
#pragma unroll
    for (int u = 0; u < kScanBatch; ++u) {
      const float x[4] = {v[u].x, v[u].y, v[u].z, v[u].w};
      if (interior) {
        bad |= poisoned(x[0]) || poisoned(x[1]) || poisoned(x[2]) || poisoned(x[3]);
      } else {
        const uintptr_t p = lo + 16 * (threadIdx.x + static_cast<uintptr_t>(b + u) * kScanThreads);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const uintptr_t q = p + 4 * k;
          if (q >= base && q < end) bad |= poisoned(x[k]);
        }
      }
    }
  }
  if (__syncthreads_or(bad) && threadIdx.x == 0) valid[item.record] = 0;
}

// Token spans of aligned paths, one warp per record (the conversion the
// reference's README describes, README.md:509-517): the path's equal-label
// runs, blank runs dropped; run k of a record is its k-th token, as the path
// collapses to the transcript.  Each 32-frame chunk finds run starts and ends
// by comparing every label with its predecessor; a ballot and a population
// count number them.  A record whose non-blank run count is not U -- a failed
// record (labels -1) among them -- gets -1 for every span.
__global__ void __launch_bounds__(256)
ffa_token_spans_kernel(const SpanRecord* __restrict__ recs, int64_t count) {
  const int64_t r = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (r >= count) return;
  const SpanRecord rec = recs[r];
  const int64_t* labels = rec.labels;
  int64_t* spans = rec.spans;
  const unsigned lt = (1u << lane) - 1u;
  int runs = 0;            // non-blank runs started before this chunk
  int64_t carry = -1;      // label of the chunk's previous frame (-1: none)
  bool invalid = false;
  for (int base = 0; base < rec.T; base += 32) {
    const int t = base + lane;
    int64_t lab = t < rec.T ? labels[t] : rec.blank;
    if (lab < 0) { invalid = true; lab = rec.blank; }
    int64_t prev = __shfl_up_sync(0xffffffffu, lab, 1);
    if (lane == 0) prev = carry;
    const bool start = t < rec.T && lab != rec.blank && lab != prev;
    const bool end = t < rec.T && prev >= 0 && prev != rec.blank && lab != prev;
    const unsigned starts = __ballot_sync(0xffffffffu, start);
    const int before = runs + __popc(starts & lt);  // runs started before frame t
    if (start && before < rec.U) spans[2 * before] = t;
    if (end && before - 1 < rec.U) spans[2 * (before - 1) + 1] = t;
    runs += __popc(starts);
    carry = __shfl_sync(0xffffffffu, lab, 31);
  }
  // The last run ends with the record (past a partial last chunk, `carry`
  // holds padding, so the last frame's label is read again).
  if (lane == 0 && rec.T > 0) {
    const int64_t last = labels[rec.T - 1];
    if (last >= 0 && last != rec.blank && runs >= 1 && runs <= rec.U) spans[2 * (runs - 1) + 1] = rec.T;
  }
  invalid = __any_sync(0xffffffffu, invalid) || runs != rec.U;
  if (!invalid) return;
  for (int k = lane; k < 2 * rec.U; k += 32) spans[k] = -1;
}

// Row log-sum-exp of logits (input formats 1 and 2), the z that turns them
// into the log_softmax emissions x - z:
//   z[t] = m + log(sum_v exp(x[t, v] - m)),  m = max_v x[t, v],
// in fp32: the terms with CUDA's __expf intrinsic (its relative error, a
// few 1e-7 on terms in (0, 1], stays below the additions' rounding of the
// sum), the log with logf.  Lane l of a row's warp takes columns
// l, l + 32, l + 64, ... and sums their terms in that order; the warp then
// adds the lanes' sums in a butterfly (so every lane holds the same sum).
// That order depends on V alone, so a row's z is the same wherever the row
// lies and whichever variant below computes it.  A row holding NaN or +inf,
// or only -inf, gets NaN (its emissions are NaN, as torch.log_softmax's
// are).  Rows are in packed frame order; record r's rows are out_off ..
// out_off + T - 1, and each warp finds the record of its first row by a
// search over the descriptors.
//
// Each warp takes kLseRowsPerWarp consecutive rows.  kN > 0 (every V of
// the launch at most 32 kN, kN <= 2): the warp loads all of its rows' values
// before it reduces any, and the rows' reductions interleave.  kN == 0: one
// row at a time, each pass over the row's columns with 16 loads per lane in
// flight (the second pass finds the row in L1).
// Rows first .. first + kLseRowsPerWarp - 1 (those below `rows`), by one warp.
template <int kFmt, int kN>
__device__ __forceinline__ void lse_rows(const RecordDev* __restrict__ recs, int count, int64_t rows,
                                         float* __restrict__ z, int64_t first, int lane) {
  using Elem = typename Input<kFmt>::Elem;
  constexpr int kRows = kLseRowsPerWarp;
  // The last record with out_off <= first, by a 32-way search: lane j tests
  // the first record of the j-th of 32 blocks of the range (at most three
  // rounds for 65535 records).  Record 0 starts at row 0.
  int lo = 0, n = count;
  while (n > 1) {
    const int step = (n + 31) / 32;
    const int cand = lo + lane * step;
    const bool ok = cand < lo + n && recs[cand].out_off <= first;
    const int j = 31 - __clz(static_cast<int>(__ballot_sync(0xffffffffu, ok)));
    lo += j * step;
    n = min(step, n - j * step);
  }
  int r = lo;
  int64_t off = recs[r].out_off;
  int64_t T = recs[r].T;
  int V = recs[r].V;
  // The row's data (records follow one another in row order).
  auto locate = [&](int64_t row) {
    while (row >= off + T && r + 1 < count) {
      ++r;
      off = recs[r].out_off;
      T = recs[r].T;
      V = recs[r].V;
    }
    return reinterpret_cast<const Elem*>(recs[r].emissions) + (row - off) * V;
  };
  if constexpr (kN == 0) {
    const int64_t end = min(rows, first + kRows);
    for (int64_t row = first; row < end; ++row) {
      const Elem* x = locate(row);
      float m = -INFINITY;
#pragma unroll 16
      for (int v = lane; v < V; v += 32) m = fmaxf(m, elem_to_float(x[v]));
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
      float s = 0.0f;
#pragma unroll 16
      for (int v = lane; v < V; v += 32) s = __fadd_rn(s, __expf(__fsub_rn(elem_to_float(x[v]), m)));
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) s = __fadd_rn(s, __shfl_xor_sync(0xffffffffu, s, o));
      if (lane == 0) z[row] = __fadd_rn(m, logf(s));
    }
  } else {
    static_assert(kN <= 2, "register-resident rows");
    float val[kRows][kN];
    int vocab[kRows];
#pragma unroll
    for (int q = 0; q < kRows; ++q) {
      const int64_t row = first + q;
      const Elem* x = row < rows ? locate(row) : nullptr;
      vocab[q] = row < rows ? V : 0;
#pragma unroll
      for (int k = 0; k < kN; ++k) {
        const int v = lane + 32 * k;
        val[q][k] = v < vocab[q] ? elem_to_float(x[v]) : -INFINITY;
      }
    }
    float mine = 0.0f;  // lane q < kRows keeps row first + q's z
#pragma unroll
    for (int q = 0; q < kRows; ++q) {
      float m = -INFINITY;
#pragma unroll
      for (int k = 0; k < kN; ++k) m = fmaxf(m, val[q][k]);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
      float s = 0.0f;
#pragma unroll
      for (int k = 0; k < kN; ++k)
        if (lane + 32 * k < vocab[q]) s = __fadd_rn(s, __expf(__fsub_rn(val[q][k], m)));
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) s = __fadd_rn(s, __shfl_xor_sync(0xffffffffu, s, o));
      if (lane == q) mine = __fadd_rn(m, logf(s));
    }
    if (lane < kRows && first + lane < rows) z[first + lane] = mine;
  }
}

// The grid holds one wave of CTAs (or fewer); each warp takes row groups
// warp, warp + all warps, ... so no tail wave runs at low occupancy.
template <int kFmt, int kN>
__global__ void __launch_bounds__(kLseThreads)
ffa_row_lse(const RecordDev* __restrict__ recs, int count, int64_t rows, float* __restrict__ z) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (kLseThreads / 32);
  for (int64_t g = static_cast<int64_t>(blockIdx.x) * (kLseThreads / 32) + (threadIdx.x >> 5);
       g * kLseRowsPerWarp < rows; g += warps)
    lse_rows<kFmt, kN>(recs, count, rows, z, g * kLseRowsPerWarp, lane);
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

namespace {
thread_local int64_t g_launches = 0;
}  // namespace
int64_t launches_so_far() { return g_launches; }

// Copies 16-byte blocks from pinned host memory (read over the bus) to the
// device, many blocks in flight per thread.
__global__ void __launch_bounds__(256) ffa_upload_kernel(const uint4* __restrict__ src, uint4* __restrict__ dst,
                                                         int64_t n) {
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    dst[i] = src[i];
}

cudaError_t launch_upload(const void* mapped_src, void* dst, size_t bytes, cudaStream_t stream) {
  const int64_t n = static_cast<int64_t>((bytes + 15) / 16);
  if (n == 0) return cudaSuccess;
  ++g_launches;
  const unsigned blocks = static_cast<unsigned>(std::min<int64_t>((n + 255) / 256, 1184));
  ffa_upload_kernel<<<blocks, 256, 0, stream>>>(static_cast<const uint4*>(mapped_src), static_cast<uint4*>(dst), n);
  return cudaGetLastError();
}

cudaError_t launch_spans(const SpanRecord* recs, int64_t count, cudaStream_t stream) {
  if (count <= 0) return cudaSuccess;
  ++g_launches;
  const unsigned blocks = static_cast<unsigned>((count * 32 + 255) / 256);
  ffa_token_spans_kernel<<<blocks, 256, 0, stream>>>(recs, count);
  return cudaGetLastError();
}
void count_launch() { ++g_launches; }

namespace {
// Kernel variants per (staging, vocabulary specialisation, input format):
// log-probabilities have a V = 32 row-staged variant besides the generic
// ones; logits inputs use the generic row-staged and gathered kernels.
constexpr int kVariants = 7;
int variant_of(bool row_mode, int row_vocab, int fmt) {
  if (fmt == 0) return !row_mode ? 0 : (row_vocab == 32 ? 2 : 1);
  return 3 + 2 * (fmt - 1) + (row_mode ? 1 : 0);
}
using ForwardKernel = void (*)(ForwardParams);
using FinishKernel = void (*)(ForwardParams, const int32_t*, const int32_t*, int, unsigned);
const ForwardKernel kForwardKernels[kVariants] = {
    ffa_viterbi_forward<false, 0, 0>, ffa_viterbi_forward<true, 0, 0>, ffa_viterbi_forward<true, 32, 0>,
    ffa_viterbi_forward<false, 0, 1>, ffa_viterbi_forward<true, 0, 1>,
    ffa_viterbi_forward<false, 0, 2>, ffa_viterbi_forward<true, 0, 2>};
const FinishKernel kFinishKernels[kVariants] = {
    ffa_finish_route<false, 0, 0>, ffa_finish_route<true, 0, 0>, ffa_finish_route<true, 32, 0>,
    ffa_finish_route<false, 0, 1>, ffa_finish_route<true, 0, 1>,
    ffa_finish_route<false, 0, 2>, ffa_finish_route<true, 0, 2>};

using FallbackKernel = void (*)(ForwardParams, const int32_t*, const int32_t*);
const FallbackKernel kFallbackKernels[kVariants] = {
    ffa_window_fallback<false, 0, 0>, ffa_window_fallback<true, 0, 0>, ffa_window_fallback<true, 32, 0>,
    ffa_window_fallback<false, 0, 1>, ffa_window_fallback<true, 0, 1>,
    ffa_window_fallback<false, 0, 2>, ffa_window_fallback<true, 0, 2>};

// Opting in to >48 KiB of dynamic shared memory is per device and kernel:
// done once, to `bytes`, then every launch fits under it.
template <typename Kernel>
cudaError_t opt_in(Kernel kernel, std::atomic<uint64_t>& opted, size_t bytes) {
  int device = 0;
  cudaError_t err = cudaGetDevice(&device);
  if (err != cudaSuccess) return err;
  const uint64_t bit = device < 64 ? uint64_t{1} << device : 0;
  if (bit != 0 && (opted.load(std::memory_order_acquire) & bit)) return cudaSuccess;
  err = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(bytes));
  if (err != cudaSuccess) return err;
  if (bit) opted.fetch_or(bit, std::memory_order_acq_rel);
  return cudaSuccess;
}

// The current device's SM count (cached per device).
int device_sm_count() {
  static std::atomic<int> cache[64];
  int device = 0;
  if (cudaGetDevice(&device) != cudaSuccess) return 148;
  int v = device < 64 ? cache[device].load(std::memory_order_relaxed) : 0;
  if (v > 0) return v;
  if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, device) != cudaSuccess || v <= 0) v = 148;
  if (device < 64) cache[device].store(v, std::memory_order_relaxed);
  return v;
}

template <int kFmt, int kN>
cudaError_t lse_launch(const RecordDev* recs, int count, int64_t rows, float* z, cudaStream_t stream) {
  // One wave: the SMs times the CTAs of this variant resident on one SM
  // (cached per device).
  static std::atomic<int> wave[64];
  int device = 0;
  cudaError_t err = cudaGetDevice(&device);
  if (err != cudaSuccess) return err;
  int ctas = device < 64 ? wave[device].load(std::memory_order_relaxed) : 0;
  if (ctas <= 0) {
    int sms = 0, per_sm = 0;
    err = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
    if (err != cudaSuccess) return err;
    err = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, ffa_row_lse<kFmt, kN>, kLseThreads, 0);
    if (err != cudaSuccess) return err;
    ctas = std::max(1, sms * per_sm);
    if (device < 64) wave[device].store(ctas, std::memory_order_relaxed);
  }
  const int64_t per_cta = static_cast<int64_t>(kLseThreads / 32) * kLseRowsPerWarp;
  const int64_t blocks = std::min<int64_t>((rows + per_cta - 1) / per_cta, ctas);
  ++g_launches;
  ffa_row_lse<kFmt, kN><<<static_cast<unsigned>(blocks), kLseThreads, 0, stream>>>(recs, count, rows, z);
  return cudaGetLastError();
}
template <int kFmt>
cudaError_t lse_dispatch(const RecordDev* recs, int count, int64_t rows, int max_vocab, float* z,
                         cudaStream_t stream) {
  if (max_vocab <= 32) return lse_launch<kFmt, 1>(recs, count, rows, z, stream);
  if (max_vocab <= 64) return lse_launch<kFmt, 2>(recs, count, rows, z, stream);
  return lse_launch<kFmt, 0>(recs, count, rows, z, stream);
}
}  // namespace

cudaError_t launch_forward(const ForwardParams& params, int num_bundles, bool row_mode,
                           int row_vocab, int fmt, unsigned smem_bytes, cudaStream_t stream) {
  if (num_bundles <= 0) return cudaSuccess;
  if (fmt < 0 || fmt > 2) return cudaErrorInvalidValue;
  static std::atomic<uint64_t> opted[kVariants];
  const int variant = variant_of(row_mode, row_vocab, fmt);
  const ForwardKernel kernel = kForwardKernels[variant];
  cudaError_t err = opt_in(kernel, opted[variant], kSmemBudget);
  if (err != cudaSuccess) return err;
  if (smem_bytes > kSmemBudget) return cudaErrorInvalidValue;
  ++g_launches;
  kernel<<<num_bundles, kCtaThreads, smem_bytes, stream>>>(params);
  return cudaGetLastError();
}

cudaError_t launch_finish(const ForwardParams& params, const int32_t* records, int count,
                          const int32_t* device_count, int ctas_per_record, int threads, bool row_mode,
                          int row_vocab, int fmt, unsigned smem_bytes, cudaStream_t stream) {
  if (count <= 0) return cudaSuccess;
  if (fmt < 0 || fmt > 2) return cudaErrorInvalidValue;
  static std::atomic<uint64_t> opted[kVariants];
  const int variant = variant_of(row_mode, row_vocab, fmt);
  const FinishKernel kernel = kFinishKernels[variant];
  cudaError_t err = opt_in(kernel, opted[variant], kFinishDynamicSmem);
  if (err != cudaSuccess) return err;
  if (smem_bytes > kFinishDynamicSmem) return cudaErrorInvalidValue;
  if (threads != kCtaThreads && threads != kCtaThreads / 2 && threads != kCtaThreads / 4)
    return cudaErrorInvalidValue;
  ++g_launches;
  kernel<<<count * ctas_per_record, threads, smem_bytes, stream>>>(params, records, device_count, ctas_per_record,
                                                                  smem_bytes);
  return cudaGetLastError();
}

cudaError_t launch_window_fallback(const ForwardParams& params, const int32_t* list, const int32_t* count,
                                   int max_count, int row_vocab, int fmt, unsigned smem_bytes, cudaStream_t stream) {
  if (max_count <= 0) return cudaSuccess;
  if (fmt < 0 || fmt > 2) return cudaErrorInvalidValue;
  static std::atomic<uint64_t> opted[kVariants];
  const int variant = variant_of(true, row_vocab, fmt);
  const FallbackKernel kernel = kFallbackKernels[variant];
  // Static shared memory: the fill warps' path scratch.
  constexpr size_t kDynamic = kSmemBudget - sizeof(int32_t) * kFillWarps * (1 << kMaxSegLog2);
  cudaError_t err = opt_in(kernel, opted[variant], kDynamic);
  if (err != cudaSuccess) return err;
  if (smem_bytes > kDynamic) return cudaErrorInvalidValue;
  const int ctas = std::min(max_count, std::max(device_sm_count(), 1));
  ++g_launches;
  kernel<<<ctas, kCtaThreads, smem_bytes, stream>>>(params, list, count);
  return cudaGetLastError();
}

cudaError_t launch_lse(const RecordDev* recs, int count, int64_t rows, int max_vocab, int fmt, float* z,
                       cudaStream_t stream) {
  if (rows <= 0) return cudaSuccess;
  if (fmt == 1) return lse_dispatch<1>(recs, count, rows, max_vocab, z, stream);
  if (fmt == 2) return lse_dispatch<2>(recs, count, rows, max_vocab, z, stream);
  return cudaErrorInvalidValue;
}

cudaError_t launch_fill(const RecordDev* recs, const FillItem* items, int num_items,
                        const uint32_t* bp, const int32_t* anchors, const OutputsDev& out,
                        const int32_t* route, int32_t* fill_done, const int16_t* path_states, const float* lse,
                        int fmt, cudaStream_t stream) {
  if (num_items <= 0) return cudaSuccess;
  ++g_launches;
  ffa_trace_fill<<<num_items, 32 * kFillWarps, 0, stream>>>(recs, items, bp, anchors, out, route,
                                                             fill_done, path_states, lse, fmt);
  return cudaGetLastError();
}

cudaError_t launch_check_targets(const RecordDev* recs, int64_t count, int32_t* status,
                                 cudaStream_t stream) {
  ++g_launches;
  ffa_check_targets_kernel<<<static_cast<unsigned>((count + 7) / 8), 256, 0, stream>>>(recs, count, status);
  return cudaGetLastError();
}

cudaError_t launch_validity(const ScanRecord* recs, int64_t count, const ScanItem* items,
                            int64_t num_items, uint8_t* valid, cudaStream_t stream) {
  const int fill_blocks = static_cast<int>((count + 255) / 256);
  ++g_launches;
  ffa_fill_u8<<<fill_blocks, 256, 0, stream>>>(valid, count, 1);
  cudaError_t err = cudaGetLastError();
  if (err != cudaSuccess || num_items <= 0) return err;
  ++g_launches;
  ffa_validity_scan<<<static_cast<unsigned>(num_items), kScanThreads, 0, stream>>>(recs, items, valid);
  return cudaGetLastError();
}

}  // namespace ffa
