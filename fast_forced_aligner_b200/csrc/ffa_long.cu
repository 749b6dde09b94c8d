// ffa_long.cu -- conventional DP of long records on thread-block clusters.
//
// A record with more CTC states than one CTA holds (kMaxStates < S <=
// kMaxLongStates; the reference stops at S = 4095, alignment.py:250) runs on
// one cluster of C = ceil(S / 512 K) CTAs: CTA c owns states [512 K c,
// 512 K (c + 1)), K per thread (8, or 16 where that lets every record of the
// launch run at once: clusters of more than 9 CTAs fit only 7 at a time on a
// B200).  Each CTA runs, frame by frame, the same
// max-plus step as every other DP of this library (dp_frame: stay > step >
// skip by strict '>', one fp32 add per cell, alignment.cu:418-424, with the
// ancestor deltas of the segment maps).  The only dependence between CTAs is
// the left neighbour's last state at the previous frame (a state reads s-1
// and s-2, and a CTA's first state is a blank, which has no skip), so:
//   - after each frame, CTA c's last thread publishes that state for CTA c+1:
//     one 8-byte store into a kLinkRing-frame ring in CTA c+1's shared
//     memory (distributed shared memory, no global round trip);
//   - CTA c+1's first thread reads it when it steps the next frame, and
//     reports the frames it has consumed back into CTA c's shared memory once
//     per frame group, so a producer runs at most kLinkRing frames ahead.
// Every wait is bounded (kWaitNs); a CTA whose wait gave up stops waiting and
// the record ends with status 5.  After the last frame the terminal states
// and any failure reach the last CTA, which applies the terminal rule
// (alignment.cu:496-510) and walks the segment maps into the anchors; the
// traceback fill then runs as for any whole record.
#include <cuda_runtime.h>

#include <atomic>
#include <cmath>
#include <cstdint>

#include "ffa_device.cuh"
#include "ffa_internal.h"

namespace ffa {
using namespace dev;
namespace {

constexpr unsigned kFull = 0xffffffffu;

struct LongShared {
  Boundary bnd[2][kMaxWarps];  // last-state hand-off between the CTA's warps
  int chk_bad[kMaxWarps];
  int chk_rep[kMaxWarps];
  int status;
  unsigned cta_fault;          // a wait of this CTA gave up
  unsigned fault;              // last CTA: a wait of some CTA of the cluster gave up
  float term_last, term_prev;  // last CTA: alpha[S-1], alpha[S-2] at the last frame
  unsigned long long link[kLinkRing];  // left neighbour's last state, frame t at t % kLinkRing
  unsigned long long ack;              // frames the right neighbour has consumed
  unsigned long long full[kRowRing];   // emission chunk landed (row staging)
};
constexpr size_t kLongHeader = (sizeof(LongShared) + 127) / 128 * 128;

// One frame's boundary as a 64-bit word: alpha's bits, the ancestor delta
// (at most 2 states per frame over a segment of at most 1024 frames: < 2^12)
// and the frame number's low 20 bits.  A CTA runs ahead of its left
// neighbour only while its first warp is above the reachable band, i.e. for
// fewer than 32768 frames, so a slot never holds a stale word whose frame
// bits equal those of the frame its reader waits for.
constexpr unsigned kFrameBits = 20;
constexpr unsigned kFrameMask = (1u << kFrameBits) - 1;
__device__ __forceinline__ unsigned long long pack_link(int t, float alpha, int delta) {
  return static_cast<unsigned long long>(__float_as_uint(alpha)) << 32 |
         static_cast<unsigned long long>(static_cast<unsigned>(delta) & 0xfffu) << kFrameBits |
         (static_cast<unsigned>(t) & kFrameMask);
}

template <int K, bool kRow, int kV, int kFmt>
__global__ void __launch_bounds__(kCtaThreads, 1)
ffa_long_forward(const __grid_constant__ LongParams P) {
  using In = Input<kFmt>;
  using Elem = typename In::Elem;
  constexpr int KT = K / 2;
  extern __shared__ __align__(128) unsigned char smem_raw[];
  LongShared& sh = *reinterpret_cast<LongShared*>(smem_raw);
  const unsigned rank = cluster_rank(), C = cluster_size();
  const int r = P.records[blockIdx.x / C];
  const RecordDev rec = P.recs[r];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int T = rec.T, U = rec.U, blank = rec.blank;
  const int V = kV > 0 ? kV : rec.V;
  const int S = 2 * U + 1;
  const int64_t* tgt = rec.targets;
  // Thread index within the record: thread g owns states K g .. K g + K-1.
  const int g = static_cast<int>(rank) * kCtaThreads + tid;

  // ---- status: mask, then target validation (alignment.cu:836, 852-874).
  // Every CTA computes it, so the whole cluster agrees without exchanging it.
  int status = P.mask != nullptr && !P.mask[r] ? 2 : 0;
  if (P.check_inputs) {
    int bad = 0, rep = 0;
    for (int k = tid; k < U; k += kCtaThreads) {
      const int64_t token = tgt[k];
      bad |= (token < 0 || token >= V || token == blank) ? 1 : 0;
      if (k > 0) rep += token == tgt[k - 1] ? 1 : 0;
    }
    bad = __reduce_or_sync(kFull, bad);
    rep = __reduce_add_sync(kFull, rep);
    if (lane == 0) { sh.chk_bad[warp] = bad; sh.chk_rep[warp] = rep; }
    __syncthreads();
    if (tid == 0) {
      int b = 0;
      int64_t q = 0;
      for (int w = 0; w < kMaxWarps; ++w) { b |= sh.chk_bad[w]; q += sh.chk_rep[w]; }
      sh.status = b ? 3 : (static_cast<int64_t>(U) + q > T ? 4 : status);
    }
    __syncthreads();
    status = sh.status;
  }
  if (rank == 0 && tid == 0) {
    // Diagnostics start at zero (alignment.py:101-129): long records always
    // take the conventional DP.
    P.out.stitched[r] = 0;
    P.out.repair_passes[r] = 0;
    P.out.repaired_frames[r] = 0;
    for (int j = 0; j < 3; ++j) { P.out.shortcut_stats[3 * r + j] = 0; P.out.routing_stats[3 * r + j] = 0; }
    if (P.out.reuse_stats) for (int j = 0; j < 4; ++j) P.out.reuse_stats[4 * r + j] = 0;
    if (status >= 2) { P.out.objective[r] = -INFINITY; P.out.status[r] = status; }
  }
  if (status >= 2) return;  // every CTA of the cluster returns here

  // Labels of this thread's states (odd k: token K/2 g + k/2) and which of
  // them a skip may enter (alignment.cu:407).
  int col[KT];
  unsigned skip = 0;
  {
    const int first = KT * g;
    int prev = (first >= 1 && first - 1 < U) ? clamp_label(tgt[first - 1], V) : -1;
#pragma unroll
    for (int q = 0; q < KT; ++q) {
      const int u = first + q;
      col[q] = u < U ? clamp_label(tgt[u], V) : blank;
      if (u < U && u >= 1 && col[q] != blank && col[q] != prev) skip |= 1u << q;
      prev = col[q];
    }
  }

  // Emission rows: TMA bulk copies of kChunkFrames rows into a kRowRing ring
  // (row staging), or per-thread cp.async gathers of the thread's columns;
  // logits are normalised as they are read (x - z, Input<kFmt>).
  const Elem* e = reinterpret_cast<const Elem*>(rec.emissions);
  Elem* ring = reinterpret_cast<Elem*>(smem_raw + kLongHeader);
  float* gring = reinterpret_cast<float*>(smem_raw + kLongHeader) + tid;
  HalfWords hw{};
  if constexpr (In::kHalf && !kRow) hw.set(rec.emissions);
  static_assert(kChunkGroups * kGroup == 32, "log-sum-exp blocks");
  LseStream lse{};
  if constexpr (In::kLogits) lse.start(P.lse + rec.out_off, T, 0, lane);
  const int nchunks = (T + kChunkFrames - 1) / kChunkFrames;
  auto issue_chunk = [&](int c) {  // kRow: by thread 0
    const int rows = min(kChunkFrames, T - c * kChunkFrames);
    const unsigned bytes = static_cast<unsigned>(rows) * V * static_cast<unsigned>(sizeof(Elem));
    unsigned long long* bar = &sh.full[c % kRowRing];
    mbar_expect_tx(bar, bytes);
    tma_bulk_load(ring + (c % kRowRing) * kChunkFrames * V, e + static_cast<int64_t>(c) * kChunkFrames * V,
                  bytes, bar);
  };
  auto gather = [&](int f) {  // !kRow: KT + 1 private 4-byte copies of frame f
    if (f < T) {
      float* dst = gring + (f % kGroup) * (KT + 1) * kCtaThreads;
      if constexpr (In::kHalf) {
        const int64_t i = static_cast<int64_t>(f) * V;
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

  if (tid == 0) {
    // No frame has arrived: a frame field no reader can be waiting for.
    for (int k = 0; k < kLinkRing; ++k) sh.link[k] = pack_link(static_cast<int>(kFrameMask), -INFINITY, 0);
    sh.ack = 0;
    sh.cta_fault = 0;
    sh.fault = 0;
    sh.term_last = -INFINITY;
    sh.term_prev = -INFINITY;
    if constexpr (kRow) {
      for (int k = 0; k < kRowRing; ++k) mbar_init(&sh.full[k], 1);
      fence_mbar_init();
      for (int c = 0; c < kRowRing && c < nchunks; ++c) issue_chunk(c);
    }
  }
  if constexpr (!kRow) {
#pragma unroll
    for (int f = 0; f < kGroup - 1; ++f) gather(f);
  }
  // Every CTA's ring is initialised before any neighbour writes into it.
  cluster_sync();

  const bool consumer = rank > 0 && tid == 0;
  const bool producer = rank + 1 < C && tid == kCtaThreads - 1;
  const unsigned right_link = producer ? cluster_addr(&sh.link[0], rank + 1) : 0u;
  const unsigned left_ack = consumer ? cluster_addr(&sh.ack, rank - 1) : 0u;
  bool tma_fault = false, link_fault = false;

  // Producer: frame t's last state into the right neighbour's ring, once that
  // neighbour has consumed frame t - kLinkRing from the same slot (the
  // neighbour's count is re-read only when the copy last read is too old).
  long long acked = 0;
  auto link_put = [&](int t, float alpha, int delta) {
    const long long need = static_cast<long long>(t) - kLinkRing + 1;
    if (need > acked) {
      acked = static_cast<long long>(ld_cluster_u64(&sh.ack));
      if (need > acked && !link_fault) {
        const unsigned long long start = global_ns();
        while ((acked = static_cast<long long>(ld_cluster_u64(&sh.ack))) < need)
          if (global_ns() - start > kWaitNs) { link_fault = true; break; }
      }
    }
    st_cluster_u64(right_link + static_cast<unsigned>(t % kLinkRing) * 8u, pack_link(t, alpha, delta));
  };
  // Consumer, warp 0: lane l < kGroup holds the word of frame tg - 1 + l as it
  // stood when the group started (the producer usually runs ahead, so a
  // group's boundaries cost one load per lane); lane 0 waits only for a frame
  // that had not arrived.
  const bool link_warp = rank > 0 && warp == 0;
  unsigned long long linkw = 0;
  auto link_prefetch = [&](int tg) {
    const int f = tg - 1 + lane;
    linkw = (lane < kGroup && f >= 0) ? ld_cluster_u64(&sh.link[f % kLinkRing]) : 0ull;
  };
  auto link_wait = [&](int t, unsigned long long w) {
    const unsigned long long* slot = &sh.link[t % kLinkRing];
    const unsigned want = static_cast<unsigned>(t) & kFrameMask;
    if ((static_cast<unsigned>(w) & kFrameMask) != want) {
      w = ld_cluster_u64(slot);
      if ((static_cast<unsigned>(w) & kFrameMask) != want && !link_fault) {
        const unsigned long long start = global_ns();
        while (((w = ld_cluster_u64(slot)) & kFrameMask) != want)
          if (global_ns() - start > kWaitNs) { link_fault = true; break; }
      }
    }
    return w;
  };

  float a[K];
  int d[K];
#pragma unroll
  for (int k = 0; k < K; ++k) { a[k] = -INFINITY; d[k] = 0; }
  const int hmask = (1 << rec.seg_log2) - 1;
  const int row_words = bp_row_words(S);
  uint8_t* bp_rows = reinterpret_cast<uint8_t*>(P.bp + rec.bp_off);
  const bool stores_codes = K * g < row_words * 16;
  const int64_t map_stride = state_stride(S);
  const bool stores_maps = K * g < map_stride;
  uint16_t* maps = P.maps + rec.map_off + K * g;
  // Reachable band [S - 2(T - t), 2t + 1], tested per warp and frame group
  // exactly as in the first pass; warps wholly past the last state never run.
  const int w_lo = K * (g - lane);
  const int w_hi = w_lo + 32 * K - 1;
  const unsigned band_lo = static_cast<unsigned>(max(w_lo - 1, 0));
  const int64_t hi64 = static_cast<int64_t>(w_hi) - S + 2 * static_cast<int64_t>(T);
  const bool never = hi64 < 0 || w_lo >= S;
  const unsigned band_hi = never ? 0u : (hi64 > 0xffffffffLL ? 0xffffffffu : static_cast<unsigned>(hi64));

  // Frame f's emissions of this thread's states (row j of the staged group
  // `rows`); logits become x - z.  Called by whole warps.
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
        const bool odd = hw.row_odd(f, V);
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
    if (!stores_maps) return;
    uint32_t* dst = reinterpret_cast<uint32_t*>(maps + static_cast<int64_t>(t >> rec.seg_log2) * map_stride);
#pragma unroll
    for (int q = 0; q < KT; ++q)
      dst[q] = static_cast<uint32_t>(d[2 * q]) | (static_cast<uint32_t>(d[2 * q + 1]) << 16);
  };
  auto frame = [&](int t, int j, const Elem* rows) {
    float eb, et[KT];
    load(t, j, rows, eb, et);
    float p1 = __shfl_up_sync(kFull, a[K - 1], 1);
    int pd = __shfl_up_sync(kFull, d[K - 1], 1);
    unsigned long long lw = 0;
    if (link_warp) lw = __shfl_sync(kFull, linkw, j);  // frame t - 1's word as prefetched
    if (lane == 0) {
      if (warp > 0) {
        const Boundary nb = sh.bnd[t & 1][warp - 1];
        p1 = nb.alpha;
        pd = nb.delta;
      } else if (consumer) {
        lw = link_wait(t - 1, lw);
        p1 = __uint_as_float(static_cast<unsigned>(lw >> 32));
        pd = static_cast<int>((lw >> kFrameBits) & 0xfffu);
      } else {
        p1 = -INFINITY;
        pd = 0;
      }
    }
    if (j == 0 && (t & hmask) == 0) {  // a new traceback segment starts at t
#pragma unroll
      for (int k = 0; k < K; ++k) d[k] = 0;
      pd = 0;
    }
    const unsigned bits = dp_frame<K>(a, d, p1, pd, eb, et, skip);
    if (stores_codes) store_codes<K>(bp_rows + static_cast<int64_t>(t) * row_words * 4, g, bits);
    if (j == kGroup - 1 && (t & hmask) == hmask) store_map(t);
    if (lane == 31) sh.bnd[(t + 1) & 1][warp] = Boundary{a[K - 1], d[K - 1]};
    // Published before the barrier (measured faster than after it from three
    // CTAs per cluster on: the neighbour's group prefetch then finds it).
    if (producer) link_put(t, a[K - 1], d[K - 1]);
    __syncthreads();
  };

  const int ngroups = (T + kGroup - 1) / kGroup;
  for (int gi = 0; gi < ngroups; ++gi) {
    const Elem* rows = nullptr;
    if constexpr (In::kLogits)
      if (gi > 0 && gi % kChunkGroups == 0) lse.advance(gi * kGroup, lane);
    if constexpr (kRow) {
      const int c = gi / kChunkGroups;
      if (gi % kChunkGroups == 0 && !tma_fault && !mbar_wait(&sh.full[c % kRowRing], (c / kRowRing) & 1))
        tma_fault = true;
      rows = ring + ((c % kRowRing) * kChunkFrames + (gi % kChunkGroups) * kGroup) * V;
    }
    const int tg = gi * kGroup;
    const unsigned g2 = 2u * static_cast<unsigned>(tg);
    const bool seeded = gi == 0;
    const bool group_active = seeded || (!never && g2 + 2u * (kGroup - 1) >= band_lo && g2 <= band_hi);
    if (!group_active) {
      // Out of band: above it the states stay -inf, or turn NaN for good on
      // a NaN or +inf emission (as the full DP holds them); below it they
      // can no longer reach the end.  The producer still publishes every
      // frame, so its neighbour never waits on a frame it skipped.
      const bool above = !never && g2 + 2u * (kGroup - 1) < band_lo;
#pragma unroll 1
      for (int j = 0; j < kGroup && tg + j < T; ++j) {
        if (above || !kRow) {
          float eb, et[KT];
          load(tg + j, j, rows, eb, et);
          if (above) {
#pragma unroll
            for (int k = 0; k < K; ++k)
              if (poisons((k & 1) ? et[k >> 1] : eb)) a[k] = NAN;
          }
        }
        if (producer) link_put(tg + j, a[K - 1], d[K - 1]);
        __syncthreads();
      }
    } else if (seeded) {
      // Frame 0: alpha[s] = e[0, l[s]] for s < 2, else -inf (alignment.cu:409).
      float eb, et[KT];
      load(0, 0, rows, eb, et);
      if (g == 0) {
        a[0] = eb;
        if (S > 1) a[1] = et[0];
      }
      if (lane == 31) sh.bnd[1][warp] = Boundary{a[K - 1], 0};
      if (producer) link_put(0, a[K - 1], 0);
      __syncthreads();
      if (link_warp) link_prefetch(0);
#pragma unroll 1
      for (int j = 1; j < kGroup && j < T; ++j) frame(j, j, rows);
    } else {
      if (link_warp) link_prefetch(tg);
#pragma unroll
      for (int j = 0; j < kGroup; ++j)
        if (tg + j < T) frame(tg + j, j, rows);
    }
    // Frames below tg + kGroup - 1 are consumed: their ring slots may be reused.
    if (consumer) st_cluster_u64(left_ack, static_cast<unsigned long long>(tg + kGroup - 1));
    if constexpr (kRow) {
      const int c = gi / kChunkGroups;
      if (tid == 0 && (gi % kChunkGroups == kChunkGroups - 1 || gi == ngroups - 1) && c + kRowRing < nchunks) {
        fence_proxy_async();
        issue_chunk(c + kRowRing);
      }
    }
  }
  if constexpr (!kRow) cp_async_wait<0>();
  if constexpr (kRow) {
    // After a failed wait, give the copies still in flight a short, bounded
    // chance to land before the CTA's shared memory goes away.
    if (tma_fault && tid == 0)
      for (int c = max(0, nchunks - kRowRing); c < nchunks; ++c)
        mbar_wait(&sh.full[c % kRowRing], (c / kRowRing) & 1, kDrainNs);
  }
  if (((T - 1) & hmask) != hmask) store_map(T - 1);  // the last, partial segment

  // Terminal states and failures to the last CTA.
  const int last = S - 1;
#pragma unroll
  for (int q = 0; q < K; ++q) {
    const int s = K * g + q;
    if (s == last) st_cluster_f32(cluster_addr(&sh.term_last, C - 1), a[q]);
    if (s == last - 1) st_cluster_f32(cluster_addr(&sh.term_prev, C - 1), a[q]);
  }
  if (tma_fault || link_fault) atomicOr(&sh.cta_fault, 1u);
  __syncthreads();
  if (tid == 0 && sh.cta_fault) st_cluster_u32(cluster_addr(&sh.fault, C - 1), 1u);
  __threadfence();  // backpointers and maps visible to the last CTA's walk
  cluster_sync();
  if (rank != C - 1 || tid != 0) return;

  // Terminal rule: S-1 unless S>1 and alpha[S-2] >= alpha[S-1]
  // (alignment.cu:497-499); status from the objective (:507-510).
  int end_state = last;
  float best = sh.term_last;
  if (S > 1 && sh.term_prev >= best) { end_state = last - 1; best = sh.term_prev; }
  const bool fault = sh.fault != 0;
  const bool finite = isfinite(best);
  P.out.objective[r] = best;
  P.out.status[r] = fault ? kStatusDeviceFault : (finite ? 0 : 1);
  if (!finite || fault) return;
  // The path's state at every segment end, from the maps (the clamp never
  // acts on maps a completed DP wrote; it keeps every read in the arena).
  const uint16_t* mp = P.maps + rec.map_off;
  int32_t* anc = P.anchors + rec.seg_off;
  int s = end_state;
  for (int seg = (T - 1) >> rec.seg_log2; seg >= 0; --seg) {
    anc[seg] = s;
    s = min(max(s - mp[static_cast<int64_t>(seg) * map_stride + s], 0), S - 1);
  }
}

}  // namespace

size_t long_header_bytes() { return kLongHeader; }

namespace {
using LongKernel = void (*)(LongParams);
// Kernel variant and its index among the (K, staging, input format)
// instantiations: per K, log-probabilities gathered / row-staged / row-staged
// at V = 32, then fp32 and bf16 logits gathered / row-staged.
constexpr int kLongVariants = 14;
LongKernel long_kernel(int k, bool row_mode, int row_vocab, int fmt, int* variant) {
  const int per_k = fmt == 0 ? (!row_mode ? 0 : (row_vocab == 32 ? 2 : 1)) : 3 + 2 * (fmt - 1) + (row_mode ? 1 : 0);
  const int v = (k == 16 ? 7 : 0) + per_k;
  *variant = v;
  static const LongKernel table[kLongVariants] = {
      ffa_long_forward<8, false, 0, 0>,  ffa_long_forward<8, true, 0, 0>,  ffa_long_forward<8, true, 32, 0>,
      ffa_long_forward<8, false, 0, 1>,  ffa_long_forward<8, true, 0, 1>,
      ffa_long_forward<8, false, 0, 2>,  ffa_long_forward<8, true, 0, 2>,
      ffa_long_forward<16, false, 0, 0>, ffa_long_forward<16, true, 0, 0>, ffa_long_forward<16, true, 32, 0>,
      ffa_long_forward<16, false, 0, 1>, ffa_long_forward<16, true, 0, 1>,
      ffa_long_forward<16, false, 0, 2>, ffa_long_forward<16, true, 0, 2>};
  return table[v];
}
cudaLaunchConfig_t long_config(int count, int cluster, unsigned smem, cudaStream_t stream,
                               cudaLaunchAttribute* attr) {
  attr->id = cudaLaunchAttributeClusterDimension;
  attr->val.clusterDim.x = static_cast<unsigned>(cluster);
  attr->val.clusterDim.y = 1;
  attr->val.clusterDim.z = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(count * cluster));
  cfg.blockDim = dim3(kCtaThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cfg;
}
// Per device and variant, once: the shared-memory budget and clusters beyond
// the portable 8 CTAs.
cudaError_t prepare_long(LongKernel kernel, int variant, int device) {
  static std::atomic<uint64_t> opted[kLongVariants];
  const uint64_t bit = device < 64 ? uint64_t{1} << device : 0;
  if (bit != 0 && (opted[variant].load(std::memory_order_acquire) & bit)) return cudaSuccess;
  cudaError_t err = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(kSmemBudget));
  if (err != cudaSuccess) return err;
  err = cudaFuncSetAttribute(kernel, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
  if (err != cudaSuccess) return err;
  if (bit) opted[variant].fetch_or(bit, std::memory_order_acq_rel);
  return cudaSuccess;
}
}  // namespace

int long_capacity(int k, int cluster, bool row_mode, int row_vocab, int fmt, unsigned smem_bytes) {
  if ((k != 8 && k != 16) || cluster < 1 || cluster > kMaxClusterCtas || smem_bytes > kSmemBudget ||
      fmt < 0 || fmt > 2)
    return 0;
  int variant = 0;
  const LongKernel kernel = long_kernel(k, row_mode, row_vocab, fmt, &variant);
  int device = 0;
  if (cudaGetDevice(&device) != cudaSuccess) return 0;
  // Cached per (device, variant, cluster size): the count + 1 (0 = unknown).
  static std::atomic<int> known[kLongVariants][64][kMaxClusterCtas + 1];
  const int slot = device < 64 ? device : 63;
  const int cached = known[variant][slot][cluster].load(std::memory_order_acquire);
  if (cached > 0 && device < 64) return cached - 1;
  if (prepare_long(kernel, variant, device) != cudaSuccess) return 0;
  cudaLaunchAttribute attr;
  cudaLaunchConfig_t cfg = long_config(1, cluster, smem_bytes, nullptr, &attr);
  int clusters = 0;
  if (cudaOccupancyMaxActiveClusters(&clusters, kernel, &cfg) != cudaSuccess) {
    (void)cudaGetLastError();
    clusters = 0;
  }
  if (device < 64) known[variant][slot][cluster].store(clusters + 1, std::memory_order_release);
  return clusters;
}

cudaError_t launch_long(const LongParams& params, int count, int cluster, int k, bool row_mode,
                        int row_vocab, int fmt, unsigned smem_bytes, cudaStream_t stream) {
  if (count <= 0) return cudaSuccess;
  if ((k != 8 && k != 16) || cluster < 1 || cluster > kMaxClusterCtas || smem_bytes > kSmemBudget ||
      fmt < 0 || fmt > 2)
    return cudaErrorInvalidValue;
  if (long_capacity(k, cluster, row_mode, row_vocab, fmt, smem_bytes) < 1) return cudaErrorInvalidClusterSize;
  int variant = 0;
  const LongKernel kernel = long_kernel(k, row_mode, row_vocab, fmt, &variant);
  cudaLaunchAttribute attr;
  cudaLaunchConfig_t cfg = long_config(count, cluster, smem_bytes, stream, &attr);
  count_launch();
  return cudaLaunchKernelEx(&cfg, kernel, params);
}

}  // namespace ffa
