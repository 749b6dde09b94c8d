// ffa_window.cu -- the window route of the optimized mode (sm_100a).
//
//   ffa_window_viterbi   one warp per record: the conventional max-plus
//                        Viterbi DP (alignment.cu:354-523) restricted to a
//                        64-state window that slides up the trellis, with
//                        the greedy bound of every frame (the largest
//                        emission over the transcript alphabet, the maximum
//                        the reference's greedy_shortcuts finds,
//                        alignment.cu:29-153) certifying that no state left
//                        outside the window could have been on the full DP's
//                        path.  Emission rows arrive by TMA bulk copies;
//                        backpointers, segment maps and the traceback stay in
//                        shared memory, and the warp writes the record's
//                        labels, scores, objective, status and diagnostics.
//
// Why the window result is the conventional result.  Let m[t] be the largest
// emission of frame t over the record's alphabet (every state's label is in
// it), all m[t] <= 0 (log-probabilities), and M(t) = m[0] + ... + m[t].  Any
// path's score after frame t is at most its score at t plus m[t+1] + ... +
// m[T-1]; so a path through state s at frame t scores at most
// M(T-1) - lambda(t, s), with lambda(t, s) = M(t) - alpha(t, s) >= 0 the
// "prefix loss".  The window DP runs the reference recurrence (one fp32
// round-to-nearest add per cell, stay > step > skip by strict '>') on the
// states inside the window, with -inf for every state outside it, so its
// values never exceed the full DP's.  A state leaves the window in two ways:
// slid out below (its prefix loss at that frame is recorded), or reached above
// the top from the window's top state (that state's prefix loss is recorded:
// an exit one frame later has at least that loss, less one rounding step).
// Suppose the full DP's path P leaves the window for the first time at frame
// t; up to t the window DP made P's decisions with P's exact values (an
// alternative the window lacks is -inf, no more than its full value, and a
// full-DP loser stays a loser), so the recorded loss bounds P's prefix loss
// there.  The full DP's objective is the fp32 sequential sum of P's
// emissions: at most M(T-1) - lambda_exit plus the rounding of the remaining
// additions, each below 2^-24 of a partial sum's magnitude -- and with all
// emissions <= 0 those partial sums lie between 0 and the objective, which
// is at least the window's own (OPT).  So if every recorded loss exceeds
// L = M(T-1) - OPT by more than those rounding terms, P never left the
// window: the window DP returned the full DP's path, scores and objective bit
// for bit, ties included.  A record that is not so certified -- or holds NaN
// or +inf in an alphabet column, or a positive emission -- runs the full
// conventional DP (ffa_window_fallback in ffa_kernels.cu).
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <climits>
#include <cmath>
#include <cstdint>

#include "ffa_device.cuh"
#include "ffa_internal.h"

namespace ffa {
using namespace dev;
namespace {

static_assert(kWinStates == 64 && kWinChunk == 32, "window geometry: 32 lanes x 2 states, 32-frame segments");
static_assert(kGreedyChunk == 4 * 32, "a greedy chunk is four frames per lane");
constexpr unsigned kFull = 0xffffffffu;

// An order-preserving key of a float for an unsigned max (NaN never occurs
// in a certified record; it only steers the window's position).
__device__ __forceinline__ unsigned order_key(float v) {
  const unsigned u = __float_as_uint(v);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

__device__ __forceinline__ double warp_min(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmin(v, __shfl_xor_sync(kFull, v, o));
  return v;
}

// The reference's greedy chunk test (alignment.cu:93-153) on one chunk of
// frames [a, b), by the whole warp: lane j holds the greedy labels lab[q] of
// frames a + 4j + q (the unique finite maximum over the alphabet; every frame
// of the chunk has one).  The label sequence must match exactly one placement
// s .. s + r[b-1] among the record's states (a legal CTC walk: the state
// advances by 0 on a repeated label, by 1 into or out of a blank, by 2
// between tokens).  Returns kGreedyAccepted, kGreedyMultiple (several
// placements) or 0.  label_of(s): the label column of state s.  Tokens of a
// label L: tokens.at(j, L) for j in [tokens.begin(L), tokens.end(L)) is a
// token position u holding L, or -1.
template <typename LabelOf, typename Tokens>
__device__ int greedy_verdict(const int (&lab)[4], int a, int b, int T, int S, int blank, const Tokens& tokens,
                              LabelOf label_of, int lane) {
  // r[t] - r[a] by a warp scan of the increments.
  int inc[4], own = 0;
  unsigned chg = 0;
  int prev = __shfl_up_sync(kFull, lab[3], 1);
  if (lane == 0) prev = lab[0];
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const int t = a + 4 * lane + q;
    int d = 0;
    if (t > a && t < b && lab[q] != prev) {
      d = (lab[q] == blank || prev == blank) ? 1 : 2;
      chg |= 1u << q;
    }
    prev = lab[q];
    own += d;
    inc[q] = own;
  }
  int scan = own;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int v = __shfl_up_sync(kFull, scan, o);
    if (lane >= o) scan += v;
  }
  const int before = scan - own;               // increments of the frames before this lane's four
  const int R = __shfl_sync(kFull, scan, 31);  // r[b-1]
#pragma unroll
  for (int q = 0; q < 4; ++q) inc[q] += before;
  const int ga = __shfl_sync(kFull, lab[0], 0);
  const int hi_start = a == 0 ? 1 : S - 1;  // the first chunk starts at state 0 or 1 (alignment.cu:119)
  auto in_range = [&](int s) {
    const int term = s + R;
    return s >= 0 && s <= hi_start && term < S && !(b == T && term < S - 2);
  };
  const unsigned changers = __ballot_sync(kFull, chg != 0);
  int matches = 0;
  if (changers == 0) {
    // One label throughout: every state holding it in range is a placement.
    if (ga == blank) {
      const int lo = b == T ? max(0, S - 2) : 0, hi = min(hi_start, S - 1);
      matches = hi < lo ? 0 : (hi / 2 - (lo + 1) / 2 + 1);  // even states in [lo, hi]
    } else {
      for (int j = tokens.begin(ga) + lane; j < tokens.end(ga); j += 32) {
        const int u = tokens.at(j, ga);
        matches += u >= 0 && in_range(2 * u + 1) ? 1 : 0;
      }
      matches = __reduce_add_sync(kFull, matches);
    }
    return matches == 1 ? kGreedyAccepted : (matches > 1 ? kGreedyMultiple : 0);
  }
  // The first change (label gc at offset rc) fixes the placement once its
  // state is chosen: the start is a token state of label g[a] when g[a] is a
  // token, else the blank just below a token state of label gc.
  const int lc = __ffs(changers) - 1;
  int q0 = __ffs(chg) - 1;
  q0 = __shfl_sync(kFull, q0, lc);
  int gcv = 0, rcv = 0;
#pragma unroll
  for (int q = 0; q < 4; ++q)
    if (q == q0) { gcv = lab[q]; rcv = inc[q]; }
  const int gc = __shfl_sync(kFull, gcv, lc), rc = __shfl_sync(kFull, rcv, lc);
  const int lb = ga != blank ? ga : gc;
  const int shift = ga != blank ? 1 : 0;  // start = 2u + shift for a token u of label lb
  const int n1 = tokens.end(lb);
  for (int j0 = tokens.begin(lb); j0 < n1; j0 += 32) {
    const int j = j0 + lane;
    int s0 = 0;
    bool cand = false;
    const int u = j < n1 ? tokens.at(j, lb) : -1;
    if (u >= 0) {
      s0 = 2 * u + shift;
      cand = in_range(s0) && s0 + rc < S && label_of(s0 + rc) == gc;  // passes the first change
    }
    unsigned cands = __ballot_sync(kFull, cand);
    while (cands) {
      const int q = __ffs(cands) - 1;
      cands &= cands - 1;
      const int st0 = __shfl_sync(kFull, s0, q);
      bool ok = true;  // every label change lands on a state holding the new label
#pragma unroll
      for (int k = 0; k < 4; ++k)
        if ((chg >> k) & 1u) ok &= st0 + inc[k] < S && label_of(st0 + inc[k]) == lab[k];
      if (__all_sync(kFull, ok)) ++matches;
    }
  }
  return matches == 1 ? kGreedyAccepted : (matches > 1 ? kGreedyMultiple : 0);
}

// A record's tokens grouped by label (ffa_greedy_prep's lists).
struct LabelLists {
  const uint16_t* lpos;
  const uint16_t* lstart;
  __device__ __forceinline__ int begin(int L) const { return lstart[L]; }
  __device__ __forceinline__ int end(int L) const { return lstart[L + 1]; }
  __device__ __forceinline__ int at(int j, int) const { return lpos[j]; }
};
// A record's tokens as its label columns (cols[u]), scanned for a label.
struct LabelScan {
  const int* cols;
  int U;
  __device__ __forceinline__ int begin(int) const { return 0; }
  __device__ __forceinline__ int end(int) const { return U; }
  __device__ __forceinline__ int at(int j, int L) const { return cols[j] == L ? j : -1; }
};

// The reference accepts a chunk only if the fp32 sum of its frames' maxima,
// added in frame order, is finite (alignment.cu:135-138).  With every
// |maximum| at most kSumSafe the sum of at most kGreedyChunk of them cannot
// overflow; otherwise it is formed exactly.
constexpr float kSumSafe = 1.0e36f;

// max with NaN propagated (PTX max.NaN): a NaN anywhere in a reduction shows.
__device__ __forceinline__ float max_nan(float a, float b) {
  float r;
  asm("max.NaN.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
  return r;
}

// Greedy bound and label of one frame from its row over the alphabet
// (alo, ahi): the largest emission (NaN columns never compare greater or
// equal), whether it is unique, its column, and whether an alphabet column is
// NaN or +inf.
struct GreedyFrame {
  float best;
  int arg, ties;
  bool nonfinite;
};
// A 32-column fp32 row already in registers.
__device__ __forceinline__ GreedyFrame greedy_row32(const float4 (&v4)[8], unsigned alo) {
  GreedyFrame f{-INFINITY, 0, 0, false};
  float bn = -INFINITY;
  {
    float xs[32];
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      xs[4 * k] = v4[k].x; xs[4 * k + 1] = v4[k].y; xs[4 * k + 2] = v4[k].z; xs[4 * k + 3] = v4[k].w;
    }
    float bf[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
    float bq[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
    for (int k = 0; k < 32; ++k) {
      const float v = ((alo >> k) & 1u) ? xs[k] : -INFINITY;
      bf[k & 3] = fmaxf(bf[k & 3], v);
      bq[k & 3] = max_nan(bq[k & 3], v);
    }
    f.best = fmaxf(fmaxf(bf[0], bf[1]), fmaxf(bf[2], bf[3]));
    bn = max_nan(max_nan(bq[0], bq[1]), max_nan(bq[2], bq[3]));
    int tq[4] = {0, 0, 0, 0};
#pragma unroll
    for (int k = 0; k < 32; ++k) {
      const bool hit = ((alo >> k) & 1u) && xs[k] == f.best;
      tq[k & 3] += hit ? 1 : 0;
      f.arg = hit ? k : f.arg;
    }
    f.ties = tq[0] + tq[1] + tq[2] + tq[3];
  }
  f.nonfinite = !(bn < INFINITY);
  return f;
}

// Any row of V <= 64 columns, read column by column.  Logits are compared as
// the emissions they stand for, x - z (rounding may tie two of them), and
// `best` is then that emission.
template <int kFmt>
__device__ __forceinline__ GreedyFrame greedy_row(const typename Input<kFmt>::Elem* row, int V, unsigned alo,
                                                  unsigned ahi, float z) {
  GreedyFrame f{-INFINITY, 0, 0, false};
  float bn = -INFINITY;
  {
    for (int col = 0; col < V; ++col) {
      const bool in = col < 32 ? ((alo >> col) & 1u) : ((ahi >> (col - 32)) & 1u);
      if (!in) continue;
      float v = elem_to_float(row[col]);
      bn = max_nan(bn, v);
      if constexpr (Input<kFmt>::kLogits) v = __fsub_rn(v, z);
      if (v > f.best) { f.best = v; f.arg = col; f.ties = 1; }
      else if (v == f.best) ++f.ties;
    }
  }
  f.nonfinite = !(bn < INFINITY);
  return f;
}

// The greedy preparation: a warp per record of the launch.  The transcript
// alphabet (label columns, blank included) as a 64-bit mask, and the token
// positions grouped by label (a counting sort: lanes holding equal labels
// form a group, whose first lane updates the label's count).  The reference
// runs no greedy chunk of a record of status >= 2 (alignment.cu:35): the
// same mask and target checks as the DP kernels' (alignment.cu:836,
// 852-874) mark such a record with an empty alphabet, and its statistics stay
// zero.
__global__ void __launch_bounds__(32 * kGreedyWarps)
ffa_greedy_prep(const __grid_constant__ GreedyParams P) {
  const int warp = static_cast<int>(threadIdx.x >> 5), lane = static_cast<int>(threadIdx.x & 31);
  const int64_t index = static_cast<int64_t>(blockIdx.x) * kGreedyWarps + warp;
  if (index >= P.num_records) return;
  const int r = P.records[index];
  const RecordDev rec = P.recs[r];
  const int T = rec.T, U = rec.U, V = rec.V, blank = rec.blank;
  uint16_t* lpos = P.lpos + P.tok_off[r];
  uint16_t* lstart = P.lstart + static_cast<int64_t>(kGreedyLabels) * r;
  __shared__ uint16_t cursor_s[kGreedyWarps][kGreedyLabels];
  __shared__ uint8_t label_s[kGreedyWarps][kMaxStates / 2];  // U < kMaxStates / 2 here
  uint16_t* cursor = cursor_s[warp];
  uint8_t* labs = label_s[warp];
  for (int c = lane; c < kGreedyLabels; c += 32) cursor[c] = 0;
  // The transcript's label columns (clamped into the row), four 32-token
  // blocks of loads in flight at a time; invalid IDs (status 3).
  int bad = 0;
  for (int base = 0; base < U; base += 128) {
    int64_t token[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int k = base + 32 * q + lane;
      token[q] = k < U ? __ldg(rec.targets + k) : 0;
    }
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int k = base + 32 * q + lane;
      if (k < U) {
        bad |= (token[q] < 0 || token[q] >= V || token[q] == blank) ? 1 : 0;
        labs[k] = static_cast<uint8_t>(clamp_label(token[q], V));
      }
    }
  }
  __syncwarp();
  // Alphabet, adjacent repeats (status 4; with every ID valid the labels are
  // the IDs) and each label's token count.
  uint64_t alpha = uint64_t{1} << blank;
  int rep = 0;
  for (int base = 0; base < U; base += 32) {
    const int k = base + lane;
    const int c = k < U ? labs[k] : 0x100 + lane;
    if (k < U) {
      alpha |= uint64_t{1} << c;
      if (k > 0 && labs[k - 1] == c) ++rep;
    }
    const unsigned grp = __match_any_sync(kFull, c);
    if (k < U && lane == __ffs(grp) - 1) cursor[c] = static_cast<uint16_t>(cursor[c] + __popc(grp));
    __syncwarp();
  }
  bool rejected = P.mask != nullptr && !P.mask[r];
  if (P.check_inputs) {
    bad = __reduce_or_sync(kFull, bad);
    rep = __reduce_add_sync(kFull, rep);
    rejected |= bad != 0 || static_cast<int64_t>(U) + rep > T;
  }
  const unsigned lo = __reduce_or_sync(kFull, static_cast<unsigned>(alpha));
  const unsigned hi = __reduce_or_sync(kFull, static_cast<unsigned>(alpha >> 32));
  if (lane == 0) {
    P.alphabet[r] = rejected ? 0 : static_cast<uint64_t>(hi) << 32 | lo;
    for (int j = 0; j < 3; ++j) P.shortcut_stats[3 * r + j] = 0;
  }
  // Exclusive prefix over labels (V <= 64: two per lane).
  const int c0 = 2 * lane, c1 = c0 + 1;
  const int n0 = c0 < V ? cursor[c0] : 0, n1 = c1 < V ? cursor[c1] : 0;
  int incl = n0 + n1;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int v = __shfl_up_sync(kFull, incl, o);
    if (lane >= o) incl += v;
  }
  const int excl = incl - n0 - n1;
  __syncwarp();
  if (c0 <= V) { lstart[c0] = static_cast<uint16_t>(excl); cursor[c0] = static_cast<uint16_t>(excl); }
  if (c1 <= V) { lstart[c1] = static_cast<uint16_t>(excl + n0); cursor[c1] = static_cast<uint16_t>(excl + n0); }
  if (lane == 0) lstart[V] = static_cast<uint16_t>(U);  // (V = 64 lies past the lanes' pairs)
  __syncwarp();
  for (int base = 0; base < U; base += 32) {
    const int k = base + lane;
    const int c = k < U ? labs[k] : 0x100 + lane;
    const unsigned grp = __match_any_sync(kFull, c);
    const int at = k < U ? cursor[c] + __popc(grp & ((1u << lane) - 1u)) : 0;
    __syncwarp();
    if (k < U) {
      lpos[at] = static_cast<uint16_t>(k);
      if (lane == __ffs(grp) - 1) cursor[c] = static_cast<uint16_t>(cursor[c] + __popc(grp));
    }
    __syncwarp();
  }
}

// The greedy pass: a warp per kGreedyChunk-frame chunk of a record of the
// window route.  Lane j scans the rows of frames a + 4j .. a + 4j + 3 over the
// record's alphabet (16-byte loads of whole rows, streamed): each frame's
// greedy bound m[t] (to the bound arena) and greedy label (the unique finite
// maximum, as alignment.cu:60-91 finds it); then the chunk's verdict
// (greedy_verdict) and flags go to one byte.
template <int kFmt, int kV>
__global__ void __launch_bounds__(32 * kGreedyWarps, 4)
ffa_greedy_pass(const __grid_constant__ GreedyParams P) {
  using In = Input<kFmt>;
  using Elem = typename In::Elem;
  const int warp = static_cast<int>(threadIdx.x >> 5), lane = static_cast<int>(threadIdx.x & 31);
  const int64_t index = static_cast<int64_t>(blockIdx.x) * kGreedyWarps + warp;
  if (index >= P.count) return;
  const GreedyItem item = P.items[index];
  const int r = item.record;
  const RecordDev rec = P.recs[r];
  const int T = rec.T, U = rec.U, blank = rec.blank;
  const int V = kV > 0 ? kV : rec.V;
  const int S = 2 * U + 1;
  const uint64_t alpha = __ldg(P.alphabet + r);
  const unsigned alo = static_cast<unsigned>(alpha), ahi = static_cast<unsigned>(alpha >> 32);
  const Elem* e = reinterpret_cast<const Elem*>(rec.emissions);
  const int a = item.chunk * kGreedyChunk, b = min(T, a + kGreedyChunk);
  int lab[4];
  bool poison = false, positive = false, rejected = false, large = false;
  // z of frame t (logits).
  auto lse_of = [&](int t) { return In::kLogits ? __ldg(P.lse + rec.out_off + t) : 0.0f; };
  // Frame t's bound, flags and greedy label from its row's scan (for logits,
  // greedy_row's maximum is already x - z).
  auto take = [&](int q, const GreedyFrame& f) {
    const int t = a + 4 * lane + q;
    lab[q] = -1;
    if (t >= b) return;
    bool nonfinite = f.nonfinite;
    const float m = f.best;
    if constexpr (In::kLogits) nonfinite |= !isfinite(lse_of(t));
    P.bound[rec.out_off + t] = m;
    poison |= nonfinite;
    positive |= m > 0.0f;
    large |= !(fabsf(m) <= kSumSafe);
    const bool ok = f.ties == 1 && isfinite(m);
    rejected |= !ok;
    lab[q] = ok ? f.arg : 0xff;
  };
  if constexpr (kV == 32 && kFmt == 0) {
    // A row's eight 16-byte loads in flight at a time (streamed: read once);
    // few registers keep many warps resident, which covers the latency.
#pragma unroll 1
    for (int q = 0; q < 4; ++q) {
      float4 v4[8];
      const int t = min(a + 4 * lane + q, b - 1);
      const float4* row = reinterpret_cast<const float4*>(e + static_cast<int64_t>(t) * 32);
#pragma unroll
      for (int k = 0; k < 8; ++k) v4[k] = __ldcs(row + k);
      take(q, greedy_row32(v4, alo));
    }
  } else {
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int t = min(a + 4 * lane + q, b - 1);
      take(q, greedy_row<kFmt>(e + static_cast<int64_t>(t) * V, V, alo, ahi, lse_of(t)));
    }
  }
  poison = __any_sync(kFull, poison);
  positive = __any_sync(kFull, positive);
  int verdict = 0;
  if (!__any_sync(kFull, rejected)) {
    const int64_t* targets = rec.targets;
    auto label_of = [&](int s) { return (s & 1) ? clamp_label(__ldg(targets + (s >> 1)), V) : blank; };
    const LabelLists lists{P.lpos + P.tok_off[r], P.lstart + static_cast<int64_t>(kGreedyLabels) * r};
    verdict = greedy_verdict(lab, a, b, T, S, blank, lists, label_of, lane);
    if (verdict == kGreedyAccepted && __any_sync(kFull, large)) {
      // The chunk's sum of maxima in frame order (the lanes' bounds above).
      __syncwarp();
      float total = 0.0f;
      if (lane == 0)
        for (int t = a; t < b; ++t) total = __fadd_rn(total, P.bound[rec.out_off + t]);
      if (!__shfl_sync(kFull, isfinite(total) ? 1 : 0, 0)) verdict = 0;
    }
  }
  if (lane == 0) {
    P.verdicts[P.greedy_first[r] + item.chunk] =
        static_cast<uint8_t>(verdict | (poison ? kGreedyPoison : 0) | (positive ? kGreedyPositive : 0));
    // The reference's statistics (alignment.cu:130-146): accepted chunks and
    // their frames; chunks with several placements.
    unsigned long long* stats = reinterpret_cast<unsigned long long*>(P.shortcut_stats + 3 * r);
    if (alpha != 0 && verdict == kGreedyAccepted) {
      atomicAdd(stats, 1ull);
      atomicAdd(stats + 1, static_cast<unsigned long long>(b - a));
    } else if (alpha != 0 && verdict == kGreedyMultiple) {
      atomicAdd(stats + 2, 1ull);
    }
  }
}

// The greedy pass of the records whose alphabet a 64-bit mask cannot hold
// (more than 64 columns, or rows that are not staged): their shortcut
// statistics only (the window route never takes them).  A CTA per
// kGreedyChunk-frame chunk, kWideGreedyWarps warps.  Shared memory holds the
// record's token columns (for the placement search) and its alphabet: the
// distinct label columns in increasing order, from a bitmap of the row's
// columns (or, past kWideBitmapWords words, every label column as it comes:
// a repeated column is the same column, never a tie).  A frame's greedy
// label is found by 8 lanes, each reading every 8th alphabet column of the
// frame's row and keeping the largest emission, its column and whether a
// different column reached it too -- the reference's unique finite maximum
// over the alphabet (alignment.cu:60-91), NaN never compared greater or
// equal.  Four frames share a warp's loads, two such groups are in flight
// (16 loads per lane), and each warp takes 32 frames of the chunk.  Warp 0
// then applies the verdict (greedy_verdict, finding a label's tokens by
// scanning the token columns) and the finite-sum rule.  A record of status
// >= 2 (mask, target checks: alignment.cu:35) runs no chunk.  Its
// statistics were zeroed by the first pass, which this launch follows.
constexpr int kWideGreedyWarps = 4;
constexpr int kWideThreads = 32 * kWideGreedyWarps;
template <int kFmt>
__global__ void __launch_bounds__(kWideThreads)
ffa_greedy_wide(const __grid_constant__ GreedyParams P, int max_tokens, int bitmap_words) {
  using In = Input<kFmt>;
  using Elem = typename In::Elem;
  static_assert(kGreedyChunk == 32 * kWideGreedyWarps, "a warp takes 32 frames of a chunk");
  extern __shared__ int wide_smem[];
  int* cols = wide_smem;                  // the U token columns, then the blank
  int* alph = cols + (max_tokens + 1);    // the alphabet (increasing columns)
  unsigned* bits = reinterpret_cast<unsigned*>(alph + (max_tokens + 1));  // bitmap_words
  __shared__ int lab_s[kGreedyChunk];
  __shared__ float best_s[kGreedyChunk];
  __shared__ int ok_s[kGreedyChunk];
  __shared__ int rep_s, scan_s[kWideGreedyWarps];
  const int tid = static_cast<int>(threadIdx.x), warp = tid >> 5, lane = tid & 31;
  const GreedyItem item = P.items[blockIdx.x];
  const int r = item.record;
  const RecordDev rec = P.recs[r];
  const int T = rec.T, U = rec.U, V = rec.V, blank = rec.blank;
  const int S = 2 * U + 1;
  if (P.mask != nullptr && !P.mask[r]) return;
  const int words = (V + 31) >> 5;
  const bool dedup = words <= bitmap_words;
  if (tid == 0) rep_s = 0;
  if (dedup)
    for (int w = tid; w < words; w += kWideThreads) bits[w] = 0;
  __syncthreads();
  // Token columns, invalid IDs (status 3), adjacent repeats (status 4).
  int bad = 0, rep = 0;
  for (int j = tid; j <= U; j += kWideThreads) {
    int c = blank;
    if (j < U) {
      const int64_t token = __ldg(rec.targets + j);
      bad |= (token < 0 || token >= V || token == blank) ? 1 : 0;
      if (j > 0) rep += __ldg(rec.targets + j - 1) == token ? 1 : 0;
      c = clamp_label(token, V);
    }
    cols[j] = c;
    if (dedup) atomicOr(&bits[c >> 5], 1u << (c & 31));
  }
  rep = __reduce_add_sync(kFull, rep);
  if (lane == 0 && rep != 0) atomicAdd(&rep_s, rep);
  bad = __syncthreads_or(bad);
  if (P.check_inputs && (bad != 0 || static_cast<int64_t>(U) + rep_s > T)) return;
  // The alphabet: thread i compacts bitmap words [i per, (i + 1) per) after
  // the columns of the words before them (a block scan of their counts).
  int A = U + 1;
  const int* cols_in = cols;
  if (dedup) {
    const int per = (words + kWideThreads - 1) / kWideThreads;
    const int w0 = min(words, tid * per), w1 = min(words, w0 + per);
    int n = 0;
    for (int w = w0; w < w1; ++w) n += __popc(bits[w]);
    int incl = n;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int v = __shfl_up_sync(kFull, incl, o);
      if (lane >= o) incl += v;
    }
    if (lane == 31) scan_s[warp] = incl;
    __syncthreads();
    int at = incl - n;
    for (int k = 0; k < warp; ++k) at += scan_s[k];
    A = 0;
    for (int k = 0; k < kWideGreedyWarps; ++k) A += scan_s[k];
    for (int w = w0; w < w1; ++w)
      for (unsigned m = bits[w]; m != 0; m &= m - 1) alph[at++] = 32 * w + __ffs(m) - 1;
    __syncthreads();
    cols_in = alph;
  }

  const Elem* e = reinterpret_cast<const Elem*>(rec.emissions);
  const int a = item.chunk * kGreedyChunk, b = min(T, a + kGreedyChunk);
  const int g = lane >> 3, sub = lane & 7;
  // Two frames per lane group at a time (offsets f and f + 4 in the chunk);
  // each batch loads up to 8 alphabet columns of both rows before folding
  // them in.
#pragma unroll 1
  for (int i = 0; i < 8; i += 2) {
    const int f0 = 32 * warp + 4 * i + g;
    int fr[2];
    const Elem* row[2];
    float z[2], best[2];
    int arg[2];
    bool tie[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      fr[h] = f0 + 4 * h;
      const int t = min(a + fr[h], b - 1);
      row[h] = e + static_cast<int64_t>(t) * V;
      z[h] = In::kLogits ? __ldg(P.lse + rec.out_off + t) : 0.0f;
      best[h] = -INFINITY;
      arg[h] = INT_MAX;
      tie[h] = false;
    }
    for (int j0 = sub; j0 < A; j0 += 64) {
      int c[8];
      float v[2][8];
#pragma unroll
      for (int k = 0; k < 8; ++k) c[k] = j0 + 8 * k < A ? cols_in[j0 + 8 * k] : -1;
#pragma unroll
      for (int h = 0; h < 2; ++h)
#pragma unroll
        for (int k = 0; k < 8; ++k) v[h][k] = c[k] >= 0 ? elem_to_float(__ldg(row[h] + c[k])) : -INFINITY;
#pragma unroll
      for (int h = 0; h < 2; ++h)
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          float x = v[h][k];
          if constexpr (In::kLogits) x = __fsub_rn(x, z[h]);
          const bool gt = c[k] >= 0 && x > best[h];
          const bool eq = c[k] >= 0 && x == best[h] && c[k] != arg[h];
          tie[h] = gt ? false : (tie[h] || eq);
          arg[h] = gt ? c[k] : arg[h];
          best[h] = gt ? x : best[h];
        }
    }
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      // The 8 lanes of the frame combine (a -inf maximum is rejected anyway).
#pragma unroll
      for (int o = 4; o > 0; o >>= 1) {
        const float ob = __shfl_xor_sync(kFull, best[h], o);
        const int oa = __shfl_xor_sync(kFull, arg[h], o);
        const bool ot = __shfl_xor_sync(kFull, tie[h] ? 1 : 0, o) != 0;
        const bool gt = ob > best[h], eq = ob == best[h];
        tie[h] = gt ? ot : (eq ? (tie[h] || ot || oa != arg[h]) : tie[h]);
        arg[h] = gt ? oa : (eq ? min(arg[h], oa) : arg[h]);
        best[h] = gt ? ob : best[h];
      }
      if (sub == 0 && a + fr[h] < b) {
        lab_s[fr[h]] = arg[h];
        best_s[fr[h]] = best[h];
        ok_s[fr[h]] = !tie[h] && isfinite(best[h]) ? 1 : 0;
      }
    }
  }
  __syncthreads();
  if (warp != 0) return;
  int lab[4];
  bool ok = true;
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const int f = 4 * lane + q;
    lab[q] = a + f < b ? lab_s[f] : -1;
    ok &= a + f >= b || ok_s[f] != 0;
  }
  if (!__all_sync(kFull, ok)) return;
  auto label_of = [&](int s) { return (s & 1) ? cols[s >> 1] : blank; };
  int verdict = greedy_verdict(lab, a, b, T, S, blank, LabelScan{cols, U}, label_of, lane);
  if (verdict == kGreedyAccepted) {
    // The fp32 sum of the chunk's maxima in frame order must be finite
    // (alignment.cu:135-138).
    float total = 0.0f;
    if (lane == 0)
      for (int f = 0; f < b - a; ++f) total = __fadd_rn(total, best_s[f]);
    if (!__shfl_sync(kFull, isfinite(total) ? 1 : 0, 0)) verdict = 0;
  }
  if (lane == 0) {
    unsigned long long* stats = reinterpret_cast<unsigned long long*>(P.shortcut_stats + 3 * r);
    if (verdict == kGreedyAccepted) {
      atomicAdd(stats, 1ull);
      atomicAdd(stats + 1, static_cast<unsigned long long>(b - a));
    } else if (verdict == kGreedyMultiple) {
      atomicAdd(stats + 2, 1ull);
    }
  }
}

// A lane's K states: base + K lane + k (even k: blanks, odd k: tokens), their
// scores and their ancestors (each state's path state at the frame before
// the current traceback segment).
template <int K>
struct WinLane {
  float a[K];
  int anc[K];
};

// One frame of the recurrence (alignment.cu:414-429) for a lane's K states:
// stay, then step if strictly greater, then skip if strictly greater and
// legal; one fp32 round-to-nearest add per cell.  seg: the frame starts a
// traceback segment (ancestors restart from the predecessors).  s0: the
// lane's first state.  Returns the frame's 2K code bits (state k at bits 2k).
template <int K>
__device__ __forceinline__ uint32_t win_step(WinLane<K>& x, float eb, const float (&et)[K / 2],
                                             const bool (&sk)[K / 2], bool first_lane, int s0, bool seg) {
  float p1 = __shfl_up_sync(kFull, x.a[K - 1], 1);  // state s0 - 1, the lane below's last
  int pa = __shfl_up_sync(kFull, x.anc[K - 1], 1);
  if (seg) {
#pragma unroll
    for (int k = 0; k < K; ++k) x.anc[k] = s0 + k;
    pa = s0 - 1;
  }
  p1 = first_lane ? -INFINITY : p1;  // below the window: -inf
  float na[K];
  int nn[K];
  uint32_t bits = 0;
#pragma unroll
  for (int k = 0; k < K; ++k) {
    const float x1 = k >= 1 ? x.a[k - 1] : p1;
    const int n1 = k >= 1 ? x.anc[k - 1] : pa;
    const bool c = x1 > x.a[k];
    float b = c ? x1 : x.a[k];
    int n = c ? n1 : x.anc[k];
    uint32_t code = c ? 1u : 0u;
    if (k & 1) {
      const float x2 = k >= 2 ? x.a[k - 2] : p1;
      const int n2 = k >= 2 ? x.anc[k - 2] : pa;
      const bool j2 = sk[k >> 1] && x2 > b;
      b = j2 ? x2 : b;
      n = j2 ? n2 : n;
      code = j2 ? 2u : code;
      na[k] = __fadd_rn(b, et[k >> 1]);
    } else {
      na[k] = __fadd_rn(b, eb);
    }
    nn[k] = n;
    bits |= code << (2 * k);
  }
#pragma unroll
  for (int k = 0; k < K; ++k) { x.a[k] = na[k]; x.anc[k] = nn[k]; }
  return bits;
}

// a[idx] of a register array without a dynamic register index.
template <int K>
__device__ __forceinline__ float pick(const float (&a)[K], int idx) {
  float v = a[0];
#pragma unroll
  for (int k = 1; k < K; ++k) v = idx == k ? a[k] : v;
  return v;
}

// The window DP of one record by one warp, K states per lane (window of 32 K
// states, sliding by 8 lanes).  sm: the record's slice of dynamic shared
// memory (win_layout); full: its kWinRing mbarriers.  wide: the 128-state
// second tier, for a record the 64-state window did not certify (its
// diagnostics and shortcut statistics are already written).  Returns false
// when a bounded wait gave up (status 5 written).
template <int kFmt, int kV, int K>
__device__ __forceinline__ bool window_record(const WindowParams& P, int r, unsigned char* sm,
                                              unsigned long long* full, int lane) {
  using In = Input<kFmt>;
  using Elem = typename In::Elem;
  constexpr bool kWide = K == 4;
  constexpr int W = 32 * K;           // window states
  constexpr int kWords = K / 2;       // code words per lane per 8-frame group
  constexpr int kFramesPerWord = 8 / kWords;
  constexpr int kShift = 8;           // a slide moves the window by 8 lanes
  constexpr int kSlide = kShift * K;  // = 8 K states
  constexpr int kHighLane = 16;       // slide when the best state lies in lane 16 or above
  const RecordDev rec = P.recs[r];
  const int T = rec.T, U = rec.U, blank = rec.blank;
  const int V = kV > 0 ? kV : rec.V;
  const int S = 2 * U + 1;
  const bool smem_codes = P.smem_codes != 0;
  const WinLayout L = win_layout(T, U, V, static_cast<int>(sizeof(Elem)), K, smem_codes);
  Elem* ring = reinterpret_cast<Elem*>(sm + L.ring);
  uint8_t* tok = sm + L.tok;
  // Backpointer codes of the window, written once per 8-frame group (a word
  // per lane), read back by the traceback: in the slice, or in global memory
  // (coalesced 128-byte stores).
  uint32_t* bp = smem_codes ? reinterpret_cast<uint32_t*>(sm + L.bp) : P.codes + win_codes_offset(rec.out_off, r);
  uint16_t* gb = reinterpret_cast<uint16_t*>(sm + L.gb);
  uint16_t* map = reinterpret_cast<uint16_t*>(sm + L.map);
  int16_t* anc = reinterpret_cast<int16_t*>(sm + L.anc);
  float* stash = reinterpret_cast<float*>(sm + L.stash);
  uint16_t* path = reinterpret_cast<uint16_t*>(sm + L.path);
  int64_t* labels = P.out.labels + rec.out_off;
  float* scores = P.out.scores + rec.out_off;
  const float kNegInf = -INFINITY;

  // ---- status: mask, then target validation (alignment.cu:836, 852-874);
  //      the transcript's label columns into shared memory ----
  int status = (P.mask != nullptr && !P.mask[r]) ? 2 : 0;
  int bad = 0, rep = 0;
  int64_t carry = 0;  // the token before this 32-token block
#pragma unroll 4
  for (int base = 0; base < U; base += 32) {
    const int k = base + lane;
    const int64_t token = k < U ? rec.targets[k] : 0;
    int64_t prev = __shfl_up_sync(kFull, token, 1);
    if (lane == 0) prev = carry;
    carry = __shfl_sync(kFull, token, 31);
    if (k < U) {
      bad |= (token < 0 || token >= V || token == blank) ? 1 : 0;
      if (k > 0) rep += token == prev ? 1 : 0;
      tok[k] = static_cast<uint8_t>(clamp_label(token, V));
    }
  }
  if (P.check_inputs) {
    bad = __reduce_or_sync(kFull, bad);
    rep = __reduce_add_sync(kFull, rep);
    if (bad) status = 3;
    else if (static_cast<int64_t>(U) + rep > T) status = 4;
  }
  if (!kWide && lane == 0) {
    // Diagnostics start at zero (alignment.py:101-129).
    P.out.stitched[r] = 0;
    P.out.repair_passes[r] = 0;
    P.out.repaired_frames[r] = 0;
    // (The greedy pass owns the shortcut statistics.)
    for (int j = 0; j < 3; ++j) P.out.routing_stats[3 * r + j] = 0;
    if (P.out.reuse_stats) for (int j = 0; j < 4; ++j) P.out.reuse_stats[4 * r + j] = 0;
  }
  if (status >= 2) {
    if (lane == 0) { P.out.status[r] = status; P.out.objective[r] = -INFINITY; }
    for (int t = lane; t < T; t += 32) { labels[t] = -1; scores[t] = -INFINITY; }
    return true;
  }
  __syncwarp();

  // ---- emission rows: kWinChunk-row TMA copies into a kWinRing ring ----
  const Elem* e = reinterpret_cast<const Elem*>(rec.emissions);
  const int nchunks = (T + kWinChunk - 1) / kWinChunk;
  auto issue = [&](int c) {  // by lane 0
    const int rows = min(kWinChunk, T - c * kWinChunk);
    const unsigned bytes = static_cast<unsigned>(rows) * V * static_cast<unsigned>(sizeof(Elem));
    unsigned long long* bar = &full[c % kWinRing];
    mbar_expect_tx(bar, bytes);
    tma_bulk_load(ring + (c % kWinRing) * kWinChunk * V, e + static_cast<int64_t>(c) * kWinChunk * V, bytes, bar);
  };
  if (lane == 0) {
    for (int k = 0; k < kWinRing; ++k) mbar_init(&full[k], 1);
    fence_mbar_init();
    fence_proxy_async();  // shared memory a previous record read is rewritten by the copies
    for (int c = 0; c < kWinRing && c < nchunks; ++c) issue(c);
  }
  LseStream lse{};
  if constexpr (In::kLogits) lse.start(P.lse + rec.out_off, T, 0, lane);

  // ---- the window: lane l owns states base + K l + k ----
  int base = 0;
  WinLane<K> x;
#pragma unroll
  for (int k = 0; k < K; ++k) { x.a[k] = kNegInf; x.anc[k] = 0; }
  auto label_of = [&](int s) { return (s & 1) ? static_cast<int>(tok[s >> 1]) : blank; };
  // Label column and skip legality of token state s1 (skip s1-2 -> s1: a
  // token unlike the blank and its predecessor, alignment.cu:407).
  auto token_info = [&](int s1, int& col, bool& sk) {
    const bool valid = s1 < S;
    const int u = s1 >> 1;
    col = valid ? static_cast<int>(tok[u]) : blank;
    sk = valid && u >= 1 && tok[u] != blank && tok[u] != tok[u - 1];
  };
  int col[K / 2];
  bool sk[K / 2];
#pragma unroll
  for (int q = 0; q < K / 2; ++q) token_info(K * lane + 2 * q + 1, col[q], sk[q]);
  const bool first_lane = lane == 0, top_lane = lane == 31;

  double Mbase = 0.0;     // sum of the greedy bounds m of the frames before this chunk
  double esc = INFINITY;  // smallest recorded prefix loss of a state that left the window (this lane's)
  bool fault = false;
  // A state s at frame t can still reach a terminal state (S-2 or S-1).
  auto reaches_end = [&](int s, int t) { return s + 2 * (T - 1 - t) >= S - 2; };
  // Whether the window's best state that can still reach the end lies in
  // lane kHighLane or above, judged at frame t (a heuristic: any choice is
  // safe): the best key among all lanes and among the lanes below, reduced
  // mid-group and compared after it.
  auto slide_keys = [&](int t, unsigned& kall, unsigned& klow) {
    const int s0 = base + K * lane;
    unsigned key = 0;
#pragma unroll
    for (int k = 0; k < K; ++k)
      if (s0 + k < S && reaches_end(s0 + k, t)) key = max(key, order_key(x.a[k]));
    kall = __reduce_max_sync(kFull, key);
    klow = __reduce_max_sync(kFull, lane < kHighLane ? key : 0u);
  };

  for (int c = 0; c < nchunks; ++c) {
    const int t0 = c * kWinChunk;
    const int rows = min(kWinChunk, T - t0);
    if (!fault && !mbar_wait(&full[c % kWinRing], (c / kWinRing) & 1)) fault = true;
    fault = __any_sync(kFull, fault);
    if (fault) break;
    const Elem* chunk = ring + (c % kWinRing) * kWinChunk * V;
    if constexpr (In::kLogits)
      if (c > 0) lse.advance(t0, lane);
    // The greedy bound of frame t0 + lane (the greedy pass wrote it).
    const float m = lane < rows ? __ldg(P.bound + rec.out_off + t0 + lane) : 0.0f;
    // M of each frame of the chunk: lane f holds m[t0] + ... + m[t0 + f] (fp64).
    double Mpre = static_cast<double>(m);
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const double v = __shfl_up_sync(kFull, Mpre, o);
      if (lane >= o) Mpre += v;
    }
    for (int g = 0; g < kWinChunk / 8 && 8 * g < rows; ++g) {
      const int tg = t0 + 8 * g;
      if (lane == 0) gb[tg >> 3] = static_cast<uint16_t>(base);
      // While states lie above the window, the top state's score is kept at
      // every frame (an exit above the window at the next frame scores at
      // most that plus the next frame's bound); otherwise -inf.
      const bool open = base + W < S;
      const bool keep_top = top_lane && open;
      if (top_lane && !open)
        for (int j = 0; j < 8; ++j) stash[8 * g + j] = kNegInf;
      const int s0 = base + K * lane;
      const bool seg0 = g == 0;  // the chunk's first frame starts a traceback segment
      const Elem* grow = chunk + 8 * g * V;
      uint32_t w[kWords];
#pragma unroll
      for (int q = 0; q < kWords; ++q) w[q] = 0;
      unsigned kall = 0, klow = 0;
      auto emissions_of = [&](int j, float& eb, float (&et)[K / 2]) {
        const Elem* row = grow + j * V;
        eb = elem_to_float(row[blank]);
#pragma unroll
        for (int q = 0; q < K / 2; ++q) et[q] = elem_to_float(row[col[q]]);
        if constexpr (In::kLogits) {
          const float z = lse.at(8 * g + j);
          eb = __fsub_rn(eb, z);
#pragma unroll
          for (int q = 0; q < K / 2; ++q) et[q] = __fsub_rn(et[q], z);
        }
      };
      if (tg > 0 && tg + 8 <= T) {
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          float eb, et[K / 2];
          emissions_of(j, eb, et);
          const uint32_t bits = win_step<K>(x, eb, et, sk, first_lane, s0, seg0 && j == 0);
          w[j / kFramesPerWord] |= bits << (2 * K * (j % kFramesPerWord));
          if (keep_top) stash[8 * g + j] = x.a[K - 1];
          // Reduce the slide keys mid-group, so that the reductions overlap
          // the group's last frames; the slide is applied after them.
          if (j == 3 && open) slide_keys(tg + 3, kall, klow);
        }
      } else {
        for (int j = 0; j < 8 && tg + j < T; ++j) {
          float eb, et[K / 2];
          emissions_of(j, eb, et);
          if (tg + j == 0) {
            // Frame 0: alpha[s] = e[0, l[s]] for s < 2 (alignment.cu:409).
#pragma unroll
            for (int k = 0; k < K; ++k) { x.a[k] = kNegInf; x.anc[k] = s0 + k; }
            if (first_lane) {
              x.a[0] = eb;
              if (S > 1) x.a[1] = et[0];
            }
          } else {
            const uint32_t bits = win_step<K>(x, eb, et, sk, first_lane, s0, seg0 && j == 0);
            w[j / kFramesPerWord] |= bits << (2 * K * (j % kFramesPerWord));
          }
          if (keep_top) stash[8 * g + j] = x.a[K - 1];
        }
      }
#pragma unroll
      for (int q = 0; q < kWords; ++q) {
        uint32_t* dst = bp + ((tg >> 3) * kWords + q) * 32 + lane;
        if (smem_codes) *dst = w[q];
        else __stcg(dst, w[q]);
      }
      const int tl = min(tg + 8, T) - 1;
      if ((tl & (kWinChunk - 1)) == kWinChunk - 1 || tl == T - 1) {
        // Segment map: each window state's path state at the frame before
        // the segment.
        uint16_t* mp = map + (tl / kWinChunk) * W + K * lane;
#pragma unroll
        for (int k = 0; k < K; ++k) mp[k] = static_cast<uint16_t>(x.anc[k]);
      }
      if (kall > order_key(kNegInf) && klow < kall) {
        // Drop the bottom kSlide states (recording their prefix losses at
        // frame tl) and take kSlide new ones at the top (-inf).
        const double Mtl = Mbase + __shfl_sync(kFull, Mpre, tl - t0);
        if (lane < kShift) {
#pragma unroll
          for (int k = 0; k < K; ++k)
            if (reaches_end(s0 + k, tl)) esc = fmin(esc, Mtl - static_cast<double>(x.a[k]));
        }
        const bool top = lane >= 32 - kShift;
#pragma unroll
        for (int k = 0; k < K; ++k) {
          x.a[k] = __shfl_down_sync(kFull, x.a[k], kShift);
          x.anc[k] = __shfl_down_sync(kFull, x.anc[k], kShift);
          if (top) x.a[k] = kNegInf;
        }
        // Every lane reads its new states' label columns from shared memory.
        base += kSlide;
#pragma unroll
        for (int q = 0; q < K / 2; ++q) token_info(base + K * lane + 2 * q + 1, col[q], sk[q]);
      }
    }
    __syncwarp();  // the top state's scores are in the stash; every lane has read the ring entry
    if (lane < rows) esc = fmin(esc, (Mbase + Mpre) - static_cast<double>(stash[lane]));
    Mbase += __shfl_sync(kFull, Mpre, 31);
    __syncwarp();
    if (lane == 0 && c + kWinRing < nchunks) {
      fence_proxy_async();
      issue(c + kWinRing);
    }
  }
  if (fault) {
    // A bounded wait gave up: status 5; give the copies still in flight a
    // short, bounded chance to land before the shared memory goes away.
    if (lane == 0) {
      for (int c = max(0, nchunks - kWinRing); c < nchunks; ++c)
        mbar_wait(&full[c % kWinRing], (c / kWinRing) & 1, kDrainNs);
      P.out.status[r] = kStatusDeviceFault;
      P.out.objective[r] = -INFINITY;
    }
    for (int t = lane; t < T; t += 32) { labels[t] = -1; scores[t] = -INFINITY; }
    return false;
  }
  if (lane == 0)
    for (int k = 0; k < kWinRing; ++k) mbar_inval(&full[k]);  // every copy has landed and been read

  // ---- terminal rule (alignment.cu:496-510) and the certificate ----
  const double M = Mbase;
  const bool covers = base + W >= S;  // S-1 and S-2 inside the window
  const int r_last = min(max(S - 1 - base, 0), W - 1), r_prev = min(max(S - 2 - base, 0), W - 1);
  const float vlast = __shfl_sync(kFull, pick<K>(x.a, r_last % K), r_last / K);
  const float vprev = S > 1 ? __shfl_sync(kFull, pick<K>(x.a, r_prev % K), r_prev / K) : kNegInf;
  const bool take_prev = S > 1 && vprev >= vlast;
  const float opt = take_prev ? vprev : vlast;
  const int term = take_prev ? S - 2 : S - 1;
  // The greedy pass's verdicts: NaN / +inf in an alphabet column, positive
  // bounds.
  const int nitems = (T + kGreedyChunk - 1) / kGreedyChunk;
  const uint8_t* verdicts = P.verdicts + P.greedy_first[r];
  bool poison = false, positive = false;
  for (int k = lane; k < nitems; k += 32) {
    const int v = verdicts[k];
    poison |= (v & kGreedyPoison) != 0;
    positive |= (v & kGreedyPositive) != 0;
  }
  poison = __any_sync(kFull, poison);
  positive = __any_sync(kFull, positive);
  const double exit_loss = warp_min(esc);
  const double loss = M - static_cast<double>(opt);
  // Rounding: T additions along the full DP's path, each within 2^-24 of
  // |OPT|; one more for an exit above the window bounded through the top
  // state; the fp64 sums of m.
  const double aopt = fabs(static_cast<double>(opt)), am = fabs(M);
  const double margin =
      static_cast<double>(T) * (ldexp(aopt, -23) + ldexp(am, -50)) + ldexp(aopt + am, -21) + 1e-9;
  const bool certified =
      covers && !poison && !positive && isfinite(opt) && isfinite(M) && exit_loss > loss + margin;
  if (!certified) {
    // The next tier takes the record: the 128-state window, then the full
    // conventional DP (the reference's routing state 2: its completed early
    // fallback).
    if (lane == 0) {
      if (kWide || poison || positive) P.out.routing_stats[3 * r] = 2;
      P.fallback_list[atomicAdd(P.fallback_count, 1)] = r;
    }
    return true;
  }

  // ---- traceback in shared memory ----
  const int nseg = nchunks;
  if (lane == 0) {
    // Anchors: the path's state at each segment's last frame, from the maps.
    int s = term;
    for (int g = nseg - 1; g >= 0; --g) {
      anc[g] = static_cast<int16_t>(s);
      if (g > 0) {
        const int tl = min(T, (g + 1) * kWinChunk) - 1;
        const int k = min(max(s - static_cast<int>(gb[tl >> 3]), 0), W - 1);
        s = map[g * W + k];
      }
    }
  }
  __syncwarp();
  // Segment g walks back from its anchor (path[t-1] = path[t] - jump(t,
  // path[t]), alignment.cu:656-659).  Codes in global memory are first
  // brought into the emission ring, free now, a batch of segments at a time
  // (independent 16-byte loads), so that each step of the walks is a
  // shared-memory read; with a ring too small for one segment's codes (a
  // vocabulary of a few columns) the walks read global memory.
  constexpr int kSegWords = (kWinChunk / 8) * kWords * 32;  // one segment's codes
  const int total_words = ((T + 7) >> 3) * kWords * 32;
  const int ring_words = kWinRing * kWinChunk * V * static_cast<int>(sizeof(Elem)) / 4;
  const int per_batch = min(32, ring_words / kSegWords);
  uint32_t* stage = reinterpret_cast<uint32_t*>(ring);
  auto walk = [&](int g, const uint32_t* codes, int first_word, bool global) {
    const int t_lo = g * kWinChunk;
    const int t_hi = min(T, t_lo + kWinChunk) - 1;
    int s = anc[g];
    path[t_hi] = static_cast<uint16_t>(s);
    for (int t = t_hi; t > t_lo; --t) {
      const int k = min(max(s - static_cast<int>(gb[t >> 3]), 0), W - 1);
      const int j = t & 7;
      const int at = ((t >> 3) * kWords + j / kFramesPerWord) * 32 + k / K - first_word;
      const uint32_t word = global ? __ldcg(codes + at) : codes[at];
      s -= static_cast<int>((word >> (2 * K * (j % kFramesPerWord) + 2 * (k % K))) & 3u);
      path[t - 1] = static_cast<uint16_t>(s);
    }
  };
  if (smem_codes) {
    for (int g = lane; g < nseg; g += 32) walk(g, bp, 0, false);
  } else if (per_batch >= 1) {
    for (int g0 = 0; g0 < nseg; g0 += per_batch) {
      const int w0 = g0 * kSegWords;
      const int w1 = min(total_words, (g0 + per_batch) * kSegWords);
      for (int i = 4 * lane; i < w1 - w0; i += 128)
        *reinterpret_cast<uint4*>(stage + i) = __ldcg(reinterpret_cast<const uint4*>(bp + w0 + i));
      __syncwarp();
      if (lane < per_batch && g0 + lane < nseg) walk(g0 + lane, stage, w0, false);
      __syncwarp();
    }
  } else {
    for (int g = lane; g < nseg; g += 32) walk(g, bp, 0, true);
  }
  __syncwarp();
  // Labels and the selected scores (alignment.cu:662-666), frame-coalesced.
#pragma unroll 4
  for (int t = lane; t < T; t += 32) {
    const int label = label_of(min(static_cast<int>(path[t]), S - 1));
    const int64_t i = static_cast<int64_t>(t) * V + label;
    float score = elem_to_float(e[i]);
    if constexpr (In::kLogits) score = __fsub_rn(score, P.lse[rec.out_off + t]);
    labels[t] = label;
    scores[t] = score;
  }
  if (lane == 0) {
    P.out.objective[r] = opt;
    P.out.status[r] = 0;
    if (kWide) P.out.routing_stats[3 * r] = 0;
  }
  return true;
}

// The 64-state window: one warp per record of the call's window route, the
// CTA's records listed by the host.
template <int kFmt, int kV>
__global__ void __launch_bounds__(32 * kWinWarps, 2)
ffa_window_viterbi(const __grid_constant__ WindowParams P) {
  extern __shared__ __align__(128) unsigned char smem_raw[];
  __shared__ unsigned long long bars[kWinWarps][kWinRing];
  const int warp = static_cast<int>(threadIdx.x >> 5), lane = static_cast<int>(threadIdx.x & 31);
  const WinCta cta = P.ctas[blockIdx.x];
  if (warp >= cta.count) return;
  const WinSlot slot = P.slots[cta.first + warp];
  window_record<kFmt, kV, 2>(P, slot.record, smem_raw + slot.smem_off, bars[warp], lane);
}

// The 128-state window for the records the 64-state window did not certify:
// one warp per CTA, striding over the device-written list (records longer
// than kWinWideMaxFrames go straight to the full DP's list).
template <int kFmt, int kV>
__global__ void __launch_bounds__(32, 1)
ffa_window_wide(const __grid_constant__ WindowParams P) {
  extern __shared__ __align__(128) unsigned char smem_raw[];
  __shared__ unsigned long long bars[kWinRing];
  const int lane = static_cast<int>(threadIdx.x);
  const int n = *P.in_count;
  for (int i = static_cast<int>(blockIdx.x); i < n; i += static_cast<int>(gridDim.x)) {
    const int r = P.in_list[i];
    if (P.recs[r].T > kWinWideMaxFrames) {
      if (lane == 0) {
        P.out.routing_stats[3 * r] = 2;
        P.fallback_list[atomicAdd(P.fallback_count, 1)] = r;
      }
      continue;
    }
    if (!window_record<kFmt, kV, 4>(P, r, smem_raw, bars, lane)) break;  // copies may be in flight
  }
}

constexpr int kWindowVariantsDecl = 4;
int window_variant(int row_vocab, int fmt) { return fmt == 0 ? (row_vocab == 32 ? 0 : 1) : 1 + fmt; }
using GreedyKernel = void (*)(GreedyParams);
const GreedyKernel kGreedyKernels[kWindowVariantsDecl] = {
    ffa_greedy_pass<0, 32>, ffa_greedy_pass<0, 0>, ffa_greedy_pass<1, 0>, ffa_greedy_pass<2, 0>};
using WideGreedyKernel = void (*)(GreedyParams, int, int);
const WideGreedyKernel kWideGreedyKernels[3] = {ffa_greedy_wide<0>, ffa_greedy_wide<1>, ffa_greedy_wide<2>};
// Alphabet bitmaps of rows up to 65,536 columns (8 KiB of shared memory).
constexpr int kWideBitmapWords = 2048;
using WindowKernel = void (*)(WindowParams);
const WindowKernel kWindowKernels[kWindowVariantsDecl] = {
    ffa_window_viterbi<0, 32>, ffa_window_viterbi<0, 0>, ffa_window_viterbi<1, 0>, ffa_window_viterbi<2, 0>};
const WindowKernel kWideKernels[kWindowVariantsDecl] = {
    ffa_window_wide<0, 32>, ffa_window_wide<0, 0>, ffa_window_wide<1, 0>, ffa_window_wide<2, 0>};

// Opt a window kernel in to the dynamic shared memory budget (once per
// device); the CTA's static shared memory (its mbarriers) stays under 1 KiB.
constexpr size_t kWinStatic = 1024;
static_assert(sizeof(unsigned long long) * kWinWarps * kWinRing <= kWinStatic, "window static shared memory");
cudaError_t window_opt_in(WindowKernel kernel, std::atomic<uint64_t>& opted) {
  int device = 0;
  cudaError_t err = cudaGetDevice(&device);
  if (err != cudaSuccess) return err;
  const uint64_t bit = device < 64 ? uint64_t{1} << device : 0;
  if (bit != 0 && (opted.load(std::memory_order_acquire) & bit)) return cudaSuccess;
  err = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(kSmemBudget - kWinStatic));
  if (err != cudaSuccess) return err;
  if (bit) opted.fetch_or(bit, std::memory_order_acq_rel);
  return cudaSuccess;
}

}  // namespace

cudaError_t launch_greedy(const GreedyParams& params, int row_vocab, int fmt, cudaStream_t stream,
                          cudaEvent_t between) {
  if (params.count <= 0 || params.num_records <= 0) return cudaSuccess;
  if (fmt < 0 || fmt > 2) return cudaErrorInvalidValue;
  count_launch();
  ffa_greedy_prep<<<static_cast<unsigned>((params.num_records + kGreedyWarps - 1) / kGreedyWarps),
                    32 * kGreedyWarps, 0, stream>>>(params);
  cudaError_t err = cudaGetLastError();
  if (err != cudaSuccess) return err;
  if (between != nullptr && (err = cudaEventRecord(between, stream)) != cudaSuccess) return err;
  count_launch();
  kGreedyKernels[window_variant(row_vocab, fmt)]<<<static_cast<unsigned>((params.count + kGreedyWarps - 1) /
                                                                         kGreedyWarps),
                                                   32 * kGreedyWarps, 0, stream>>>(params);
  return cudaGetLastError();
}

cudaError_t launch_greedy_wide(const GreedyParams& params, int max_tokens, int max_vocab, int fmt,
                               cudaStream_t stream) {
  if (params.count <= 0) return cudaSuccess;
  if (fmt < 0 || fmt > 2 || max_tokens < 0 || 2 * max_tokens + 1 > kMaxStates || max_vocab < 1)
    return cudaErrorInvalidValue;
  const int words = std::min((max_vocab + 31) / 32, kWideBitmapWords);
  const size_t smem = sizeof(int) * 2 * (static_cast<size_t>(max_tokens) + 1) + sizeof(unsigned) * words;
  count_launch();
  kWideGreedyKernels[fmt]<<<static_cast<unsigned>(params.count), kWideThreads, smem, stream>>>(params, max_tokens,
                                                                                                words);
  return cudaGetLastError();
}

cudaError_t launch_window(const WindowParams& params, int num_ctas, int row_vocab, int fmt, unsigned smem_bytes,
                          cudaStream_t stream) {
  if (num_ctas <= 0) return cudaSuccess;
  if (fmt < 0 || fmt > 2) return cudaErrorInvalidValue;
  static std::atomic<uint64_t> opted[kWindowVariantsDecl];
  const int variant = window_variant(row_vocab, fmt);
  cudaError_t err = window_opt_in(kWindowKernels[variant], opted[variant]);
  if (err != cudaSuccess) return err;
  if (smem_bytes > kSmemBudget - kWinStatic) return cudaErrorInvalidValue;
  count_launch();
  kWindowKernels[variant]<<<num_ctas, 32 * kWinWarps, smem_bytes, stream>>>(params);
  return cudaGetLastError();
}

cudaError_t launch_window_wide(const WindowParams& params, int max_count, int row_vocab, int fmt,
                               unsigned smem_bytes, cudaStream_t stream) {
  if (max_count <= 0) return cudaSuccess;
  if (fmt < 0 || fmt > 2) return cudaErrorInvalidValue;
  static std::atomic<uint64_t> opted[kWindowVariantsDecl];
  const int variant = window_variant(row_vocab, fmt);
  cudaError_t err = window_opt_in(kWideKernels[variant], opted[variant]);
  if (err != cudaSuccess) return err;
  if (smem_bytes > kSmemBudget - kWinStatic) return cudaErrorInvalidValue;
  int device = 0, sms = 0;
  if ((err = cudaGetDevice(&device)) != cudaSuccess) return err;
  if ((err = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device)) != cudaSuccess) return err;
  count_launch();
  kWideKernels[variant]<<<std::min(max_count, std::max(sms, 1)), 32, smem_bytes, stream>>>(params);
  return cudaGetLastError();
}

}  // namespace ffa
