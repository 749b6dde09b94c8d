// ffa_device.cuh -- device helpers shared by the forward kernels: barriers,
// TMA bulk copies and mbarriers, the DP frame step and the backpointer layout.
#pragma once

#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>

#include "ffa_internal.h"

namespace ffa {
namespace dev {


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

// An emission that turns an unreachable state (-inf) into NaN: -inf + NaN and
// -inf + inf are both NaN.
__device__ __forceinline__ bool poisons(float e) { return e != e || e == INFINITY; }

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
  int chk_bad[kMaxWarps];      // target validation, per warp
  int chk_rep[kMaxWarps];
  // Per piece of a run and per warp: best end score on the band, its state,
  // and whether the warp saw NaN at or above the band.
  float red_val[kMaxRunPieces][kMaxWarps];
  int red_idx[kMaxRunPieces][kMaxWarps];
  int red_nan[kMaxRunPieces][kMaxWarps];
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

// The same frame step without ancestor deltas, for runs whose path is found
// by tracing the backpointers (pieces of the optimized route).
template <int K>
__device__ __forceinline__ unsigned dp_frame_plain(float (&a)[K], float p1, float eb,
                                                   const float (&et)[K / 2], unsigned skip) {
  float na[K];
  unsigned bits = 0;
#pragma unroll
  for (int k = 0; k < K; ++k) {
    const float x1 = k >= 1 ? a[k - 1] : p1;
    const bool c = x1 > a[k];
    float b = c ? x1 : a[k];
    if (k & 1) {
      const float x2 = k >= 2 ? a[k - 2] : p1;
      const bool j2 = ((skip >> (k >> 1)) & 1u) && x2 > b;
      b = j2 ? x2 : b;
      bits |= (static_cast<unsigned>(c || j2) << k) | (static_cast<unsigned>(j2) << (K + (k >> 1)));
      na[k] = __fadd_rn(b, et[k >> 1]);
    } else {
      bits |= static_cast<unsigned>(c) << k;
      na[k] = __fadd_rn(b, eb);
    }
  }
#pragma unroll
  for (int k = 0; k < K; ++k) a[k] = na[k];
  return bits;
}

// Backpointer word geometry: 1.5*K bits per frame and thread, packed in
// 16-bit lanes of 32-bit words when they fit (two frames per word).
__host__ __device__ constexpr int frames_per_word(int K) { return 3 * K / 2 <= 16 ? 2 : 1; }

// Jump of state s (owned by a thread with K states) from one frame's bits.
template <int K>
__device__ __forceinline__ int jump_of(unsigned bits, int s) {
  const int k = s & (K - 1);
  const unsigned moved = (bits >> k) & 1u;
  const unsigned skipped = (k & 1) ? (bits >> (K + (k >> 1))) & 1u : 0u;
  return static_cast<int>(moved + skipped);
}

// One warp walks a path back through the backpointers, from state s at frame
// t_hi down to frame t_lo (path[t-1] = path[t] - jump(t, path[t]),
// alignment.cu:656-659).  The path moves at most 2 states per frame, so over
// FB frames it stays within 2*FB/K + 2 threads' words: the warp loads those
// FB x NTH words in one round trip, then steps through them with shuffles;
// every lane tracks the same state.  `at_frame(t, s)` is called (by every
// lane) with the path's state at each frame t_hi-1 .. t_lo; returns the state
// at t_lo.  bp: the record's backpointer words, NT threads per frame row.
template <int K, typename AtFrame>
__device__ __forceinline__ int warp_trace(const uint32_t* __restrict__ bp, int NT, int s, int t_hi,
                                          int t_lo, int lane, AtFrame at_frame) {
  constexpr int fpw = frames_per_word(K);
  constexpr int FB = K >= 8 ? 8 : 6;
  constexpr int NTH = 2 * FB / K + 2;
  constexpr int kShift = K == 4 ? 2 : (K == 8 ? 3 : 4);
  static_assert((1 << kShift) == K, "K is a power of two");
  for (int t = t_hi; t > t_lo;) {
    const int f = lane / NTH, dd = lane % NTH;
    const int tt = t - f;
    const int th = (s >> kShift) - dd;
    uint32_t w = 0;
    if (f < FB && tt > t_lo && th >= 0) w = bp[static_cast<int64_t>(tt / fpw) * NT + th];
    const int steps = min(FB, t - t_lo);
    const int th0 = s >> kShift;
    for (int i = 0; i < steps; ++i) {
      const int ct = t - i;
      const uint32_t word = __shfl_sync(0xffffffffu, w, i * NTH + (th0 - (s >> kShift)));
      // (The clamp never acts on backpointers a completed DP wrote; it keeps
      // every read inside the arena.)
      s = max(s - jump_of<K>(fpw == 2 ? word >> (16 * (ct & 1)) : word, s), 0);
      at_frame(ct - 1, s);
    }
    t -= steps;
  }
  return s;
}

}  // namespace dev
}  // namespace ffa
