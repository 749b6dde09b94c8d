// ffa_device.cuh -- device helpers shared by the forward kernels: barriers,
// TMA bulk copies and mbarriers, the DP frame step and the backpointer layout.
#pragma once

#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>
#include <type_traits>

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
__device__ __forceinline__ void cp_async4(void* smem_dst, const void* gmem_src) {
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
__device__ __forceinline__ void mbar_inval(unsigned long long* bar) {
  asm volatile("mbarrier.inval.shared::cta.b64 [%0];" ::"r"(smem_u32(bar)) : "memory");
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
// One TMA bulk copy global -> shared (no tensor map; this CTA's shared memory only), completed
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

// ---- thread-block clusters (long records: one cluster per record) ----------
__device__ __forceinline__ unsigned cluster_rank() {
  unsigned r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ unsigned cluster_size() {
  unsigned n;
  asm volatile("mov.u32 %0, %%cluster_nctarank;" : "=r"(n));
  return n;
}
// Address of this CTA's shared variable `p` in the shared memory of cluster
// CTA `rank` (a shared::cluster address).
__device__ __forceinline__ unsigned cluster_addr(const void* p, unsigned rank) {
  unsigned a;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(a) : "r"(smem_u32(p)), "r"(rank));
  return a;
}
__device__ __forceinline__ void st_cluster_u64(unsigned cluster_address, unsigned long long v) {
  asm volatile("st.relaxed.cluster.shared::cluster.b64 [%0], %1;" ::"r"(cluster_address), "l"(v) : "memory");
}
__device__ __forceinline__ void st_cluster_f32(unsigned cluster_address, float v) {
  asm volatile("st.relaxed.cluster.shared::cluster.f32 [%0], %1;" ::"r"(cluster_address), "f"(v) : "memory");
}
__device__ __forceinline__ void st_cluster_u32(unsigned cluster_address, unsigned v) {
  asm volatile("st.relaxed.cluster.shared::cluster.u32 [%0], %1;" ::"r"(cluster_address), "r"(v) : "memory");
}
// A load of this CTA's shared memory that sees stores other CTAs of the
// cluster made to it.
__device__ __forceinline__ unsigned long long ld_cluster_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.relaxed.cluster.shared::cta.b64 %0, [%1];" : "=l"(v) : "r"(smem_u32(p)) : "memory");
  return v;
}
// Every thread of every CTA of the cluster; orders shared and global memory
// accesses before it with those after it, cluster-wide.
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release;\n\tbarrier.cluster.wait.acquire;" ::: "memory");
}

// How the kernels read an emission (ffa_input_format).  Format 0: fp32
// log-probabilities, used as stored.  Formats 1 (fp32) and 2 (bf16): logits,
// used as their log_softmax -- the emission of (t, v) is x[t, v] - z[t] in
// one fp32 round-to-nearest subtraction, z[t] being row t's log-sum-exp that
// ffa_row_lse wrote.  Every kernel forms it the same way, so every kernel
// sees the same emission matrix.
template <int kFmt>
struct Input {
  static_assert(kFmt >= 0 && kFmt <= 2, "input format");
  using Elem = typename std::conditional<kFmt == 2, uint16_t, float>::type;
  static constexpr bool kLogits = kFmt != 0;
  static constexpr bool kHalf = kFmt == 2;
};
// A bf16 value (its 16 bits) as fp32: exact.
__device__ __forceinline__ float bf16_to_float(uint32_t bits) { return __uint_as_float(bits << 16); }
__device__ __forceinline__ float elem_to_float(float v) { return v; }
__device__ __forceinline__ float elem_to_float(uint16_t v) { return bf16_to_float(v); }
// The bf16 half of a 4-byte word at element parity `odd` (little endian).
__device__ __forceinline__ float bf16_of_word(uint32_t word, bool odd) {
  return __uint_as_float(odd ? (word & 0xffff0000u) : (word << 16));
}

// Row log-sum-exps of a run of frames from t0 (logits input): lane l holds
// z[t0 + 32 b + l] of the run's current 32-frame block b and of the next one,
// so a frame's value is one shuffle away and the next block's loads are in
// flight a block ahead.  Every lane of the warp calls at().
struct LseStream {
  const float* z;  // the record's z[0 .. T)
  int T;
  float cur, nxt;
  __device__ __forceinline__ float get(int t) const { return t < T ? __ldg(z + t) : 0.0f; }
  __device__ __forceinline__ void start(const float* zr, int frames, int t0, int lane) {
    z = zr;
    T = frames;
    cur = get(t0 + lane);
    nxt = get(t0 + 32 + lane);
  }
  // Enter the block that starts at frame `first` (the previous next block).
  __device__ __forceinline__ void advance(int first, int lane) {
    cur = nxt;
    nxt = get(first + 32 + lane);
  }
  // z of the frame at offset f from the run's start (f in the current block).
  __device__ __forceinline__ float at(int f) const { return __shfl_sync(0xffffffffu, cur, f & 31); }
};

// A record's bf16 elements as 4-byte words (per-thread column gathers copy
// whole aligned words): element i of the record -- i = t V + v -- lies in
// word (i + odd) / 2 counted from `words`, in its upper half when i + odd is
// odd.  That word is the 4-byte aligned granule holding the element, which
// no device allocation splits.
struct HalfWords {
  const uint32_t* words;  // the 4-byte word holding the record's first element
  int odd;                // 1 when that element is the word's upper half
  __device__ __forceinline__ void set(const void* base) {
    const uintptr_t a = reinterpret_cast<uintptr_t>(base);
    words = reinterpret_cast<const uint32_t*>(a & ~static_cast<uintptr_t>(3));
    odd = static_cast<int>((a >> 1) & 1);
  }
  __device__ __forceinline__ const uint32_t* word(int64_t i) const { return words + ((i + odd) >> 1); }
  // Parity of element t V + v from the parities of frame t's first element and of v.
  __device__ __forceinline__ bool row_odd(int64_t t, int V) const { return ((odd + (t & V)) & 1) != 0; }
};

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
// previous traceback segment).  Returns the frame's 2K-bit jump codes; the
// states' selections are independent of one another within a frame, and
// their codes are gathered by a balanced OR tree.
template <int K>
__device__ __forceinline__ unsigned dp_frame(float (&a)[K], int (&d)[K], float p1, int pd, float eb,
                                             const float (&et)[K / 2], unsigned skip) {
  float na[K];
  int nd[K];
  unsigned m[K];
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
      m[k] = (j2 ? 2u : (c ? 1u : 0u)) << (2 * k);
      na[k] = __fadd_rn(b, et[k >> 1]);
    } else {
      m[k] = (c ? 1u : 0u) << (2 * k);
      na[k] = __fadd_rn(b, eb);
    }
    nd[k] = n;
  }
#pragma unroll
  for (int w = 1; w < K; w *= 2)
#pragma unroll
    for (int k = 0; k + w < K; k += 2 * w) m[k] |= m[k + w];
#pragma unroll
  for (int k = 0; k < K; ++k) { a[k] = na[k]; d[k] = nd[k]; }
  return m[0];
}

// The same frame step without ancestor deltas, for runs whose path is found
// by tracing the backpointers (pieces of the optimized route).
template <int K>
__device__ __forceinline__ unsigned dp_frame_plain(float (&a)[K], float p1, float eb,
                                                   const float (&et)[K / 2], unsigned skip) {
  float na[K];
  unsigned m[K];
#pragma unroll
  for (int k = 0; k < K; ++k) {
    const float x1 = k >= 1 ? a[k - 1] : p1;
    const bool c = x1 > a[k];
    float b = c ? x1 : a[k];
    if (k & 1) {
      const float x2 = k >= 2 ? a[k - 2] : p1;
      const bool j2 = ((skip >> (k >> 1)) & 1u) && x2 > b;
      b = j2 ? x2 : b;
      m[k] = (j2 ? 2u : (c ? 1u : 0u)) << (2 * k);
      na[k] = __fadd_rn(b, et[k >> 1]);
    } else {
      m[k] = (c ? 1u : 0u) << (2 * k);
      na[k] = __fadd_rn(b, eb);
    }
  }
#pragma unroll
  for (int w = 1; w < K; w *= 2)
#pragma unroll
    for (int k = 0; k + w < K; k += 2 * w) m[k] |= m[k + w];
#pragma unroll
  for (int k = 0; k < K; ++k) a[k] = na[k];
  return m[0];
}

// Stores one thread's 2K jump-code bits of a frame into its row (K = 4, 8,
// 16: a byte, a halfword or a word at state K*tl).
template <int K>
__device__ __forceinline__ void store_codes(uint8_t* row, int tl, unsigned bits) {
  if constexpr (K == 16) reinterpret_cast<uint32_t*>(row)[tl] = bits;
  else if constexpr (K == 8) reinterpret_cast<uint16_t*>(row)[tl] = static_cast<uint16_t>(bits);
  else reinterpret_cast<uint8_t*>(row)[tl] = static_cast<uint8_t>(bits);
}

// One warp walks a path back through the backpointers, from state s at frame
// t_hi down to frame t_lo (path[t-1] = path[t] - jump(t, path[t]),
// alignment.cu:656-659).  The path drops at most 2 states per frame, so over
// 32 frames it stays within the 4-word block holding its starting state and
// the block before it: lane l loads those two 16-byte blocks of frame t - l
// (rows are whole multiples of 4 words, so the loads are aligned) in one
// round trip, and the warp then steps through the 32 frames with a shuffle
// each; every lane tracks the same state.  `at_frame(t, s)` is called (by
// every lane) with the path's state at each frame t_hi-1 .. t_lo; returns the
// state at t_lo.  bp: the record's rows, row_words words per frame.  Rows are
// read through L2 (ld.global.cg): a trace may follow rows that another CTA of
// the same launch wrote.
template <typename AtFrame>
__device__ __forceinline__ int warp_trace(const uint32_t* bp, int row_words, int s,
                                          int t_hi, int t_lo, int lane, AtFrame at_frame) {
  for (int t = t_hi; t > t_lo;) {
    const int steps = min(32, t - t_lo);
    const int qb = (s >> 6) << 2;  // first word of the block holding s
    uint4 hi = make_uint4(0u, 0u, 0u, 0u), lo = hi;
    if (lane < steps) {
      const uint4* row = reinterpret_cast<const uint4*>(bp + static_cast<int64_t>(t - lane) * row_words + qb);
      hi = __ldcg(row);
      if (qb >= 4) lo = __ldcg(row - 1);
    }
    for (int i = 0; i < steps; ++i) {
      // Word (s >> 4) is qb + d with d in [-4, 3]: position d + 4 of lo:hi
      // (the same position on every lane), taken from lane i (frame t - i).
      const int idx = (s >> 4) - qb + 4;
      const bool b0 = idx & 1, b1 = idx & 2, b2 = idx & 4;
      const uint32_t x = b1 ? (b0 ? lo.w : lo.z) : (b0 ? lo.y : lo.x);
      const uint32_t y = b1 ? (b0 ? hi.w : hi.z) : (b0 ? hi.y : hi.x);
      const uint32_t word = __shfl_sync(0xffffffffu, b2 ? y : x, i);
      // (The clamp never acts on backpointers a completed DP wrote; it keeps
      // every read inside the arena.)
      s = max(s - static_cast<int>((word >> (2 * (s & 15))) & 3u), 0);
      at_frame(t - i - 1, s);
    }
    t -= steps;
  }
  return s;
}

// The same walk with fewer bytes per frame: FB = 10 frames over 3 words
// around the path's word per round trip (lanes f*3 + dd load word w0 - dd of
// frame t - f).  Where many warps walk at once (the traceback fill of every
// segment) the memory traffic, not one walk's latency, bounds the kernel, and
// this variant moves 4 bytes per lane instead of 32.
template <typename AtFrame>
__device__ __forceinline__ int warp_trace_lean(const uint32_t* bp, int row_words, int s,
                                               int t_hi, int t_lo, int lane, AtFrame at_frame) {
  constexpr int FB = 10, NW = 3;
  for (int t = t_hi; t > t_lo;) {
    const int f = lane / NW, dd = lane % NW;
    const int tt = t - f;
    const int w0 = s >> 4;
    uint32_t w = 0;
    if (f < FB && tt > t_lo && w0 - dd >= 0) w = __ldcg(bp + static_cast<int64_t>(tt) * row_words + (w0 - dd));
    const int steps = min(FB, t - t_lo);
    for (int i = 0; i < steps; ++i) {
      const int ct = t - i;
      const uint32_t word = __shfl_sync(0xffffffffu, w, i * NW + (w0 - (s >> 4)));
      s = max(s - static_cast<int>((word >> (2 * (s & 15))) & 3u), 0);
      at_frame(ct - 1, s);
    }
    t -= steps;
  }
  return s;
}

}  // namespace dev
}  // namespace ffa
