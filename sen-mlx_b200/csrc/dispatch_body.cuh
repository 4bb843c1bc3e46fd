// dispatch_body.cuh -- building blocks of the deterministic dispatch (see
// dispatch.cu), shared by the dispatch kernels and the fused router kernel.
// topk_ids are read with ld.global.cg: in the fused router they were written
// by other CTAs of the same grid.
#pragma once

#include "common.cuh"
#include "kernels.h"

namespace senmoe {
namespace dispatch_detail {

constexpr int kThreads = kDispatchChunk;  // one pair per thread per chunk
constexpr int kWarps = kThreads / 32;

// Block-wide exclusive scan of one int per thread (1024 threads).
__device__ __forceinline__ int block_exclusive_scan(int v, int* warp_tot, int* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int inc = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int n = __shfl_up_sync(0xffffffffu, inc, o);
    if (lane >= o) inc += n;
  }
  if (lane == 31) warp_tot[warp] = inc;
  __syncthreads();
  if (warp == 0) {
    int wv = warp_tot[lane];
    int wi = wv;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int n = __shfl_up_sync(0xffffffffu, wi, o);
      if (lane >= o) wi += n;
    }
    warp_tot[lane] = wi - wv;  // exclusive warp base
    if (lane == 31) *total = wi;
  }
  __syncthreads();
  const int r = warp_tot[warp] + inc - v;
  __syncthreads();
  return r;
}

// Offsets (exclusive scan of counts) and the active-expert list, for
// E <= 1024 (one expert per thread).  cnt: shared [E] counts.
__device__ __forceinline__ void scan_counts(const int* cnt, const DispatchArgs& a, int* warp_tot, int* total) {
  const int e = threadIdx.x;
  const int c = e < a.num_experts ? cnt[e] : 0;
  const int off = block_exclusive_scan(c, warp_tot, total);
  if (e < a.num_experts) a.offsets[e] = off;
  if (e == a.num_experts - 1) a.offsets[a.num_experts] = off + c;
  const int is_active = (e < a.num_experts && c > 0 && e >= a.expert_begin && e < a.expert_end) ? 1 : 0;
  const int pos = block_exclusive_scan(is_active, warp_tot, total);
  if (is_active) a.active[pos] = e;
  if (threadIdx.x == 0) *a.active_count = *total;
  __syncthreads();
}

// Stable placement of one chunk of pairs.  cursor[e] (shared) holds the
// first free slot of expert e for this chunk and is advanced past it.
__device__ __forceinline__ void place_chunk(const DispatchArgs& a, int chunk, int* cursor, int* whist) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int E = a.num_experts;
  const int p = chunk * kThreads + threadIdx.x;
  int e = -1;
  if (p < a.num_pairs) {
    e = __ldcg(a.topk_ids + p);
    if (e < 0 || e >= E) {
      record_error(a.err, kDevBadExpert);
      e = -1;
    }
  }
  for (int i = threadIdx.x; i < kWarps * E; i += kThreads) whist[i] = 0;
  __syncthreads();
  const unsigned mask = __match_any_sync(0xffffffffu, e);
  const int rank = __popc(mask & ((1u << lane) - 1u));
  if (e >= 0 && lane == __ffs(mask) - 1) whist[warp * E + e] = __popc(mask);
  __syncthreads();
  for (int x = threadIdx.x; x < E; x += kThreads) {
    int run = cursor[x];
    for (int w = 0; w < kWarps; ++w) {
      const int c = whist[w * E + x];
      whist[w * E + x] = run;
      run += c;
    }
    cursor[x] = run;
  }
  __syncthreads();
  if (e >= 0) {
    const int slot = whist[warp * E + e] + rank;
    a.perm[slot] = p;
    a.inverse[p] = (a.keep_remote_slots || (e >= a.expert_begin && e < a.expert_end)) ? slot : -1;
  } else if (p < a.num_pairs) {
    a.inverse[p] = -1;  // rejected id: the combine skips the pair
  }
  __syncthreads();
}

__device__ __forceinline__ void histogram_chunk(const DispatchArgs& a, int p_begin, int p_end, int* cnt) {
  for (int i = threadIdx.x; i < a.num_experts; i += kThreads) cnt[i] = 0;
  __syncthreads();
  for (int p = p_begin + threadIdx.x; p < p_end; p += kThreads) {
    const int e = __ldcg(a.topk_ids + p);
    if (e >= 0 && e < a.num_experts) atomicAdd(&cnt[e], 1);
  }
  __syncthreads();
}

// Whole dispatch in one CTA of kThreads threads (num_pairs small); sm holds
// dispatch_smem_bytes(E) of shared memory.
__device__ __forceinline__ void dispatch_single_body(const DispatchArgs& a, int* sm) {
  int* cnt = sm;                         // [E]
  int* whist = sm + a.num_experts;       // [kWarps * E]
  __shared__ int warp_tot[32];
  __shared__ int total;
  histogram_chunk(a, 0, a.num_pairs, cnt);
  scan_counts(cnt, a, warp_tot, &total);
  // cursor = offsets (reuse cnt)
  for (int e = threadIdx.x; e < a.num_experts; e += kThreads) cnt[e] = a.offsets[e];
  __syncthreads();
  const int nchunks = (a.num_pairs + kThreads - 1) / kThreads;
  for (int c = 0; c < nchunks; ++c) place_chunk(a, c, cnt, whist);
}

// The whole dispatch of at most 128 pairs by one warp, with the same result
// as dispatch_single_body: a shared-memory histogram, per-lane prefix sums
// over E/32 consecutive experts (offsets, active list), then stable
// placement 32 pairs at a time in pair order (match_any rank within the 32
// plus each expert's running cursor).  cnt: shared [E], E <= 512.
__device__ __forceinline__ void dispatch_warp_body(const DispatchArgs& a, int* cnt, int lane) {
  const int E = a.num_experts, P = a.num_pairs;
  for (int e = lane; e < E; e += 32) cnt[e] = 0;
  __syncwarp();
  for (int p = lane; p < P; p += 32) {
    const int e = __ldcg(a.topk_ids + p);
    if (e >= 0 && e < E) atomicAdd(&cnt[e], 1);
  }
  __syncwarp();
  const int epl = (E + 31) / 32, e0 = lane * epl;
  int mine = 0;
  uint32_t act = 0;  // bit i: expert e0 + i is local and has pairs
  for (int i = 0; i < epl; ++i) {
    const int e = e0 + i;
    if (e < E) {
      const int c = cnt[e];
      mine += c;
      if (c > 0 && e >= a.expert_begin && e < a.expert_end) act |= 1u << i;
    }
  }
  int incl = mine, ainc = __popc(act);
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int u = __shfl_up_sync(0xffffffffu, incl, o), v = __shfl_up_sync(0xffffffffu, ainc, o);
    if (lane >= o) {
      incl += u;
      ainc += v;
    }
  }
  int run = incl - mine, apos = ainc - __popc(act);
  for (int i = 0; i < epl; ++i) {
    const int e = e0 + i;
    if (e < E) {
      const int c = cnt[e];
      a.offsets[e] = run;
      cnt[e] = run;  // from here on: the expert's next free slot
      run += c;
      if (act & (1u << i)) a.active[apos++] = e;
    }
  }
  if (lane == 31) {
    a.offsets[E] = incl;
    *a.active_count = ainc;
  }
  __syncwarp();
  for (int c0 = 0; c0 < P; c0 += 32) {
    const int p = c0 + lane;
    int e = -1;
    if (p < P) {
      e = __ldcg(a.topk_ids + p);
      if (e < 0 || e >= E) {
        record_error(a.err, kDevBadExpert);
        e = -1;
      }
    }
    const unsigned mask = __match_any_sync(0xffffffffu, e);
    const int rank = __popc(mask & ((1u << lane) - 1u));
    if (e >= 0) {
      const int slot = cnt[e] + rank;
      a.perm[slot] = p;
      a.inverse[p] = (a.keep_remote_slots || (e >= a.expert_begin && e < a.expert_end)) ? slot : -1;
    } else if (p < P) {
      a.inverse[p] = -1;  // rejected id: the combine skips the pair
    }
    __syncwarp();
    if (e >= 0 && lane == __ffs(mask) - 1) cnt[e] += __popc(mask);
    __syncwarp();
  }
}
constexpr int kWarpDispatchMaxPairs = 128;

}  // namespace dispatch_detail
}  // namespace senmoe
