// dispatch.cu -- deterministic expert-contiguous permutation of (token, slot) pairs.
//
// The reference gathers each (token, slot) pair separately (gather_qmm with
// sorted_indices=false, src/engine/mlx_lm/models/deepseek_v2.rs:441) and has
// no permutation.  This build groups pairs by expert: a stable counting sort
// of pair indices p = t*K + j by expert id, giving
//   offsets[e] .. offsets[e+1]   the slots of expert e,
//   perm[slot]                   the pair in that slot (ascending p within e),
//   inverse[p]                   the slot of pair p (-1 if e is not local,
//                                unless keep_remote_slots is set),
//   active[0 .. active_count)    local experts that received pairs, ascending.
// The result depends only on topk_ids: counts are integer atomics (order-free)
// and ranks inside a 1024-pair chunk come from warp match masks plus
// per-warp histograms, so no placement depends on thread timing.
//
// Small batches (one chunk) run in a single CTA; larger ones use three
// kernels: per-chunk histograms, one scan CTA, per-chunk stable scatter.

#include "common.cuh"
#include "kernels.h"

namespace senmoe {

namespace {

constexpr int kThreads = kDispatchChunk;  // one pair per thread per chunk
constexpr int kWarps = kThreads / 32;

// Block-wide exclusive scan of one int per thread (1024 threads).
__device__ int block_exclusive_scan(int v, int* warp_tot, int* total) {
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
__device__ void scan_counts(const int* cnt, const DispatchArgs& a, int* warp_tot, int* total) {
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
__device__ void place_chunk(const DispatchArgs& a, int chunk, int* cursor, int* whist) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int E = a.num_experts;
  const int p = chunk * kThreads + threadIdx.x;
  int e = -1;
  if (p < a.num_pairs) {
    e = a.topk_ids[p];
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

__device__ void histogram_chunk(const DispatchArgs& a, int p_begin, int p_end, int* cnt) {
  for (int i = threadIdx.x; i < a.num_experts; i += kThreads) cnt[i] = 0;
  __syncthreads();
  for (int p = p_begin + threadIdx.x; p < p_end; p += kThreads) {
    const int e = a.topk_ids[p];
    if (e >= 0 && e < a.num_experts) atomicAdd(&cnt[e], 1);
  }
  __syncthreads();
}

}  // namespace

// Whole dispatch in one CTA (num_pairs small).
__global__ void __launch_bounds__(kThreads) dispatch_single_kernel(DispatchArgs a) {
  pdl_wait();
  pdl_launch_dependents();
  extern __shared__ int sm[];
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

// Phase 1 of the large dispatch: one histogram per chunk.
__global__ void __launch_bounds__(kThreads) dispatch_hist_kernel(DispatchArgs a) {
  pdl_wait();
  pdl_launch_dependents();
  extern __shared__ int sm[];
  const int c = blockIdx.x;
  histogram_chunk(a, c * kThreads, min(a.num_pairs, (c + 1) * kThreads), sm);
  for (int e = threadIdx.x; e < a.num_experts; e += kThreads) a.chunk_hist[static_cast<size_t>(c) * a.num_experts + e] = sm[e];
}

// Phase 2: totals, offsets, active list; chunk_hist becomes per-chunk bases.
__global__ void __launch_bounds__(kThreads) dispatch_scan_kernel(DispatchArgs a, int nchunks) {
  pdl_wait();
  pdl_launch_dependents();
  extern __shared__ int sm[];
  __shared__ int warp_tot[32];
  __shared__ int total;
  for (int e = threadIdx.x; e < a.num_experts; e += kThreads) {
    int s = 0;  // NOLINT
#pragma unroll 16
    for (int c = 0; c < nchunks; ++c) s += a.chunk_hist[static_cast<size_t>(c) * a.num_experts + e];
    sm[e] = s;
  }
  __syncthreads();
  scan_counts(sm, a, warp_tot, &total);
  for (int e = threadIdx.x; e < a.num_experts; e += kThreads) {
    int run = a.offsets[e];
    // 16 chunk counts per batch of independent loads, then their prefix
    for (int c0 = 0; c0 < nchunks; c0 += 16) {
      int n[16];
#pragma unroll
      for (int i = 0; i < 16; ++i)
        n[i] = c0 + i < nchunks ? a.chunk_hist[static_cast<size_t>(c0 + i) * a.num_experts + e] : 0;
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        if (c0 + i < nchunks) a.chunk_hist[static_cast<size_t>(c0 + i) * a.num_experts + e] = run;
        run += n[i];
      }
    }
  }
}

// Phase 3: per-chunk stable placement from the chunk's bases.
__global__ void __launch_bounds__(kThreads) dispatch_place_kernel(DispatchArgs a) {
  pdl_wait();
  pdl_launch_dependents();
  extern __shared__ int sm[];
  int* cursor = sm;
  int* whist = sm + a.num_experts;
  const int c = blockIdx.x;
  for (int e = threadIdx.x; e < a.num_experts; e += kThreads)
    cursor[e] = a.chunk_hist[static_cast<size_t>(c) * a.num_experts + e];
  __syncthreads();
  place_chunk(a, c, cursor, whist);
}

size_t dispatch_smem_bytes(int num_experts) {
  return static_cast<size_t>(num_experts) * (1 + kWarps) * sizeof(int);
}

cudaError_t launch_dispatch(const DispatchArgs& a, cudaStream_t st) {
  const size_t smem = dispatch_smem_bytes(a.num_experts);
  const int nchunks = (a.num_pairs + kThreads - 1) / kThreads;
  cudaError_t e;
  if (nchunks <= 2 || a.chunk_hist == nullptr) {
    e = ensure_dynamic_smem(reinterpret_cast<const void*>(dispatch_single_kernel), smem);
    if (e != cudaSuccess) return e;
    return launch_pdl(dispatch_single_kernel, dim3(1), dim3(kThreads), smem, st, a);
  }
  e = ensure_dynamic_smem(reinterpret_cast<const void*>(dispatch_place_kernel), smem);
  if (e != cudaSuccess) return e;
  e = launch_pdl(dispatch_hist_kernel, dim3(nchunks), dim3(kThreads), a.num_experts * sizeof(int), st, a);
  if (e == cudaSuccess)
    e = launch_pdl(dispatch_scan_kernel, dim3(1), dim3(kThreads), a.num_experts * sizeof(int), st, a, nchunks);
  if (e == cudaSuccess) e = launch_pdl(dispatch_place_kernel, dim3(nchunks), dim3(kThreads), smem, st, a);
  return e;
}

}  // namespace senmoe
