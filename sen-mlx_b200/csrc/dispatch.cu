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
#include "dispatch_body.cuh"
#include "kernels.h"

namespace senmoe {

using namespace dispatch_detail;

// Whole dispatch in one CTA (num_pairs small).
__global__ void __launch_bounds__(kThreads) dispatch_single_kernel(DispatchArgs a) {
  pdl_wait();
  pdl_launch_dependents();
  extern __shared__ int sm[];
  dispatch_single_body(a, sm);
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
