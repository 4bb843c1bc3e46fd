// tiles.cuh -- the per-CTA tile list of the persistent grouped expert GEMMs.
#pragma once

#include <stdint.h>

#include "common.cuh"

namespace senmoe {

constexpr int kTileScratchInts = 4 * 512 + 64;  // per active expert: e, s0, cnt, prefix; + scan totals

// Tiles of a grouped GEMM are numbered expert-major (active list order), then
// m-tile, then chunk of bn slots (chunk_major: chunk, then m-tile); CTA c
// takes tile numbers c, c + grid, ...
// Writes this CTA's tiles (local expert, first row, first slot, slots) to
// s_tiles and returns their number (at most max_tiles; more records
// kDevTileOverflow).  Every thread of the block calls it (blockDim.x >=
// active experts, at most 512); scratch is kTileScratchInts ints of shared
// memory; it ends with __syncthreads.  The loads of the active list and the
// offsets are issued by all threads at once: a single thread walking the list
// would wait on one dependent global load per expert.
// Slots come out local: offsets[e] - offsets[expert_begin]; with slot_cap >
// 0 an expert's slots past slot_cap are dropped (kDevSlotOverflow).  With
// cnt_hi > 0 only experts of cnt_lo <= slots < cnt_hi are listed.
__device__ __forceinline__ int list_tiles(const int32_t* __restrict__ active, const int32_t* __restrict__ active_count,
                                          const int32_t* __restrict__ offsets, int expert_begin, int m_tiles, int bm,
                                          int bn, bool chunk_major, int4* s_tiles, int max_tiles, int* scratch,
                                          int* err, int slot_cap = 0, int cnt_lo = 0, int cnt_hi = 0) {
  int* s_e = scratch;
  int* s_s0 = scratch + 512;
  int* s_cnt = scratch + 1024;
  int* s_pre = scratch + 1536;  // exclusive prefix of tile counts
  int* s_wt = scratch + 2048;   // per-warp totals [32], then the grand total
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int nact = min(*active_count, 512);
  int v = 0;
  if (tid < nact) {
    const int e = active[tid];
    const int base = offsets[expert_begin];
    const int s0 = offsets[e] - base;
    int cnt = offsets[e + 1] - offsets[e];
    if (cnt_hi > 0 && (cnt < cnt_lo || cnt >= cnt_hi)) cnt = 0;  // the other kernel's expert
    if (slot_cap > 0 && s0 + cnt > slot_cap) {
      cnt = s0 < slot_cap ? slot_cap - s0 : 0;
      record_error(err, kDevSlotOverflow);
    }
    s_e[tid] = e;
    s_s0[tid] = s0;
    s_cnt[tid] = cnt;
    v = m_tiles * ((cnt + bn - 1) / bn);
  }
  // block exclusive scan of v over the first nact threads
  int incl = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int u = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += u;
  }
  if (lane == 31) s_wt[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    const int nw = (blockDim.x + 31) >> 5;
    int w = lane < nw ? s_wt[lane] : 0;
    int wi = w;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int u = __shfl_up_sync(0xffffffffu, wi, o);
      if (lane >= o) wi += u;
    }
    if (lane < nw) s_wt[lane] = wi - w;  // exclusive warp offsets
    if (lane == 31) s_wt[32] = wi;       // total tiles
  }
  __syncthreads();
  if (tid < nact) s_pre[tid] = s_wt[warp] + incl - v;
  const int total = s_wt[32];
  __syncthreads();
  const int grid = static_cast<int>(gridDim.x), me = static_cast<int>(blockIdx.x);
  const int mine = total > me ? (total - me + grid - 1) / grid : 0;
  const int n = min(mine, max_tiles);
  for (int k = tid; k < n; k += blockDim.x) {
    const int idx = me + k * grid;
    int lo = 0, hi = nact - 1;  // last i with s_pre[i] <= idx
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (s_pre[mid] <= idx) lo = mid;
      else hi = mid - 1;
    }
    const int r = idx - s_pre[lo], cnt = s_cnt[lo];
    const int nch = (cnt + bn - 1) / bn;
    const int mt = chunk_major ? r % m_tiles : r / nch;
    const int c = chunk_major ? r / m_tiles : r - mt * nch;
    s_tiles[k] = make_int4(s_e[lo] - expert_begin, mt * bm, s_s0[lo] + c * bn, min(bn, cnt - c * bn));
  }
  if (tid == 0 && mine > max_tiles) record_error(err, kDevTileOverflow);
  __syncthreads();
  return n;
}

}  // namespace senmoe
