// ep.cu -- expert parallelism over NVLink peer memory.
//
// The reference runs the MoE block on one GPU (deepseek_v2.rs:520-553); here
// its experts are split across the GPUs of one node, contiguous blocks of
// experts per rank.  Every rank holds the same tokens, runs the router and
// the full dispatch itself (both are deterministic, so every rank computes
// the same global slot order), and runs the expert products of its own
// experts only, writing their rows at their global slots of its `d` buffer.
// The tokens are split in contiguous blocks too (ep_token_begin): rank r's
// weighted combine takes its own tokens, reads each (token, slot) pair's row
// from the rank that owns the pair's expert, through CUDA IPC mappings of the
// peers' buffers, and sums the slots in order exactly as the one-GPU combine
// does.  It stores each combined row to its own y and into every peer's row
// exchange (peer stores over NVLink); ep_gather_rows_kernel then copies the
// other ranks' tokens from the exchange into y, so every rank ends with the
// same y.  Per layer a rank reads K rows for T / world tokens and sends
// T / world rows to each peer, instead of reading K rows for all T tokens.
//
// Three rank flags per layer order the exchange, all in the flag block of
// each rank's arena and all holding a call epoch:
//   ready[r]  rank r's expert rows of epoch e are complete (written by r's
//             announce kernel, right after its expert kernels, into every
//             rank's block), and r has finished reading its exchange of
//             epoch e - 1;
//   done[r]   rank r has finished reading its peers' rows of epoch e (written
//             by the last CTA of r's combine);
//   rows[r]   rank r's combined rows of epoch e are in this rank's exchange
//             (written by the last CTA of r's combine).
// A rank waits for done[*] >= e - 1 before its expert kernels overwrite d
// (ep_fence_kernel), for ready[*] >= e before reading rows or writing into a
// peer's exchange (ep_combine_kernel) and for rows[*] >= e before reading its
// exchange (ep_gather_rows_kernel).  Every wait is bounded: on timeout the
// kernel records kDevPeerTimeout and continues, so a missing peer turns into
// a status the host reads, never a hung GPU.

#include "common.cuh"
#include "kernels.h"

namespace senmoe {

namespace {

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Spins until *flag >= want (wrap-safe) or the cycle limit passes.  Once a
// peer wait has run out (*err == kDevPeerTimeout) later waits give up at
// once, so a missing rank costs one limit, not one per CTA and layer.
__device__ __forceinline__ bool wait_flag(const uint32_t* flag, uint32_t want, const int* err) {
  const long long t0 = clock64();
  while (static_cast<int32_t>(ld_acquire_sys(flag) - want) < 0) {
    if (clock64() - t0 > kWaitLimitCycles || *reinterpret_cast<const volatile int*>(err) == kDevPeerTimeout)
      return false;
    __nanosleep(64);
  }
  return true;
}

__global__ void ep_fence_kernel(EpArgs a) {
  __shared__ uint32_t s_epoch;
  if (threadIdx.x == 0) {
    const uint32_t e = *a.epoch + 1u;
    *a.epoch = e;
    s_epoch = e;
  }
  __syncthreads();
  pdl_launch_dependents();
  const int r = threadIdx.x;
  if (r < a.world && r != a.rank) {
    if (!wait_flag(a.flags + kEpDoneOffset + r, s_epoch - 1u, a.err)) record_error(a.err, kDevPeerTimeout);
  }
  pdl_wait();  // the expert kernels after this one wait on it, and through it on dispatch
}

// ready[rank] := epoch in every rank's flag block (its own included): this
// rank's expert rows of the call are complete.  One warp, launched right
// after the down projection: griddepcontrol.wait returns once the expert
// kernels have finished and their writes are visible, one system-scope fence
// orders them before the flag stores, and each peer gets one release store.
__global__ void ep_announce_kernel(EpArgs a) {
  pdl_wait();
  pdl_launch_dependents();
  const uint32_t epoch = *a.epoch;
  if (threadIdx.x == 0) __threadfence_system();
  __syncwarp();
  const int r = threadIdx.x;
  if (r < a.world) st_release_sys(a.peer_flags[r] + kEpReadyOffset + a.rank, epoch);
}

// Partitioned routing: this rank's routing rows (global pair rows
// [tok_begin[rank] * K, + n_routed * K)) -> every peer's routing arrays and,
// in the token-local form, its n_rows token rows -> its own exchange buffer
// (the peers' gathers read them there); the last CTA to finish raises
// ids[rank] in every rank's flags.  Each CTA fences its
// stores (one system-scope fence after a barrier) before it counts itself.
__global__ void __launch_bounds__(256) ep_publish_kernel(EpArgs a, const uint16_t* __restrict__ x, int n_rows,
                                                         int n_routed, int hidden) {
  pdl_wait();  // the router's ids / weights of this call are complete
  pdl_launch_dependents();
  const uint32_t epoch = *a.epoch;
  const size_t nthreads = size_t(gridDim.x) * blockDim.x, tid = size_t(blockIdx.x) * blockDim.x + threadIdx.x;
  const size_t nvec = size_t(n_rows) * hidden / 8;
  const uint4* src = reinterpret_cast<const uint4*>(x);
  uint4* dst = reinterpret_cast<uint4*>(a.peer_y[a.rank]);
  for (size_t i = tid; i < nvec; i += nthreads) dst[i] = __ldcg(src + i);
  const size_t p0 = size_t(a.tok_begin[a.rank]) * a.top_k, np = size_t(n_routed) * a.top_k;
  for (size_t i = tid; i < np; i += nthreads) {
    const int32_t id = a.peer_ids[a.rank][p0 + i];
    const float w = a.peer_wts[a.rank][p0 + i];
    for (int q = 0; q < a.world; ++q) {
      if (q == a.rank) continue;
      a.peer_ids[q][p0 + i] = id;
      a.peer_wts[q][p0 + i] = w;
    }
  }
  __shared__ bool s_last;
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    s_last = atomicAdd(a.published, 1u) == gridDim.x - 1u;
    if (s_last) __threadfence_system();
  }
  __syncthreads();
  if (s_last) {
    if (threadIdx.x == 0) *a.published = 0u;
    const int r = threadIdx.x;
    if (r < a.world) st_release_sys(a.peer_flags[r] + kEpIdsOffset + a.rank, epoch);
  }
}

// Waits until every peer's routing and token rows of this call are here.
__global__ void ep_wait_published_kernel(EpArgs a) {
  pdl_wait();
  const uint32_t epoch = *a.epoch;
  const int r = threadIdx.x;
  if (r < a.world && r != a.rank) {
    if (!wait_flag(a.flags + kEpIdsOffset + r, epoch, a.err)) record_error(a.err, kDevPeerTimeout);
  }
  __syncthreads();
  pdl_launch_dependents();
}

// Expert-rows owner of expert e: the rank r with bounds[r] <= e < bounds[r+1].
__device__ __forceinline__ int owner_of(const EpArgs& a, int e) {
  int r = 0;
#pragma unroll
  for (int i = 1; i < kEpMaxRanks; ++i) r += (i < a.world && e >= a.bounds[i]) ? 1 : 0;
  return r;
}

// y[t, :] = bf16( sum_j f32(d_owner(j)[inv[t*K + j], :]) * w[t, j]  (+ gate_t * shared[t, :]) (+ residual) )
// for this rank's tokens, with the one-GPU combine's arithmetic and slot
// order.  Grid: x covers the hidden columns (8 per thread), y strides over
// the rank's tokens.
template <int KMAX>  // compile-time bound on top_k sizing the per-thread arrays
__global__ void __launch_bounds__(256, KMAX <= 8 ? 4 : 2) ep_combine_kernel(EpArgs a, CombineArgs c, int num_tokens) {
  pdl_wait();  // d, ids, inverse and weights of this call are complete; ready[rank] is announced
  pdl_launch_dependents();
  const uint32_t epoch = *a.epoch;
  const int r = threadIdx.x;
  // every peer's rows of this call are complete (their announce kernels);
  // the flags live in this rank's own memory, so the polls stay local
  if (r < a.world && r != a.rank) {
    if (!wait_flag(a.flags + kEpReadyOffset + r, epoch, a.err)) record_error(a.err, kDevPeerTimeout);
  }
  __syncthreads();

  const int col = (blockIdx.x * blockDim.x + threadIdx.x) * 8;
  const int t_begin = a.tok_begin[a.rank];
  const int t_end = a.tok_begin[a.rank + 1];
  constexpr int kMaxK = KMAX;
  if (col < c.hidden) {
    for (int t = t_begin + blockIdx.y; t < t_end; t += gridDim.y) {
      float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      const uint16_t* src[kMaxK];
      float wj[kMaxK];
#pragma unroll
      for (int j = 0; j < kMaxK; ++j) {
        src[j] = nullptr;
        if (j < c.top_k) {
          const int p = t * c.top_k + j;
          const int slot = c.inverse[p];
          wj[j] = c.weights[p];
          if (slot >= 0) {
            const int e = a.topk_ids[p];
            const int q = owner_of(a, e);
            const int row = slot - a.offsets[a.bounds[q]];  // the owner's local row
            if (a.slot_cap > 0 && row >= a.slot_cap) record_error(a.err, kDevSlotOverflow);
            else src[j] = a.peer_d[q] + static_cast<size_t>(row) * c.hidden + col;
          }
        }
      }
      uint4 rows[kMaxK];
#pragma unroll
      for (int j = 0; j < kMaxK; ++j)
        if (src[j]) rows[j] = __ldcg(reinterpret_cast<const uint4*>(src[j]));
#pragma unroll
      for (int j = 0; j < kMaxK; ++j) {
        if (src[j]) {
          const uint4 v = rows[j];
          const float w = wj[j];
          acc[0] += bf16_lo(v.x) * w; acc[1] += bf16_hi(v.x) * w;
          acc[2] += bf16_lo(v.y) * w; acc[3] += bf16_hi(v.y) * w;
          acc[4] += bf16_lo(v.z) * w; acc[5] += bf16_hi(v.z) * w;
          acc[6] += bf16_lo(v.w) * w; acc[7] += bf16_hi(v.w) * w;
        }
      }
      const size_t lrow = static_cast<size_t>(t - c.local_row0);  // row of y / residual / shared_gate
      if (c.shared_out) {
        const float g = c.shared_gate ? c.shared_gate[lrow] : 1.0f;
        const uint4 v =
            *reinterpret_cast<const uint4*>(c.shared_out + static_cast<size_t>(t - c.shared_row0) * c.hidden + col);
        acc[0] += g * bf16_lo(v.x); acc[1] += g * bf16_hi(v.x);
        acc[2] += g * bf16_lo(v.y); acc[3] += g * bf16_hi(v.y);
        acc[4] += g * bf16_lo(v.z); acc[5] += g * bf16_hi(v.z);
        acc[6] += g * bf16_lo(v.w); acc[7] += g * bf16_hi(v.w);
      }
      if (c.residual) {
        const uint4 v = *reinterpret_cast<const uint4*>(c.residual + lrow * c.hidden + col);
        acc[0] += bf16_lo(v.x); acc[1] += bf16_hi(v.x); acc[2] += bf16_lo(v.y); acc[3] += bf16_hi(v.y);
        acc[4] += bf16_lo(v.z); acc[5] += bf16_hi(v.z); acc[6] += bf16_lo(v.w); acc[7] += bf16_hi(v.w);
      }
      uint4 o;
      o.x = uint32_t(f32_to_bf16_bits(acc[0])) | (uint32_t(f32_to_bf16_bits(acc[1])) << 16);
      o.y = uint32_t(f32_to_bf16_bits(acc[2])) | (uint32_t(f32_to_bf16_bits(acc[3])) << 16);
      o.z = uint32_t(f32_to_bf16_bits(acc[4])) | (uint32_t(f32_to_bf16_bits(acc[5])) << 16);
      o.w = uint32_t(f32_to_bf16_bits(acc[6])) | (uint32_t(f32_to_bf16_bits(acc[7])) << 16);
      *reinterpret_cast<uint4*>(c.y + lrow * c.hidden + col) = o;
      if (!a.local_tokens) {  // replicated form: every rank returns every token
        const size_t off = static_cast<size_t>(t) * c.hidden + col;
        for (int q = 0; q < a.world; ++q)
          if (q != a.rank) *reinterpret_cast<uint4*>(a.peer_y[q] + off) = o;
      }
    }
  }

  // The last CTA to finish tells every peer that this rank is done reading
  // and that its combined rows are in the peer's exchange.  The barrier
  // orders the CTA's peer loads and stores before thread 0, whose one
  // system-scope fence (cumulative) orders them before the CTA counts itself
  // finished; the last CTA fences again before raising the flags.
  __shared__ bool s_last;
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    const uint32_t total = gridDim.x * gridDim.y;
    s_last = atomicAdd(a.finished, 1u) == total - 1u;
    if (s_last) __threadfence_system();
  }
  __syncthreads();
  if (s_last) {
    if (threadIdx.x == 0) *a.finished = 0u;
    if (r < a.world) {
      st_release_sys(a.peer_flags[r] + kEpDoneOffset + a.rank, epoch);
      if (r != a.rank && !a.local_tokens) st_release_sys(a.peer_flags[r] + kEpRowsOffset + a.rank, epoch);
    }
  }
}

// y[t, :] = exchange[t, :] for the tokens other ranks own.  Grid: x covers
// the hidden columns (8 per thread), y strides over those tokens.
__global__ void __launch_bounds__(256) ep_gather_rows_kernel(EpArgs a, uint16_t* y, int hidden, int num_tokens) {
  pdl_wait();  // y's previous readers have finished; this call's epoch is set
  pdl_launch_dependents();
  const int t_begin = a.tok_begin[a.rank];
  const int t_end = a.tok_begin[a.rank + 1];
  const int others = num_tokens - (t_end - t_begin);
  if (others == 0) return;
  const uint32_t epoch = *a.epoch;
  const int r = threadIdx.x;
  if (r < a.world && r != a.rank) {
    if (!wait_flag(a.flags + kEpRowsOffset + r, epoch, a.err)) record_error(a.err, kDevPeerTimeout);
  }
  __syncthreads();
  const int col = (blockIdx.x * blockDim.x + threadIdx.x) * 8;
  if (col >= hidden) return;
  const uint16_t* ex = a.peer_y[a.rank];
  for (int u = blockIdx.y; u < others; u += gridDim.y) {
    const int t = u < t_begin ? u : u + (t_end - t_begin);
    const size_t off = static_cast<size_t>(t) * hidden + col;
    *reinterpret_cast<uint4*>(y + off) = __ldcg(reinterpret_cast<const uint4*>(ex + off));
  }
}

}  // namespace

cudaError_t launch_ep_fence(const EpArgs& a, cudaStream_t st) {
  return launch_pdl(ep_fence_kernel, dim3(1), dim3(32), 0, st, a);
}

cudaError_t launch_ep_announce(const EpArgs& a, cudaStream_t st) {
  return launch_pdl(ep_announce_kernel, dim3(1), dim3(32), 0, st, a);
}

cudaError_t launch_ep_publish(const EpArgs& a, const uint16_t* x, int n_rows, int n_routed, int hidden,
                              cudaStream_t st) {
  // enough CTAs to stream the rows at full bandwidth; at least one raises the flags
  const size_t work = size_t(n_rows) * hidden / 8 + size_t(n_routed) * a.top_k;
  int grid = static_cast<int>((work + 255) / 256);
  grid = grid < 1 ? 1 : (grid > 296 ? 296 : grid);
  return launch_pdl(ep_publish_kernel, dim3(grid), dim3(256), 0, st, a, x, n_rows, n_routed, hidden);
}

cudaError_t launch_ep_wait_published(const EpArgs& a, cudaStream_t st) {
  return launch_pdl(ep_wait_published_kernel, dim3(1), dim3(32), 0, st, a);
}

cudaError_t launch_ep_combine(const EpArgs& a, const CombineArgs& c, int num_tokens, cudaStream_t st) {
  (void)num_tokens;
  const int own = a.tok_begin[a.rank + 1] - a.tok_begin[a.rank];
  const int threads = own < 256 ? 64 : 256;  // narrow CTAs for small batches (>= 8 ranks' flag threads)
  const int gx = (c.hidden / 8 + threads - 1) / threads;
  // enough CTAs to cover the rank's tokens of a decode batch in one wave;
  // larger batches loop (each CTA announces and waits once).  A rank that
  // owns no token still launches one row of CTAs for the flag hand-over.
  const int gy = own < 1 ? 1 : (own < 1024 ? own : 1024);
  if (c.top_k <= 8) return launch_pdl(ep_combine_kernel<8>, dim3(gx, gy), dim3(threads), 0, st, a, c, num_tokens);
  return launch_pdl(ep_combine_kernel<16>, dim3(gx, gy), dim3(threads), 0, st, a, c, num_tokens);
}

cudaError_t launch_ep_gather_rows(const EpArgs& a, uint16_t* y, int hidden, int num_tokens, cudaStream_t st) {
  const int own = a.tok_begin[a.rank + 1] - a.tok_begin[a.rank];
  const int others = num_tokens - own;
  const int threads = others < 256 ? 64 : 256;
  const int gx = (hidden / 8 + threads - 1) / threads;
  const int gy = others < 1 ? 1 : (others < 1024 ? others : 1024);
  return launch_pdl(ep_gather_rows_kernel, dim3(gx, gy), dim3(threads), 0, st, a, y, hidden, num_tokens);
}

}  // namespace senmoe
