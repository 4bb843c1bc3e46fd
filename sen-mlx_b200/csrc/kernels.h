// kernels.h -- internal launch interfaces of the senmoe CUDA kernels.
#pragma once

#include <cuda.h>  // CUtensorMap (types only; the encoder is fetched at run time)
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace senmoe {

// Device-side error codes written to an error word (first writer wins).
enum DeviceError : int {
  kDevOk = 0,
  kDevBadExpert = 1,    // an expert id outside [0, E)
  kDevWaitTimeout = 2,  // a bounded mbarrier wait ran out
  kDevFp16Range = 3,    // an activation outside fp16 range met the tensor-core path
  kDevTileOverflow = 4, // a persistent CTA was handed more tiles than it can list
  kDevPeerTimeout = 5,  // a bounded wait on another rank's flag ran out
  kDevSlotOverflow = 6, // more pairs reached this rank's experts than its expert-slot capacity
};

// -------------------------------------------------------------- dispatch
struct DispatchArgs {
  const int32_t* topk_ids;  // [P] = [T*K]
  int num_pairs, num_experts;
  int expert_begin, expert_end;  // experts whose slots count as local
  int32_t* perm;            // [P] pair index of each expert-sorted slot
  int32_t* inverse;         // [P] slot of each pair (-1 for non-local experts)
  int32_t* offsets;         // [E + 1]
  int32_t* active;          // [E] local experts with tokens, ascending
  int32_t* active_count;    // [1]
  int32_t* chunk_hist;      // [nchunks, E] scratch (large dispatch only)
  int* err;
  int keep_remote_slots;    // 1: inverse keeps the slot of non-local experts too
};
// ---------------------------------------------------------------- router
struct RouterArgs {
  const uint16_t* x;        // bf16 [T, H]
  const uint16_t* weight;   // bf16 [E, H]
  float* logits;            // fp32 [T, E] (bf16-rounded values unless raw)
  int32_t* topk_ids;        // [T, K]
  float* topk_weights;      // [T, K]
  int num_tokens, hidden, num_experts, top_k;
  int norm_topk_prob;
  float routed_scaling_factor;
  int round_logits;         // 1: logits rounded to bf16 (nn::Linear output dtype)
  int* err;                 // device error word (bounded waits of the tiled router), may be null
  // Fusion (router_logits_kernel only): with tile_cnt set, the last CTA of
  // each 4-token tile runs top-k for its tokens (tile_cnt: one zeroed int per
  // tile, left zero), so no top-k launch follows.
  int* tile_cnt;
};
cudaError_t launch_router_logits(const RouterArgs& a, cudaStream_t st);
// Prefill router: logits (bf16 tensor-core MMA, fp32 accumulation, bf16
// rounded) and softmax / top-k in one launch, 32 tokens per CTA; logits are
// not written to global memory.  tX: x bf16 [T, H], tW: Wg bf16 [E, H], both
// 64-column boxes with SWIZZLE_128B (32 and 128 rows).  H % 64 == 0, E <= 512.
// Each CTA streams all of Wg; up to one CTA per SM (the 8-stage ring).  With
// more than 128 experts and fewer 32-token tiles than SMs, one CTA per (tile,
// 128-expert chunk) writes the logits to a.logits [T, E] and a top-k launch
// follows (same results).
constexpr int kRouterTcTokensPerCta = 32;
bool router_tc_supported(int hidden, int num_experts, int top_k);
size_t router_tc_smem_bytes(int num_experts, bool split = false);
cudaError_t launch_router_tc(const CUtensorMap& tX, const CUtensorMap& tW, const RouterArgs& a, cudaStream_t st);
cudaError_t launch_router_topk(const RouterArgs& a, cudaStream_t st);
// ------------------------------------- single-token fused layer (batch 1)
struct SingleTokenArgs {
  const uint16_t* x;              // bf16 [H]
  const uint16_t* router_weight;  // bf16 [E, H]
  const uint32_t* w[3];           // gate, up, down codes (MLX layout, 4-bit)
  const uint16_t* s[3];           // bf16 scales
  const uint16_t* b[3];           // bf16 biases
  const uint16_t* residual;       // bf16 [H] added before rounding, or null
  uint16_t* y;                    // bf16 [H]
  float* logits;                  // fp32 [E]: bf16-rounded router logits
  int32_t* topk_ids;              // [K]
  float* topk_weights;            // [K]
  uint16_t* h;                    // bf16 [K, I] scratch
  unsigned int* grid_bar;         // grid barrier word, zero before the first call
  int* err;
  int hidden, inter, num_experts, top_k, bits;
  int norm_topk_prob;
  float routed_scaling_factor;
  int act;
  // filled by single_token_plan: row split units, the most rows per CTA,
  // shared-memory bytes (gate/up part, down part, total with h)
  int unit_c, unit_d, rows_c, rows_d, smem_c, smem_d, smem;
};
// Fills the plan fields; false if the shape is not supported (4-bit, H with
// 8 code words per lane, I with 2 or 3, E <= 512, K <= 16 and <= sms, the
// shared memory within 200 KB).
bool single_token_plan(SingleTokenArgs& a, int sms);
// One persistent grid of `sms` CTAs (all resident: the caller gives the SM count).
cudaError_t launch_single_token_layer(const SingleTokenArgs& a, int sms, cudaStream_t st);
// sigmoid_bf16 against the exact form over every bf16 input (synchronous, current device).
cudaError_t selftest_sigmoid(int64_t* mismatches, int64_t* exact_form);
// Top-k of every token plus the single-chunk dispatch in one CTA, for small
// batches (<= kTopkDispatchMaxTokens tokens, <= 2048 pairs); d.topk_ids must
// be a.topk_ids.  Measured on the 48-layer decode stack: one launch fewer
// wins at 1-8 tokens (about 1 %); at 32-64 tokens the one CTA's top-k of
// every token costs more than the launch (+2 %, +5 %).
constexpr int kTopkDispatchMaxTokens = 8;
bool router_topk_dispatch_supported(int num_tokens, int num_pairs, int num_experts);
cudaError_t launch_router_topk_dispatch(const RouterArgs& a, const DispatchArgs& d, cudaStream_t st);
bool router_supported(int hidden, int num_experts, int top_k);

// Gemma-4 router (router_gemma.cu, gemma4.rs:716-736): rms_norm with weight
// f32(scale) * root (root = H^-1/2), the affine-quantized projection, top-k,
// softmax over the k, * per_expert_scale.  One CTA per token.
struct GemmaRouterArgs {
  const uint16_t* x;                 // bf16 [T, H]
  const uint32_t* proj_w;            // [E, H * bits / 32]
  const uint16_t* proj_s;            // bf16 [E, H / group]
  const uint16_t* proj_b;
  const uint16_t* scale;             // bf16 [H]
  const uint16_t* per_expert_scale;  // bf16 [E]
  int32_t* topk_ids;                 // [T, K]
  float* topk_weights;               // [T, K]
  int num_tokens, hidden, num_experts, top_k, bits, group_size;
  float eps, root;
};
bool gemma_router_supported(int hidden, int num_experts, int top_k, int bits, int group_size);
cudaError_t launch_gemma_router(const GemmaRouterArgs& a, cudaStream_t st);

constexpr int kDispatchChunk = 1024;
cudaError_t launch_dispatch(const DispatchArgs& a, cudaStream_t st);
size_t dispatch_smem_bytes(int num_experts);

// ------------------------------------------------------------ expert GEMV
enum ItemMode : int { kItemsGrouped = 0, kItemsGather = 1 };
struct QGemvArgs {
  const uint16_t* x;        // bf16 [tokens, kdim]
  const uint32_t* w[2];     // per projection: u32 [E_local, rows, kdim*bits/32]
  const uint16_t* s[2];     // bf16 [E_local, rows, kdim/64]
  const uint16_t* b[2];
  int kdim, rows, rows_per_cta;
  int mode;                 // ItemMode
  // grouped items: CTA x-index i serves active[i]'s slots offsets[e]..offsets[e+1];
  // slot s is row s - offsets[expert_begin] of out (and of x when x_by_slot)
  const int32_t* active;
  const int32_t* active_count;
  const int32_t* offsets;
  const int32_t* perm;
  int k_div;                // token of slot s = perm[s] / k_div
  int x_by_slot;            // 1: x row of slot s is s itself (the down projection)
  int expert_begin;
  // gather items: CTA x-index i serves index i, token i / rep, expert gather_idx[i]
  // (gather_idx null: expert 0 for every index)
  const uint32_t* gather_idx;
  long long rep;
  int num_experts;
  uint16_t* out;            // bf16 [slots, out_stride], row r of slot s at out[s*out_stride + r]
  long long out_stride;
  int act;                  // 0 SwiGLU, 1 GeGLU (two-projection form only)
  int* err;
};
size_t qgemv_smem_bytes(int nproj, int rows_per_cta, int kdim, int bits);
// grid: x = items (active experts or indices), y = row blocks.
cudaError_t launch_qgemv(const QGemvArgs& a, int nproj, int bits, int num_items, cudaStream_t st);
bool qgemv_supported(int kdim, int bits);

// --------------------------------------------------------------- combine
struct CombineArgs {
  const uint16_t* d;        // bf16 [P, H] expert outputs in slot order
  const int32_t* inverse;   // [T*K]
  const float* weights;     // [T*K]
  const uint16_t* shared_out;  // bf16 [rows, H] or null; row i holds token shared_row0 + i
  int shared_row0;
  const float* shared_gate;    // fp32 [T] gate per token (already sigmoid) or null
  const uint16_t* residual;    // bf16 [T, H] added before rounding (fused residual) or null
  uint16_t* y;              // bf16 [T, H]
  // Token-local expert parallelism: y, residual and shared_gate hold only
  // this rank's tokens, row i = global token local_row0 + i (0 otherwise).
  int local_row0;
  float* y_f32;             // optional fp32 copy
  int hidden, top_k;
};
cudaError_t launch_combine(const CombineArgs& a, int num_tokens, cudaStream_t st);

// -------------------------------------------------- tensor-core GEMM
struct TcGemmArgs {
  const uint16_t* s[2];     // bf16 scales per projection [E_local, rows, kdim/64]
  const uint16_t* b[2];     // bf16 biases
  int rows, kdim, m_tiles;  // rows = output features per expert (multiple of 128)
  const int32_t* active;
  const int32_t* active_count;
  const int32_t* offsets;
  int expert_begin;
  uint16_t* out;            // [slots, out_stride]: fp16 (two-projection form) or bf16 (one)
  long long out_stride;
  int act;                  // 0 SwiGLU, 1 GeGLU (two-projection form)
  int* err;
  // Group-scaled two-projection form: per slot row the B operand's 64-column
  // group sums x 2^-24 ([slots + 16, kdim/64] fp32, from gather_rows); the
  // one-projection form computes its own.
  const float* xsum;
  // Slots are local: slot s of the tile list is row s - offsets[expert_begin]
  // of the activation, h and out buffers, which hold slot_cap rows (0: no
  // limit); rows past slot_cap are not computed (kDevSlotOverflow).
  int slot_cap;
  // With cnt_hi > 0 only experts whose slot count c (before any slot_cap
  // clipping) satisfies cnt_lo <= c < cnt_hi get tiles: a call splits its
  // experts between the warp-MMA and the tcgen05 kernels by their load.
  int cnt_lo, cnt_hi;
};
size_t tc_smem_bytes(int bits, int nproj, int bn, int kdim);
bool tc_supported(int rows, int kdim, int bits, int nproj, int bn);
// tiles_upper: an upper bound on the tile count (the grid is sized from it).
cudaError_t launch_tc_gemm(const CUtensorMap& tA0, const CUtensorMap& tA1, const CUtensorMap& tB,
                           const TcGemmArgs& a, int bits, int nproj, int bn, int tiles_upper, cudaStream_t st);
// 2-D tiled tensor map (row-major [outer, inner], no interleave, zero OOB fill).
cudaError_t make_tmap_2d(CUtensorMap* map, const void* base, CUtensorMapDataType dtype, uint64_t inner,
                         uint64_t outer, uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer,
                         bool swizzle128);
// x_sorted[s - s0, :] = fp16(x[perm[s] / k_div, :]) for s < num_slots (x bf16, rows of
// `hidden`; s0 = offsets[eb], 0 without offsets); a value outside fp16 range
// records kDevFp16Range in *err.  With slot_cap > 0 rows past it are skipped
// (kDevSlotOverflow).
// With `offsets` non-null only the slots of experts [eb, ee), i.e. slots
// offsets[eb] .. offsets[ee], are gathered (the layer always passes them:
// slots past offsets[E] hold no placed pair when the dispatch rejected an
// out-of-range expert id).  `order` selects the k order of
// the consuming kernel: kOrderTc (tcgen05, kperm8), kOrderMma (warp-MMA
// dequantising form, kperm256, 256-column stages; hidden % 256 == 0) or
// kOrderMmaG4 (warp-MMA group-scaled form, kperm_g4 with odd columns / 16;
// hidden % 64 == 0).
enum ActivationOrder { kOrderTc = 0, kOrderMma = 1, kOrderMmaG4 = 2 };
// Where the gather finds token rows: x itself (world == 0), or, for
// token-local expert parallelism, the owner rank's exchange buffer over
// NVLink: token g of rank q (begin[q] <= g < begin[q+1]) is row g - begin[q]
// of base[q] (plain peer loads; no TMA reads peer memory).
constexpr int kPeerRowsMax = 8;
struct PeerRows {
  const uint16_t* base[kPeerRowsMax];
  int begin[kPeerRowsMax + 1];
  int world;
};
// With kOrderMmaG4 and `group_sums` non-null, group_sums[s * hidden/64 + G]
// also receives 2^-24 * (the fp32 sum of x[perm[s]/k_div, 64 G .. 64 G + 63])
// for every gathered slot: the group sums the group-scaled gate/up kernel
// post-scales with.  With `one_group` non-null (int32 [4]) the kernel also
// writes a one-group tile list for the consuming GEMMs: offsets {0,
// num_slots}, active {0}, count 1 (the shared expert as a grouped GEMM of
// one expert over every gathered row).  With cnt_hi > 0 (needs `ids`, the
// [T, K] expert ids perm indexes, and `offsets`) only the slots of experts
// with cnt_lo <= slots < cnt_hi are gathered: one call per kernel class when
// a forward splits its experts between the warp-MMA and tcgen05 kernels.
cudaError_t launch_gather_rows(const uint16_t* x, const int32_t* perm, int k_div, uint16_t* x_sorted,
                               int num_slots, int hidden, int* err, cudaStream_t st,
                               const int32_t* offsets = nullptr, int eb = 0, int ee = 0, int order = kOrderTc,
                               float* group_sums = nullptr, int32_t* one_group = nullptr,
                               const PeerRows* peer_rows = nullptr, int slot_cap = 0,
                               const int32_t* ids = nullptr, int cnt_lo = 0, int cnt_hi = 0);

// ------------------------------------------- warp-MMA expert GEMM (decode)
// Same arguments as the tcgen05 GEMM (TcGemmArgs; out holds h as fp16 in
// the activation order of the form for the two-projection form, bf16 d for
// the one-projection form).  tA*: packed codes [E_local*rows, words] u32,
// 32-word x 128-row boxes, SWIZZLE_128B; tB: fp16 [slots, kdim] in the
// form's activation order, 64-column x 8*nt-row boxes, SWIZZLE_128B.
// nt in {1, 2, 4}: 8*nt slots per tile.  g4 selects the group-scaled form
// (kOrderMmaG4 activations; 4-bit, nt <= 2, scale / bias arrays 4-byte
// aligned: mma_g4_supported), else the dequantising form (kOrderMma).
size_t mma_smem_bytes(int bits, int nproj, int nt, bool g4);
bool mma_supported(int rows, int kdim, int bits);
bool mma_g4_supported(int bits, int nt, const TcGemmArgs& a);
cudaError_t launch_mma_gemm(const CUtensorMap& tA0, const CUtensorMap& tA1, const CUtensorMap& tB,
                            const TcGemmArgs& a, int bits, int nproj, int nt, bool g4, int tiles_upper,
                            cudaStream_t st);
// Group-scaled down (4-bit, 8 slots per tile) in tiles of two 128-row blocks
// (a.m_tiles = rows / 256; tA with 128-row boxes): the same bits as
// launch_mma_gemm's 128-row tiles, two MMA chains per warp.
bool mma_down_pair_supported(int bits, int nt, const TcGemmArgs& a);
cudaError_t launch_mma_down_pair(const CUtensorMap& tA, const CUtensorMap& tB, const TcGemmArgs& a, int bits, int nt,
                                 int tiles_upper, cudaStream_t st);
// Group-scaled form at two CTAs per SM: 64-row tiles (a.m_tiles = rows / 64;
// tA* with 64-row boxes), 8 slots per tile, 4-bit.
cudaError_t launch_mma_q4(const CUtensorMap& tA0, const CUtensorMap& tA1, const CUtensorMap& tB,
                          const TcGemmArgs& a, int bits, int nproj, int tiles_upper, cudaStream_t st);

// ------------------------------------------------- expert parallelism
constexpr int kEpMaxRanks = 8;
constexpr int kEpReadyOffset = 0;   // u32 index of ready[0] in a rank's flag block
constexpr int kEpDoneOffset = 8;    // u32 index of done[0]
constexpr int kEpRowsOffset = 16;   // u32 index of rows[0]: rank r's combined rows are in this rank's exchange
constexpr int kEpIdsOffset = 24;    // u32 index of ids[0]: rank r's routing and token rows are published
constexpr size_t kEpFlagBytes = 128; // ready[8], done[8], rows[8], ids[8]
// Token ownership of the expert-parallel combine: rank r combines tokens
// [ep_token_begin(T, world, r), ep_token_begin(T, world, r + 1)).
__host__ __device__ inline int ep_token_begin(int num_tokens, int world, int r) {
  return static_cast<int>(static_cast<long long>(num_tokens) * r / world);
}
struct EpArgs {
  int rank, world;
  int bounds[kEpMaxRanks + 1];         // rank r owns experts [bounds[r], bounds[r+1])
  // Tokens rank r combines: global tokens [tok_begin[r], tok_begin[r+1]).
  // Replicated form: contiguous blocks of the shared batch (ep_token_begin);
  // token-local form: each rank's own tokens, in rank order.
  int tok_begin[kEpMaxRanks + 1];
  int local_tokens;                    // 1: token-local form (no combined-row exchange)
  const uint16_t* peer_d[kEpMaxRanks]; // expert rows [P, H] of each rank, mapped here (own included)
  uint16_t* peer_y[kEpMaxRanks];       // combined-row exchange [Tmax, H] of each rank, mapped here (own included)
  uint32_t* peer_flags[kEpMaxRanks];   // flag block of each rank, mapped here (own included)
  uint32_t* flags;                     // this rank's flag block
  uint32_t* epoch;                     // this rank's call counter
  uint32_t* finished;                  // combine CTA completion counter
  uint32_t* published;                 // publish CTA completion counter (token-local form)
  const int32_t* topk_ids;             // [T*K]
  // the call's expert offsets [E + 1] (the same on every rank): rank q's row
  // of global slot s is s - offsets[bounds[q]], below slot_cap (0: no limit)
  const int32_t* offsets;
  int slot_cap;
  // token-local form: every rank's routing arrays (global pair rows), mapped here
  int32_t* peer_ids[kEpMaxRanks];
  float* peer_wts[kEpMaxRanks];
  int top_k;
  int* err;
};
// Waits (bounded) until every peer has finished reading this rank's rows of
// the previous call; advances the call epoch.  Launch before the expert kernels.
cudaError_t launch_ep_fence(const EpArgs& a, cudaStream_t st);
// Announces this rank's expert rows of the call (ready[rank] in every rank's
// flags).  Launch right after the expert kernels.
cudaError_t launch_ep_announce(const EpArgs& a, cudaStream_t st);
// Waits (bounded) for every peer's rows and runs the weighted combine of
// this rank's tokens, reading each pair's row from its owner
// (CombineArgs.d unused); every combined row goes to c.y and to each
// peer's exchange, and the last CTA raises rows[rank] in every peer's flags.
cudaError_t launch_ep_combine(const EpArgs& a, const CombineArgs& c, int num_tokens, cudaStream_t st);
// Partitioned routing, after the router of this rank's n_routed tokens
// (routing rows at global pair rows tok_begin[rank]*K ...): copies the
// routing rows into every peer's routing arrays and the token rows x
// [n_rows, H] (token-local form; 0 rows in the replicated form) into this
// rank's exchange, read by the peers' gathers, then raises ids[rank] in
// every rank's flags.
cudaError_t launch_ep_publish(const EpArgs& a, const uint16_t* x, int n_rows, int n_routed, int hidden,
                              cudaStream_t st);
// Waits (bounded) until every peer has published (ids[*] >= epoch).  Launch
// before the dispatch of the global pair list.
cudaError_t launch_ep_wait_published(const EpArgs& a, cudaStream_t st);
// Waits (bounded) for every peer's combined rows and copies the tokens this
// rank does not own from its exchange into y [T, H].  Launch after the combine.
cudaError_t launch_ep_gather_rows(const EpArgs& a, uint16_t* y, int hidden, int num_tokens, cudaStream_t st);

// Launch with programmatic dependent launch enabled: the kernel may start
// while its predecessor in the stream is still running; it must call
// pdl_wait() (griddepcontrol.wait) before touching the predecessor's output.
// Works the same inside a CUDA-graph capture.
template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                              Args&&... args) {
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...);
}

// Raises a kernel's dynamic shared-memory limit to at least `bytes` on the
// current device.  Only the first call per (kernel, device, size) reaches the
// driver, so launches inside a CUDA-graph capture after a warm-up call make
// no attribute calls.
cudaError_t ensure_dynamic_smem(const void* kernel, size_t bytes);

// sigmoid of a per-token logit, in place.
cudaError_t launch_sigmoid_inplace(float* v, int n, cudaStream_t st);

}  // namespace senmoe
