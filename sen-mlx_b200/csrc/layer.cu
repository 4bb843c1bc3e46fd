// layer.cu -- the C ABI (include/senmoe.h): layer life cycle, forward, and
// the stand-alone router / dispatch / gather_qmm entry points.
//
// SenMoeLayer mirrors DeepseekMoe (src/engine/mlx_lm/models/deepseek_v2.rs:485-553):
// it borrows the caller's device weights in MLX layout and owns only its
// scratch, allocated once at create time for config.max_tokens.  forward is
// stream-ordered, allocation-free and never synchronises the host.

#include <cuda_runtime.h>

#include <cmath>
#include <map>
#include <mutex>
#include <utility>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <new>
#include <string>
#include <vector>

#include "../../include/senmoe.h"
#include "kernels.h"

using namespace senmoe;

namespace senmoe {
cudaError_t ensure_dynamic_smem(const void* kernel, size_t bytes) {
  static std::mutex mu;
  static std::map<std::pair<const void*, int>, size_t> done;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  std::lock_guard<std::mutex> lock(mu);
  size_t& cur = done[{kernel, dev}];
  if (bytes <= cur) return cudaSuccess;
  e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(bytes));
  if (e == cudaSuccess) cur = bytes;
  return e;
}
}  // namespace senmoe

namespace {

thread_local std::string g_last_error;

int fail(int status, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return status;
}

#define SENMOE_CUDA(call)                                                                            \
  do {                                                                                               \
    cudaError_t e_ = (call);                                                                         \
    if (e_ != cudaSuccess)                                                                           \
      return fail(e_ == cudaErrorNotSupported ? SENMOE_ERR_UNSUPPORTED : SENMOE_ERR_CUDA, "%s: %s (%s:%d)", \
                  #call, cudaGetErrorString(e_), __FILE__, __LINE__);                                \
  } while (0)

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Rows of one CTA for the grouped GEMV: gate/up rows (two projections) and
// down rows.  Both keep one CTA's slice under ~70 KB of shared memory.
constexpr int kGateUpRows = 16;
constexpr int kDownRows = 64;

// Tensor-core path: token tiles (N) offered, and the average tokens per
// touched expert from which the tensor cores beat the CUDA-core GEMV.  Tiles
// stop at 128 tokens: TMEM also holds the dequantised A stages, and a
// 256-token tile of gate and up would fill it with accumulators alone.
constexpr int kTcTiles[4] = {16, 32, 64, 128};
constexpr int kTcMaxTile = 3;  // index of the widest tile
// Measured on B200 (4-layer config-1 and config-4 stacks, CUDA-graph replay,
// each path forced): the warp-MMA kernel is fastest for decode-size groups,
// the tcgen05 GEMM from 16 tokens per expert at 4 bits (config 1: 192 against
// 200 us per layer at 256 tokens, 146 against 135 at 128) and from 24 at
// 8 bits, whose dequantisation costs the tcgen05 kernel about twice the ALU
// work; the CUDA-core GEMV is kept for shapes the tensor paths do not support
// and as the forced reference path.
inline double tc_min_tokens_per_expert(int bits) { return bits == 4 ? 16.0 : 24.0; }
// The per-call choice above sees only the mean load per expert.  Skewed
// routing (a few experts holding most pairs) is better served by both
// kernels at once: from kHybridMinPairs pairs, a call on the warp-MMA path
// sends experts with at least kHybridHotSlots slots to the tcgen05 GEMM
// (128-slot tiles, so their weights stream once) and the rest to the
// warp-MMA kernel; each kernel lists only its own experts.  Below that size
// the two extra launches cost more than any skew recovers.
constexpr int kHybridMinPairs = 2048;
constexpr int kHybridHotSlots = 32;
constexpr double kMmaMinTokensPerExpert = 0.0;
enum ExpertPath { kPathAuto = 0, kPathGemv = 1, kPathTensorCore = 2, kPathMma = 3,
                  kPathSingleToken = 4 /* reported only: the one-token fused launch */ };
// SenMoeConfig.reserved[1]: warp-MMA form, 0 = group-scaled where supported
// (4-bit, up to 16 slots per tile; two CTAs per SM at 8 slots), 1 = always
// dequantise to fp16, 2 = group-scaled, one CTA per SM at every tile width,
// 3 = as 2 with 128-row down tiles instead of 256-row ones at 8 slots (same
// bits)
enum MmaForm { kMmaFormAuto = 0, kMmaFormDequant = 1, kMmaFormG4Single = 2, kMmaFormG4Down128 = 3 };
// From this many tokens the router runs as one tensor-core launch (logits
// and top-k, 32 tokens per CTA, so at least 16 CTAs) instead of the CUDA-core
// logits + top-k pair.
constexpr int kRouterTcMinTokens = 512;
// From this many tokens the CUDA-core router runs top-k in its own last CTAs
// (measured: a separate top-k launch is as fast below that).
constexpr int kFusedTopkMinTokens = 128;
// Replicated expert parallelism routes each rank's own block of tokens (and
// exchanges the routing rows) only where the tensor-core router over all
// tokens takes more than one wave of CTAs: each CTA streams all of Wg, so
// below that a smaller block is no faster, and the exchange adds a wait for
// the slowest rank (measured at 2 GPUs with the split from 16 tokens per rank:
// decode 128 tokens 25.1k -> 23.4k tokens/s, prefill 4096 180.5k -> 175.5k).
bool partition_routing(int64_t tokens, int sms) {
  return tokens >= kRouterTcMinTokens && (tokens + kRouterTcTokensPerCta - 1) / kRouterTcTokensPerCta > sms;
}

int tc_tile_index(double tokens_per_expert) {
  for (int i = 0; i < kTcMaxTile; ++i)
    if (tokens_per_expert <= kTcTiles[i]) return i;
  return kTcMaxTile;
}

}  // namespace

struct SenMoeLayer {
  SenMoeConfig cfg{};
  SenMoeWeights w{};
  int device = 0;
  int max_pairs = 0;
  int nchunks_max = 0;
  int slot_cap = 0;  // rows of the per-pair buffers (local expert slots); max_pairs unless capped
  // scratch (one allocation, carved)
  void* arena = nullptr;
  float* logits = nullptr;       // [Tmax, E]
  int32_t* ids = nullptr;        // [Tmax*K]
  float* wts = nullptr;          // [Tmax*K]
  int32_t* perm = nullptr;       // [Tmax*K]
  int32_t* inv = nullptr;        // [Tmax*K]
  int32_t* offsets = nullptr;    // [E+1]
  int32_t* active = nullptr;     // [E]
  int32_t* active_count = nullptr;
  int* err = nullptr;
  int32_t* chunk_hist = nullptr; // [nchunks, E]
  uint16_t* h = nullptr;         // [Tmax*K, I]
  uint16_t* d = nullptr;         // [Tmax*K, H]
  uint16_t* sh_h = nullptr;      // [Tmax, Is]
  uint16_t* sh_out = nullptr;    // [Tmax, H]
  float* sh_gate = nullptr;      // [Tmax]
  uint32_t* zeros_idx = nullptr; // [Tmax] expert 0 for the shared expert
  // tensor-core path
  bool tc_ok = false;
  uint16_t* xs = nullptr;        // fp16 [Tmax*K, H] activations gathered into slot order
  uint16_t* h16 = nullptr;       // fp16 [Tmax*K, I] SwiGLU output (B operand of the down GEMM)
  float* xsum = nullptr;         // [Tmax*K + 16, H/64] group sums of xs (group-scaled gate/up)
  CUtensorMap tm_gate{}, tm_up{}, tm_down{};  // packed codes, [rows, words]
  CUtensorMap tm_gate64{}, tm_up64{}, tm_down64{};  // the same with 64-row boxes (two-CTA form)
  bool q4_ok = false;
  int sms = 148;  // SMs of the layer's device
  CUtensorMap tm_xs[4]{}, tm_h[4]{};          // activation tiles per token-tile width
  int* route_cnt = nullptr;      // fused top-k tile counters [ceil(Tmax/4)] (null: separate top-k)
  // tensor-core prefill router (Wg tensor map; x's is encoded per call)
  bool rtc_ok = false;
  CUtensorMap tm_router{};
  // warp-MMA path
  bool mma_ok = false;
  CUtensorMap tm_xs8{}, tm_h8{};              // 8-slot activation tiles
  // shared expert on the tensor-core kernels: a grouped GEMM of one expert
  // over the rows gathered from x (sh_tc_ok / sh_mma_ok: the shapes allow it)
  bool sh_tc_ok = false, sh_mma_ok = false;
  uint16_t* xs_sh = nullptr;     // fp16 [Tmax, H] gathered rows of x
  uint16_t* hsh16 = nullptr;     // fp16 [Tmax, Is] activation (B operand of the shared down GEMM)
  float* xsum_sh = nullptr;      // [Tmax + 16, H/64] group sums (group-scaled form)
  int32_t* sh_iota = nullptr;    // [Tmax] identity permutation
  int32_t* sh_group = nullptr;   // [4] one-group tile list (written by the shared gather)
  CUtensorMap tm_shg{}, tm_shu{}, tm_shd{};   // shared gate / up / down codes
  CUtensorMap tm_xsh[4]{}, tm_hsh[4]{}, tm_xsh8{}, tm_hsh8{};
  // expert parallelism (senmoe_layer_connect_peers)
  size_t arena_bytes = 0, o_d = 0, o_flags = 0, o_yx = 0, o_ids = 0, o_wts = 0;
  uint32_t* ep_flags = nullptr;  // ready[8], done[8], rows[8]: written by peers
  uint32_t* ep_local = nullptr;  // [0] call epoch, [1] combine CTA counter, [2] publish CTA counter
  int ep_world = 0, ep_rank = 0; // ep_world 0: not connected
  int ep_bounds[kEpMaxRanks + 1] = {};
  const uint16_t* ep_peer_d[kEpMaxRanks] = {};
  uint16_t* ep_peer_y[kEpMaxRanks] = {};     // row exchanges [Tmax, H]: combined rows (replicated
                                             // form) or each rank's own token rows (token-local form)
  int32_t* ep_peer_ids[kEpMaxRanks] = {};    // routing arrays [Tmax*K] of every rank (token-local form)
  float* ep_peer_wts[kEpMaxRanks] = {};
  uint32_t* ep_peer_flags[kEpMaxRanks] = {};
  void* ep_opened[kEpMaxRanks] = {};  // IPC mappings to close
  // per-stage timing
  bool profiling = false;
  bool profiled_once = false;
  cudaEvent_t ev[SENMOE_NUM_STAGES + 1] = {};
  // the shared expert runs on a side stream forked from the caller's at the
  // start of a forward and joined before the combine (its kernels overlap
  // the router, dispatch and routed experts)
  cudaStream_t side = nullptr;
  cudaEvent_t fork_ev = nullptr, join_ev = nullptr;
  // a skewed batch split between the warp-MMA and tcgen05 kernels runs the
  // tcgen05 part (its gather and both products) on this stream, so each
  // kernel's last-round SMs take the other's tiles
  cudaStream_t hyb = nullptr;
  cudaEvent_t hyb_fork = nullptr, hyb_join = nullptr;
  // one token on one GPU: the fused single-launch block (layer_single.cu)
  bool single_ok = false;
  SingleTokenArgs single{};
  unsigned int* gbar = nullptr;  // its grid-barrier word
};

static size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

static int validate_config(const SenMoeConfig* c) {
  if (!c) return fail(SENMOE_ERR_BAD_ARG, "config is NULL");
  const int H = c->hidden_size, I = c->moe_intermediate_size, E = c->n_routed_experts, K = c->num_experts_per_tok;
  if (H <= 0 || I <= 0 || E <= 0 || K <= 0 || K > E)
    return fail(SENMOE_ERR_BAD_ARG, "bad sizes H=%d I=%d E=%d K=%d", H, I, E, K);
  if (c->bits != 4 && c->bits != 8)
    return fail(SENMOE_ERR_UNSUPPORTED, "bits=%d: only 4- and 8-bit affine quantization is supported", c->bits);
  if (c->group_size != 64)
    return fail(SENMOE_ERR_UNSUPPORTED, "group_size=%d: only 64 is supported", c->group_size);
  if (c->router_kind != SENMOE_ROUTER_SOFTMAX_TOPK)
    return fail(SENMOE_ERR_UNSUPPORTED, "router_kind=%d not supported", c->router_kind);
  if (c->activation != SENMOE_ACT_SWIGLU && c->activation != SENMOE_ACT_GEGLU)
    return fail(SENMOE_ERR_BAD_ARG, "activation=%d", c->activation);
  if (!router_supported(H, E, K))
    return fail(SENMOE_ERR_UNSUPPORTED, "router: need H %% 8 == 0, H <= 4096, E <= 512, K <= 16 (H=%d E=%d K=%d)",
                H, E, K);
  if (!qgemv_supported(H, c->bits) || !qgemv_supported(I, c->bits))
    return fail(SENMOE_ERR_UNSUPPORTED, "expert GEMV: H=%d / I=%d not supported at %d bits", H, I, c->bits);
  if (c->shared_intermediate < 0 || (c->shared_intermediate > 0 && !qgemv_supported(c->shared_intermediate, c->bits)))
    return fail(SENMOE_ERR_UNSUPPORTED, "shared_intermediate=%d not supported", c->shared_intermediate);
  if (c->max_tokens <= 0) return fail(SENMOE_ERR_BAD_ARG, "max_tokens=%d", c->max_tokens);
  if ((long long)c->max_tokens * K > (1ll << 30)) return fail(SENMOE_ERR_BAD_ARG, "max_tokens*K too large");
  if (c->expert_begin < 0 || c->expert_end > E || c->expert_begin >= c->expert_end)
    return fail(SENMOE_ERR_BAD_ARG, "local expert range [%d, %d) outside [0, %d)", c->expert_begin, c->expert_end, E);
  return SENMOE_OK;
}

static int validate_weights(const SenMoeConfig* c, const SenMoeWeights* w) {
  if (!w) return fail(SENMOE_ERR_BAD_ARG, "weights is NULL");
  // router_weight may be NULL (a layer used only through senmoe_layer_experts_forward)
  if (w->router_weight && !aligned16(w->router_weight))
    return fail(SENMOE_ERR_BAD_ARG, "router_weight %p is not 16-byte aligned", w->router_weight);
  const void* req[] = {w->gate_weight, w->gate_scales, w->gate_biases, w->up_weight, w->up_scales,
                       w->up_biases,   w->down_weight, w->down_scales, w->down_biases};
  for (const void* p : req) {
    if (!p) return fail(SENMOE_ERR_BAD_ARG, "a required weight pointer is NULL");
    if (!aligned16(p)) return fail(SENMOE_ERR_BAD_ARG, "weight pointer %p is not 16-byte aligned", p);
  }
  if (c->shared_intermediate > 0) {
    const void* sh[] = {w->shared_gate_weight, w->shared_gate_scales, w->shared_gate_biases,
                        w->shared_up_weight,   w->shared_up_scales,   w->shared_up_biases,
                        w->shared_down_weight, w->shared_down_scales, w->shared_down_biases};
    for (const void* p : sh) {
      if (!p) return fail(SENMOE_ERR_BAD_ARG, "a shared-expert weight pointer is NULL");
      if (!aligned16(p)) return fail(SENMOE_ERR_BAD_ARG, "shared-expert pointer %p is not 16-byte aligned", p);
    }
    if (c->shared_gate && !w->shared_gate_vector)
      return fail(SENMOE_ERR_BAD_ARG, "shared_gate set but shared_gate_vector is NULL");
  }
  // Bulk copies move whole row blocks: the scale/bias rows of a block must be
  // 16-byte multiples.
  // Every block start (expert stride, full blocks) and the ragged last block
  // must be 16-byte multiples.
  auto blocks_ok = [](long long rows, long long kdim, long long rows_per_cta) {
    const long long g2 = kdim / 64 * 2;
    return (rows * g2) % 16 == 0 && (rows_per_cta * g2) % 16 == 0 && ((rows % rows_per_cta) * g2) % 16 == 0;
  };
  const int H = c->hidden_size, I = c->moe_intermediate_size, Is = c->shared_intermediate;
  if (!blocks_ok(I, H, kGateUpRows) || !blocks_ok(H, I, kDownRows) ||
      (Is > 0 && (!blocks_ok(Is, H, kGateUpRows) || !blocks_ok(H, Is, kDownRows))))
    return fail(SENMOE_ERR_UNSUPPORTED, "scale/bias blocks of H=%d I=%d Is=%d are not 16-byte multiples", H, I, Is);
  return SENMOE_OK;
}

extern "C" {

const char* senmoe_last_error(void) { return g_last_error.c_str(); }

const char* senmoe_version(void) { return "senmoe 1 sm_100a"; }

int senmoe_selftest_sigmoid(int64_t* mismatches, int64_t* exact_form) {
  g_last_error.clear();
  if (!mismatches || !exact_form) return fail(SENMOE_ERR_BAD_ARG, "output pointer is NULL");
  const cudaError_t e = selftest_sigmoid(mismatches, exact_form);
  if (e != cudaSuccess) return fail(SENMOE_ERR_CUDA, "selftest_sigmoid: %s", cudaGetErrorString(e));
  return SENMOE_OK;
}

int senmoe_layer_create(const SenMoeConfig* config, const SenMoeWeights* weights, int device,
                        SenMoeLayer** out_layer) {
  g_last_error.clear();
  if (!out_layer) return fail(SENMOE_ERR_BAD_ARG, "out_layer is NULL");
  *out_layer = nullptr;
  int rc = validate_config(config);
  if (rc) return rc;
  if ((rc = validate_weights(config, weights))) return rc;
  int cur = 0;
  SENMOE_CUDA(cudaGetDevice(&cur));
  SENMOE_CUDA(cudaSetDevice(device));

  SenMoeLayer* L = new (std::nothrow) SenMoeLayer();
  if (!L) return fail(SENMOE_ERR_NO_MEMORY, "host allocation failed");
  L->cfg = *config;
  L->w = *weights;
  L->device = device;
  const SenMoeConfig& c = L->cfg;
  const size_t T = c.max_tokens, K = c.num_experts_per_tok, E = c.n_routed_experts;
  const size_t H = c.hidden_size, I = c.moe_intermediate_size, Is = c.shared_intermediate;
  const size_t P = T * K;
  L->max_pairs = static_cast<int>(P);
  L->nchunks_max = static_cast<int>((P + kDispatchChunk - 1) / kDispatchChunk);
  // per-pair buffers hold this rank's slots only: up to every pair, or the
  // configured expert-slot capacity (expert parallelism)
  const size_t C = (c.reserved[2] > 0 && size_t(c.reserved[2]) < P) ? size_t(c.reserved[2]) : P;
  L->slot_cap = static_cast<int>(C);

  // carve one arena (256-byte aligned pieces)
  size_t off = 0;
  auto take = [&](size_t bytes) { size_t o = off; off = align_up(off + bytes, 256); return o; };
  const size_t o_logits = take(T * E * 4), o_ids = take(P * 4), o_wts = take(P * 4), o_perm = take(P * 4),
               o_inv = take(P * 4), o_offs = take((E + 1) * 4), o_act = take(E * 4), o_cnt = take(4),
               o_err = take(4), o_hist = take(size_t(L->nchunks_max) * E * 4), o_h = take(C * I * 2),
               o_d = take(C * H * 2), o_shh = take(Is ? T * Is * 2 : 0), o_sho = take(Is ? T * H * 2 : 0),
               o_shg = take(Is ? T * 4 : 0), o_zero = take(Is ? T * 4 : 0), o_xs = take(C * H * 2),
               o_h16 = take(C * I * 2), o_flags = take(kEpFlagBytes), o_local = take(16),
               o_route = take((T + 3) / 4 * 4), o_yx = take(T * H * 2),
               o_xsum = take((C + 16) * (H / 64) * 4), o_xssh = take(Is ? T * H * 2 : 0),
               o_hsh = take(Is ? T * Is * 2 : 0), o_xsumsh = take(Is ? (T + 16) * (H / 64) * 4 : 0),
               o_iota = take(Is ? T * 4 : 0), o_shgrp = take(Is ? 16 : 0), o_gbar = take(16);
  cudaError_t e = cudaMalloc(&L->arena, off);
  if (e != cudaSuccess) {
    delete L;
    cudaSetDevice(cur);
    return fail(SENMOE_ERR_NO_MEMORY, "cudaMalloc(%zu) for layer scratch failed: %s", off, cudaGetErrorString(e));
  }
  char* base = static_cast<char*>(L->arena);
  L->logits = reinterpret_cast<float*>(base + o_logits);
  L->ids = reinterpret_cast<int32_t*>(base + o_ids);
  L->wts = reinterpret_cast<float*>(base + o_wts);
  L->perm = reinterpret_cast<int32_t*>(base + o_perm);
  L->inv = reinterpret_cast<int32_t*>(base + o_inv);
  L->offsets = reinterpret_cast<int32_t*>(base + o_offs);
  L->active = reinterpret_cast<int32_t*>(base + o_act);
  L->active_count = reinterpret_cast<int32_t*>(base + o_cnt);
  L->err = reinterpret_cast<int*>(base + o_err);
  L->chunk_hist = reinterpret_cast<int32_t*>(base + o_hist);
  L->h = reinterpret_cast<uint16_t*>(base + o_h);
  L->d = reinterpret_cast<uint16_t*>(base + o_d);
  if (Is) {
    L->sh_h = reinterpret_cast<uint16_t*>(base + o_shh);
    L->sh_out = reinterpret_cast<uint16_t*>(base + o_sho);
    L->sh_gate = reinterpret_cast<float*>(base + o_shg);
    L->zeros_idx = reinterpret_cast<uint32_t*>(base + o_zero);
    L->xs_sh = reinterpret_cast<uint16_t*>(base + o_xssh);
    L->hsh16 = reinterpret_cast<uint16_t*>(base + o_hsh);
    L->xsum_sh = reinterpret_cast<float*>(base + o_xsumsh);
    L->sh_iota = reinterpret_cast<int32_t*>(base + o_iota);
    L->sh_group = reinterpret_cast<int32_t*>(base + o_shgrp);
  }
  L->xs = reinterpret_cast<uint16_t*>(base + o_xs);
  L->h16 = reinterpret_cast<uint16_t*>(base + o_h16);
  L->route_cnt = reinterpret_cast<int*>(base + o_route);
  L->xsum = reinterpret_cast<float*>(base + o_xsum);
  L->ep_flags = reinterpret_cast<uint32_t*>(base + o_flags);
  L->ep_local = reinterpret_cast<uint32_t*>(base + o_local);
  L->gbar = reinterpret_cast<unsigned int*>(base + o_gbar);
  L->arena_bytes = off;
  L->o_d = o_d;
  L->o_flags = o_flags;
  L->o_yx = o_yx;
  L->o_ids = o_ids;
  L->o_wts = o_wts;
  {  // tensor maps for the tensor-core paths (host-side encoding only)
    const int bits = c.bits, El = c.expert_end - c.expert_begin;
    const uint64_t gw = uint64_t(H) * bits / 32, dw = uint64_t(I) * bits / 32;
    // packed codes: 128-row x 128-byte boxes (32 words), SWIZZLE_128B; a
    // row shorter than a box would need a box wider than the tensor
    bool maps = gw >= 32 && dw >= 32 && I % 128 == 0 && H % 128 == 0;
    maps = maps && make_tmap_2d(&L->tm_gate, L->w.gate_weight, CU_TENSOR_MAP_DATA_TYPE_UINT32, gw,
                                uint64_t(El) * I, gw * 4, 32, 128, true) == cudaSuccess;
    maps = maps && make_tmap_2d(&L->tm_up, L->w.up_weight, CU_TENSOR_MAP_DATA_TYPE_UINT32, gw, uint64_t(El) * I,
                                gw * 4, 32, 128, true) == cudaSuccess;
    maps = maps && make_tmap_2d(&L->tm_down, L->w.down_weight, CU_TENSOR_MAP_DATA_TYPE_UINT32, dw,
                                uint64_t(El) * H, dw * 4, 32, 128, true) == cudaSuccess;
    for (int i = 0; i < 4 && maps; ++i) {
      maps = make_tmap_2d(&L->tm_xs[i], L->xs, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, H, C, H * 2, 64, kTcTiles[i],
                          true) == cudaSuccess &&
             make_tmap_2d(&L->tm_h[i], L->h16, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, I, C, I * 2, 64, kTcTiles[i],
                          true) == cudaSuccess;
    }
    L->tc_ok = maps && tc_supported(int(I), int(H), bits, 2, 128) && tc_supported(int(H), int(I), bits, 1, 128);
    L->mma_ok = maps && mma_supported(int(I), int(H), bits) && mma_supported(int(H), int(I), bits) &&
                make_tmap_2d(&L->tm_xs8, L->xs, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, H, C, H * 2, 64, 8, true) ==
                    cudaSuccess &&
                make_tmap_2d(&L->tm_h8, L->h16, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, I, C, I * 2, 64, 8, true) ==
                    cudaSuccess;
  }
  cudaDeviceGetAttribute(&L->sms, cudaDevAttrMultiProcessorCount, device);
  if (L->mma_ok && c.bits == 4) {
    const int El = c.expert_end - c.expert_begin;
    const uint64_t gw = uint64_t(H) / 8, dw = uint64_t(I) / 8;
    L->q4_ok = make_tmap_2d(&L->tm_gate64, L->w.gate_weight, CU_TENSOR_MAP_DATA_TYPE_UINT32, gw, uint64_t(El) * I,
                            gw * 4, 32, 64, true) == cudaSuccess &&
               make_tmap_2d(&L->tm_up64, L->w.up_weight, CU_TENSOR_MAP_DATA_TYPE_UINT32, gw, uint64_t(El) * I,
                            gw * 4, 32, 64, true) == cudaSuccess &&
               make_tmap_2d(&L->tm_down64, L->w.down_weight, CU_TENSOR_MAP_DATA_TYPE_UINT32, dw, uint64_t(El) * H,
                            dw * 4, 32, 64, true) == cudaSuccess;
  }
  if (Is) {  // the shared expert on the warp-MMA / tcgen05 kernels (one expert, rows Is and H)
    const int bits = c.bits;
    const uint64_t gw = uint64_t(H) * bits / 32, dw = uint64_t(Is) * bits / 32;
    bool maps = gw >= 32 && dw >= 32 && Is % 128 == 0 && H % 128 == 0 &&
                make_tmap_2d(&L->tm_shg, L->w.shared_gate_weight, CU_TENSOR_MAP_DATA_TYPE_UINT32, gw, Is, gw * 4, 32,
                             128, true) == cudaSuccess &&
                make_tmap_2d(&L->tm_shu, L->w.shared_up_weight, CU_TENSOR_MAP_DATA_TYPE_UINT32, gw, Is, gw * 4, 32,
                             128, true) == cudaSuccess &&
                make_tmap_2d(&L->tm_shd, L->w.shared_down_weight, CU_TENSOR_MAP_DATA_TYPE_UINT32, dw, H, dw * 4, 32,
                             128, true) == cudaSuccess;
    for (int i = 0; i < 4 && maps; ++i)
      maps = make_tmap_2d(&L->tm_xsh[i], L->xs_sh, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, H, T, H * 2, 64, kTcTiles[i],
                          true) == cudaSuccess &&
             make_tmap_2d(&L->tm_hsh[i], L->hsh16, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, Is, T, Is * 2, 64, kTcTiles[i],
                          true) == cudaSuccess;
    L->sh_tc_ok = maps && tc_supported(int(Is), int(H), bits, 2, 128) && tc_supported(int(H), int(Is), bits, 1, 128);
    L->sh_mma_ok = maps && mma_supported(int(Is), int(H), bits) && mma_supported(int(H), int(Is), bits) &&
                   make_tmap_2d(&L->tm_xsh8, L->xs_sh, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, H, T, H * 2, 64, 8, true) ==
                       cudaSuccess &&
                   make_tmap_2d(&L->tm_hsh8, L->hsh16, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, Is, T, Is * 2, 64, 8, true) ==
                       cudaSuccess;
  }
  if (L->w.router_weight && !Is && c.expert_begin == 0 && c.expert_end == c.n_routed_experts) {
    SingleTokenArgs& sa = L->single;
    sa.router_weight = static_cast<const uint16_t*>(L->w.router_weight);
    sa.w[0] = static_cast<const uint32_t*>(L->w.gate_weight);
    sa.w[1] = static_cast<const uint32_t*>(L->w.up_weight);
    sa.w[2] = static_cast<const uint32_t*>(L->w.down_weight);
    sa.s[0] = static_cast<const uint16_t*>(L->w.gate_scales);
    sa.s[1] = static_cast<const uint16_t*>(L->w.up_scales);
    sa.s[2] = static_cast<const uint16_t*>(L->w.down_scales);
    sa.b[0] = static_cast<const uint16_t*>(L->w.gate_biases);
    sa.b[1] = static_cast<const uint16_t*>(L->w.up_biases);
    sa.b[2] = static_cast<const uint16_t*>(L->w.down_biases);
    sa.logits = L->logits;
    sa.topk_ids = L->ids;
    sa.topk_weights = L->wts;
    sa.h = L->h;
    sa.grid_bar = L->gbar;
    sa.err = L->err;
    sa.hidden = int(H);
    sa.inter = int(I);
    sa.num_experts = int(E);
    sa.top_k = int(K);
    sa.bits = c.bits;
    sa.norm_topk_prob = c.norm_topk_prob;
    sa.routed_scaling_factor = c.routed_scaling_factor;
    sa.act = c.activation;
    L->single_ok = single_token_plan(sa, L->sms);
  }
  L->rtc_ok = L->w.router_weight && router_tc_supported(int(H), int(E), int(K)) && E >= 128 &&
              make_tmap_2d(&L->tm_router, L->w.router_weight, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, H, E, H * 2, 64, 128,
                           true) == cudaSuccess;
  e = cudaMemset(L->arena, 0, off);
  if (e == cudaSuccess && Is) {  // identity permutation of the shared expert's gather
    std::vector<int32_t> iota(T);
    for (size_t i = 0; i < T; ++i) iota[i] = static_cast<int32_t>(i);
    e = cudaMemcpy(L->sh_iota, iota.data(), T * 4, cudaMemcpyHostToDevice);
  }
  if (e == cudaSuccess && Is) {
    e = cudaStreamCreateWithFlags(&L->side, cudaStreamNonBlocking);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&L->fork_ev, cudaEventDisableTiming);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&L->join_ev, cudaEventDisableTiming);
  }
  if (e == cudaSuccess && L->tc_ok && L->mma_ok) {
    e = cudaStreamCreateWithFlags(&L->hyb, cudaStreamNonBlocking);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&L->hyb_fork, cudaEventDisableTiming);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&L->hyb_join, cudaEventDisableTiming);
  }
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  cudaSetDevice(cur);
  if (e != cudaSuccess) {
    senmoe_layer_destroy(L);
    return fail(SENMOE_ERR_CUDA, "scratch initialisation failed: %s", cudaGetErrorString(e));
  }
  *out_layer = L;
  return SENMOE_OK;
}

int senmoe_layer_destroy(SenMoeLayer* layer) {
  g_last_error.clear();
  if (!layer) return SENMOE_OK;
  int cur = 0;
  cudaGetDevice(&cur);
  cudaSetDevice(layer->device);
  for (auto& ev : layer->ev)
    if (ev) cudaEventDestroy(ev);
  if (layer->fork_ev) cudaEventDestroy(layer->fork_ev);
  if (layer->join_ev) cudaEventDestroy(layer->join_ev);
  if (layer->side) cudaStreamDestroy(layer->side);
  if (layer->hyb_fork) cudaEventDestroy(layer->hyb_fork);
  if (layer->hyb_join) cudaEventDestroy(layer->hyb_join);
  if (layer->hyb) cudaStreamDestroy(layer->hyb);
  for (void* p : layer->ep_opened)
    if (p) cudaIpcCloseMemHandle(p);
  cudaError_t e = cudaFree(layer->arena);
  cudaSetDevice(cur);
  delete layer;
  if (e != cudaSuccess) return fail(SENMOE_ERR_CUDA, "cudaFree: %s", cudaGetErrorString(e));
  return SENMOE_OK;
}

// Expected tokens per touched local expert for `pairs` (token, slot) pairs.
static double tokens_per_expert(const SenMoeLayer* L, int64_t pairs) {
  const SenMoeConfig& c = L->cfg;
  const int64_t e_local = c.expert_end - c.expert_begin;
  // expert-parallel ranks see only their experts' share of the pairs
  if (L->ep_world > 0) pairs = pairs * e_local / c.n_routed_experts;
  if (pairs < 1) pairs = 1;
  return double(pairs) / double(pairs < e_local ? pairs : e_local);
}

// Expert-product kernels one forward of `pairs` pairs takes (ExpertPath).
// One token on one GPU with the automatic kernel choice takes the fused
// single-launch block (layer_single.cu); a forward with debug outputs or
// stage profiling keeps the staged kernels.
static bool single_token_path(const SenMoeLayer* L, int64_t tokens) {
  return tokens == 1 && L->single_ok && L->ep_world == 0 && L->cfg.reserved[0] == kPathAuto &&
         L->cfg.reserved[1] == kMmaFormAuto;
}

static int expert_path_for(const SenMoeLayer* L, int64_t pairs) {
  const int forced = L->cfg.reserved[0];
  if (forced == kPathTensorCore && L->tc_ok) return kPathTensorCore;
  if (forced == kPathMma && L->mma_ok) return kPathMma;
  if (forced == kPathGemv) return kPathGemv;
  if (forced != kPathAuto) return kPathGemv;  // forced path not available for this shape
  const double pe = tokens_per_expert(L, pairs);
  if (pe >= tc_min_tokens_per_expert(L->cfg.bits) && L->tc_ok) return kPathTensorCore;
  if (pe >= kMmaMinTokensPerExpert && L->mma_ok) return kPathMma;
  if (pe >= kMmaMinTokensPerExpert && L->tc_ok) return kPathTensorCore;
  return kPathGemv;
}

// ext_ids / ext_w: routing [T, K] from the caller (Experts::forward), or
// null to run the layer's router.
// tokens_per_rank (host, [ep_world], token-local expert parallelism): x and
// y hold this rank's num_tokens tokens only, which are global tokens
// [sum of the earlier ranks' counts, + num_tokens) of the call.
static int layer_forward(SenMoeLayer* L, const void* x, int64_t num_tokens, void* y, const SenMoeDebug* debug,
                         bool residual, senmoe_stream_t stream, const int32_t* ext_ids = nullptr,
                         const float* ext_w = nullptr, const int64_t* tokens_per_rank = nullptr) {
  g_last_error.clear();
  if (!L) return fail(SENMOE_ERR_BAD_ARG, "layer is NULL");
  const SenMoeConfig& c = L->cfg;
  const bool local = tokens_per_rank != nullptr && L->ep_world > 0;
  int tok_begin[kEpMaxRanks + 1] = {};
  int64_t total = num_tokens;
  if (local) {
    total = 0;
    for (int r = 0; r < L->ep_world; ++r) {
      if (tokens_per_rank[r] < 0 || tokens_per_rank[r] > c.max_tokens)
        return fail(SENMOE_ERR_BAD_ARG, "tokens_per_rank[%d]=%lld outside [0, max_tokens=%d]", r,
                    (long long)tokens_per_rank[r], c.max_tokens);
      tok_begin[r] = static_cast<int>(total);
      total += tokens_per_rank[r];
      tok_begin[r + 1] = static_cast<int>(total);
    }
    if (tokens_per_rank[L->ep_rank] != num_tokens)
      return fail(SENMOE_ERR_BAD_ARG, "tokens_per_rank[%d]=%lld is not this rank's num_tokens=%lld", L->ep_rank,
                  (long long)tokens_per_rank[L->ep_rank], (long long)num_tokens);
    if (ext_ids || debug) return fail(SENMOE_ERR_UNSUPPORTED, "token-local forward takes no routing or debug outputs");
  }
  if (num_tokens < 0 || total > c.max_tokens)
    return fail(SENMOE_ERR_BAD_ARG, "num_tokens=%lld (%lld in all) outside [0, max_tokens=%d]", (long long)num_tokens,
                (long long)total, c.max_tokens);
  if (total == 0) return SENMOE_OK;  // every rank sees the same total: all skip together
  if (num_tokens > 0 && (!x || !y)) return fail(SENMOE_ERR_BAD_ARG, "x or y is NULL");
  if ((x && !aligned16(x)) || (y && !aligned16(y))) return fail(SENMOE_ERR_BAD_ARG, "x and y must be 16-byte aligned");
  if (!ext_ids && !L->w.router_weight)
    return fail(SENMOE_ERR_BAD_ARG, "the layer has no router weight: use senmoe_layer_experts_forward");
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  int32_t* const ids = ext_ids ? const_cast<int32_t*>(ext_ids) : L->ids;   // read-only when given
  float* const wts = ext_w ? const_cast<float*>(ext_w) : L->wts;
  // T: tokens of the call (all ranks' in the token-local form); T_loc, row0:
  // the tokens x holds and the global index of its first row
  const int T = static_cast<int>(total), K = c.num_experts_per_tok, E = c.n_routed_experts;
  const int T_loc = static_cast<int>(num_tokens), row0 = local ? tok_begin[L->ep_rank] : 0;
  const int H = c.hidden_size, I = c.moe_intermediate_size, Is = c.shared_intermediate;
  const int P = T * K;
  if (!local) tok_begin[0] = 0;
  if (local && expert_path_for(L, P) == kPathGemv)
    return fail(SENMOE_ERR_UNSUPPORTED, "token-local expert parallelism needs the tensor-core expert kernels (the "
                                        "CUDA-core GEMV path reads tokens from x)");
  // with a capped expert-slot buffer (fewer rows than pairs) only the
  // expert-parallel tensor-core paths run: they skip and report rows past
  // the cap, where the one-GPU combine and the GEMV would index past it
  const int slot_cap = L->slot_cap < P ? L->slot_cap : 0;
  if (slot_cap && (L->ep_world == 0 || expert_path_for(L, P) == kPathGemv))
    return fail(SENMOE_ERR_UNSUPPORTED, "%d pairs with an expert-slot capacity of %d: a capped layer needs expert "
                "parallelism and the tensor-core expert kernels", P, L->slot_cap);
  // Stage events are recorded only outside a stream capture (inside one a
  // plain record only links the capture's streams).
  bool profile = L->profiling;
  if (profile) {
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    SENMOE_CUDA(cudaStreamIsCapturing(st, &cs));
    profile = cs == cudaStreamCaptureStatusNone;
  }
  auto mark = [&](int stage) -> cudaError_t { return profile ? cudaEventRecord(L->ev[stage], st) : cudaSuccess; };
  SENMOE_CUDA(mark(0));

  // One token on one GPU: the whole block in one persistent launch
  // (layer_single.cu), equal bit for bit to the CUDA-core GEMV path.  Stage
  // profiling, debug outputs, forced kernels and capped slots keep the
  // staged launches.
  if (single_token_path(L, T) && !local && !ext_ids && !debug && !profile && slot_cap == 0) {
    SingleTokenArgs sa = L->single;
    sa.x = static_cast<const uint16_t*>(x);
    sa.residual = residual ? static_cast<const uint16_t*>(x) : nullptr;
    sa.y = static_cast<uint16_t*>(y);
    SENMOE_CUDA(launch_single_token_layer(sa, L->sms, st));
    return SENMOE_OK;
  }

  const bool ep = L->ep_world > 0;
  EpArgs ea{};
  if (ep) {
    ea.rank = L->ep_rank;
    ea.world = L->ep_world;
    for (int r = 0; r <= L->ep_world; ++r) {
      ea.bounds[r] = L->ep_bounds[r];
      ea.tok_begin[r] = local ? tok_begin[r] : ep_token_begin(T, L->ep_world, r);
    }
    ea.local_tokens = local ? 1 : 0;
    for (int r = 0; r < L->ep_world; ++r) {
      ea.peer_d[r] = L->ep_peer_d[r];
      ea.peer_y[r] = L->ep_peer_y[r];
      ea.peer_flags[r] = L->ep_peer_flags[r];
      ea.peer_ids[r] = L->ep_peer_ids[r];
      ea.peer_wts[r] = L->ep_peer_wts[r];
    }
    ea.flags = L->ep_flags;
    ea.epoch = L->ep_local;
    ea.finished = L->ep_local + 1;
    ea.published = L->ep_local + 2;
    ea.topk_ids = ids;
    ea.offsets = L->offsets;
    ea.slot_cap = slot_cap;
    ea.top_k = K;
    ea.err = L->err;
  }
  // 5. shared expert (deepseek_v2.rs:550-552), optionally sigmoid-gated.
  // On the tensor-core kernels it is a grouped GEMM of one expert over the
  // rows of x this rank combines (all of them on one GPU): sh_out row i is
  // token sh_t0 + i.  Otherwise the CUDA-core GEMV over every token.
  int sh_t0 = 0;  // sh_out row i is token sh_t0 + i
  auto run_shared = [&](cudaStream_t s5) -> int {
    // the tokens this rank combines (global indices own_t0 ..); the
    // token-local form holds exactly those in x
    const int sh_n = local ? T_loc : ep ? ea.tok_begin[L->ep_rank + 1] - ea.tok_begin[L->ep_rank] : T;
    const int own_t0 = local ? row0 : ep ? ea.tok_begin[L->ep_rank] : 0;
    const int forced = c.reserved[0];
    int sh_path = kPathGemv;
    if (forced == kPathTensorCore && L->sh_tc_ok) sh_path = kPathTensorCore;
    else if (forced == kPathMma && L->sh_mma_ok) sh_path = kPathMma;
    // kernel and tile width follow the call's token count T, the same on every
    // expert-parallel rank and on one GPU, so each token's shared output is
    // bit-identical however the tokens are split
    else if (forced == kPathAuto)
      sh_path = (T >= tc_min_tokens_per_expert(c.bits) && L->sh_tc_ok) ? kPathTensorCore
                : L->sh_mma_ok                                  ? kPathMma
                : L->sh_tc_ok                                   ? kPathTensorCore
                                                                : kPathGemv;
    if (sh_path != kPathGemv) {
      sh_t0 = own_t0;  // the GEMV below writes every token's row instead
      TcGemmArgs sa{};
      sa.s[0] = static_cast<const uint16_t*>(L->w.shared_gate_scales);
      sa.b[0] = static_cast<const uint16_t*>(L->w.shared_gate_biases);
      sa.s[1] = static_cast<const uint16_t*>(L->w.shared_up_scales);
      sa.b[1] = static_cast<const uint16_t*>(L->w.shared_up_biases);
      sa.rows = Is;
      sa.kdim = H;
      sa.m_tiles = Is / 128;
      sa.offsets = L->sh_group;       // {0, sh_n}, written by the gather below
      sa.active = L->sh_group + 2;    // {0}
      sa.active_count = L->sh_group + 3;
      sa.expert_begin = 0;
      sa.out = L->hsh16;
      sa.out_stride = Is;
      sa.act = c.activation;
      sa.err = L->err;
      sa.xsum = L->xsum_sh;
      TcGemmArgs sd = sa;
      sd.s[0] = sd.s[1] = static_cast<const uint16_t*>(L->w.shared_down_scales);
      sd.b[0] = sd.b[1] = static_cast<const uint16_t*>(L->w.shared_down_biases);
      sd.rows = H;
      sd.kdim = Is;
      sd.m_tiles = H / 128;
      sd.out = L->sh_out;
      sd.out_stride = H;
      const uint16_t* xs_src = static_cast<const uint16_t*>(x) + static_cast<size_t>(sh_t0 - row0) * H;
      if (sh_n > 0 && sh_path == kPathMma) {
        const int nt = T <= 8 ? 1 : (T <= 16 ? 2 : 4);
        const CUtensorMap& tb_x = nt == 1 ? L->tm_xsh8 : L->tm_xsh[nt == 2 ? 0 : 1];
        const CUtensorMap& tb_h = nt == 1 ? L->tm_hsh8 : L->tm_hsh[nt == 2 ? 0 : 1];
        const bool g4 = mma_g4_supported(c.bits, nt, sa) &&
                        (c.reserved[1] == kMmaFormG4Single || c.reserved[1] == kMmaFormG4Down128 ||
                         (c.reserved[1] == kMmaFormAuto && nt == 1));
        SENMOE_CUDA(launch_gather_rows(xs_src, L->sh_iota, 1, L->xs_sh, sh_n, H, L->err, st, nullptr, 0, 0,
                                       g4 ? kOrderMmaG4 : kOrderMma, g4 ? L->xsum_sh : nullptr, L->sh_group));
        SENMOE_CUDA(launch_mma_gemm(L->tm_shg, L->tm_shu, tb_x, sa, c.bits, 2, nt, g4,
                                    (sh_n / (8 * nt) + 1) * sa.m_tiles, s5));
        SENMOE_CUDA(launch_mma_gemm(L->tm_shd, L->tm_shd, tb_h, sd, c.bits, 1, nt, g4,
                                    (sh_n / (8 * nt) + 1) * sd.m_tiles, s5));
      } else if (sh_n > 0) {
        const int ti = tc_tile_index(double(T)), bn = kTcTiles[ti];
        SENMOE_CUDA(launch_gather_rows(xs_src, L->sh_iota, 1, L->xs_sh, sh_n, H, L->err, st, nullptr, 0, 0,
                                       kOrderTc, nullptr, L->sh_group));
        SENMOE_CUDA(launch_tc_gemm(L->tm_shg, L->tm_shu, L->tm_xsh[ti], sa, c.bits, 2, bn,
                                   (sh_n / bn + 1) * sa.m_tiles, s5));
        SENMOE_CUDA(launch_tc_gemm(L->tm_shd, L->tm_shd, L->tm_hsh[ti], sd, c.bits, 1, bn,
                                   (sh_n / bn + 1) * sd.m_tiles, s5));
      }
    } else {
      sh_t0 = row0;  // every token x holds, row i = global token row0 + i
      QGemvArgs sg{};
      sg.x = static_cast<const uint16_t*>(x);
      sg.w[0] = L->w.shared_gate_weight;
      sg.s[0] = static_cast<const uint16_t*>(L->w.shared_gate_scales);
      sg.b[0] = static_cast<const uint16_t*>(L->w.shared_gate_biases);
      sg.w[1] = L->w.shared_up_weight;
      sg.s[1] = static_cast<const uint16_t*>(L->w.shared_up_scales);
      sg.b[1] = static_cast<const uint16_t*>(L->w.shared_up_biases);
      sg.kdim = H;
      sg.rows = Is;
      sg.rows_per_cta = kGateUpRows;
      sg.mode = kItemsGather;
      sg.gather_idx = L->zeros_idx;
      sg.rep = 1;
      sg.num_experts = 1;
      sg.out = L->sh_h;
      sg.out_stride = Is;
      sg.act = c.activation;
      sg.err = L->err;
      SENMOE_CUDA(launch_qgemv(sg, 2, c.bits, T_loc, s5));
      QGemvArgs sd = sg;
      sd.x = L->sh_h;
      sd.w[0] = L->w.shared_down_weight;
      sd.s[0] = static_cast<const uint16_t*>(L->w.shared_down_scales);
      sd.b[0] = static_cast<const uint16_t*>(L->w.shared_down_biases);
      sd.kdim = Is;
      sd.rows = H;
      sd.rows_per_cta = kDownRows;
      sd.out = L->sh_out;
      sd.out_stride = H;
      SENMOE_CUDA(launch_qgemv(sd, 1, c.bits, T_loc, s5));
    }
    if (c.shared_gate) {
      RouterArgs gr{};
      gr.x = static_cast<const uint16_t*>(x);  // every token x holds (combine: row t - local_row0)
      gr.hidden = H;
      gr.top_k = K;
      gr.err = L->err;
      gr.num_tokens = T_loc;
      gr.weight = static_cast<const uint16_t*>(L->w.shared_gate_vector);
      gr.logits = L->sh_gate;
      gr.num_experts = 1;
      gr.round_logits = 0;
      gr.tile_cnt = nullptr;  // a plain dot product: no top-k
      if (T_loc > 0) {        // per token of x (combine: row t - local_row0)
        SENMOE_CUDA(launch_router_logits(gr, s5));
        SENMOE_CUDA(launch_sigmoid_inplace(L->sh_gate, T_loc, s5));
      }
    }
    return SENMOE_OK;
  };
  // With stage profiling the shared expert runs in its own stage, after the
  // routed experts; otherwise it is forked onto the layer's side stream
  // here, so that its kernels overlap the router, dispatch and routed expert
  // launches (it reads only x), and joined before the combine.
  const bool overlap_shared = Is > 0 && !profile && L->side;
  if (overlap_shared) {
    SENMOE_CUDA(cudaEventRecord(L->fork_ev, st));
    SENMOE_CUDA(cudaStreamWaitEvent(L->side, L->fork_ev, 0));
    const int rc = run_shared(L->side);
    if (rc != SENMOE_OK) return rc;
    SENMOE_CUDA(cudaEventRecord(L->join_ev, L->side));
  }

  // Routing is partitioned by token: the token-local form routes the tokens
  // x holds; the replicated form, where partition_routing says so, routes the
  // block of tokens its combine owns.  Either way the rows are published to
  // every rank before the dispatch of all pairs.
  const bool part = local || (ep && !ext_ids && L->rtc_ok && partition_routing(T, L->sms));
  const int r_begin = local ? row0 : part ? ea.tok_begin[L->ep_rank] : 0;
  const int r_count = local ? T_loc : part ? ea.tok_begin[L->ep_rank + 1] - r_begin : T;
  const uint16_t* r_x = static_cast<const uint16_t*>(x) + static_cast<size_t>(local ? 0 : r_begin) * H;
  // the call epoch first (the publish carries it)
  if (part) SENMOE_CUDA(launch_ep_fence(ea, st));

  // 1. router (deepseek_v2.rs:528-543), over the tokens routed here; the
  // kernel is picked by the call's token count T, so each token's routing is
  // bit-identical however the tokens are split across ranks
  RouterArgs ra{};
  ra.x = r_x;
  ra.weight = static_cast<const uint16_t*>(L->w.router_weight);
  ra.logits = L->logits;
  ra.topk_ids = L->ids + static_cast<size_t>(r_begin) * K;
  ra.topk_weights = L->wts + static_cast<size_t>(r_begin) * K;
  ra.num_tokens = r_count;
  ra.hidden = H;
  ra.num_experts = E;
  ra.top_k = K;
  ra.norm_topk_prob = c.norm_topk_prob;
  ra.routed_scaling_factor = c.routed_scaling_factor;
  ra.round_logits = 1;
  ra.err = L->err;

  // 2. dispatch
  DispatchArgs da{};
  da.topk_ids = ids;
  da.num_pairs = P;
  da.num_experts = E;
  da.expert_begin = c.expert_begin;
  da.expert_end = c.expert_end;
  da.perm = L->perm;
  da.inverse = L->inv;
  da.offsets = L->offsets;
  da.active = L->active;
  da.active_count = L->active_count;
  da.chunk_hist = L->chunk_hist;
  da.err = L->err;
  da.keep_remote_slots = ep ? 1 : 0;  // the combine reads remote slots from their owners
  // token-local form: every rank's routing rows are needed before the
  // dispatch of the call's global pair list
  auto exchange_routing = [&]() -> cudaError_t {
    if (!part) return cudaSuccess;
    // the token-local form also publishes its token rows (the peers' gathers read them)
    cudaError_t e = launch_ep_publish(ea, static_cast<const uint16_t*>(x), local ? T_loc : 0, r_count, H, st);
    return e == cudaSuccess ? launch_ep_wait_published(ea, st) : e;
  };
  if (ext_ids) {
    SENMOE_CUDA(mark(1));  // routing given by the caller
    SENMOE_CUDA(launch_dispatch(da, st));
  } else if (r_count == 0) {  // a rank with no tokens to route
    SENMOE_CUDA(exchange_routing());
    SENMOE_CUDA(mark(1));
    SENMOE_CUDA(launch_dispatch(da, st));
  } else if (L->rtc_ok && T >= kRouterTcMinTokens) {
    // prefill sizes: logits on the tensor cores and top-k in one launch
    CUtensorMap tm_x;
    SENMOE_CUDA(make_tmap_2d(&tm_x, r_x, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, H, r_count, uint64_t(H) * 2, 64, 32, true));
    SENMOE_CUDA(launch_router_tc(tm_x, L->tm_router, ra, st));
    SENMOE_CUDA(exchange_routing());
    SENMOE_CUDA(mark(1));
    SENMOE_CUDA(launch_dispatch(da, st));
  } else if (L->route_cnt && T >= kFusedTopkMinTokens) {
    // one launch: logits, then top-k by the last CTA of each 4-token tile
    RouterArgs rf = ra;
    rf.tile_cnt = L->route_cnt;
    SENMOE_CUDA(launch_router_logits(rf, st));
    SENMOE_CUDA(exchange_routing());
    SENMOE_CUDA(mark(1));
    SENMOE_CUDA(launch_dispatch(da, st));
  } else if (!part && router_topk_dispatch_supported(static_cast<int>(T), P, E)) {
    // 1-8 tokens: logits, then top-k and the dispatch in one CTA
    SENMOE_CUDA(launch_router_logits(ra, st));
    SENMOE_CUDA(launch_router_topk_dispatch(ra, da, st));
    SENMOE_CUDA(mark(1));
  } else {
    SENMOE_CUDA(launch_router_logits(ra, st));
    SENMOE_CUDA(launch_router_topk(ra, st));
    SENMOE_CUDA(exchange_routing());
    SENMOE_CUDA(mark(1));
    SENMOE_CUDA(launch_dispatch(da, st));
  }
  // d is about to be overwritten: wait until the peers have read the last
  // call's rows (a partitioned routing did so first of all)
  if (ep && !part) SENMOE_CUDA(launch_ep_fence(ea, st));
  // token-local form: the gathers read each token's row from its owner's exchange
  PeerRows prow{};
  if (local) {
    prow.world = L->ep_world;
    for (int r = 0; r < L->ep_world; ++r) prow.base[r] = L->ep_peer_y[r];
    for (int r = 0; r <= L->ep_world; ++r) prow.begin[r] = tok_begin[r];
  }
  const PeerRows* prow_p = local ? &prow : nullptr;

  // 3-4. expert products over the touched local experts: h [P, I], d [P, H]
  const int E_local = c.expert_end - c.expert_begin;
  const int max_items = P < E_local ? P : E_local;
  const double per_expert = tokens_per_expert(L, P);
  const int path = expert_path_for(L, P);
  if (path == kPathMma) {
    const int nt = per_expert <= 8.0 ? 1 : (per_expert <= 16.0 ? 2 : 4);  // slots per tile: 8 * nt
    const CUtensorMap& tb_x = nt == 1 ? L->tm_xs8 : L->tm_xs[nt == 2 ? 0 : 1];
    const CUtensorMap& tb_h = nt == 1 ? L->tm_h8 : L->tm_h[nt == 2 ? 0 : 1];
    TcGemmArgs ga{};
    ga.s[0] = static_cast<const uint16_t*>(L->w.gate_scales);
    ga.b[0] = static_cast<const uint16_t*>(L->w.gate_biases);
    ga.s[1] = static_cast<const uint16_t*>(L->w.up_scales);
    ga.b[1] = static_cast<const uint16_t*>(L->w.up_biases);
    ga.rows = I;
    ga.kdim = H;
    ga.m_tiles = I / 128;
    ga.active = L->active;
    ga.active_count = L->active_count;
    ga.offsets = L->offsets;
    ga.expert_begin = c.expert_begin;
    ga.out = L->h16;
    ga.out_stride = I;
    ga.act = c.activation;
    ga.err = L->err;
    // group-scaled form (4-bit, up to 16 slots per tile) unless the
    // dequantising form is forced
    // Form (measured on the 48-layer decode stack): the group-scaled form
    // wins at 8-slot tiles, the dequantising form from 16 slots on (the
    // group-scaled post-scale grows with the slot count, dequantisation
    // does not); the two-CTA kernel only while the 128-row gate/up tiles
    // cannot fill the SMs (about one token per expert).
    const bool g4 = mma_g4_supported(c.bits, nt, ga) &&
                    (c.reserved[1] == kMmaFormG4Single || c.reserved[1] == kMmaFormG4Down128 ||
                     (c.reserved[1] == kMmaFormAuto && nt == 1));
    const bool q4 = g4 && nt == 1 && L->q4_ok && c.reserved[1] == kMmaFormAuto && max_items * (I / 128) < L->sms;
    // down in 256-row tiles (two 128-row blocks per warp: two MMA chains, as
    // in gate/up, where a 128-row down tile gives each warp only one) while
    // the expected tiles (uniform routing) still give every SM five or more;
    // with fewer the half as many tiles fill the SMs worse (measured, 48-layer
    // config-1 graphs: -3 % per layer at 32-128 tokens, +1.4 % at 8)
    const int64_t local_pairs = ep ? static_cast<int64_t>(P) * E_local / c.n_routed_experts : P;
    const double touched = E_local * (1.0 - std::pow(1.0 - 1.0 / E_local, static_cast<double>(local_pairs)));
    const bool down_pair = g4 && nt == 1 && !q4 && H % 256 == 0 && touched * (H / 256) >= 5.0 * L->sms &&
                           c.reserved[1] != kMmaFormG4Down128;
    const bool hybrid = P >= kHybridMinPairs && L->tc_ok && c.reserved[0] == kPathAuto && !q4;
    const int hot = kHybridHotSlots, hot_max = 0x7fffffff;
    ga.cnt_lo = 0;
    ga.cnt_hi = hybrid ? hot : 0;
    // the loaded experts' gather and products on the layer's second stream,
    // beside the warp-MMA kernels (disjoint slots of xs, h and d); joined
    // before the combine.  Stage profiling keeps them in line.
    const bool overlap_hybrid = hybrid && !profile && L->hyb;
    cudaStream_t hs = overlap_hybrid ? L->hyb : st;
    if (overlap_hybrid) {
      SENMOE_CUDA(cudaEventRecord(L->hyb_fork, st));
      SENMOE_CUDA(cudaStreamWaitEvent(hs, L->hyb_fork, 0));
    }
    SENMOE_CUDA(launch_gather_rows(static_cast<const uint16_t*>(x), L->perm, K, L->xs, P, H, L->err, st,
                                   L->offsets, c.expert_begin, c.expert_end,
                                   g4 ? kOrderMmaG4 : kOrderMma, g4 ? L->xsum : nullptr, nullptr, prow_p, slot_cap,
                                   ids, ga.cnt_lo, ga.cnt_hi));
    if (hybrid)  // the loaded experts' slots, in the tcgen05 kernel's order
      SENMOE_CUDA(launch_gather_rows(static_cast<const uint16_t*>(x), L->perm, K, L->xs, P, H, L->err, hs,
                                     L->offsets, c.expert_begin, c.expert_end, kOrderTc, nullptr, nullptr, prow_p,
                                     slot_cap, ids, hot, hot_max));
    ga.xsum = L->xsum;
    ga.slot_cap = slot_cap;
    // the loaded experts on the tcgen05 GEMM (gate/up, then down)
    TcGemmArgs ha = ga;
    ha.m_tiles = I / 128;
    ha.cnt_lo = hot;
    ha.cnt_hi = hot_max;
    const int hot_upper = P / kTcTiles[kTcMaxTile] + P / hot;  // slot tiles of the loaded experts, at most
    SENMOE_CUDA(mark(2));
    if (q4) {
      ga.m_tiles = I / 64;
      SENMOE_CUDA(launch_mma_q4(L->tm_gate64, L->tm_up64, tb_x, ga, c.bits, 2, (P / 8 + max_items) * ga.m_tiles, st));
    } else {
      SENMOE_CUDA(launch_mma_gemm(L->tm_gate, L->tm_up, tb_x, ga, c.bits, 2, nt, g4,
                                  (P / (8 * nt) + max_items) * ga.m_tiles, st));
    }
    if (hybrid)
      SENMOE_CUDA(launch_tc_gemm(L->tm_gate, L->tm_up, L->tm_xs[kTcMaxTile], ha, c.bits, 2, kTcTiles[kTcMaxTile],
                                 hot_upper * ha.m_tiles, hs));
    SENMOE_CUDA(mark(3));
    TcGemmArgs gd = ga;
    gd.s[0] = static_cast<const uint16_t*>(L->w.down_scales);
    gd.b[0] = static_cast<const uint16_t*>(L->w.down_biases);
    gd.s[1] = gd.s[0];
    gd.b[1] = gd.b[0];
    gd.rows = H;
    gd.kdim = I;
    gd.m_tiles = H / 128;
    gd.out = L->d;
    gd.out_stride = H;
    if (q4) {
      gd.m_tiles = H / 64;
      SENMOE_CUDA(launch_mma_q4(L->tm_down64, L->tm_down64, tb_h, gd, c.bits, 1, (P / 8 + max_items) * gd.m_tiles,
                                st));
    } else if (down_pair) {
      gd.m_tiles = H / 256;
      SENMOE_CUDA(launch_mma_down_pair(L->tm_down, tb_h, gd, c.bits, nt, (P / (8 * nt) + max_items) * gd.m_tiles, st));
    } else {
      SENMOE_CUDA(launch_mma_gemm(L->tm_down, L->tm_down, tb_h, gd, c.bits, 1, nt, g4,
                                  (P / (8 * nt) + max_items) * gd.m_tiles, st));
    }
    if (hybrid) {
      TcGemmArgs hd = gd;
      hd.m_tiles = H / 128;
      hd.cnt_lo = hot;
      hd.cnt_hi = hot_max;
      SENMOE_CUDA(launch_tc_gemm(L->tm_down, L->tm_down, L->tm_h[kTcMaxTile], hd, c.bits, 1, kTcTiles[kTcMaxTile],
                                 hot_upper * hd.m_tiles, hs));
    }
    if (overlap_hybrid) {
      SENMOE_CUDA(cudaEventRecord(L->hyb_join, hs));
      SENMOE_CUDA(cudaStreamWaitEvent(st, L->hyb_join, 0));
    }
    SENMOE_CUDA(mark(4));
  } else if (path == kPathTensorCore) {
    const int ti = tc_tile_index(per_expert), bn = kTcTiles[ti];
    SENMOE_CUDA(launch_gather_rows(static_cast<const uint16_t*>(x), L->perm, K, L->xs, P, H, L->err, st,
                                   L->offsets, c.expert_begin, c.expert_end, kOrderTc, nullptr, nullptr, prow_p,
                                   slot_cap));
    SENMOE_CUDA(mark(2));
    TcGemmArgs ga{};
    ga.s[0] = static_cast<const uint16_t*>(L->w.gate_scales);
    ga.b[0] = static_cast<const uint16_t*>(L->w.gate_biases);
    ga.s[1] = static_cast<const uint16_t*>(L->w.up_scales);
    ga.b[1] = static_cast<const uint16_t*>(L->w.up_biases);
    ga.rows = I;
    ga.kdim = H;
    ga.m_tiles = I / 128;
    ga.active = L->active;
    ga.active_count = L->active_count;
    ga.offsets = L->offsets;
    ga.expert_begin = c.expert_begin;
    ga.out = L->h16;
    ga.out_stride = I;
    ga.act = c.activation;
    ga.err = L->err;
    ga.slot_cap = slot_cap;
    SENMOE_CUDA(launch_tc_gemm(L->tm_gate, L->tm_up, L->tm_xs[ti], ga, c.bits, 2, bn,
                               (P / bn + max_items) * ga.m_tiles, st));
    SENMOE_CUDA(mark(3));
    TcGemmArgs gd = ga;
    gd.s[0] = static_cast<const uint16_t*>(L->w.down_scales);
    gd.b[0] = static_cast<const uint16_t*>(L->w.down_biases);
    gd.s[1] = gd.s[0];
    gd.b[1] = gd.b[0];
    gd.rows = H;
    gd.kdim = I;
    gd.m_tiles = H / 128;
    gd.out = L->d;
    gd.out_stride = H;
    SENMOE_CUDA(launch_tc_gemm(L->tm_down, L->tm_down, L->tm_h[ti], gd, c.bits, 1, bn,
                               (P / bn + max_items) * gd.m_tiles, st));
    SENMOE_CUDA(mark(4));
  } else {
    SENMOE_CUDA(mark(2));
    QGemvArgs g{};
    g.x = static_cast<const uint16_t*>(x);
    g.w[0] = L->w.gate_weight;
    g.s[0] = static_cast<const uint16_t*>(L->w.gate_scales);
    g.b[0] = static_cast<const uint16_t*>(L->w.gate_biases);
    g.w[1] = L->w.up_weight;
    g.s[1] = static_cast<const uint16_t*>(L->w.up_scales);
    g.b[1] = static_cast<const uint16_t*>(L->w.up_biases);
    g.kdim = H;
    g.rows = I;
    g.rows_per_cta = kGateUpRows;
    g.mode = kItemsGrouped;
    g.active = L->active;
    g.active_count = L->active_count;
    g.offsets = L->offsets;
    g.perm = L->perm;
    g.k_div = K;
    g.x_by_slot = 0;
    g.expert_begin = c.expert_begin;
    g.out = L->h;
    g.out_stride = I;
    g.act = c.activation;
    g.err = L->err;
    SENMOE_CUDA(launch_qgemv(g, 2, c.bits, max_items, st));
    SENMOE_CUDA(mark(3));

    QGemvArgs dn = g;
    dn.x = L->h;
    dn.w[0] = L->w.down_weight;
    dn.s[0] = static_cast<const uint16_t*>(L->w.down_scales);
    dn.b[0] = static_cast<const uint16_t*>(L->w.down_biases);
    dn.kdim = I;
    dn.rows = H;
    dn.rows_per_cta = kDownRows;
    dn.x_by_slot = 1;
    dn.out = L->d;
    dn.out_stride = H;
    SENMOE_CUDA(launch_qgemv(dn, 1, c.bits, max_items, st));
    SENMOE_CUDA(mark(4));
  }

  // expert parallelism: this rank's rows are complete; peers may read them
  if (ep) SENMOE_CUDA(launch_ep_announce(ea, st));

  // 5. the shared expert: joined from the side stream, or run now
  if (Is > 0 && !overlap_shared) {
    const int rc = run_shared(st);
    if (rc != SENMOE_OK) return rc;
  }
  if (overlap_shared) SENMOE_CUDA(cudaStreamWaitEvent(st, L->join_ev, 0));

  SENMOE_CUDA(mark(5));

  // 6. weighted combine (deepseek_v2.rs:546-548) -> y
  CombineArgs ca{};
  ca.d = L->d;
  ca.inverse = L->inv;
  ca.weights = wts;
  ca.shared_out = Is > 0 ? L->sh_out : nullptr;
  ca.shared_row0 = sh_t0;
  ca.local_row0 = row0;
  ca.shared_gate = (Is > 0 && c.shared_gate) ? L->sh_gate : nullptr;
  ca.y = static_cast<uint16_t*>(y);
  ca.residual = residual ? static_cast<const uint16_t*>(x) : nullptr;
  ca.y_f32 = nullptr;
  ca.hidden = H;
  ca.top_k = K;
  if (ep) {
    SENMOE_CUDA(launch_ep_combine(ea, ca, T, st));
    if (!local) SENMOE_CUDA(launch_ep_gather_rows(ea, ca.y, H, T, st));
  } else
    SENMOE_CUDA(launch_combine(ca, T, st));
  SENMOE_CUDA(mark(6));
  if (profile) L->profiled_once = true;

  if (debug) {
    if (debug->topk_ids)
      SENMOE_CUDA(cudaMemcpyAsync(debug->topk_ids, ids, size_t(P) * 4, cudaMemcpyDeviceToDevice, st));
    if (debug->topk_weights)
      SENMOE_CUDA(cudaMemcpyAsync(debug->topk_weights, wts, size_t(P) * 4, cudaMemcpyDeviceToDevice, st));
    if (debug->perm) SENMOE_CUDA(cudaMemcpyAsync(debug->perm, L->perm, size_t(P) * 4, cudaMemcpyDeviceToDevice, st));
    if (debug->offsets)
      SENMOE_CUDA(cudaMemcpyAsync(debug->offsets, L->offsets, size_t(E + 1) * 4, cudaMemcpyDeviceToDevice, st));
  }
  return SENMOE_OK;
}

int senmoe_layer_forward(SenMoeLayer* L, const void* x, int64_t num_tokens, void* y, const SenMoeDebug* debug,
                         senmoe_stream_t stream) {
  return layer_forward(L, x, num_tokens, y, debug, false, stream);
}

int senmoe_layer_forward_residual(SenMoeLayer* L, const void* x, int64_t num_tokens, void* h_out,
                                  senmoe_stream_t stream) {
  return layer_forward(L, x, num_tokens, h_out, nullptr, true, stream);
}

int senmoe_layer_forward_tokens(SenMoeLayer* L, const void* x, int64_t num_tokens, void* y,
                                const int64_t* tokens_per_rank, int32_t residual, senmoe_stream_t stream) {
  g_last_error.clear();
  if (!L) return fail(SENMOE_ERR_BAD_ARG, "layer is NULL");
  if (!tokens_per_rank) return fail(SENMOE_ERR_BAD_ARG, "tokens_per_rank is NULL");
  if (L->ep_world == 0) {  // not connected: one rank holding every token
    if (tokens_per_rank[0] != num_tokens)
      return fail(SENMOE_ERR_BAD_ARG, "tokens_per_rank[0]=%lld is not num_tokens=%lld",
                  (long long)tokens_per_rank[0], (long long)num_tokens);
    return layer_forward(L, x, num_tokens, y, nullptr, residual != 0, stream);
  }
  return layer_forward(L, x, num_tokens, y, nullptr, residual != 0, stream, nullptr, nullptr, tokens_per_rank);
}

int senmoe_layer_expert_path(const SenMoeLayer* L, int64_t num_tokens) {
  g_last_error.clear();
  if (!L) return -fail(SENMOE_ERR_BAD_ARG, "layer is NULL");
  if (num_tokens <= 0) return kPathGemv;
  if (single_token_path(L, num_tokens)) return kPathSingleToken;
  return expert_path_for(L, num_tokens * L->cfg.num_experts_per_tok);
}

int senmoe_layer_set_profiling(SenMoeLayer* L, int enable) {
  g_last_error.clear();
  if (!L) return fail(SENMOE_ERR_BAD_ARG, "layer is NULL");
  int cur = 0;
  SENMOE_CUDA(cudaGetDevice(&cur));
  SENMOE_CUDA(cudaSetDevice(L->device));
  if (enable && !L->ev[0]) {
    for (auto& e : L->ev) SENMOE_CUDA(cudaEventCreate(&e));
  }
  L->profiling = enable != 0;
  L->profiled_once = false;
  SENMOE_CUDA(cudaSetDevice(cur));
  return SENMOE_OK;
}

int senmoe_layer_stage_times(SenMoeLayer* L, float* ms, int n) {
  g_last_error.clear();
  if (!L || !ms || n < 0) return -fail(SENMOE_ERR_BAD_ARG, "bad arguments");
  if (!L->profiled_once) return -fail(SENMOE_ERR_BAD_ARG, "no profiled forward since profiling was enabled");
  cudaError_t e = cudaEventSynchronize(L->ev[SENMOE_NUM_STAGES]);
  if (e != cudaSuccess) return -fail(SENMOE_ERR_CUDA, "cudaEventSynchronize: %s", cudaGetErrorString(e));
  const int m = n < SENMOE_NUM_STAGES ? n : SENMOE_NUM_STAGES;
  for (int i = 0; i < m; ++i) {
    e = cudaEventElapsedTime(&ms[i], L->ev[i], L->ev[i + 1]);
    if (e != cudaSuccess) return -fail(SENMOE_ERR_CUDA, "cudaEventElapsedTime: %s", cudaGetErrorString(e));
  }
  return m;
}

int senmoe_layer_check(SenMoeLayer* L, senmoe_stream_t stream) {
  g_last_error.clear();
  if (!L) return fail(SENMOE_ERR_BAD_ARG, "layer is NULL");
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  int host_err = 0;
  SENMOE_CUDA(cudaMemcpyAsync(&host_err, L->err, sizeof(int), cudaMemcpyDeviceToHost, st));
  SENMOE_CUDA(cudaStreamSynchronize(st));
  if (host_err) {
    SENMOE_CUDA(cudaMemsetAsync(L->err, 0, sizeof(int), st));
    SENMOE_CUDA(cudaStreamSynchronize(st));
    if (host_err == kDevBadExpert) return fail(SENMOE_ERR_DEVICE, "a kernel saw an expert id outside [0, E)");
    if (host_err == kDevWaitTimeout) return fail(SENMOE_ERR_TIMEOUT, "a bounded device-side wait ran out");
    if (host_err == kDevPeerTimeout)
      return fail(SENMOE_ERR_TIMEOUT, "a wait for another expert-parallel rank ran out (a rank missed a forward, "
                                      "or ran a different sequence of forwards)");
    if (host_err == kDevSlotOverflow)
      return fail(SENMOE_ERR_DEVICE, "more pairs reached this rank's experts than its expert-slot capacity (%d); "
                                     "the excess was skipped", L->slot_cap);
    if (host_err == kDevFp16Range)
      return fail(SENMOE_ERR_DEVICE, "an activation outside fp16 range reached the tensor-core path (use the "
                                     "CUDA-core path, expert path 1, for such inputs)");
    return fail(SENMOE_ERR_DEVICE, "device error code %d", host_err);
  }
  return SENMOE_OK;
}

int senmoe_layer_peer_info(const SenMoeLayer* L, SenMoePeerInfo* out) {
  g_last_error.clear();
  if (!L || !out) return fail(SENMOE_ERR_BAD_ARG, "layer or out is NULL");
  static_assert(sizeof(cudaIpcMemHandle_t) == sizeof(out->ipc_handle), "IPC handle size");
  int cur = 0;
  SENMOE_CUDA(cudaGetDevice(&cur));
  SENMOE_CUDA(cudaSetDevice(L->device));
  cudaIpcMemHandle_t h;
  const cudaError_t e = cudaIpcGetMemHandle(&h, L->arena);
  cudaSetDevice(cur);
  if (e != cudaSuccess) return fail(SENMOE_ERR_CUDA, "cudaIpcGetMemHandle: %s", cudaGetErrorString(e));
  std::memset(out, 0, sizeof(*out));
  std::memcpy(out->ipc_handle, &h, sizeof(h));
  out->rows_offset = static_cast<int64_t>(L->o_d);
  out->flags_offset = static_cast<int64_t>(L->o_flags);
  out->arena_bytes = static_cast<int64_t>(L->arena_bytes);
  out->expert_begin = L->cfg.expert_begin;
  out->expert_end = L->cfg.expert_end;
  out->device = L->device;
  return SENMOE_OK;
}

int senmoe_layer_connect_peers(SenMoeLayer* L, int32_t rank, int32_t world_size, const SenMoePeerInfo* peers) {
  g_last_error.clear();
  if (!L || !peers) return fail(SENMOE_ERR_BAD_ARG, "layer or peers is NULL");
  if (L->ep_world) return fail(SENMOE_ERR_BAD_ARG, "layer is already connected");
  if (world_size < 1 || world_size > kEpMaxRanks || rank < 0 || rank >= world_size)
    return fail(SENMOE_ERR_BAD_ARG, "rank %d / world_size %d (at most %d ranks)", rank, world_size, kEpMaxRanks);
  const SenMoeConfig& c = L->cfg;
  if (peers[0].expert_begin != 0 || peers[world_size - 1].expert_end != c.n_routed_experts)
    return fail(SENMOE_ERR_BAD_ARG, "expert ranges must start at 0 and end at %d", c.n_routed_experts);
  for (int r = 0; r < world_size; ++r) {
    const SenMoePeerInfo& p = peers[r];
    if (p.expert_begin >= p.expert_end || (r > 0 && p.expert_begin != peers[r - 1].expert_end))
      return fail(SENMOE_ERR_BAD_ARG, "rank %d expert range [%d, %d) does not continue the previous one", r,
                  p.expert_begin, p.expert_end);
    if (p.arena_bytes != static_cast<int64_t>(L->arena_bytes) || p.rows_offset != static_cast<int64_t>(L->o_d) ||
        p.flags_offset != static_cast<int64_t>(L->o_flags))
      return fail(SENMOE_ERR_BAD_ARG, "rank %d arena layout differs (configs must match apart from the expert range)",
                  r);
  }
  if (peers[rank].expert_begin != c.expert_begin || peers[rank].expert_end != c.expert_end)
    return fail(SENMOE_ERR_BAD_ARG, "peers[%d] is not this layer's entry", rank);
  int cur = 0;
  SENMOE_CUDA(cudaGetDevice(&cur));
  SENMOE_CUDA(cudaSetDevice(L->device));
  char* bases[kEpMaxRanks] = {};
  for (int r = 0; r < world_size; ++r) {
    if (r == rank) {
      bases[r] = static_cast<char*>(L->arena);
      continue;
    }
    cudaIpcMemHandle_t h;
    std::memcpy(&h, peers[r].ipc_handle, sizeof(h));
    void* p = nullptr;
    const cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) {
      for (int q = 0; q < r; ++q)
        if (q != rank && bases[q]) cudaIpcCloseMemHandle(bases[q]);
      cudaSetDevice(cur);
      return fail(SENMOE_ERR_CUDA, "cudaIpcOpenMemHandle(rank %d): %s", r, cudaGetErrorString(e));
    }
    bases[r] = static_cast<char*>(p);
  }
  cudaSetDevice(cur);
  for (int r = 0; r < world_size; ++r) {
    L->ep_peer_d[r] = reinterpret_cast<const uint16_t*>(bases[r] + L->o_d);
    L->ep_peer_y[r] = reinterpret_cast<uint16_t*>(bases[r] + L->o_yx);
    L->ep_peer_flags[r] = reinterpret_cast<uint32_t*>(bases[r] + L->o_flags);
    L->ep_peer_ids[r] = reinterpret_cast<int32_t*>(bases[r] + L->o_ids);
    L->ep_peer_wts[r] = reinterpret_cast<float*>(bases[r] + L->o_wts);
    L->ep_opened[r] = r == rank ? nullptr : bases[r];
    L->ep_bounds[r] = peers[r].expert_begin;
  }
  L->ep_bounds[world_size] = c.n_routed_experts;
  L->ep_rank = rank;
  L->ep_world = world_size;
  return SENMOE_OK;
}

int senmoe_router(const void* x, int64_t num_tokens, const void* router_weight, int32_t hidden, int32_t num_experts,
                  int32_t top_k, int32_t norm_topk_prob, float routed_scaling_factor, float* logits_scratch,
                  int32_t* topk_ids, float* topk_weights, senmoe_stream_t stream) {
  g_last_error.clear();
  if (num_tokens < 0 || num_tokens > (1ll << 28)) return fail(SENMOE_ERR_BAD_ARG, "num_tokens=%lld", (long long)num_tokens);
  if (!router_supported(hidden, num_experts, top_k))
    return fail(SENMOE_ERR_UNSUPPORTED, "router: H=%d E=%d K=%d unsupported", hidden, num_experts, top_k);
  if (num_tokens == 0) return SENMOE_OK;
  if (!x || !router_weight || !logits_scratch || !topk_ids || !topk_weights)
    return fail(SENMOE_ERR_BAD_ARG, "NULL pointer");
  if (!aligned16(x) || !aligned16(router_weight)) return fail(SENMOE_ERR_BAD_ARG, "x / router_weight not 16-byte aligned");
  RouterArgs ra{};
  ra.x = static_cast<const uint16_t*>(x);
  ra.weight = static_cast<const uint16_t*>(router_weight);
  ra.logits = logits_scratch;
  ra.topk_ids = topk_ids;
  ra.topk_weights = topk_weights;
  ra.num_tokens = static_cast<int>(num_tokens);
  ra.hidden = hidden;
  ra.num_experts = num_experts;
  ra.top_k = top_k;
  ra.norm_topk_prob = norm_topk_prob;
  ra.routed_scaling_factor = routed_scaling_factor;
  ra.round_logits = 1;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  SENMOE_CUDA(launch_router_logits(ra, st));
  SENMOE_CUDA(launch_router_topk(ra, st));
  return SENMOE_OK;
}

int senmoe_layer_experts_forward(SenMoeLayer* L, const void* x, int64_t num_tokens, const int32_t* topk_ids,
                                 const float* topk_weights, void* y, senmoe_stream_t stream) {
  g_last_error.clear();
  if (num_tokens > 0 && (!topk_ids || !topk_weights)) return fail(SENMOE_ERR_BAD_ARG, "topk_ids / topk_weights NULL");
  return layer_forward(L, x, num_tokens, y, nullptr, false, stream, topk_ids, topk_weights);
}

int senmoe_gemma_router(const SenMoeGemmaRouter* r, const void* x, int64_t num_tokens, int32_t* topk_ids,
                        float* topk_weights, senmoe_stream_t stream) {
  g_last_error.clear();
  if (!r) return fail(SENMOE_ERR_BAD_ARG, "router is NULL");
  if (num_tokens < 0 || num_tokens > (1ll << 28)) return fail(SENMOE_ERR_BAD_ARG, "num_tokens=%lld", (long long)num_tokens);
  if (!gemma_router_supported(r->hidden_size, r->num_experts, r->top_k, r->bits, r->group_size))
    return fail(SENMOE_ERR_UNSUPPORTED, "gemma router: H=%d E=%d K=%d bits=%d group=%d unsupported", r->hidden_size,
                r->num_experts, r->top_k, r->bits, r->group_size);
  if (!(r->rms_norm_eps >= 0.0f)) return fail(SENMOE_ERR_BAD_ARG, "rms_norm_eps must be >= 0");
  if (num_tokens == 0) return SENMOE_OK;
  if (!x || !r->proj_weight || !r->proj_scales || !r->proj_biases || !r->scale || !r->per_expert_scale ||
      !topk_ids || !topk_weights)
    return fail(SENMOE_ERR_BAD_ARG, "NULL pointer");
  GemmaRouterArgs a{};
  a.x = static_cast<const uint16_t*>(x);
  a.proj_w = r->proj_weight;
  a.proj_s = static_cast<const uint16_t*>(r->proj_scales);
  a.proj_b = static_cast<const uint16_t*>(r->proj_biases);
  a.scale = static_cast<const uint16_t*>(r->scale);
  a.per_expert_scale = static_cast<const uint16_t*>(r->per_expert_scale);
  a.topk_ids = topk_ids;
  a.topk_weights = topk_weights;
  a.num_tokens = static_cast<int>(num_tokens);
  a.hidden = r->hidden_size;
  a.num_experts = r->num_experts;
  a.top_k = r->top_k;
  a.bits = r->bits;
  a.group_size = r->group_size;
  a.eps = r->rms_norm_eps;
  a.root = powf(static_cast<float>(r->hidden_size), -0.5f);  // (hidden_size as f32).powf(-0.5), gemma4.rs:705
  SENMOE_CUDA(launch_gemma_router(a, reinterpret_cast<cudaStream_t>(stream)));
  return SENMOE_OK;
}

int senmoe_dispatch(const int32_t* topk_ids, int64_t num_tokens, int32_t top_k, int32_t num_experts, int32_t* perm,
                    int32_t* inverse, int32_t* offsets, int32_t* scratch, senmoe_stream_t stream) {
  g_last_error.clear();
  if (num_tokens < 0 || top_k <= 0 || num_experts <= 0 || num_experts > 1024 || num_tokens * top_k > (1ll << 30))
    return fail(SENMOE_ERR_BAD_ARG, "bad sizes T=%lld K=%d E=%d", (long long)num_tokens, top_k, num_experts);
  if (num_tokens == 0) return SENMOE_OK;
  if (!topk_ids || !perm || !inverse || !offsets || !scratch) return fail(SENMOE_ERR_BAD_ARG, "NULL pointer");
  DispatchArgs da{};
  da.topk_ids = topk_ids;
  da.num_pairs = static_cast<int>(num_tokens * top_k);
  da.num_experts = num_experts;
  da.expert_begin = 0;
  da.expert_end = num_experts;
  da.perm = perm;
  da.inverse = inverse;
  da.offsets = offsets;
  da.active = scratch;
  da.active_count = scratch + num_experts;
  da.err = scratch + num_experts + 1;
  da.chunk_hist = nullptr;  // single-CTA form
  SENMOE_CUDA(launch_dispatch(da, reinterpret_cast<cudaStream_t>(stream)));
  return SENMOE_OK;
}

// The quantized product behind gather_qmm and the dense quantized Linear:
// out[i, :] = bf16( x[i / (n_indices / x_rows), :] @ dequant(w[idx[i]])^T ),
// idx null = expert 0 for every row (the dense form, num_experts == 1);
// need_idx: the caller's form requires an index list.
static int quantized_product(const char* who, const void* x, int64_t x_rows, const uint32_t* w, const void* scales,
                             const void* biases, const uint32_t* idx, bool need_idx, int64_t n_indices,
                             int64_t in_features, int64_t out_features, int32_t num_experts, int32_t group_size,
                             int32_t bits, void* out, senmoe_stream_t stream) {
  if (bits != 4 && bits != 8) return fail(SENMOE_ERR_UNSUPPORTED, "%s: bits=%d", who, bits);
  if (group_size != 64) return fail(SENMOE_ERR_UNSUPPORTED, "%s: group_size=%d", who, group_size);
  if (x_rows <= 0 || n_indices < 0 || n_indices % x_rows || num_experts <= 0 || out_features <= 0 ||
      n_indices > (1ll << 31) - 1)
    return fail(SENMOE_ERR_BAD_ARG, "%s: x_rows=%lld n_indices=%lld (must be a multiple)", who, (long long)x_rows,
                (long long)n_indices);
  if (in_features <= 0 || in_features > (1 << 20) || !qgemv_supported(static_cast<int>(in_features), bits))
    return fail(SENMOE_ERR_UNSUPPORTED, "%s: in_features=%lld unsupported at %d bits", who,
                (long long)in_features, bits);
  if (n_indices == 0) return SENMOE_OK;
  if (!x || !w || !scales || !biases || !out || (need_idx && !idx)) return fail(SENMOE_ERR_BAD_ARG, "NULL pointer");
  if (!aligned16(x) || !aligned16(w) || !aligned16(scales) || !aligned16(biases))
    return fail(SENMOE_ERR_BAD_ARG, "%s: x / w / scales / biases must be 16-byte aligned", who);
  // Bulk copies move [rows_per_cta, groups] scale blocks: every block start
  // and size must be a 16-byte multiple.
  const int groups = static_cast<int>(in_features / 64);
  int rows_per_cta = 16;
  while ((rows_per_cta * groups * 2) % 16) rows_per_cta *= 2;
  if ((out_features * groups * 2) % 16 || ((out_features % rows_per_cta) * groups * 2) % 16)
    return fail(SENMOE_ERR_UNSUPPORTED, "%s: out_features=%lld with in_features=%lld leaves scale rows that are "
                "not 16-byte multiples", who, (long long)out_features, (long long)in_features);
  QGemvArgs g{};
  g.x = static_cast<const uint16_t*>(x);
  g.w[0] = w;
  g.s[0] = static_cast<const uint16_t*>(scales);
  g.b[0] = static_cast<const uint16_t*>(biases);
  g.kdim = static_cast<int>(in_features);
  g.rows = static_cast<int>(out_features);
  g.rows_per_cta = rows_per_cta;
  g.mode = kItemsGather;
  g.gather_idx = idx;
  g.rep = n_indices / x_rows;
  g.num_experts = num_experts;
  g.out = static_cast<uint16_t*>(out);
  g.out_stride = out_features;
  g.err = nullptr;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  SENMOE_CUDA(launch_qgemv(g, 1, bits, static_cast<int>(n_indices), st));
  return SENMOE_OK;
}

int senmoe_gather_qmm(const void* x, int64_t x_rows, const uint32_t* w, const void* scales, const void* biases,
                      const uint32_t* rhs_indices, int64_t n_indices, int64_t in_features, int64_t out_features,
                      int32_t num_experts, int32_t transpose, int32_t group_size, int32_t bits,
                      int32_t sorted_indices, void* out, senmoe_stream_t stream) {
  (void)sorted_indices;
  g_last_error.clear();
  if (!transpose)
    return fail(SENMOE_ERR_UNSUPPORTED, "gather_qmm: transpose=false is not supported (the reference only uses "
                                        "transpose=true)");
  return quantized_product("gather_qmm", x, x_rows, w, scales, biases, rhs_indices, true, n_indices, in_features,
                           out_features, num_experts, group_size, bits, out, stream);
}

int senmoe_quantized_linear(const void* x, int64_t num_tokens, const uint32_t* w, const void* scales,
                            const void* biases, int64_t in_features, int64_t out_features, int32_t group_size,
                            int32_t bits, void* y, senmoe_stream_t stream) {
  g_last_error.clear();
  if (num_tokens < 0) return fail(SENMOE_ERR_BAD_ARG, "quantized_linear: num_tokens=%lld", (long long)num_tokens);
  if (num_tokens == 0) return SENMOE_OK;
  return quantized_product("quantized_linear", x, num_tokens, w, scales, biases, nullptr, false, num_tokens,
                           in_features, out_features, 1, group_size, bits, y, stream);
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Allocation-free forward.
//
// Some callers cannot allocate device memory when they need a MoE forward:
// code that runs while a CUDA stream capture is open (cudaMalloc is illegal
// there), serving loops whose HBM is fully reserved up front by another
// allocator (a caching pool that owns all free memory), and plugin hosts that
// forbid device allocation on their hot path.  senmoe_moe_forward_noalloc
// serves them: it takes the config and weights directly (no layer handle, no
// create-time allocation) and places all of its scratch in the file-scope
// array below, which every GPU that loads this library holds until exit.
//
// Set-up: the first call on each device looks up the array's device address
// with cudaGetSymbolAddress (a host-side use of the array's name is only a
// stand-in, not a device address); make that first call before any stream
// capture.  Every call shares the array and it keeps the last call's
// contents, so calls whose work overlaps on the GPU (different streams, or
// concurrent host threads) race with each other: serialise them.
// ---------------------------------------------------------------------------

namespace {

constexpr size_t kNoAllocScratchBytes = size_t(4) << 20;  // 4 MiB per device
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

constexpr int kNoAllocMaxDevices = 64;
std::mutex g_noalloc_mu;
void* g_noalloc_ptr[kNoAllocMaxDevices] = {};

// Scratch bytes one forward of T tokens needs (same pieces as a layer's arena).
size_t noalloc_bytes(const SenMoeConfig& c, size_t T, size_t* offs /* [16] */) {
  const size_t K = c.num_experts_per_tok, E = c.n_routed_experts, H = c.hidden_size;
  const size_t I = c.moe_intermediate_size, Is = c.shared_intermediate, P = T * K;
  const size_t nchunks = (P + kDispatchChunk - 1) / kDispatchChunk;
  const size_t sizes[16] = {T * E * 4, P * 4, P * 4, P * 4, P * 4, (E + 1) * 4, E * 4, 4, 4,
                            nchunks * E * 4, P * I * 2, P * H * 2, Is ? T * Is * 2 : 0, Is ? T * H * 2 : 0,
                            Is ? T * 4 : 0, Is ? T * 4 : 0};
  size_t off = 0;
  for (int i = 0; i < 16; ++i) {
    offs[i] = off;
    off = align_up(off + sizes[i], 256);
  }
  return off;
}

}  // namespace

extern "C" int senmoe_moe_forward_noalloc(const SenMoeConfig* config, const SenMoeWeights* weights, const void* x,
                                          int64_t num_tokens, void* y, senmoe_stream_t stream) {
  g_last_error.clear();
  int rc = validate_config(config);
  if (rc) return rc;
  if ((rc = validate_weights(config, weights))) return rc;
  if (num_tokens < 0 || num_tokens > config->max_tokens)
    return fail(SENMOE_ERR_BAD_ARG, "num_tokens=%lld outside [0, max_tokens=%d]", (long long)num_tokens,
                config->max_tokens);
  if (num_tokens == 0) return SENMOE_OK;
  size_t offs[16];
  const size_t need = noalloc_bytes(*config, static_cast<size_t>(num_tokens), offs);
  if (need > kNoAllocScratchBytes)
    return fail(SENMOE_ERR_BAD_ARG,
                "senmoe_moe_forward_noalloc: %lld tokens need %zu bytes of scratch, above its fixed %zu-byte "
                "array (use a layer handle for this size)",
                (long long)num_tokens, need, kNoAllocScratchBytes);

  int dev = 0;
  SENMOE_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kNoAllocMaxDevices) return fail(SENMOE_ERR_UNSUPPORTED, "device %d out of range", dev);
  void* base = nullptr;
  {
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    if (!g_noalloc_ptr[dev]) {
      void* p = nullptr;
      const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
      if (e != cudaSuccess || !p)
        return fail(SENMOE_ERR_CUDA, "cudaGetSymbolAddress(g_noalloc_scratch) on device %d: %s", dev,
                    cudaGetErrorString(e));
      g_noalloc_ptr[dev] = p;
    }
    base = g_noalloc_ptr[dev];
  }

  // A stack-only layer view over the static array; the forward itself is the
  // layer forward, unchanged.
  SenMoeLayer L;
  L.cfg = *config;
  L.w = *weights;
  L.device = dev;
  L.max_pairs = static_cast<int>(num_tokens * config->num_experts_per_tok);
  L.nchunks_max = (L.max_pairs + kDispatchChunk - 1) / kDispatchChunk;
  char* b = static_cast<char*>(base);
  L.logits = reinterpret_cast<float*>(b + offs[0]);
  L.ids = reinterpret_cast<int32_t*>(b + offs[1]);
  L.wts = reinterpret_cast<float*>(b + offs[2]);
  L.perm = reinterpret_cast<int32_t*>(b + offs[3]);
  L.inv = reinterpret_cast<int32_t*>(b + offs[4]);
  L.offsets = reinterpret_cast<int32_t*>(b + offs[5]);
  L.active = reinterpret_cast<int32_t*>(b + offs[6]);
  L.active_count = reinterpret_cast<int32_t*>(b + offs[7]);
  L.err = reinterpret_cast<int*>(b + offs[8]);
  L.chunk_hist = reinterpret_cast<int32_t*>(b + offs[9]);
  L.h = reinterpret_cast<uint16_t*>(b + offs[10]);
  L.d = reinterpret_cast<uint16_t*>(b + offs[11]);
  if (config->shared_intermediate > 0) {
    L.sh_h = reinterpret_cast<uint16_t*>(b + offs[12]);
    L.sh_out = reinterpret_cast<uint16_t*>(b + offs[13]);
    L.sh_gate = reinterpret_cast<float*>(b + offs[14]);
    L.zeros_idx = reinterpret_cast<uint32_t*>(b + offs[15]);
  }
  // The array keeps the previous call's bytes: clear what must start at zero
  // (the device error word and the shared expert's all-zero index list).
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  SENMOE_CUDA(cudaMemsetAsync(L.err, 0, sizeof(int), st));
  if (L.zeros_idx) SENMOE_CUDA(cudaMemsetAsync(L.zeros_idx, 0, size_t(num_tokens) * 4, st));
  return layer_forward(&L, x, num_tokens, y, nullptr, false, stream);
}
