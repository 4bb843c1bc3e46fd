/*
 * senmoe.h -- C ABI of the B200 (sm_100a) mixture-of-experts block.
 *
 * Drop-in boundary for sen-mlx's MoE hot path.  Every entry point is plain C:
 * device pointers, sizes and a cudaStream_t, an int status (0 = ok) and a
 * thread-local message from senmoe_last_error().  No entry point aborts,
 * traps or allocates on the forward path.
 *
 * Reference interfaces replaced (paths inside the sen-mlx project):
 *   senmoe_gather_qmm       <- gather_qmm / mlx_sys::mlx_gather_qmm
 *                              src/engine/mlx_lm/utils/moe.rs:33-77
 *   senmoe_quantized_linear <- nn::QuantizedLinear::forward (the quantized projections
 *                              next to the block, deepseek_v2.rs:190-205, 367-394)
 *   senmoe_layer_create     <- DeepseekMoe::new + SwitchGlu/SwitchLinear weight slots
 *                              src/engine/mlx_lm/models/deepseek_v2.rs:400-428, 485-518
 *   senmoe_layer_forward    <- DeepseekMoe::forward(&mut self, x: &Array) -> Result<Array>
 *                              src/engine/mlx_lm/models/deepseek_v2.rs:520-553
 *   senmoe_router           <- the router half of DeepseekMoe::forward, :526-543
 *   senmoe_gemma_router     <- gemma4::Router::forward(&mut self, x) -> (indices, weights)
 *                              src/engine/mlx_lm/models/gemma4.rs:716-736
 *   senmoe_layer_experts_forward
 *                           <- gemma4::Experts::forward(&self, x, indices, weights)
 *                              src/engine/mlx_lm/models/gemma4.rs:842-848 (also the expert
 *                              half of DeepseekMoe::forward, deepseek_v2.rs:544-552)
 *   senmoe_dispatch         <- (no counterpart: the reference gathers per (token, slot)
 *                              with sorted_indices=false, deepseek_v2.rs:441; this is the
 *                              build's expert-contiguous permutation)
 *   senmoe_layer_destroy    <- Drop of the MLX Param<Array>s (deepseek_v2.rs:408-413)
 *   senmoe_last_error       <- Exception::custom(...) text, utils/moe.rs:66-74
 *
 * Weight layout is MLX's affine-quantized layout, unchanged
 * (src/engine/mlx_native.rs:3381-3389, 3473-3477): for a [E, out, in]
 * projection, weight is uint32 [E, out, in*bits/32] with 32/bits codes per
 * word (lower columns in lower bits), scales and biases are bf16
 * [E, out, in/group]; w = q * scale + bias.  bits is 4 or 8, group is 64.
 *
 * Numerics: fp32 accumulation; bf16 rounding at the points where the MLX
 * graph rounds (logits, softmax scores, gate/up, silu, silu*up, down);
 * router weights and the weighted combine in fp32; y is bf16.
 */
#ifndef SENMOE_H_
#define SENMOE_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define SENMOE_ABI_VERSION 1

typedef struct CUstream_st* senmoe_stream_t; /* == cudaStream_t */

typedef enum SenMoeStatus {
  SENMOE_OK = 0,
  SENMOE_ERR_BAD_ARG = 1,     /* shape, alignment or index rejected on the host */
  SENMOE_ERR_CUDA = 2,        /* a CUDA runtime call failed */
  SENMOE_ERR_NCCL = 3,        /* an NCCL call failed (expert parallelism) */
  SENMOE_ERR_TIMEOUT = 4,     /* a bounded device- or host-side wait ran out */
  SENMOE_ERR_UNSUPPORTED = 5, /* valid in MLX, not supported by this build */
  SENMOE_ERR_NO_MEMORY = 6,   /* scratch allocation at create time failed */
  SENMOE_ERR_DEVICE = 7       /* a kernel reported bad data (expert index out of range) */
} SenMoeStatus;

typedef enum SenMoeRouter {
  SENMOE_ROUTER_SOFTMAX_TOPK = 0, /* DeepSeek/Qwen: softmax over E, top-k, optional renorm */
  SENMOE_ROUTER_TOPK_SOFTMAX = 1  /* Gemma-4: rms_norm, quantized proj, top-k, softmax over k,
                                     x per-expert scale (senmoe_gemma_router) */
} SenMoeRouter;

typedef enum SenMoeActivation {
  SENMOE_ACT_SWIGLU = 0, /* silu(gate) * up   (deepseek_v2.rs:472-474) */
  SENMOE_ACT_GEGLU = 1   /* gelu_approx(gate) * up (gemma4.rs:817-819) */
} SenMoeActivation;

/* Field names follow the reference's config.json / ModelArgs
 * (deepseek_v2.rs:103-118). */
typedef struct SenMoeConfig {
  int32_t hidden_size;             /* H */
  int32_t moe_intermediate_size;   /* I */
  int32_t n_routed_experts;        /* E (global expert count) */
  int32_t num_experts_per_tok;     /* K */
  int32_t bits;                    /* 4 or 8 */
  int32_t group_size;              /* 64 */
  int32_t router_kind;             /* SenMoeRouter */
  int32_t activation;              /* SenMoeActivation */
  int32_t norm_topk_prob;          /* 0/1 */
  float routed_scaling_factor;     /* 1.0 = off */
  int32_t shared_intermediate;     /* moe_intermediate_size * n_shared_experts; 0 = none */
  int32_t shared_gate;             /* 1: y += sigmoid(x . shared_gate_w) * shared(x) */
  int32_t max_tokens;              /* T_max: scratch is sized for this at create time */
  int32_t expert_begin;            /* first expert held by this rank (0 on one GPU) */
  int32_t expert_end;              /* one past the last local expert (E on one GPU) */
  int32_t reserved[3];             /* [0]: expert kernels, 0 auto, 1 CUDA-core GEMV, 2 tcgen05 GEMM,
                                      3 warp-MMA GEMM; [1]: warp-MMA form, 0 group-scaled where
                                      supported (4-bit), 1 dequantise every weight, 2 group-scaled
                                      with one CTA per SM, 3 as 2 with 128-row down tiles instead
                                      of 256-row ones (same results); [2]: expert-slot
                                      capacity, the most
                                      (token, expert) pairs that reach this rank's experts in one
                                      call (0: max_tokens * K).  Under expert parallelism a rank
                                      holds only its own experts' pairs, about 1/world of them, so
                                      its per-pair scratch can be that much smaller; a call whose
                                      local pairs exceed it skips the excess and reports
                                      SENMOE_ERR_DEVICE from senmoe_layer_check.  A call with more
                                      pairs in all than the capacity needs expert parallelism and
                                      the tensor-core expert kernels (SENMOE_ERR_UNSUPPORTED) */
} SenMoeConfig;

/* Device pointers, caller-owned, valid for the layer's lifetime.  Expert
 * tensors hold experts [expert_begin, expert_end) only. */
typedef struct SenMoeWeights {
  const void* router_weight;      /* bf16 [E, H]  (mlp.gate.weight, unquantized); NULL: the
                                     layer serves senmoe_layer_experts_forward only */
  const uint32_t* gate_weight;    /* u32 [E_local, I, H*bits/32] (switch_mlp.gate_proj) */
  const void* gate_scales;        /* bf16 [E_local, I, H/group] */
  const void* gate_biases;
  const uint32_t* up_weight;      /* switch_mlp.up_proj, same shapes as gate */
  const void* up_scales;
  const void* up_biases;
  const uint32_t* down_weight;    /* u32 [E_local, H, I*bits/32] (switch_mlp.down_proj) */
  const void* down_scales;        /* bf16 [E_local, H, I/group] */
  const void* down_biases;
  const uint32_t* shared_gate_weight; /* shared_experts.gate_proj: u32 [Is, H*bits/32] */
  const void* shared_gate_scales;
  const void* shared_gate_biases;
  const uint32_t* shared_up_weight;
  const void* shared_up_scales;
  const void* shared_up_biases;
  const uint32_t* shared_down_weight; /* u32 [H, Is*bits/32] */
  const void* shared_down_scales;
  const void* shared_down_biases;
  const void* shared_gate_vector;     /* bf16 [H], only when shared_gate */
} SenMoeWeights;

/* Optional device outputs of one forward (any field may be NULL). */
typedef struct SenMoeDebug {
  int32_t* topk_ids;      /* [T, K] expert ids, slot order = score desc, id asc */
  float* topk_weights;    /* [T, K] fp32 router weights after renorm/scaling */
  int32_t* perm;          /* [T*K] pair index (t*K + j) of each expert-sorted slot */
  int32_t* offsets;       /* [E + 1] slot range of each expert */
} SenMoeDebug;

typedef struct SenMoeLayer SenMoeLayer;

/* Message of the last failing call on this thread ("" when none). */
const char* senmoe_last_error(void);
/* "senmoe <abi> sm_100a" */
const char* senmoe_version(void);
/* Self-check of the expert epilogues' sigmoid on the current device
 * (synchronous): its fast form against 1 / (1 + expf(-g)) rounded to bf16,
 * for every bf16 gate value g but NaNs.  *mismatches must come back 0;
 * *exact_form counts the inputs that took the exact form. */
int senmoe_selftest_sigmoid(int64_t* mismatches, int64_t* exact_form);

/* Layer life cycle.  create validates the config, checks pointer alignment,
 * and allocates the layer's scratch on `device` for config->max_tokens. */
int senmoe_layer_create(const SenMoeConfig* config, const SenMoeWeights* weights, int device,
                        SenMoeLayer** out_layer);
int senmoe_layer_destroy(SenMoeLayer* layer);

/* y[T, H] = DeepseekMoe::forward(x[T, H]), bf16, stream-ordered, no host
 * synchronisation and no allocation; 0 <= T <= max_tokens. */
int senmoe_layer_forward(SenMoeLayer* layer, const void* x, int64_t num_tokens, void* y,
                         const SenMoeDebug* debug, senmoe_stream_t stream);

/* h_out[T, H] = bf16(x + DeepseekMoe::forward(x)): the residual add of
 * DecoderLayer::forward (deepseek_v2.rs:613-620, `h.add(&r)`) fused into
 * the combine, so a decoder stack chains layers without an extra pass. */
int senmoe_layer_forward_residual(SenMoeLayer* layer, const void* x, int64_t num_tokens, void* h_out,
                                  senmoe_stream_t stream);

/* Per-stage timing (the build's counterpart of the reference's tracing of
 * prefill/decode rates, src/engine/mlx_native.rs:916-936).  When enabled,
 * forward records CUDA events between its stages on the stream (outside a
 * CUDA-graph capture; inside one the events are skipped).  senmoe_layer_stage_times waits for the last
 * forward's final event and writes that forward's per-stage milliseconds to
 * ms[0 .. n): router, dispatch, gate/up, down, shared expert, combine.
 * Returns the number of stages written (or a negative status). */
#define SENMOE_NUM_STAGES 6
/* Events are recorded only by forwards issued outside a stream capture. */
int senmoe_layer_set_profiling(SenMoeLayer* layer, int enable);
int senmoe_layer_stage_times(SenMoeLayer* layer, float* ms, int n);

/* Which expert-product kernels a forward of num_tokens tokens runs: 1 = the
 * CUDA-core dequant-GEMV, 2 = the tcgen05 grouped GEMM (prefill-size groups of
 * tokens per expert), 3 = the warp-MMA grouped GEMM (decode-size groups),
 * 4 = one token on one GPU: the whole block in one fused launch whose expert
 * products use the GEMV's arithmetic (a forward with debug outputs or stage
 * profiling runs the staged kernels of path 3 instead);
 * SenMoeConfig.reserved[0] can force one of 1-3 (0 = choose by tokens per
 * expert). */
int senmoe_layer_expert_path(const SenMoeLayer* layer, int64_t num_tokens);

/* Synchronises `stream` and reports any error a kernel recorded on the
 * device since the previous check (bad expert index, timed-out wait). */
int senmoe_layer_check(SenMoeLayer* layer, senmoe_stream_t stream);

/* ---- Expert parallelism (no counterpart in the reference, which runs the
 * block on one Apple GPU).  One process per GPU; rank r creates its layer with
 * expert_begin/expert_end set to its contiguous block of experts (rank order
 * = expert order) and weight tensors holding only those experts, all ranks
 * with the same config otherwise.  Each rank publishes its SenMoePeerInfo,
 * the host exchanges them (e.g. torch.distributed all_gather), and every rank
 * connects with the full table.  After that, forward on every rank takes the
 * SAME tokens x (replicated), and every rank returns the same y: each rank
 * computes only its experts' rows, combines its own contiguous block of the
 * tokens reading every row from its owner over NVLink (CUDA IPC mappings), in
 * slot order, with the one-GPU combine's arithmetic, and sends the combined
 * rows to every peer.  All ranks must run the same sequence of forwards
 * (same num_tokens); a rank that does not shows up as SENMOE_ERR_TIMEOUT from
 * senmoe_layer_check on the others (every cross-GPU wait is bounded). */
#define SENMOE_MAX_RANKS 8

typedef struct SenMoePeerInfo {
  uint8_t ipc_handle[64];  /* cudaIpcMemHandle_t of the layer's scratch arena */
  int64_t rows_offset;     /* byte offset of the expert-output rows in the arena */
  int64_t flags_offset;    /* byte offset of the rank flag block in the arena */
  int64_t arena_bytes;     /* arena size (must match on every rank) */
  int32_t expert_begin;
  int32_t expert_end;
  int32_t device;          /* CUDA ordinal in the publishing process (diagnostics) */
  int32_t reserved;
} SenMoePeerInfo;

/* Token-local expert parallelism (the prefill form of the expert split; no
 * counterpart in the reference): each rank passes ITS OWN tokens x [T_r, H]
 * -- data-parallel tokens, e.g. its own sequences -- and gets y [T_r, H] =
 * DeepseekMoe::forward(x) (+ x when residual != 0, DecoderLayer::forward's
 * residual add) for them.  tokens_per_rank[q] = T_q (host memory, the same
 * array on every rank); the call's tokens are the ranks' tokens in rank
 * order and sum(T_q) <= max_tokens.  Each rank routes only its own tokens,
 * publishes its routing rows and token rows to the peers, runs its experts
 * over every rank's pairs (reading each token's row from its owner over
 * NVLink) and combines its own tokens in slot order, reading each pair's row
 * from the expert's owner: the result is bit-identical to one GPU running
 * the concatenated tokens whenever both take the same router kernel (it is
 * picked by the token count routed: CUDA-core below 512 tokens, tensor-core
 * from 512), within the block tolerance otherwise.  Needs the tensor-core
 * expert kernels (SENMOE_ERR_UNSUPPORTED for the GEMV path).  A layer that
 * is not connected runs it as senmoe_layer_forward (tokens_per_rank[0] ==
 * num_tokens).  Same ordering rules as the replicated form. */
int senmoe_layer_forward_tokens(SenMoeLayer* layer, const void* x, int64_t num_tokens, void* y,
                                const int64_t* tokens_per_rank, int32_t residual, senmoe_stream_t stream);

/* This rank's table entry. */
int senmoe_layer_peer_info(const SenMoeLayer* layer, SenMoePeerInfo* out);

/* Opens the peers' arenas and switches forward to the expert-parallel form.
 * peers[r] is rank r's entry, r < world_size <= SENMOE_MAX_RANKS; the expert
 * ranges must tile [0, n_routed_experts) in rank order and peers[rank] must be
 * this layer's own entry.  world_size == 1 is allowed (no peers).  Call once,
 * with no forward of the layer in flight; the mappings close on destroy. */
int senmoe_layer_connect_peers(SenMoeLayer* layer, int32_t rank, int32_t world_size, const SenMoePeerInfo* peers);

/* Router alone: ids/weights [T, K] for x [T, H] (bf16), router weight
 * [E, H] (bf16).  Same rounding and slot order as the layer. */
int senmoe_router(const void* x, int64_t num_tokens, const void* router_weight, int32_t hidden,
                  int32_t num_experts, int32_t top_k, int32_t norm_topk_prob, float routed_scaling_factor,
                  float* logits_scratch /* [T, E] fp32 device */, int32_t* topk_ids, float* topk_weights,
                  senmoe_stream_t stream);

/* Gemma-4 router (Router::forward, gemma4.rs:716-736), field names after
 * its parameters (gemma4.rs:683-700):
 *   normed = rms_norm(x, f32(scale) * hidden_size^-1/2, rms_norm_eps)   fp32
 *   scores = proj(normed)        affine-quantized [E, H] linear (MLX layout,
 *                                8-bit in the checkpoint), fp32
 *   ids    = top-k of scores     (score desc, id asc: MLX leaves the order open)
 *   w      = softmax(scores[ids]) * f32(per_expert_scale[ids])
 * x bf16 [T, H]; proj_weight u32 [E, H*bits/32], proj_scales/biases bf16
 * [E, H/group_size]; scale bf16 [H]; per_expert_scale bf16 [E]; topk_ids
 * int32 [T, K], topk_weights fp32 [T, K] (device memory). */
typedef struct SenMoeGemmaRouter {
  int32_t hidden_size;
  int32_t num_experts;
  int32_t top_k;             /* <= 16 */
  int32_t bits;              /* 4 or 8 */
  int32_t group_size;        /* 64 */
  float rms_norm_eps;
  const uint32_t* proj_weight;
  const void* proj_scales;
  const void* proj_biases;
  const void* scale;
  const void* per_expert_scale;
} SenMoeGemmaRouter;
int senmoe_gemma_router(const SenMoeGemmaRouter* router, const void* x, int64_t num_tokens, int32_t* topk_ids,
                        float* topk_weights, senmoe_stream_t stream);

/* Experts::forward (gemma4.rs:842-848): the layer's experts over routing the
 * caller computed, y[t] = bf16( sum_j f32(expert_ids[t,j](x[t])) * w[t,j] )
 * (+ the layer's shared experts; fused residual: no).  topk_ids int32 [T, K]
 * in [0, n_routed_experts), topk_weights fp32 [T, K], device memory.  A layer
 * used only this way may be created with router_weight = NULL. */
int senmoe_layer_experts_forward(SenMoeLayer* layer, const void* x, int64_t num_tokens, const int32_t* topk_ids,
                                 const float* topk_weights, void* y, senmoe_stream_t stream);

/* Dispatch alone: stable counting sort of the T*K pairs by expert.
 * perm [T*K], inverse [T*K] (slot of each pair), offsets [E + 1]; scratch is
 * int32 [E + 2] device memory: scratch[0 .. n) lists the experts that
 * received pairs (ascending), scratch[E] = n, scratch[E + 1] = nonzero if an
 * id was outside [0, E) (the caller zeroes it before the call).  E <= 1024. */
int senmoe_dispatch(const int32_t* topk_ids, int64_t num_tokens, int32_t top_k, int32_t num_experts,
                    int32_t* perm, int32_t* inverse, int32_t* offsets, int32_t* scratch, senmoe_stream_t stream);

/* gather_qmm, transpose=true (utils/moe.rs:33-43):
 *   out[i, :] = bf16( x[i / (n_indices / x_rows), :] @ dequant(w[rhs_indices[i]])^T )
 * x bf16 [x_rows, in_features]; w u32 [num_experts, out_features, in*bits/32];
 * scales/biases bf16 [num_experts, out_features, in/group]; out bf16
 * [n_indices, out_features].  n_indices must be a multiple of x_rows (x
 * broadcasts over the trailing index dim, the SwitchGlu gate/up form) or equal
 * to it (the down form).  transpose == 0 returns SENMOE_ERR_UNSUPPORTED (the
 * reference only calls the transposed form, moe.rs:43, deepseek_v2.rs:437).
 * sorted_indices is accepted and ignored (it is a performance hint in MLX). */
int senmoe_gather_qmm(const void* x, int64_t x_rows, const uint32_t* w, const void* scales, const void* biases,
                      const uint32_t* rhs_indices, int64_t n_indices, int64_t in_features, int64_t out_features,
                      int32_t num_experts, int32_t transpose, int32_t group_size, int32_t bits,
                      int32_t sorted_indices, void* out, senmoe_stream_t stream);

/* The dense quantized Linear next to the block (nn::QuantizedLinear without
 * bias, as DeepSeek builds its projections: deepseek_v2.rs:213, :382; the
 * step either side of the MoE block in decode):
 *   y[t, :] = bf16( x[t, :] @ dequant(w)^T )
 * x bf16 [T, in_features]; w u32 [out_features, in*bits/32]; scales/biases
 * bf16 [out_features, in/group]; y bf16 [T, out_features].  Same arithmetic
 * as senmoe_gather_qmm (one expert). */
int senmoe_quantized_linear(const void* x, int64_t num_tokens, const uint32_t* w, const void* scales,
                            const void* biases, int64_t in_features, int64_t out_features, int32_t group_size,
                            int32_t bits, void* y, senmoe_stream_t stream);

/* Allocation-free forward (no counterpart in the reference; this build adds
 * it for callers that cannot allocate device memory at call time: code inside
 * an open CUDA stream capture, serving loops whose HBM another allocator has
 * fully reserved, plugin hosts that forbid device allocation on the hot path).
 * DeepseekMoe::forward without a layer handle: all scratch lives in one fixed
 * 4 MiB device array inside the library (held by every GPU that loads it until
 * exit).  It always runs the CUDA-core dequant-GEMV expert kernels and the
 * router's logits and top-k as separate launches (the tensor-core paths need
 * tensor maps that a layer encodes over its own scratch at create time), so
 * its output agrees with senmoe_layer_forward within the block tolerance
 * (max abs 2e-2, relative L2 5e-3), not bit for bit, and at decode batches
 * it is slower (about 8x in gate/up at 64 tokens of config 0).
 * Size limit: the scratch of one call is the sum of these pieces, each
 * rounded up to 256 bytes, and must not exceed 4 MiB (P = num_tokens * K):
 *   T*E*4, four of P*4, (E+1)*4, E*4, 4, 4, ceil(P/1024)*E*4, P*I*2, P*H*2,
 *   and with a shared expert T*Is*2, T*H*2, T*4, T*4.
 * That is 91 tokens at config 0 (H=2048 E=128 K=8 I=768) and 71 at H=2048
 * E=512 K=10 I=512 with a 512-wide shared expert; larger calls return
 * SENMOE_ERR_BAD_ARG.  config->max_tokens bounds num_tokens as for a layer.
 * The first call on a device resolves the array's address (once per device,
 * kept for the life of the process) and should come before any stream
 * capture; after cudaDeviceReset that address is stale, so do not call this
 * entry point again in that process.  All calls share the array, which keeps
 * the last call's contents: calls that overlap on the GPU race, so serialise
 * them.  Device-side errors (an expert id out of range) are not reported on
 * this path: each call clears the array's error word and nothing reads it. */
int senmoe_moe_forward_noalloc(const SenMoeConfig* config, const SenMoeWeights* weights, const void* x,
                               int64_t num_tokens, void* y, senmoe_stream_t stream);

#ifdef __cplusplus
} /* extern "C" */
#endif
#endif /* SENMOE_H_ */
