/*
 * moe_oracle.c -- TEST INFRASTRUCTURE ONLY.
 *
 * CPU restatement of sen-mlx's mixture-of-experts block, used as the parity
 * checker for the sm_100a kernels and as the timed CPU baseline.  Nothing in
 * the product library links, loads or calls this file; only tests/, the
 * smoke() entry and bench.py's CPU-baseline leg do.
 *
 * PARITY STATUS: unpinned against MLX itself.  The reference runs all of its
 * MoE arithmetic inside the MLX C++/Metal library (mlx-rs 0.25.3 / mlx-sys
 * 0.2.0, git tag v0.25.3 of oxiglade/mlx-rs), which is not vendored in the
 * reference tree and cannot be built here (no Rust toolchain, no MLX sources,
 * Apple Metal only).  What is pinned: the reference's one known-answer test
 * for the primitive (src/engine/mlx_lm/utils/moe.rs:89-146), restated with its
 * exact input formulas in tests/golden/, and an independent numpy restatement
 * (oracle/numpy_ref.py) that must agree with this file.
 *
 * Reference graph followed (paths inside the reference project):
 *   router           src/engine/mlx_lm/models/deepseek_v2.rs:526-548
 *   Gemma router     src/engine/mlx_lm/models/gemma4.rs:716-736 (orc_gemma_router)
 *   Gemma experts    src/engine/mlx_lm/models/gemma4.rs:809-848 (GeGLU, weighted sum)
 *   SwitchGlu        src/engine/mlx_lm/models/deepseek_v2.rs:466-478
 *   SwitchLinear     src/engine/mlx_lm/models/deepseek_v2.rs:431-443
 *   gather_qmm       src/engine/mlx_lm/utils/moe.rs:20-77
 *   shared experts   src/engine/mlx_lm/models/deepseek_v2.rs:381-393, 550-552
 *   quant defaults   src/engine/mlx_native.rs:3381-3389 (group 64, 4 bits)
 *
 * Rounding model ("MLX mode", mode == 0).  MLX ops return their inputs' dtype,
 * and MLX's C++ type promotion treats a 0-d float32 array (mlx-rs `array!(f32)`)
 * as a strong float32, so:
 *   logits = bf16(x . Wg)                      deepseek_v2.rs:528 (nn::Linear)
 *   scores = bf16(softmax_fp32(logits))        :529 (precise=true)
 *   top-k on scores (order: score desc, id asc; MLX leaves it unspecified)
 *   w      = scores[top-k]                     :536 (bf16)
 *   den    = f32(bf16(sum_k w)) + 1e-20f       :538 (bf16 sum, f32 add)
 *   w      = f32(w) / den                      :539 (bf16 / f32 -> f32)
 *   w     *= routed_scaling_factor (f32)       :541-543
 *   g,u    = bf16(gather_qmm(x, Wg/Wu))        :472-473
 *   h      = bf16(bf16(g * bf16(sigmoid(g))) * u)  nn::silu then multiply
 *   d      = bf16(gather_qmm(h, Wd))           :475
 *   y      = sum_k f32(d_k) * w_k  (f32)       :546-548 (bf16 * f32 -> f32)
 *   y     += f32(shared(x))                    :550-552
 * gather_qmm itself: per 64-wide group, scale*sum(q*x) + bias*sum(x),
 * accumulated in wide precision and rounded once to bf16 (MLX's qmv path,
 * which the reference always takes: M == 1 per (token, slot)).
 * mode == 1 ("fp32 mode") skips every intermediate bf16 rounding.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define ORC_OK 0
#define ORC_BAD_ARG 1
#define ORC_BAD_INDEX 2
#define ORC_NO_MEM 3

/* ------------------------------------------------------------------ bf16 */
static inline float bf2f(uint16_t b) {
  uint32_t u = (uint32_t)b << 16;
  float f;
  memcpy(&f, &u, 4);
  return f;
}
static inline uint16_t f2bf(float f) { /* round to nearest even */
  uint32_t u;
  memcpy(&u, &f, 4);
  if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40u);
  u += 0x7fffu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}
static inline float rbf(float f) { return bf2f(f2bf(f)); }

void orc_f32_to_bf16(const float* in, uint16_t* out, int64_t n) {
  for (int64_t i = 0; i < n; ++i) out[i] = f2bf(in[i]);
}
void orc_bf16_to_f32(const uint16_t* in, float* out, int64_t n) {
  for (int64_t i = 0; i < n; ++i) out[i] = bf2f(in[i]);
}

int orc_num_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}
void orc_set_num_threads(int n) {
#ifdef _OPENMP
  if (n > 0) omp_set_num_threads(n);
#else
  (void)n;
#endif
}

/* ------------------------------------------------------ seeded normals */
/* Counter-based N(0,1) * std: element i depends only on (seed, i), so the
 * fill is reproducible under any thread count.  splitmix64 -> Box-Muller. */
static inline uint64_t splitmix64(uint64_t z) {
  z += 0x9e3779b97f4a7c15ull;
  z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
  z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
  return z ^ (z >> 31);
}
void orc_fill_normal(uint64_t seed, float* out, int64_t n, float std) {
  const uint64_t base = splitmix64(seed);
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < n; ++i) {
    const uint64_t r = splitmix64(base ^ ((uint64_t)i * 0xd1b54a32d192ed03ull));
    const double u1 = ((double)(r >> 40) + 1.0) * (1.0 / 16777217.0); /* (0, 1] */
    const double u2 = (double)(r & 0xffffffull) * (1.0 / 16777216.0); /* [0, 1) */
    out[i] = (float)(sqrt(-2.0 * log(u1)) * cos(6.283185307179586 * u2)) * std;
  }
}

/* ------------------------------------------------------------ quantizer */
/* MLX-style affine quantizer (restated from MLX's published affine_quantize):
 * per group of `group` consecutive columns, the extreme of larger magnitude
 * ("edge") is represented exactly; scale may be negative.  Packing: 32/bits
 * codes per uint32, lower columns in lower bits.  This only manufactures
 * synthetic weights: the kernels and the oracle consume the same packed
 * tensors, so its exact rounding does not affect parity. */
int orc_quantize_affine(const float* w, int64_t rows, int64_t cols, int32_t group, int32_t bits,
                        uint32_t* wq, uint16_t* scales, uint16_t* biases) {
  if (!(bits == 4 || bits == 8) || group <= 0 || cols % group || (cols * bits) % 32) return ORC_BAD_ARG;
  const int64_t ngroups = cols / group;
  const int per_word = 32 / bits;
  const float n_bins = (float)((1 << bits) - 1);
  const int64_t words_per_row = cols * bits / 32;
#pragma omp parallel for schedule(static)
  for (int64_t r = 0; r < rows; ++r) {
    const float* wr = w + r * cols;
    uint32_t* qr = wq + r * words_per_row;
    memset(qr, 0, sizeof(uint32_t) * (size_t)words_per_row);
    for (int64_t g = 0; g < ngroups; ++g) {
      const float* wg = wr + g * group;
      float mx = wg[0], mn = wg[0];
      for (int i = 1; i < group; ++i) {
        mx = wg[i] > mx ? wg[i] : mx;
        mn = wg[i] < mn ? wg[i] : mn;
      }
      const int use_min = fabsf(mn) > fabsf(mx);
      float scale = (mx - mn) / n_bins;
      if (scale < 1e-7f) scale = 1e-7f;
      scale = use_min ? scale : -scale;
      const float edge = use_min ? mn : mx;
      const float q0 = rintf(edge / scale);
      float bias = 0.0f;
      if (q0 != 0.0f) {
        scale = edge / q0;
        bias = edge;
      }
      for (int i = 0; i < group; ++i) {
        float q = rintf((wg[i] - bias) / scale);
        q = q < 0.0f ? 0.0f : (q > n_bins ? n_bins : q);
        const int64_t c = g * group + i;
        qr[c / per_word] |= ((uint32_t)q) << ((c % per_word) * bits);
      }
      scales[r * ngroups + g] = f2bf(scale);
      biases[r * ngroups + g] = f2bf(bias);
    }
  }
  return ORC_OK;
}

static inline uint32_t code_at(const uint32_t* row, int64_t c, int32_t bits) {
  const int per_word = 32 / bits;
  return (row[c / per_word] >> ((c % per_word) * bits)) & ((1u << bits) - 1u);
}

/* w[r][c] = q * scale + bias, evaluated in fp32 (utils/moe.rs:28-31).
 * Unpacks word by word (lower columns in lower bits); the same arithmetic
 * as (float)code_at(row, c, bits) * sc + bi per element. */
static void dequant_row(const uint32_t* wq, const uint16_t* s, const uint16_t* b, int64_t r, int64_t cols,
                        int32_t group, int32_t bits, float* out) {
  const int64_t ngroups = cols / group;
  const int per_word = 32 / bits, words_per_group = group / per_word;
  const uint32_t mask = (1u << bits) - 1u;
  const uint32_t* row = wq + r * (cols * bits / 32);
  for (int64_t g = 0; g < ngroups; ++g) {
    const float sc = bf2f(s[r * ngroups + g]), bi = bf2f(b[r * ngroups + g]);
    const uint32_t* wp = row + g * words_per_group;
    float* o = out + g * group;
    if (bits == 4) { /* constant trip counts, so the compiler can vectorise */
      for (int w = 0; w < words_per_group; ++w)
        for (int j = 0; j < 8; ++j) o[w * 8 + j] = (float)((wp[w] >> (j * 4)) & 15u) * sc + bi;
    } else if (bits == 8) {
      for (int w = 0; w < words_per_group; ++w)
        for (int j = 0; j < 4; ++j) o[w * 4 + j] = (float)((wp[w] >> (j * 8)) & 255u) * sc + bi;
    } else {
      for (int w = 0; w < words_per_group; ++w) {
        const uint32_t word = wp[w];
        for (int j = 0; j < per_word; ++j) o[w * per_word + j] = (float)((word >> (j * bits)) & mask) * sc + bi;
      }
    }
  }
}

int orc_dequantize_affine(const uint32_t* wq, const uint16_t* s, const uint16_t* b, int64_t rows, int64_t cols,
                          int32_t group, int32_t bits, float* out) {
  if (!(bits == 4 || bits == 8) || group <= 0 || cols % group) return ORC_BAD_ARG;
#pragma omp parallel for schedule(static)
  for (int64_t r = 0; r < rows; ++r) dequant_row(wq, s, b, r, cols, group, bits, out + r * cols);
  return ORC_OK;
}

/* dot of a dequantized row with x, accumulated per group in double:
 * sum_g scale_g * sum(q x) + bias_g * sum(x) -- MLX qmv's factorisation. */
static double qdot_row(const uint32_t* wq, const uint16_t* s, const uint16_t* b, int64_t r, int64_t cols,
                       int32_t group, int32_t bits, const float* x) {
  const int64_t ngroups = cols / group;
  const uint32_t* row = wq + r * (cols * bits / 32);
  double acc = 0.0;
  for (int64_t g = 0; g < ngroups; ++g) {
    double qx = 0.0, sx = 0.0;
    for (int64_t i = 0; i < group; ++i) {
      const int64_t c = g * group + i;
      qx += (double)code_at(row, c, bits) * (double)x[c];
      sx += (double)x[c];
    }
    acc += (double)bf2f(s[r * ngroups + g]) * qx + (double)bf2f(b[r * ngroups + g]) * sx;
  }
  return acc;
}

/* gather_qmm (utils/moe.rs:20-43), transpose=true form:
 *   y[i, :] = bf16( x[i / (n_idx / x_rows), :] @ dequant(w[idx[i]])^T )
 * x is [x_rows, in] bf16 and broadcasts over the trailing index dim when
 * n_idx is a multiple of x_rows (the SwitchGlu gate/up call); x_rows == n_idx
 * is the per-pair form (the down call).  w [E, out, in*bits/32],
 * scales/biases [E, out, in/group]. */
int orc_gather_qmm(const uint16_t* x, int64_t x_rows, const uint32_t* w, const uint16_t* scales,
                   const uint16_t* biases, const int32_t* idx, int64_t n_idx, int64_t in, int64_t out,
                   int32_t num_experts, int32_t group, int32_t bits, uint16_t* y) {
  if (!(bits == 4 || bits == 8) || group <= 0 || in % group || x_rows <= 0 || n_idx % x_rows) return ORC_BAD_ARG;
  for (int64_t i = 0; i < n_idx; ++i)
    if (idx[i] < 0 || idx[i] >= num_experts) return ORC_BAD_INDEX;
  const int64_t rep = n_idx / x_rows;
  const int64_t wstride = out * (in * bits / 32), sstride = out * (in / group);
  int err = ORC_OK;
#pragma omp parallel
  {
    float* xf = (float*)malloc(sizeof(float) * (size_t)in);
    if (!xf) {
#pragma omp atomic write
      err = ORC_NO_MEM;
    } else {
#pragma omp for schedule(dynamic, 1)
      for (int64_t i = 0; i < n_idx; ++i) {
        const uint16_t* xr = x + (i / rep) * in;
        for (int64_t c = 0; c < in; ++c) xf[c] = bf2f(xr[c]);
        const int64_t e = idx[i];
        for (int64_t o = 0; o < out; ++o)
          y[i * out + o] = f2bf((float)qdot_row(w + e * wstride, scales + e * sstride, biases + e * sstride, o, in,
                                                group, bits, xf));
      }
      free(xf);
    }
  }
  return err;
}

/* --------------------------------------------------------------- block */
typedef struct {
  int32_t hidden;              /* H */
  int32_t intermediate;        /* I  (moe_intermediate_size) */
  int32_t num_experts;         /* E  (n_routed_experts) */
  int32_t top_k;               /* K  (num_experts_per_tok) */
  int32_t bits;                /* 4 or 8 */
  int32_t group_size;          /* 64 */
  int32_t norm_topk_prob;      /* deepseek_v2.rs:115, :537 */
  float routed_scaling_factor; /* deepseek_v2.rs:112, :541 */
  int32_t shared_intermediate; /* moe_intermediate_size * n_shared_experts; 0 = none */
  int32_t shared_gate;         /* 1: y += sigmoid(x . w_sg) * shared(x) (no reference counterpart) */
  int32_t mode;                /* 0 = MLX bf16 rounding points, 1 = fp32 */
  int32_t activation;          /* 0 SwiGLU (deepseek_v2.rs:472-474), 1 GeGLU (gemma4.rs:817-819) */
} OrcConfig;

typedef struct {
  const uint16_t* router_w; /* [E, H] bf16, unquantized (deepseek_v2.rs:495-497) */
  const uint32_t *gate_w, *up_w, *down_w;
  const uint16_t *gate_s, *gate_b, *up_s, *up_b, *down_s, *down_b;
  const uint32_t *sh_gate_w, *sh_up_w, *sh_down_w; /* [Is, H*bits/32], [H, Is*bits/32] */
  const uint16_t *sh_gate_s, *sh_gate_b, *sh_up_s, *sh_up_b, *sh_down_s, *sh_down_b;
  const uint16_t* sh_gate_vec; /* [H] bf16, only when shared_gate */
} OrcWeights;

static inline float maybe_rbf(float v, int mode) { return mode == 0 ? rbf(v) : v; }
static inline float sigmoidf_(float v) { return 1.0f / (1.0f + expf(-v)); }
/* nn::gelu_approximate, the tanh form 0.5 g (1 + tanh(sqrt(2/pi) (g + 0.044715 g^3))). */
static inline float gelu_tanh_(float g) {
  return 0.5f * g * (1.0f + tanhf(0.7978845608028654f * (g + 0.044715f * g * g * g)));
}

/* Router: deepseek_v2.rs:528-543.  ids[t*K+j] / weights[t*K+j] in canonical
 * slot order (score desc, expert id asc).  scores_out (optional) [T, E]. */
int orc_router(const OrcConfig* cfg, const OrcWeights* wt, const uint16_t* x, int64_t T, int32_t* ids,
               float* weights, float* scores_out) {
  const int64_t H = cfg->hidden, E = cfg->num_experts, K = cfg->top_k;
  if (K <= 0 || K > E || H <= 0) return ORC_BAD_ARG;
  int err = ORC_OK;
#pragma omp parallel
  {
    float* sc = (float*)malloc(sizeof(float) * (size_t)E);
    unsigned char* taken = (unsigned char*)malloc((size_t)E);
    if (!sc || !taken) {
#pragma omp atomic write
      err = ORC_NO_MEM;
    } else {
#pragma omp for schedule(static)
      for (int64_t t = 0; t < T; ++t) {
        const uint16_t* xr = x + t * H;
        float mx = -INFINITY;
        for (int64_t e = 0; e < E; ++e) {
          const uint16_t* wr = wt->router_w + e * H;
          double acc = 0.0;
          for (int64_t h = 0; h < H; ++h) acc += (double)bf2f(xr[h]) * (double)bf2f(wr[h]);
          sc[e] = maybe_rbf((float)acc, cfg->mode);
          mx = sc[e] > mx ? sc[e] : mx;
        }
        double sum = 0.0;
        for (int64_t e = 0; e < E; ++e) {
          sc[e] = expf(sc[e] - mx);
          sum += sc[e];
        }
        for (int64_t e = 0; e < E; ++e) {
          sc[e] = maybe_rbf((float)(sc[e] / sum), cfg->mode);
          if (scores_out) scores_out[t * E + e] = sc[e];
        }
        memset(taken, 0, (size_t)E);
        for (int64_t j = 0; j < K; ++j) { /* select max, lowest id on ties */
          int64_t best = -1;
          for (int64_t e = 0; e < E; ++e)
            if (!taken[e] && (best < 0 || sc[e] > sc[best])) best = e;
          taken[best] = 1;
          ids[t * K + j] = (int32_t)best;
          weights[t * K + j] = sc[best];
        }
        if (cfg->norm_topk_prob) {
          float s = 0.0f;
          for (int64_t j = 0; j < K; ++j) s += weights[t * K + j];
          const float den = maybe_rbf(s, cfg->mode) + 1e-20f;
          for (int64_t j = 0; j < K; ++j) weights[t * K + j] = weights[t * K + j] / den;
        }
        if (fabsf(cfg->routed_scaling_factor - 1.0f) > 1.1920929e-7f)
          for (int64_t j = 0; j < K; ++j) weights[t * K + j] *= cfg->routed_scaling_factor;
      }
    }
    free(sc);
    free(taken);
  }
  return err;
}

/* Dispatch: stable counting sort of the T*K (token, slot) pairs by expert.
 * perm[s] = pair index p = t*K + j of the s-th expert-sorted slot;
 * offsets[e] .. offsets[e+1] is expert e's run; inv[p] = s.
 * The reference has no dispatch (gather_qmm with sorted_indices=false,
 * deepseek_v2.rs:441); this canonical permutation is the build's definition. */
int orc_dispatch(const int32_t* ids, int64_t T, int32_t K, int32_t E, int32_t* perm, int32_t* offsets,
                 int32_t* inv) {
  const int64_t P = T * K;
  if (E <= 0 || K <= 0 || T < 0) return ORC_BAD_ARG;
  for (int32_t e = 0; e <= E; ++e) offsets[e] = 0;
  for (int64_t p = 0; p < P; ++p) {
    if (ids[p] < 0 || ids[p] >= E) return ORC_BAD_INDEX;
    offsets[ids[p] + 1]++;
  }
  for (int32_t e = 0; e < E; ++e) offsets[e + 1] += offsets[e];
  int32_t* cursor = (int32_t*)malloc(sizeof(int32_t) * (size_t)E);
  if (!cursor) return ORC_NO_MEM;
  for (int32_t e = 0; e < E; ++e) cursor[e] = offsets[e];
  for (int64_t p = 0; p < P; ++p) {
    const int32_t s = cursor[ids[p]]++;
    perm[s] = (int32_t)p;
    if (inv) inv[p] = s;
  }
  free(cursor);
  return ORC_OK;
}

/* Gated expert MLP (SwiGLU: deepseek_v2.rs:466-478 and the dense twin
 * :389-392; GeGLU: gemma4.rs:809-823) over the slots of one expert.  xs: n rows of in=H floats (already bf16 values),
 * padded with zero rows to a multiple of ORC_TB; hbuf: ceil(n/ORC_TB)*ORC_TB rows of I; out: n rows of H floats,
 * rounded per mode.  Weights are one expert's slice.
 * Each dot product sums fp32 products per 64-column group (8 partial sums
 * in column order) and the groups in double; ORC_TB tokens share one pass
 * over a dequantized weight row, each token keeping exactly that order. */
#define ORC_TB 4
/* AVX2 clone where the host CPU has it (same arithmetic: no contraction, no
 * reassociation), the baseline x86-64 build otherwise */
__attribute__((target_clones("avx2", "default")))
static void glu_expert(const OrcConfig* cfg, int64_t H, int64_t I, const uint32_t* gw, const uint16_t* gs,
                          const uint16_t* gb, const uint32_t* uw, const uint16_t* us, const uint16_t* ub,
                          const uint32_t* dw, const uint16_t* ds, const uint16_t* db, const float* xs, int64_t n,
                          float* hbuf, float* rowg, float* rowu, float* out) {
  const int32_t G = cfg->group_size, B = cfg->bits, mode = cfg->mode;
  const int64_t nb = (n + ORC_TB - 1) / ORC_TB * ORC_TB;
  for (int64_t i = 0; i < I; ++i) {
    dequant_row(gw, gs, gb, i, H, G, B, rowg);
    dequant_row(uw, us, ub, i, H, G, B, rowu);
    for (int64_t r0 = 0; r0 < nb; r0 += ORC_TB) {
      double ag[ORC_TB] = {0}, au[ORC_TB] = {0};
      for (int64_t c0 = 0; c0 < H; c0 += G) { /* fp32 within a group, double across groups */
        float pg[ORC_TB][8] = {{0}}, pu[ORC_TB][8] = {{0}};
        for (int64_t c = c0; c < c0 + G; c += 8)
          for (int t = 0; t < ORC_TB; ++t) {
            const float* xr = xs + (r0 + t) * H + c;
            for (int k = 0; k < 8; ++k) {
              pg[t][k] += rowg[c + k] * xr[k];
              pu[t][k] += rowu[c + k] * xr[k];
            }
          }
        for (int t = 0; t < ORC_TB; ++t)
          for (int k = 0; k < 8; ++k) {
            ag[t] += pg[t][k];
            au[t] += pu[t][k];
          }
      }
      for (int t = 0; t < ORC_TB; ++t) {
        const float g = maybe_rbf((float)ag[t], mode), u = maybe_rbf((float)au[t], mode);
        /* SwiGLU: nn::silu(g) = g * sigmoid(g), one bf16 rounding per op;
         * GeGLU: nn::gelu_approximate(g) rounded once to bf16 (assumed: one
         * fused activation op, as MLX compiles its elementwise chains) */
        const float a = cfg->activation == 1 ? maybe_rbf(gelu_tanh_(g), mode)
                                             : maybe_rbf(g * maybe_rbf(sigmoidf_(g), mode), mode);
        hbuf[(r0 + t) * I + i] = maybe_rbf(a * u, mode);
      }
    }
  }
  for (int64_t o = 0; o < H; ++o) {
    dequant_row(dw, ds, db, o, I, G, B, rowg);
    for (int64_t r0 = 0; r0 < nb; r0 += ORC_TB) {
      double acc[ORC_TB] = {0};
      for (int64_t c0 = 0; c0 < I; c0 += G) {
        float p[ORC_TB][8] = {{0}};
        for (int64_t c = c0; c < c0 + G; c += 8)
          for (int t = 0; t < ORC_TB; ++t) {
            const float* hr = hbuf + (r0 + t) * I + c;
            for (int k = 0; k < 8; ++k) p[t][k] += rowg[c + k] * hr[k];
          }
        for (int t = 0; t < ORC_TB; ++t)
          for (int k = 0; k < 8; ++k) acc[t] += p[t][k];
      }
      for (int t = 0; t < ORC_TB && r0 + t < n; ++t) out[(r0 + t) * H + o] = maybe_rbf((float)acc[t], mode);
    }
  }
}

/* Block body: the router's (or the caller's) routing, then the experts and the
 * weighted combine.  ext_ids / ext_w: [T, K] routing from the caller, or NULL
 * to run orc_router. */
static int moe_forward_impl(const OrcConfig* cfg, const OrcWeights* wt, const uint16_t* x, int64_t T,
                            const int32_t* ext_ids, const float* ext_w, float* y_f32, uint16_t* y_bf16,
                            int32_t* ids_out, float* w_out, int32_t* perm_out, int32_t* offsets_out) {
  const int64_t H = cfg->hidden, I = cfg->intermediate, E = cfg->num_experts, K = cfg->top_k;
  const int32_t G = cfg->group_size, B = cfg->bits;
  if (T < 0 || H <= 0 || I <= 0 || H % G || I % G || !(B == 4 || B == 8)) return ORC_BAD_ARG;
  if (T == 0) return ORC_OK;
  const int64_t P = T * K;
  int err = ORC_OK;
  int32_t* ids = (int32_t*)malloc(sizeof(int32_t) * (size_t)P);
  float* wts = (float*)malloc(sizeof(float) * (size_t)P);
  int32_t* perm = (int32_t*)malloc(sizeof(int32_t) * (size_t)P);
  int32_t* inv = (int32_t*)malloc(sizeof(int32_t) * (size_t)P);
  int32_t* offs = (int32_t*)malloc(sizeof(int32_t) * (size_t)(E + 1));
  float* xf = (float*)malloc(sizeof(float) * (size_t)(T * H));
  float* d = (float*)malloc(sizeof(float) * (size_t)(P * H)); /* expert outputs, slot order */
  if (!ids || !wts || !perm || !inv || !offs || !xf || !d) {
    err = ORC_NO_MEM;
    goto done;
  }
  for (int64_t i = 0; i < T * H; ++i) xf[i] = bf2f(x[i]);
  if (ext_ids) {  /* routing given by the caller (Experts::forward, gemma4.rs:842-848) */
    memcpy(ids, ext_ids, sizeof(int32_t) * (size_t)P);
    memcpy(wts, ext_w, sizeof(float) * (size_t)P);
  } else if ((err = orc_router(cfg, wt, x, T, ids, wts, NULL))) {
    goto done;
  }
  if ((err = orc_dispatch(ids, T, (int32_t)K, (int32_t)E, perm, offs, inv))) goto done;

  const int64_t wsg = I * (H * B / 32), ssg = I * (H / G); /* gate/up strides per expert */
  const int64_t wsd = H * (I * B / 32), ssd = H * (I / G); /* down strides per expert */
#pragma omp parallel
  {
    int64_t maxn = 0;
    for (int64_t e = 0; e < E; ++e) maxn = offs[e + 1] - offs[e] > maxn ? offs[e + 1] - offs[e] : maxn;
    maxn = (maxn + ORC_TB - 1) / ORC_TB * ORC_TB; /* glu_expert reads whole blocks of ORC_TB rows */
    float* xs = (float*)calloc((size_t)(maxn * H + 1), sizeof(float));
    float* hb = (float*)malloc(sizeof(float) * (size_t)(maxn * I + 1));
    float* rg = (float*)malloc(sizeof(float) * (size_t)(H > I ? H : I));
    float* ru = (float*)malloc(sizeof(float) * (size_t)H);
    float* ob = (float*)malloc(sizeof(float) * (size_t)(maxn * H + 1));
    if (!xs || !hb || !rg || !ru || !ob) {
#pragma omp atomic write
      err = ORC_NO_MEM;
    } else {
#pragma omp for schedule(dynamic, 1)
      for (int64_t e = 0; e < E; ++e) {
        const int64_t s0 = offs[e], n = offs[e + 1] - offs[e];
        if (n == 0) continue;
        for (int64_t r = 0; r < n; ++r) memcpy(xs + r * H, xf + (perm[s0 + r] / K) * H, sizeof(float) * (size_t)H);
        for (int64_t r = n; r % ORC_TB; ++r) memset(xs + r * H, 0, sizeof(float) * (size_t)H);
        glu_expert(cfg, H, I, wt->gate_w + e * wsg, wt->gate_s + e * ssg, wt->gate_b + e * ssg,
                      wt->up_w + e * wsg, wt->up_s + e * ssg, wt->up_b + e * ssg, wt->down_w + e * wsd,
                      wt->down_s + e * ssd, wt->down_b + e * ssd, xs, n, hb, rg, ru, ob);
        memcpy(d + s0 * H, ob, sizeof(float) * (size_t)(n * H));
      }
    }
    free(xs);
    free(hb);
    free(rg);
    free(ru);
    free(ob);
  }
  if (err) goto done;

  /* combine in slot order j = 0..K-1 (deepseek_v2.rs:546-548), f32 */
#pragma omp parallel for schedule(static)
  for (int64_t t = 0; t < T; ++t)
    for (int64_t h = 0; h < H; ++h) {
      float acc = 0.0f;
      for (int64_t j = 0; j < K; ++j) acc += d[(int64_t)inv[t * K + j] * H + h] * wts[t * K + j];
      y_f32[t * H + h] = acc;
    }

  /* shared experts (deepseek_v2.rs:550-552); optional sigmoid gate */
  if (cfg->shared_intermediate > 0) {
    const int64_t Is = cfg->shared_intermediate;
#pragma omp parallel
    {
      float* xs = (float*)calloc((size_t)(ORC_TB * H), sizeof(float));
      float* hb = (float*)malloc(sizeof(float) * (size_t)(ORC_TB * Is));
      float* rg = (float*)malloc(sizeof(float) * (size_t)(H > Is ? H : Is));
      float* ru = (float*)malloc(sizeof(float) * (size_t)H);
      float* ob = (float*)malloc(sizeof(float) * (size_t)(ORC_TB * H));
      if (!xs || !hb || !rg || !ru || !ob) {
#pragma omp atomic write
        err = ORC_NO_MEM;
      } else {
#pragma omp for schedule(dynamic, 1)
        for (int64_t t0 = 0; t0 < T; t0 += ORC_TB) { /* ORC_TB tokens per pass over the shared weights */
          const int64_t n = T - t0 < ORC_TB ? T - t0 : ORC_TB;
          memcpy(xs, xf + t0 * H, sizeof(float) * (size_t)(n * H));
          memset(xs + n * H, 0, sizeof(float) * (size_t)((ORC_TB - n) * H));
          glu_expert(cfg, H, Is, wt->sh_gate_w, wt->sh_gate_s, wt->sh_gate_b, wt->sh_up_w, wt->sh_up_s,
                        wt->sh_up_b, wt->sh_down_w, wt->sh_down_s, wt->sh_down_b, xs, n, hb, rg, ru, ob);
          for (int64_t t = t0; t < t0 + n; ++t) {
            float gate = 1.0f;
            if (cfg->shared_gate) {
              double a = 0.0;
              for (int64_t h = 0; h < H; ++h) a += (double)xf[t * H + h] * (double)bf2f(wt->sh_gate_vec[h]);
              gate = sigmoidf_((float)a);
            }
            for (int64_t h = 0; h < H; ++h) y_f32[t * H + h] += gate * ob[(t - t0) * H + h];
          }
        }
      }
      free(xs);
      free(hb);
      free(rg);
      free(ru);
      free(ob);
    }
    if (err) goto done;
  }
  if (y_bf16)
    for (int64_t i = 0; i < T * H; ++i) y_bf16[i] = f2bf(y_f32[i]);
  if (ids_out) memcpy(ids_out, ids, sizeof(int32_t) * (size_t)P);
  if (w_out) memcpy(w_out, wts, sizeof(float) * (size_t)P);
  if (perm_out) memcpy(perm_out, perm, sizeof(int32_t) * (size_t)P);
  if (offsets_out) memcpy(offsets_out, offs, sizeof(int32_t) * (size_t)(E + 1));
done:
  free(ids);
  free(wts);
  free(perm);
  free(inv);
  free(offs);
  free(xf);
  free(d);
  return err;
}

/* Full block: DeepseekMoe::forward (deepseek_v2.rs:520-553).
 * Outputs: y_f32 [T, H] (the reference's f32 result), y_bf16 (optional),
 * ids/weights [T, K] in canonical slot order, perm [T*K], offsets [E+1]
 * (optional).  Weights are for all E experts. */
int orc_moe_forward(const OrcConfig* cfg, const OrcWeights* wt, const uint16_t* x, int64_t T, float* y_f32,
                    uint16_t* y_bf16, int32_t* ids_out, float* w_out, int32_t* perm_out, int32_t* offsets_out) {
  return moe_forward_impl(cfg, wt, x, T, NULL, NULL, y_f32, y_bf16, ids_out, w_out, perm_out, offsets_out);
}

/* Experts::forward (gemma4.rs:842-848; the DeepSeek block's expert half,
 * deepseek_v2.rs:544-552): the experts of the given routing ids / weights
 * [T, K] and their weighted sum in f32 (+ the shared experts of cfg).  The
 * router weights of wt are not used. */
int orc_experts_forward(const OrcConfig* cfg, const OrcWeights* wt, const uint16_t* x, int64_t T,
                        const int32_t* ids, const float* weights, float* y_f32, uint16_t* y_bf16) {
  if (!ids || !weights) return ORC_BAD_ARG;
  return moe_forward_impl(cfg, wt, x, T, ids, weights, y_f32, y_bf16, NULL, NULL, NULL, NULL);
}

/* ---------------------------------------------------------- Gemma router */
typedef struct {
  int32_t hidden;       /* H */
  int32_t num_experts;  /* E */
  int32_t top_k;        /* K */
  int32_t group_size;   /* of the quantized projection (64) */
  int32_t bits;         /* 8 in the shipped checkpoint (gemma4.rs:691-694) */
  float eps;            /* rms_norm_eps */
} OrcGemmaRouterConfig;

typedef struct {
  const uint32_t* proj_w;             /* [E, H*bits/32] */
  const uint16_t *proj_s, *proj_b;    /* [E, H/group] bf16 */
  const uint16_t* scale;              /* [H] bf16, the bare learned norm weight */
  const uint16_t* per_expert_scale;   /* [E] bf16 */
} OrcGemmaRouterWeights;

/* Router::forward (gemma4.rs:716-736):
 *   w      = f32(scale) * H^-1/2          (bf16 array x array!(f32): f32)
 *   normed = fast::rms_norm(x, w, eps)    x bf16, w f32 -> f32 out:
 *            x * 1/sqrt(mean(x^2) + eps) (fp32), then * w
 *   scores = proj(normed)                 quantized linear, f32 in -> f32
 *   top-k of scores (order: score desc, id asc; MLX leaves it unspecified)
 *   w_k    = softmax_fp32(scores[top-k]) * f32(per_expert_scale[top-k])
 * ids / weights [T, K]; scores_out [T, E] optional. */
int orc_gemma_router(const OrcGemmaRouterConfig* rc, const OrcGemmaRouterWeights* rw, const uint16_t* x, int64_t T,
                     int32_t* ids, float* weights, float* scores_out) {
  const int64_t H = rc->hidden, E = rc->num_experts, K = rc->top_k;
  const int32_t G = rc->group_size, B = rc->bits;
  if (K <= 0 || K > E || H <= 0 || G <= 0 || H % G || !(B == 4 || B == 8)) return ORC_BAD_ARG;
  const float root = powf((float)H, -0.5f);
  int err = ORC_OK;
#pragma omp parallel
  {
    float* xn = (float*)malloc(sizeof(float) * (size_t)H);
    float* sc = (float*)malloc(sizeof(float) * (size_t)E);
    unsigned char* taken = (unsigned char*)malloc((size_t)E);
    if (!xn || !sc || !taken) {
#pragma omp atomic write
      err = ORC_NO_MEM;
    } else {
#pragma omp for schedule(static)
      for (int64_t t = 0; t < T; ++t) {
        const uint16_t* xr = x + t * H;
        float ss = 0.0f;
        for (int64_t h = 0; h < H; ++h) ss += bf2f(xr[h]) * bf2f(xr[h]);
        const float inv = 1.0f / sqrtf(ss / (float)H + rc->eps);
        for (int64_t h = 0; h < H; ++h) xn[h] = (bf2f(xr[h]) * inv) * (bf2f(rw->scale[h]) * root);
        for (int64_t e = 0; e < E; ++e) sc[e] = (float)qdot_row(rw->proj_w, rw->proj_s, rw->proj_b, e, H, G, B, xn);
        if (scores_out)
          for (int64_t e = 0; e < E; ++e) scores_out[t * E + e] = sc[e];
        memset(taken, 0, (size_t)E);
        for (int64_t j = 0; j < K; ++j) { /* select max, lowest id on ties */
          int64_t best = -1;
          for (int64_t e = 0; e < E; ++e)
            if (!taken[e] && (best < 0 || sc[e] > sc[best])) best = e;
          taken[best] = 1;
          ids[t * K + j] = (int32_t)best;
        }
        const float mx = sc[ids[t * K]];  /* the first pick is the maximum */
        float sum = 0.0f;
        for (int64_t j = 0; j < K; ++j) {
          weights[t * K + j] = expf(sc[ids[t * K + j]] - mx);
          sum += weights[t * K + j];
        }
        for (int64_t j = 0; j < K; ++j)
          weights[t * K + j] = (weights[t * K + j] / sum) * bf2f(rw->per_expert_scale[ids[t * K + j]]);
      }
    }
    free(xn);
    free(sc);
    free(taken);
  }
  return err;
}
