/*
 * rec_oracle.c — CPU restatement of the rec decode hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the checker for the CUDA path in
 * rec_b200/csrc; only tests/, __graft_entry__.smoke() and bench.py's
 * cpu_baseline / --impl reference legs load it.  Nothing in the product path
 * links or calls it.
 *
 * What it restates (recursive-oss/rec, paths inside the project):
 *   - MLX affine quantization used by nn.quantize and the quantized KV cache
 *     (engine/src/rec_mlx/quantized.py:26-36, model.py:45-82); restated from
 *     mlx 0.32.0's published affine_quantize algorithm (not vendored here).
 *   - int4 g64 GEMV y = sum_g s_g*sum(x*q) + b_g*sum(x)  (megakernel.py:189-232)
 *   - RMSNorm w*bf16(x*rsqrt(mean x^2+eps))               (megakernel.py:726-744)
 *   - RoPE on pairs (i, i+64), theta_i = pos*base^(-i/64) (megakernel.py:248-266,
 *     model.py:159-176)
 *   - quantize-on-append of K/V, group 64 along head_dim   (model.py:45-82)
 *   - GQA decode attention over the quantized cache, split-KV partials and a
 *     log-sum-exp merge                                    (megakernel.py:276-318,
 *     619-693; scores/sink semantics model.py:108-139)
 *   - router: softmax -> top-k -> renormalise, or sigmoid + bias selection
 *                                                          (model.py:245-254,
 *     megakernel.py:406-435,696-725, rank_routing.py:12-32)
 *   - SwiGLU experts with the reference's bf16 rounding points and the
 *     sequential bf16 expert mix                           (megakernel.py:747-798,
 *     944-969, mixed_bits.py:32-54)
 *   - lm_head GEMV + argmax with lowest-index ties        (resident_block.py:12-59)
 *   - penalty / temperature / top-k / top-p sampler with an injected uniform.
 *
 * Every floating-point operation is written out with its rounding, in the
 * canonical order the CUDA kernels use (compile with -ffp-contract=off and
 * FMA hardware: fmaf() is the IEEE fused multiply-add).  With identical
 * inputs the CUDA path and this file agree bit for bit.
 *
 * Parity against MLX itself is unpinned: mlx/mlx-lm are not installable in
 * this environment and the reference ships no golden vectors.
 */
#include <float.h>
#include <math.h>
#include <omp.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#include "../include/rec_b200.h"

#define ORC_API __attribute__((visibility("default")))

/* ------------------------------------------------------------------ types */
static inline float u2f(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }
static inline uint32_t f2u(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }

static inline float bf(uint16_t v) { return u2f((uint32_t)v << 16); }
static inline uint16_t to_bf(float f) {
  uint32_t u = f2u(f);
  if ((u & 0x7fffffffu) > 0x7f800000u) return 0x7fff; /* canonical NaN */
  u += 0x7fffu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}
static inline float rbf(float f) { return bf(to_bf(f)); }

static inline float hf(uint16_t h) {
  uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
  uint32_t exp = (h >> 10) & 0x1fu, man = h & 0x3ffu;
  if (exp == 0) {
    if (man == 0) return u2f(sign);
    float v = (float)man * 5.9604644775390625e-8f; /* 2^-24, exact */
    return sign ? -v : v;
  }
  if (exp == 31) return u2f(sign | 0x7f800000u | (man << 13));
  return u2f(sign | ((exp + 112u) << 23) | (man << 13));
}
static inline uint16_t to_hf(float f) {
  /* round to nearest even */
  uint32_t u = f2u(f), sign = (u >> 16) & 0x8000u;
  uint32_t a = u & 0x7fffffffu;
  if (a > 0x7f800000u) return (uint16_t)(sign | 0x7e00u);
  if (a >= 0x477ff000u) return (uint16_t)(sign | 0x7c00u); /* overflow -> inf */
  if (a < 0x38800000u) {                                    /* subnormal half */
    float v = u2f(a) * 16777216.0f;                          /* * 2^24, exact */
    uint32_t m = (uint32_t)rintf(v);
    return (uint16_t)(sign | m);
  }
  uint32_t exp = (a >> 23) - 112u, man = a & 0x7fffffu;
  uint32_t h = (exp << 10) | (man >> 13);
  uint32_t rem = man & 0x1fffu;
  if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h += 1;
  return (uint16_t)(sign | h);
}
static inline float sbv(uint16_t v, int sd) { return sd == REC_SCALE_FP16 ? hf(v) : bf(v); }
static inline uint16_t to_sb(float f, int sd) { return sd == REC_SCALE_FP16 ? to_hf(f) : to_bf(f); }

ORC_API uint16_t orc_to_bf(float f) { return to_bf(f); }
ORC_API uint16_t orc_to_hf(float f) { return to_hf(f); }
ORC_API float orc_hf(uint16_t h) { return hf(h); }

/* -------------------------------------------------------------- exp */
/* Cody-Waite reduction with a 16-bit head of ln2, degree-7 Taylor polynomial
 * in Horner form with fused multiply-adds, 2^n applied in two halves. */
ORC_API float orc_exp(float x) {
  if (!(x > -104.0f)) return (x != x) ? x : 0.0f;
  if (x > 88.8f) return u2f(0x7f800000u);
  const float log2e = 1.44269504088896341f;
  const float ln2_hi = 0.693145751953125f;
  const float ln2_lo = 1.42860682030941723e-6f;
  float n = rintf(x * log2e);
  float r = fmaf(-n, ln2_hi, x);
  r = fmaf(-n, ln2_lo, r);
  float p = 1.98412698412698413e-4f;
  p = fmaf(p, r, 1.38888888888888889e-3f);
  p = fmaf(p, r, 8.33333333333333333e-3f);
  p = fmaf(p, r, 4.16666666666666667e-2f);
  p = fmaf(p, r, 1.66666666666666667e-1f);
  p = fmaf(p, r, 0.5f);
  p = fmaf(p, r, 1.0f);
  p = fmaf(p, r, 1.0f);
  int e = (int)n;
  int e1 = e / 2, e2 = e - e1;
  p = p * u2f((uint32_t)(e1 + 127) << 23);
  return p * u2f((uint32_t)(e2 + 127) << 23);
}
static inline float rexp(float x) { return orc_exp(x); }
ORC_API void orc_exp_n(const float* x, float* y, int64_t n) {
  for (int64_t i = 0; i < n; ++i) y[i] = orc_exp(x[i]);
}
/* Attention exp for x <= 0 (rec_b200/csrc/attn_core.cuh aexp): n from
 * fma(x, log2e, 1.5*2^23), the same reduction and polynomial as orc_exp,
 * 2^n in one step; x <= -87 (and -inf) gives 0. */
ORC_API float orc_aexp(float x) {
  if (!(x > -87.0f)) return 0.0f;
  const float t = fmaf(x, 1.44269504088896341f, 12582912.0f);
  const float n = t - 12582912.0f;
  float r = fmaf(-n, 0.693145751953125f, x);
  r = fmaf(-n, 1.42860682030941723e-6f, r);
  float p = 1.98412698412698413e-4f;
  p = fmaf(p, r, 1.38888888888888889e-3f);
  p = fmaf(p, r, 8.33333333333333333e-3f);
  p = fmaf(p, r, 4.16666666666666667e-2f);
  p = fmaf(p, r, 1.66666666666666667e-1f);
  p = fmaf(p, r, 0.5f);
  p = fmaf(p, r, 1.0f);
  p = fmaf(p, r, 1.0f);
  const uint32_t sc = (f2u(t) + (uint32_t)(127 - 0x4B400000)) << 23;
  return p * u2f(sc);
}
static inline float aexp(float x) { return orc_aexp(x); }
ORC_API void orc_aexp_n(const float* x, float* y, int64_t n) {
  for (int64_t i = 0; i < n; ++i) y[i] = orc_aexp(x[i]);
}
static inline float rsigmoid(float g) {
  float tail = 1.0f / (1.0f + rexp(fabsf(g)));
  return g < 0.0f ? tail : 1.0f - tail;
}

/* Butterfly sum over w lanes: v[l] += v[l^off] for off = w/2..1. */
static void bfly(float* v, int w) {
  float t[32];
  for (int off = w / 2; off >= 1; off >>= 1) {
    for (int l = 0; l < w; ++l) t[l] = v[l] + v[l ^ off];
    memcpy(v, t, sizeof(float) * w);
  }
}

/* ------------------------------------------------- affine quantization */
/* mx.quantize(w, group_size=64, bits, mode="affine") for one group of fp32
 * values; codes packed little-endian into uint32 words. */
static void quant_group(const float* w, int bits, int sd, uint32_t* codes, uint16_t* s_out,
                        uint16_t* b_out) {
  const int G = 64;
  float wmax = w[0], wmin = w[0];
  for (int i = 1; i < G; ++i) {
    wmax = w[i] > wmax ? w[i] : wmax;
    wmin = w[i] < wmin ? w[i] : wmin;
  }
  const float n_bins = (float)((1 << bits) - 1);
  float scale = (wmax - wmin) / n_bins;
  scale = scale > 1e-7f ? scale : 1e-7f;
  int side = fabsf(wmin) > fabsf(wmax);
  scale = side ? scale : -scale;
  float edge = side ? wmin : wmax;
  float q0 = rintf(edge / scale);
  float bias = 0.0f;
  if (q0 != 0.0f) {
    scale = edge / q0;
    bias = edge;
  }
  int per = 32 / bits;
  for (int i = 0; i < G / per; ++i) codes[i] = 0;
  for (int i = 0; i < G; ++i) {
    float q = rintf((w[i] - bias) / scale);
    q = q < 0.0f ? 0.0f : (q > n_bins ? n_bins : q);
    codes[i / per] |= (uint32_t)q << (bits * (i % per));
  }
  *s_out = to_sb(scale, sd);
  *b_out = to_sb(bias, sd);
}

ORC_API void orc_quantize_affine(const float* w, int64_t n_groups, int bits, int sd, uint32_t* codes,
                                 uint16_t* scales, uint16_t* biases) {
  int words = 64 * bits / 32;
#pragma omp parallel for schedule(static)
  for (int64_t g = 0; g < n_groups; ++g)
    quant_group(w + g * 64, bits, sd, codes + g * words, scales + g, biases + g);
}

/* ------------------------------------------------------------ RMSNorm */
/* Sum of squares: H/8 chunks of 8 (sequential), groups of 32 chunks by
 * butterfly, group sums in order.  inv = 1/sqrt(ss/H + eps). */
static float rms_inv(const uint16_t* h, int H, float eps) {
  int groups = H / 256;
  float total = 0.0f;
  for (int g = 0; g < groups; ++g) {
    float v[32];
    for (int l = 0; l < 32; ++l) {
      float a = 0.0f;
      for (int i = 0; i < 8; ++i) {
        float x = bf(h[(g * 32 + l) * 8 + i]);
        a = fmaf(x, x, a);
      }
      v[l] = a;
    }
    bfly(v, 32);
    total = total + v[0];
  }
  float mean = total / (float)H;
  return 1.0f / sqrtf(mean + eps);
}
static void rmsnorm(const uint16_t* h, const uint16_t* w, int H, float eps, uint16_t* out) {
  float inv = rms_inv(h, H, eps);
  for (int i = 0; i < H; ++i) out[i] = to_bf(bf(w[i]) * rbf(bf(h[i]) * inv));
}
ORC_API void orc_rmsnorm(const uint16_t* h, const uint16_t* w, int H, float eps, uint16_t* out) {
  rmsnorm(h, w, H, eps, out);
}

/* ---------------------------------------------------------- int4 GEMV */
/* x in 16-bit fixed point with one power-of-two scale per vector:
 * E = exponent of max|x|, F = min(14 - E, 100), xi = rint(x * 2^F). */
typedef struct {
  int F;
  float up, down;
} FixScale;

static FixScale fix_scale(const uint16_t* x, int K) {
  float m = 0.0f;
  for (int i = 0; i < K; ++i) {
    float a = fabsf(bf(x[i]));
    m = a > m ? a : m;
  }
  int E = (int)((f2u(m) >> 23) & 0xFF) - 127;
  int F = 14 - E;
  if (F > 100) F = 100;
  FixScale fs = {F, u2f((uint32_t)(F + 127) << 23), u2f((uint32_t)(127 - F) << 23)};
  return fs;
}

/* Prepared vector: xi per element, X per group (float of an exact sum). */
typedef struct {
  int32_t* xi;
  float* X;
  FixScale fs;
} PrepX;

static PrepX prep_x(const uint16_t* x, int K) {
  PrepX p;
  p.fs = fix_scale(x, K);
  p.xi = (int32_t*)malloc(sizeof(int32_t) * K);
  p.X = (float*)malloc(sizeof(float) * (K / 64));
  for (int i = 0; i < K; ++i) p.xi[i] = (int32_t)rintf(bf(x[i]) * p.fs.up);
  for (int g = 0; g < K / 64; ++g) {
    int32_t s = 0;
    for (int j = 0; j < 64; ++j) s += p.xi[g * 64 + j];
    p.X[g] = (float)s;
  }
  return p;
}
static void free_prep(PrepX* p) {
  free(p->xi);
  free(p->X);
}

/* Exact integer dot of group g of a row with xi. */
static int32_t group_dot(const uint32_t* wrow, const int32_t* xi, int g) {
  int64_t d = 0;
  for (int j = 0; j < 64; ++j) {
    int e = g * 64 + j;
    d += (int64_t)((wrow[e >> 3] >> (4 * (e & 7))) & 15u) * xi[e];
  }
  return (int32_t)d;
}

/* One row in the canonical lane order (see rec_b200/csrc/qdot.cuh). */
static float rowdot(const uint32_t* wrow, const uint16_t* srow, const uint16_t* brow, int sd, int K,
                    const PrepX* px) {
  int wide = (K % 2048) == 0;
  int T = wide ? 32 : 4, SEG = wide ? K / 2048 : 1, GPL = wide ? 1 : (K / 64) / 4;
  float total = 0.0f;
  for (int seg = 0; seg < SEG; ++seg) {
    float v[32];
    for (int l = 0; l < T; ++l) {
      float acc = 0.0f;
      for (int m = 0; m < GPL; ++m) {
        int g = wide ? 32 * seg + l : l + 4 * m;
        int32_t D = group_dot(wrow, px->xi, g);
        acc = fmaf(sbv(srow[g], sd), (float)D, acc);
        acc = fmaf(sbv(brow[g], sd), px->X[g], acc);
      }
      v[l] = acc;
    }
    bfly(v, T);
    total = seg == 0 ? v[0] : total + v[0];
  }
  return total * px->fs.down;
}

static void gemv(const RecQMat* m, int sd, int64_t row0, int64_t n, int K, const uint16_t* x,
                 float* yf, uint16_t* y) {
  PrepX px = prep_x(x, K);
  const uint32_t* W = (const uint32_t*)m->w;
  const uint16_t* S = (const uint16_t*)m->scales;
  const uint16_t* B = (const uint16_t*)m->biases;
#pragma omp parallel for schedule(static)
  for (int64_t r = 0; r < n; ++r) {
    int64_t row = row0 + r;
    float v = rowdot(W + row * (K / 8), S + row * (K / 64), B + row * (K / 64), sd, K, &px);
    if (yf) yf[r] = v;
    if (y) y[r] = to_bf(v);
  }
  free_prep(&px);
}

ORC_API void orc_gemv_int4(const uint32_t* w, const uint16_t* s, const uint16_t* b, int sd,
                           int64_t n, int K, const uint16_t* x, uint16_t* y) {
  RecQMat m = {w, s, b};
  gemv(&m, sd, 0, n, K, x, NULL, y);
}

/* --------------------------------------------------------- embedding */
static void embed(const RecQMat* m, int sd, int H, int token, int bits, uint16_t* h) {
  const uint32_t* W = (const uint32_t*)m->w + (int64_t)token * (H * bits / 32);
  const uint16_t* S = (const uint16_t*)m->scales + (int64_t)token * (H / 64);
  const uint16_t* B = (const uint16_t*)m->biases + (int64_t)token * (H / 64);
  for (int i = 0; i < H; ++i) {
    float q = bits == 8 ? (float)((W[i / 4] >> (8 * (i % 4))) & 255u) : (float)((W[i / 8] >> (4 * (i % 8))) & 15u);
    h[i] = to_bf(fmaf(sbv(S[i / 64], sd), q, sbv(B[i / 64], sd)));
  }
}

/* ------------------------------------------------------------- RoPE */
/* cos/sin of pos*base^(-i/64), computed in double and rounded to float. */
ORC_API void orc_rope_table(float theta, int32_t pos0, int32_t n, float* cs) {
  for (int p = 0; p < n; ++p)
    for (int i = 0; i < 64; ++i) {
      double inv = pow((double)theta, -(double)i / 64.0);
      double a = (double)(pos0 + p) * inv;
      cs[(int64_t)p * 128 + i] = (float)cos(a);
      cs[(int64_t)p * 128 + 64 + i] = (float)sin(a);
    }
}
static void rope_head(uint16_t* x, const float* cs) {
  for (int i = 0; i < 64; ++i) {
    float a = bf(x[i]), b = bf(x[i + 64]), c = cs[i], s = cs[64 + i];
    float lo = fmaf(a, c, -(b * s));
    float hi = fmaf(a, s, b * c);
    x[i] = to_bf(lo);
    x[i + 64] = to_bf(hi);
  }
}
/* per-head RMSNorm over 128 (q_norm/k_norm): lane l holds dims 4l..4l+3,
 * sequential squares, butterfly, inv = 1/sqrt(ss/128 + eps). */
static void head_norm(uint16_t* x, const uint16_t* w, float eps) {
  float v[32];
  for (int l = 0; l < 32; ++l) {
    float a = 0.0f;
    for (int j = 0; j < 4; ++j) {
      float t = bf(x[4 * l + j]);
      a = fmaf(t, t, a);
    }
    v[l] = a;
  }
  bfly(v, 32);
  float inv = 1.0f / sqrtf(v[0] / 128.0f + eps);
  for (int d = 0; d < 128; ++d) x[d] = to_bf(bf(w[d]) * rbf(bf(x[d]) * inv));
}

/* ------------------------------------------------- KV quantized append */
/* K codes `bits` wide, V codes `vbits` wide (the reference's mixed cache keeps
 * K at 8 and V at 4 bits, model.py:35-37,40-82). */
static void kv_store(const RecKVLayer* kv, int Hkv, int C, int bits, int vbits, int pos, const uint16_t* k,
                     const uint16_t* v) {
  if (bits == 16) { /* bf16 rows, stored as they are */
    for (int g = 0; g < Hkv; ++g) {
      int64_t slot = (int64_t)g * C + pos;
      memcpy((uint16_t*)kv->k_codes + slot * 128, k + g * 128, 256);
      memcpy((uint16_t*)kv->v_codes + slot * 128, v + g * 128, 256);
    }
    return;
  }
  int words = 128 * bits / 32, vwords = 128 * vbits / 32;
  for (int g = 0; g < Hkv; ++g)
    for (int half = 0; half < 2; ++half) {
      int64_t slot = (int64_t)g * C + pos;
      float wk[64], wv[64];
      for (int i = 0; i < 64; ++i) {
        wk[i] = bf(k[g * 128 + half * 64 + i]);
        wv[i] = bf(v[g * 128 + half * 64 + i]);
      }
      quant_group(wk, bits, REC_SCALE_BF16, (uint32_t*)kv->k_codes + slot * words + half * (words / 2),
                  (uint16_t*)kv->k_scales + slot * 2 + half, (uint16_t*)kv->k_biases + slot * 2 + half);
      quant_group(wv, vbits, REC_SCALE_BF16, (uint32_t*)kv->v_codes + slot * vwords + half * (vwords / 2),
                  (uint16_t*)kv->v_scales + slot * 2 + half, (uint16_t*)kv->v_biases + slot * 2 + half);
    }
}
ORC_API void orc_kv_store(const RecKVLayer* kv, int Hkv, int C, int bits, int pos, const uint16_t* k,
                          const uint16_t* v) {
  kv_store(kv, Hkv, C, bits, bits, pos, k, v);
}

/* ---------------------------------------------------------- attention */
#define ATT_BLOCK 256
#define ATT_TILE 32
#define ATT_SUPER 64 /* blocks per super-chunk */
/* blocks per work item: 1 while the context fits one super-chunk, 4 beyond */
static int att_item_blocks(int nblocks) { return nblocks <= ATT_SUPER ? 1 : 4; }
#define ATT_WARPS 8  /* tiles of a block = warps of an item */
#define NEG_INF (-INFINITY)

typedef struct {
  float m, l;
  float acc[128];
} Partial;

static void p_empty(Partial* p) {
  p->m = NEG_INF;
  p->l = 0.0f;
  memset(p->acc, 0, sizeof(p->acc));
}
/* a <- merge(a, b) */
static void p_merge(Partial* a, const Partial* b) {
  if (b->m == NEG_INF) return;
  if (a->m == NEG_INF) {
    *a = *b;
    return;
  }
  float m = a->m > b->m ? a->m : b->m;
  float a1 = rexp(a->m - m), a2 = rexp(b->m - m);
  a->l = fmaf(a->l, a1, b->l * a2);
  for (int d = 0; d < 128; ++d) a->acc[d] = fmaf(a->acc[d], a1, b->acc[d] * a2);
  a->m = m;
}

static inline uint32_t kv_code(const uint32_t* row, int bits, int d) {
  return bits == 4 ? (row[d >> 3] >> (4 * (d & 7))) & 15u : (row[d >> 2] >> (8 * (d & 3))) & 255u;
}

/* Prepared query of one head: qs = bf16(q / sqrt(128)); 16-bit fixed point
 * qi = rint(qs * 2^F), F = min(14 - exponent(max|qs| * (1 + 2^-7)), 100); QS[g] = float of
 * the exact sum of qi over group g; down = 2^-F. */
typedef struct {
  int32_t qi[128];
  float QS[2];
  float down;
  float qf[128]; /* bf16 cache: qs = fp32(q) / sqrt(128) in fp32, unrounded */
} QPrep;

static void prep_query(const uint16_t* q, QPrep* Q) {
  float qs[128], mx = 0.0f;
  for (int d = 0; d < 128; ++d) {
    Q->qf[d] = bf(q[d]) * 0.0883883476483184405f;
    qs[d] = rbf(Q->qf[d]);
    float a = fabsf(qs[d]);
    mx = a > mx ? a : mx;
  }
  /* the factor 1 + 2^-7 keeps |qi| <= 32512: both byte limbs are signed */
  uint32_t u = f2u(mx * 1.0078125f);
  int E = (int)((u >> 23) & 0xFF) - 127;
  int F = 14 - E;
  if (F > 100) F = 100;
  float up = ldexpf(1.0f, F);
  int32_t S[2] = {0, 0};
  for (int d = 0; d < 128; ++d) {
    Q->qi[d] = (int32_t)rintf(qs[d] * up);
    S[d >> 6] += Q->qi[d];
  }
  Q->QS[0] = (float)S[0];
  Q->QS[1] = (float)S[1];
  Q->down = ldexpf(1.0f, -F);
}

/* score = bf16(fma(b1, QS1, fma(s1, D1, fma(b0, QS0, s0*D0))) * 2^-F) with
 * D_g = sum over group g of qi * code, exact. */
static float att_score(const QPrep* Q, const uint32_t* krow, const uint16_t* ks, const uint16_t* kb, int bits) {
  int32_t D[2] = {0, 0};
  for (int d = 0; d < 128; ++d) D[d >> 6] += Q->qi[d] * (int32_t)kv_code(krow, bits, d);
  float t = fmaf(bf(kb[0]), Q->QS[0], bf(ks[0]) * (float)D[0]);
  t = fmaf(bf(ks[1]), (float)D[1], t);
  t = fmaf(bf(kb[1]), Q->QS[1], t);
  return rbf(t * Q->down);
}

/* Canonical tile sum (attn_core.cuh tile_sum): thread tq of a head holds
 * v[2nt + j] = x[8nt + 2tq + j]; S_tq = ((v0+v1)+(v2+v3))+((v4+v5)+(v6+v7));
 * result (S0+S1)+(S2+S3). */
static float tile_sum(const float* x) {
  float S[4];
  for (int tq = 0; tq < 4; ++tq) {
    float v[8];
    for (int nt = 0; nt < 4; ++nt)
      for (int j = 0; j < 2; ++j) v[2 * nt + j] = x[8 * nt + 2 * tq + j];
    S[tq] = ((v[0] + v[1]) + (v[2] + v[3])) + ((v[4] + v[5]) + (v[6] + v[7]));
  }
  return (S[0] + S[1]) + (S[2] + S[3]);
}

/* Folds the tile of one q head over tokens [t0, t0+32) ∩ [lo, T) into the
 * running state st (attn_core.cuh tile_fold; lo > 0: the first position of a
 * sliding window; a tile with no such token leaves st unchanged):
 *   m' = max(m, max score); alpha = aexp(m - m'); p_j = aexp(s_j - m') (0 beyond T);
 *   l' = fma(l, alpha, tile_sum(p));
 *   per V group (64 dims): w_j = p_j * scale_j, x_j = p_j * bias_j (0 beyond T);
 *      F = min(14 - exponent(max|w| * (1 + 2^-7)), 100); wq_j = rint(w_j * 2^F);
 *      acc_d' = fma(acc_d, alpha, fma(float(sum_j wq_j * code_jd), 2^-F, tile_sum(x))). */
/* The tile over a bf16 cache (attn_bf16.cuh tile_fold_bf16): the score of
 * tile row r sums its 32 four-dim chunks from chunk r on, (c + r) mod 32, in
 * fp32 fused multiply-adds (no bf16 rounding); l adds the butterfly sum of p
 * over the 32 rows; acc_d = fma(acc_d, alpha, PV_d), PV_d a fused
 * multiply-add chain over the valid rows in order. */
static void att_tile_bf16(const QPrep* Q, const RecKVLayer* kv, int g, int C, int t0, int T, int base, int lo,
                          Partial* st) {
  const uint16_t* K = (const uint16_t*)kv->k_codes;
  const uint16_t* V = (const uint16_t*)kv->v_codes;
  int nvalid = T - t0;
  if (nvalid > ATT_TILE) nvalid = ATT_TILE;
  const int first = lo > t0 ? lo - t0 : 0;
  if (nvalid <= first) return;
  float s[ATT_TILE], p[ATT_TILE];
  float mt = NEG_INF;
  for (int r = 0; r < ATT_TILE; ++r) {
    s[r] = NEG_INF;
    if (r < first || r >= nvalid) continue;
    const uint16_t* krow = K + ((int64_t)g * C + t0 - base + r) * 128;
    float a = 0.0f;
    for (int c = 0; c < 32; ++c) {
      const int cc = (c + r) & 31;
      for (int i = 0; i < 4; ++i) a = fmaf(Q->qf[4 * cc + i], bf(krow[4 * cc + i]), a);
    }
    s[r] = a;
    mt = fmaxf(mt, a);
  }
  const float mn = fmaxf(st->m, mt);
  const float alpha = aexp(st->m - mn);
  float v[32];
  for (int r = 0; r < ATT_TILE; ++r) v[r] = p[r] = (r >= first && r < nvalid) ? aexp(s[r] - mn) : 0.0f;
  bfly(v, 32);
  st->l = fmaf(st->l, alpha, v[0]);
  for (int d = 0; d < 128; ++d) {
    float pv = 0.0f;
    for (int r = first; r < nvalid; ++r) pv = fmaf(p[r], bf(V[((int64_t)g * C + t0 - base + r) * 128 + d]), pv);
    st->acc[d] = fmaf(st->acc[d], alpha, pv);
  }
  st->m = mn;
}

static void att_tile(const QPrep* Q, const RecKVLayer* kv, int g, int C, int bits, int vbits, int t0, int T,
                     int base, int lo, Partial* st) {
  if (bits == 16) {
    att_tile_bf16(Q, kv, g, C, t0, T, base, lo, st);
    return;
  }
  int words = 128 * bits / 32, vwords = 128 * vbits / 32;
  const uint32_t* KC = (const uint32_t*)kv->k_codes;
  const uint32_t* VC = (const uint32_t*)kv->v_codes;
  const uint16_t *KS = (const uint16_t*)kv->k_scales, *KB = (const uint16_t*)kv->k_biases;
  const uint16_t *VS = (const uint16_t*)kv->v_scales, *VB = (const uint16_t*)kv->v_biases;
  int nvalid = T - t0;
  if (nvalid > ATT_TILE) nvalid = ATT_TILE;
  const int first = lo > t0 ? lo - t0 : 0;
  if (nvalid <= first) return;
  float s[ATT_TILE], p[ATT_TILE];
  float mt = NEG_INF;
  for (int j = 0; j < ATT_TILE; ++j) {
    int64_t slot = (int64_t)g * C + t0 - base + j;
    s[j] = j >= first && j < nvalid ? att_score(Q, KC + slot * words, KS + slot * 2, KB + slot * 2, bits) : NEG_INF;
    mt = fmaxf(mt, s[j]);
  }
  const float mn = fmaxf(st->m, mt);
  const float alpha = aexp(st->m - mn);
  for (int j = 0; j < ATT_TILE; ++j) p[j] = aexp(s[j] - mn);
  st->l = fmaf(st->l, alpha, tile_sum(p));
  for (int gr = 0; gr < 2; ++gr) {
    float w[ATT_TILE], x[ATT_TILE];
    float mx = 0.0f;
    for (int j = 0; j < ATT_TILE; ++j) {
      int64_t slot = (int64_t)g * C + t0 - base + j;
      w[j] = j >= first && j < nvalid ? p[j] * bf(VS[slot * 2 + gr]) : 0.0f;
      x[j] = j >= first && j < nvalid ? p[j] * bf(VB[slot * 2 + gr]) : 0.0f;
      mx = fmaxf(mx, fabsf(w[j]));
    }
    int E = (int)((f2u(mx * 1.0078125f) >> 23) & 0xFF) - 127;
    int F = 14 - E;
    if (F > 100) F = 100;
    float up = ldexpf(1.0f, F), down = ldexpf(1.0f, -F);
    int32_t wq[ATT_TILE];
    for (int j = 0; j < ATT_TILE; ++j) wq[j] = (int32_t)rintf(w[j] * up);
    const float B = tile_sum(x);
    for (int d = 64 * gr; d < 64 * gr + 64; ++d) {
      int32_t acc = 0;
      for (int j = first; j < nvalid; ++j) {
        int64_t slot = (int64_t)g * C + t0 - base + j;
        acc += wq[j] * (int32_t)kv_code(VC + slot * vwords, vbits, d);
      }
      st->acc[d] = fmaf(st->acc[d], alpha, fmaf((float)acc, down, B));
    }
  }
  st->m = mn;
}

/* Partial of one q head over item it (blocks [nbi*it, nbi*it+nbi) ∩ blocks < T):
 * warp w folds tiles 8b + w of the item's blocks in order into its running
 * state; the eight warp states are folded as a tree ((w0 w1)(w2 w3))((w4 w5)(w6 w7)). */
static void att_item(const QPrep* Q, const RecKVLayer* kv, int g, int C, int bits, int vbits, int it, int T,
                     int base, int lo, Partial* out) {
  const int nbi = att_item_blocks((T + ATT_BLOCK - 1) / ATT_BLOCK);
  Partial st[ATT_WARPS];
  for (int w = 0; w < ATT_WARPS; ++w) {
    p_empty(&st[w]);
    for (int b = it * nbi; b < (it + 1) * nbi; ++b) {
      int t0 = b * ATT_BLOCK + w * ATT_TILE;
      if (t0 >= T) break;
      att_tile(Q, kv, g, C, bits, vbits, t0, T, base, lo, &st[w]);
    }
  }
  for (int step = 1; step < ATT_WARPS; step *= 2)
    for (int w = 0; w < ATT_WARPS; w += 2 * step) p_merge(&st[w], &st[w + step]);
  *out = st[0];
}

/* Super-chunk partials of every q head for super-chunks [s_lo, s_hi) of a
 * context of T tokens (items and blocks numbered as for the whole context):
 * supers[h * (s_hi - s_lo) + s - s_lo] = items of super s (64 blocks) merged
 * in order.  The cache holds tokens from `base` on (token t in slot t - base
 * of each head's C rows): a rank of a split session passes its own slice. */
static void attention_supers(const uint16_t* q, const RecKVLayer* kv, int Hq, int Hkv, int C, int bits, int vbits,
                             int T, int base, int lo, int s_lo, int s_hi, Partial* supers) {
  int nblocks = (T + ATT_BLOCK - 1) / ATT_BLOCK;
  int nbi = att_item_blocks(nblocks), per_super = ATT_SUPER / nbi;
  int nitems = (nblocks + nbi - 1) / nbi;
  int ns = s_hi - s_lo;
#pragma omp parallel for schedule(dynamic)
  for (int h = 0; h < Hq; ++h) {
    QPrep Q;
    prep_query(q + h * 128, &Q);
    int g = h / (Hq / Hkv);
    for (int s = s_lo; s < s_hi; ++s) {
      Partial* S = &supers[h * ns + s - s_lo];
      p_empty(S);
      for (int it = s * per_super; it < (s + 1) * per_super && it < nitems; ++it) {
        Partial P;
        att_item(&Q, kv, g, C, bits, vbits, it, T, base, lo, &P);
        p_merge(S, &P);
      }
    }
  }
}

ORC_API void orc_attention_supers_shard(const uint16_t* q, const RecKVLayer* kv, int Hq, int Hkv, int C, int bits,
                                        int T, int base, int s_lo, int s_hi, Partial* supers) {
  attention_supers(q, kv, Hq, Hkv, C, bits, bits, T, base, 0, s_lo, s_hi, supers);
}

/* A sliding-window layer: tokens [lo, T) only, lo = max(0, T - window)
 * (attn.cuh window_start); items below lo stay empty. */
ORC_API void orc_attention_supers_window(const uint16_t* q, const RecKVLayer* kv, int Hq, int Hkv, int C, int bits,
                                         int T, int window, Partial* supers, int n_super) {
  const int lo = window > 0 && T > window ? T - window : 0;
  attention_supers(q, kv, Hq, Hkv, C, bits, bits, T, 0, lo, 0, n_super, supers);
}

/* The same with V codes vbits wide (a mixed cache). */
ORC_API void orc_attention_supers_kv(const uint16_t* q, const RecKVLayer* kv, int Hq, int Hkv, int C, int bits,
                                     int vbits, int T, int window, Partial* supers, int n_super) {
  const int lo = window > 0 && T > window ? T - window : 0;
  attention_supers(q, kv, Hq, Hkv, C, bits, vbits, T, 0, lo, 0, n_super, supers);
}

/* Super-chunk partials of every q head over tokens [0, T) of one layer's
 * cache: supers[h * n_super + s]. */
ORC_API void orc_attention_supers(const uint16_t* q, const RecKVLayer* kv, int Hq, int Hkv, int C,
                                  int bits, int T, Partial* supers, int n_super) {
  orc_attention_supers_shard(q, kv, Hq, Hkv, C, bits, T, 0, 0, n_super, supers);
}

ORC_API void orc_attention_final(const Partial* supers, int Hq, int n_super, const uint16_t* sinks,
                                 uint16_t* out) {
  for (int h = 0; h < Hq; ++h) {
    Partial F;
    p_empty(&F);
    if (sinks) {
      F.m = bf(sinks[h]);
      F.l = 1.0f;
    }
    for (int s = 0; s < n_super; ++s) p_merge(&F, &supers[h * n_super + s]);
    for (int d = 0; d < 128; ++d) out[h * 128 + d] = to_bf(F.acc[d] / F.l);
  }
}

ORC_API int orc_partial_bytes(void) { return (int)sizeof(Partial); }

/* -------------------------------------------------------------- router */
/* bf16 router logits: lane l owns 8-element chunks l, l+32, ...; sequential
 * fused multiply-adds, butterfly, round to bf16. */
static float router_logit(const uint16_t* wrow, const uint16_t* x, int H) {
  float v[32];
  for (int l = 0; l < 32; ++l) {
    float a = 0.0f;
    for (int c = l; c < H / 8; c += 32)
      for (int i = 0; i < 8; ++i) a = fmaf(bf(wrow[c * 8 + i]), bf(x[c * 8 + i]), a);
    v[l] = a;
  }
  bfly(v, 32);
  return rbf(v[0]);
}

/* Selection + weights.  Softmax: p = exp(l - max) / sum (lane l sums experts
 * l, l+32, ... in order, then butterfly).  Sigmoid: p = sigmoid(l), choice
 * = p + bias.  top-k by choice, ties -> lower index; weights
 * = p_sel / (sum_sel + 1e-20) with the sum taken in rank order. */
/* top-k of `choice` (ties -> lower index), weights = p_sel/(sum + 1e-20) with
 * the sum taken in rank order (rank_routing.py:12-32, megakernel.py:696-725). */
ORC_API void orc_select_topk(const float* p, const float* choice, int E, int k, int32_t* ids,
                             float* weights) {
  int taken[1024] = {0};
  for (int r = 0; r < k; ++r) {
    /* a NaN choice ranks below every number; ties keep the lower index */
    int best = -1;
    for (int e = 0; e < E; ++e)
      if (!taken[e] && (best < 0 || (!isnan(choice[e]) && (isnan(choice[best]) || choice[e] > choice[best]))))
        best = e;
    taken[best] = 1;
    ids[r] = best;
  }
  float sum = 0.0f;
  for (int r = 0; r < k; ++r) sum = sum + p[ids[r]];
  sum = sum + 1e-20f;
  for (int r = 0; r < k; ++r) weights[r] = p[ids[r]] / sum;
}

/* bf16 expert mix of H elements: out[i] = mix over r of down[r*H + i]. */
ORC_API void orc_mix(const uint16_t* down, int H, const float* w, int k, uint16_t* out);

ORC_API void orc_route(const float* logits, int E, int k, int mode, const float* bias, int32_t* ids,
                       float* weights) {
  float p[1024], choice[1024];
  if (mode == REC_ROUTER_SOFTMAX) {
    float mx = NEG_INF;
    for (int e = 0; e < E; ++e) mx = logits[e] > mx ? logits[e] : mx;
    float v[32];
    for (int l = 0; l < 32; ++l) {
      float a = 0.0f;
      for (int e = l; e < E; e += 32) a = a + rexp(logits[e] - mx);
      v[l] = a;
    }
    bfly(v, 32);
    for (int e = 0; e < E; ++e) {
      p[e] = rexp(logits[e] - mx) / v[0];
      choice[e] = p[e];
    }
  } else {
    for (int e = 0; e < E; ++e) {
      p[e] = rsigmoid(logits[e]);
      choice[e] = p[e] + bias[e];
    }
  }
  orc_select_topk(p, choice, E, k, ids, weights);
}

ORC_API void orc_router_logits(const uint16_t* W, const uint16_t* x, int E, int H, float* logits) {
  for (int e = 0; e < E; ++e) logits[e] = router_logit(W + (int64_t)e * H, x, H);
}

/* SwiGLU: sig = bf16(sigmoid(g)), act = bf16(bf16(g*sig)*u) (megakernel.py:770-774). */
static inline uint16_t swiglu(float g, float u) {
  float sig = rbf(rsigmoid(g));
  return to_bf(rbf(g * sig) * u);
}
ORC_API uint16_t orc_swiglu(uint16_t g, uint16_t u) { return swiglu(bf(g), bf(u)); }

/* Expert mix for one element: m = bf16(d_0*bf16(w_0)) + 0, then for r >= 1
 * m = bf16(bf16(d_r*bf16(w_r)) + 0 + m) (mixed_bits.py:42-54). */
static inline float mix_elem(const uint16_t* d, int stride, const float* w, int k) {
  float m = 0.0f;
  for (int r = 0; r < k; ++r) {
    float t = rbf(bf(d[r * stride]) * rbf(w[r])) + 0.0f;
    m = r == 0 ? t : rbf(t + m);
  }
  return m;
}

ORC_API void orc_mix(const uint16_t* down, int H, const float* w, int k, uint16_t* out) {
  for (int i = 0; i < H; ++i) out[i] = to_bf(mix_elem(down + i, H, w, k));
}

/* SwiGLU MLP of one matrix triple on normalised x (a dense layer, or the
 * shared expert): out = down(bf16(bf16(g*sig)*u)), I rows
 * (model.py:216-224; the dense down is one GEMV of K = I). */
static void mlp(const RecQMat* gm, const RecQMat* um, const RecQMat* dm, int sd, int H, int I, const uint16_t* xn,
                uint16_t* out) {
  uint16_t* g = (uint16_t*)malloc(sizeof(uint16_t) * I);
  uint16_t* u = (uint16_t*)malloc(sizeof(uint16_t) * I);
  uint16_t* act = (uint16_t*)malloc(sizeof(uint16_t) * I);
  gemv(gm, sd, 0, I, H, xn, NULL, g);
  gemv(um, sd, 0, I, H, xn, NULL, u);
  for (int i = 0; i < I; ++i) act[i] = swiglu(bf(g[i]), bf(u[i]));
  gemv(dm, sd, 0, H, I, act, NULL, out);
  free(g);
  free(u);
  free(act);
}

/* MoE FFN on normalised x: writes the bf16 mix (without residual). */
static void moe_ffn(const RecModelDesc* md, const RecLayerWeights* L, const uint16_t* xn,
                    const int32_t* ids, const float* w, uint16_t* mix, uint16_t* act_out,
                    uint16_t* down_out) {
  int H = md->hidden, I = md->moe_inter, k = md->top_k, sd = md->scale_dtype;
  uint16_t* act = (uint16_t*)malloc(sizeof(uint16_t) * k * I);
  uint16_t* dn = (uint16_t*)malloc(sizeof(uint16_t) * k * H);
  uint16_t* g = (uint16_t*)malloc(sizeof(uint16_t) * I);
  uint16_t* u = (uint16_t*)malloc(sizeof(uint16_t) * I);
  for (int r = 0; r < k; ++r) {
    gemv(&L->gate, sd, (int64_t)ids[r] * I, I, H, xn, NULL, g);
    gemv(&L->up, sd, (int64_t)ids[r] * I, I, H, xn, NULL, u);
    for (int i = 0; i < I; ++i) act[r * I + i] = swiglu(bf(g[i]), bf(u[i]));
    gemv(&L->down, sd, (int64_t)ids[r] * H, H, I, act + r * I, NULL, dn + r * H);
  }
  for (int i = 0; i < H; ++i) mix[i] = to_bf(mix_elem(dn + i, H, w, k));
  if (act_out) memcpy(act_out, act, sizeof(uint16_t) * k * I);
  if (down_out) memcpy(down_out, dn, sizeof(uint16_t) * k * H);
  free(act);
  free(dn);
  free(g);
  free(u);
}

/* The FFN block of one layer on the residual h -> h_out:
 *   dense layer (REC_LAYER_DENSE): h + bf16 MLP output;
 *   MoE layer: router, experts, bf16 mix in rank order; with a shared expert
 *   (md->shared_inter > 0) mlp = bf16(mix + shared) (megakernel.py:955-958);
 *   h_out = bf16(h + mlp).
 * ids / w / act / down describe the routed experts (untouched for a dense
 * layer). */
ORC_API void orc_moe(const RecModelDesc* md, const RecLayerWeights* L, const uint16_t* h,
                     int32_t* ids, float* w, uint16_t* act, uint16_t* down, uint16_t* h_out) {
  int H = md->hidden, E = md->n_experts;
  uint16_t* xn = (uint16_t*)malloc(sizeof(uint16_t) * H);
  float* logits = (float*)malloc(sizeof(float) * E);
  uint16_t* mix = (uint16_t*)malloc(sizeof(uint16_t) * H);
  rmsnorm(h, (const uint16_t*)L->post_norm, H, md->rms_eps, xn);
  if (L->kind & REC_LAYER_DENSE) {
    mlp(&L->gate, &L->up, &L->down, md->scale_dtype, H, md->dense_inter, xn, mix);
  } else {
    orc_router_logits((const uint16_t*)L->router, xn, E, H, logits);
    orc_route(logits, E, md->top_k, md->router_mode, (const float*)L->expert_bias, ids, w);
    moe_ffn(md, L, xn, ids, w, mix, act, down);
    if (md->shared_inter > 0) {
      uint16_t* sh = (uint16_t*)malloc(sizeof(uint16_t) * H);
      mlp(&L->shared_gate, &L->shared_up, &L->shared_down, md->scale_dtype, H, md->shared_inter, xn, sh);
      for (int i = 0; i < H; ++i) mix[i] = to_bf(bf(mix[i]) + bf(sh[i]));
      free(sh);
    }
  }
  for (int i = 0; i < H; ++i) h_out[i] = to_bf(bf(h[i]) + bf(mix[i]));
  free(xn);
  free(logits);
  free(mix);
}

/* ------------------------------------------------------- argmax / head */
static int32_t argmax_bf16(const uint16_t* x, int64_t n) {
  float best = NEG_INF;
  int32_t idx = -1;
  for (int64_t i = 0; i < n; ++i) {
    float v = bf(x[i]);
    if (v > best || idx < 0) {
      if (v != v) continue;
      best = v;
      idx = (int32_t)i;
    }
  }
  return idx;
}
ORC_API int32_t orc_argmax_bf16(const uint16_t* x, int64_t n) { return argmax_bf16(x, n); }

/* Natural logarithm in the kernels' canonical form (rec_b200/csrc/common.cuh
 * rlog): x = m*2^e, m in [sqrt(1/2), sqrt(2)); atanh series in
 * f = (m-1)/(m+1) through f^13 by Horner in f^2. */
ORC_API float orc_log(float x) {
  if (x != x) return x;
  if (x == 0.0f) return -INFINITY;
  if (x < 0.0f) return NAN;
  if (isinf(x)) return x;
  uint32_t u;
  memcpy(&u, &x, 4);
  int e = 0;
  if (u < 0x00800000u) {
    float y = x * 16777216.0f;
    memcpy(&u, &y, 4);
    e = -24;
  }
  e += (int)(u >> 23) - 127;
  uint32_t mu = (u & 0x007fffffu) | 0x3f800000u;
  float m;
  memcpy(&m, &mu, 4);
  if (m > 1.41421353816986084f) {
    m = m * 0.5f;
    e += 1;
  }
  float f = (m - 1.0f) / (m + 1.0f);
  float f2 = f * f;
  float p = 7.69230769230769231e-2f;
  p = fmaf(p, f2, 9.09090909090909091e-2f);
  p = fmaf(p, f2, 1.11111111111111111e-1f);
  p = fmaf(p, f2, 1.42857142857142857e-1f);
  p = fmaf(p, f2, 2.00000000000000000e-1f);
  p = fmaf(p, f2, 3.33333333333333333e-1f);
  p = p * f2;
  float f2x = 2.0f * f;
  float lnm = fmaf(f2x, p, f2x);
  float ef = (float)e;
  return fmaf(ef, 0.693145751953125f, fmaf(ef, 1.42860682030941723e-6f, lnm));
}
static inline float rlog(float x) { return orc_log(x); }
ORC_API void orc_log_n(const float* x, float* y, int64_t n) {
  for (int64_t i = 0; i < n; ++i) y[i] = orc_log(x[i]);
}
static inline float gumbel(float u) { return -rlog(-rlog(u)); }

typedef struct {
  float x;
  int32_t i;
} Cand;
/* descending (x, index) */
static int cand_desc(const void* pa, const void* pb) {
  const Cand *a = (const Cand*)pa, *b = (const Cand*)pb;
  if (a->x != b->x) return a->x > b->x ? -1 : 1;
  return a->i > b->i ? -1 : (a->i < b->i ? 1 : 0);
}

#define SAMPLE_THREADS 1024
#define SAMPLE_CLUSTER 8
#define SAMPLE_MAX_CAND 1024

/* Sampling head of one row (rec_b200/csrc/sample.cuh states the rule):
 * penalties over the history, then greedy argmax, or Gumbel-max with the
 * injected uniforms u[V] over all logits (top_k = 0) or over the reference's
 * joint top-k / top-p filter (engine.py:279-301, masked_sampling.py:98-125,
 * filtered_sampling.py:7-22, sampling.py:48-52).  allow (optional, bit i & 31
 * of word i >> 5 per id) is the grammar mask.  Returns -1 when more than
 * 1,024 logits tie at the top-k threshold, no id is allowed, or no candidate
 * is finite. */
ORC_API int32_t orc_sample_masked(const uint16_t* logits, int64_t V, const int32_t* hist, int n_hist,
                                  const RecSampling* sp, const float* u, const uint32_t* allow) {
  const int pen = sp->repetition_penalty != 1.0f || sp->presence_penalty != 0.0f;
  /* grammar mask: disallowed ids are -inf after the penalties; top-k counts
   * the allowed ids (rec_b200/csrc/sample.cuh) */
  int top_k = sp->top_k;
  if (allow) {
    int64_t n_allowed = 0;
    for (int64_t i = 0; i < V; ++i) n_allowed += (allow[i >> 5] >> (i & 31)) & 1u;
    if (n_allowed == 0) return -1;
    if (n_allowed < top_k) top_k = (int)n_allowed;
  }
  uint8_t* seen = (uint8_t*)calloc((size_t)V, 1);
  if (pen)
    for (int i = 0; i < n_hist; ++i)
      if (hist[i] >= 0 && hist[i] < V) seen[hist[i]] = 1;
  float* x = (float*)malloc(sizeof(float) * V);
  for (int64_t i = 0; i < V; ++i) {
    float v = bf(logits[i]);
    if (seen[i]) {
      if (sp->repetition_penalty != 1.0f)
        v = v < 0.0f ? v * sp->repetition_penalty : v / sp->repetition_penalty;
      if (sp->presence_penalty != 0.0f) v = v - sp->presence_penalty;
    }
    x[i] = v + 0.0f;
    if (allow && !((allow[i >> 5] >> (i & 31)) & 1u)) x[i] = -INFINITY;
  }
  free(seen);
  float M = -INFINITY;
  int32_t Mi = -1; /* -1: no finite candidate */
  for (int64_t i = 0; i < V; ++i)
    if (x[i] > M) {
      M = x[i];
      Mi = (int32_t)i;
    }
  if (sp->temperature == 0.0f) {
    free(x);
    return Mi;
  }
  /* S: 8 chunks of Q = ceil(V / 8192) * 1024 ids; in chunk c thread t sums
   * ids cQ + t, cQ + t + 1024, ...; warp butterflies; warps in order; chunks
   * in order (one CTA of a cluster per chunk on the GPU) */
  const int64_t Q = (V + SAMPLE_CLUSTER * SAMPLE_THREADS - 1) / (SAMPLE_CLUSTER * SAMPLE_THREADS) * SAMPLE_THREADS;
  float tot = 0.0f;
  for (int c = 0; c < SAMPLE_CLUSTER; ++c) {
    const int64_t lo = c * Q < V ? c * Q : V, hi = lo + Q < V ? lo + Q : V;
    float part = 0.0f;
    for (int w = 0; w < SAMPLE_THREADS / 32; ++w) {
      float lanes[32];
      for (int l = 0; l < 32; ++l) {
        float acc = 0.0f;
        for (int64_t i = lo + w * 32 + l; i < hi; i += SAMPLE_THREADS) acc = acc + rexp(x[i] - M);
        lanes[l] = acc;
      }
      bfly(lanes, 32);
      part = part + lanes[0];
    }
    tot = tot + part;
  }
  const float lse = M + rlog(tot);
  const float inv_t = 1.0f / sp->temperature;
  int32_t out = -1;
  if (top_k == 0) {
    const int t1 = sp->temperature == 1.0f && sp->top_p >= 1.0f;
    float bv = -INFINITY;
    int32_t bi = 0x7fffffff;
    for (int64_t i = 0; i < V; ++i) {
      float z = t1 ? x[i] + gumbel(u[i]) : (x[i] - lse) * inv_t + gumbel(u[i]);
      if (z > bv) {
        bv = z;
        bi = (int32_t)i;
      }
    }
    free(x);
    return bi == 0x7fffffff ? -1 : bi;
  }
  /* top-k threshold: the k-th largest x */
  Cand* all = (Cand*)malloc(sizeof(Cand) * V);
  for (int64_t i = 0; i < V; ++i) {
    all[i].x = x[i];
    all[i].i = (int32_t)i;
  }
  qsort(all, (size_t)V, sizeof(Cand), cand_desc);
  const float theta = all[top_k - 1].x;
  int greater = 0, n = 0;
  while (n < V && all[n].x >= theta) {
    if (all[n].x > theta) ++greater;
    ++n;
  }
  if (n > SAMPLE_MAX_CAND) {
    free(all);
    free(x);
    return -1;
  }
  /* keep_p along the descending (x, index) order */
  int* keep_p = (int*)malloc(sizeof(int) * n);
  float* lp = (float*)malloc(sizeof(float) * n);
  const int use_p = sp->top_p < 1.0f;
  float U = 0.0f;
  for (int q = 0; q < n; ++q) {
    lp[q] = all[q].x - lse;
    keep_p[q] = !use_p || U < sp->top_p;
    U = U + rexp(lp[q]);
  }
  int first = -1;
  for (int q = n - 1; q >= greater; --q)
    if (keep_p[q]) {
      first = q;
      break;
    }
  const int allowed = top_k - greater;
  const int lo = first < 0 ? n : (first - allowed + 1 > greater ? first - allowed + 1 : greater);
  float bv = -INFINITY;
  int32_t bi = 0x7fffffff;
  for (int q = 0; q < n; ++q) {
    int keep = q < greater ? keep_p[q] : (q >= lo && q <= first);
    if (!keep) continue;
    float z = lp[q] * inv_t + gumbel(u[all[q].i]);
    if (z > bv || (z == bv && all[q].i < bi)) {
      bv = z;
      bi = all[q].i;
    }
  }
  out = bi == 0x7fffffff ? -1 : bi;
  free(keep_p);
  free(lp);
  free(all);
  free(x);
  return out;
}

/* Log-probability of `id` as the reference reports it (engine.py:294-296,
 * masked_sampling.py:126-128): report = x / T (T > 0) or x, x the penalised,
 * grammar-masked logits of orc_sample_masked; logprob = report[id] -
 * logsumexp(report).  Order of rec_b200/csrc/capi_logprob.cu: M = max;
 * thread t of 1024 sums exp(report_i - M) over i = t, t + 1024, ... in
 * order; a butterfly over each warp of 32 threads; the 32 warp sums in
 * order; lse = M + log S.  NaN for an id outside [0, V); -inf when no logit
 * is finite. */
ORC_API float orc_token_logprob(const uint16_t* logits, int64_t V, const int32_t* hist, int n_hist,
                                const RecSampling* sp, const uint32_t* allow, int32_t id) {
  const int pen = sp->repetition_penalty != 1.0f || sp->presence_penalty != 0.0f;
  uint8_t* seen = (uint8_t*)calloc((size_t)V, 1);
  if (pen)
    for (int i = 0; i < n_hist; ++i)
      if (hist[i] >= 0 && hist[i] < V) seen[hist[i]] = 1;
  float* y = (float*)malloc(sizeof(float) * V);
  for (int64_t i = 0; i < V; ++i) {
    float v;
    if (allow && !((allow[i >> 5] >> (i & 31)) & 1u)) {
      v = -INFINITY;
    } else {
      v = bf(logits[i]);
      if (seen[i]) {
        if (sp->repetition_penalty != 1.0f)
          v = v < 0.0f ? v * sp->repetition_penalty : v / sp->repetition_penalty;
        if (sp->presence_penalty != 0.0f) v = v - sp->presence_penalty;
      }
      v = v + 0.0f;
      if (sp->temperature > 0.0f) v = v / sp->temperature;
    }
    y[i] = v;
  }
  free(seen);
  float M = -INFINITY;
  for (int64_t i = 0; i < V; ++i) M = y[i] > M ? y[i] : M;
  float out;
  if (id < 0 || id >= V) {
    out = NAN;
  } else if (M == -INFINITY) {
    out = -INFINITY;
  } else {
    float S = 0.0f;
    for (int w = 0; w < 32; ++w) {
      float v[32];
      for (int l = 0; l < 32; ++l) {
        float a = 0.0f;
        for (int64_t i = 32 * w + l; i < V; i += 1024) a = a + rexp(y[i] - M);
        v[l] = a;
      }
      bfly(v, 32);
      S = S + v[0];
    }
    out = y[id] - (M + rlog(S));
  }
  free(y);
  return out;
}

ORC_API int32_t orc_sample(const uint16_t* logits, int64_t V, const int32_t* hist, int n_hist,
                           const RecSampling* sp, const float* u) {
  return orc_sample_masked(logits, V, hist, n_hist, sp, u, NULL);
}

/* --------------------------------------------------------- decode step */
/* One full decode step.  kv: n_layers layer caches of capacity C; h_trace
 * (optional) bf16[L+1, H]; logits bf16[V]. */
/* OpenMP threads of the oracle's parallel loops (rows, attention items).
 * Set explicitly by the CPU timing legs: a launcher may have exported
 * OMP_NUM_THREADS=1 before the runtime read it.  Returns the count in use. */
ORC_API int orc_set_threads(int n) {
  if (n > 0) omp_set_num_threads(n);
  return omp_get_max_threads();
}

ORC_API int orc_decode_step(const RecModelDesc* md, const RecLayerWeights* layers,
                            const RecGlobalWeights* gw, const RecKVLayer* kv, int C, int token,
                            int pos, uint16_t* logits, uint16_t* trace) {
  int H = md->hidden, Hq = md->n_q_heads, Hkv = md->n_kv_heads, D = 128;
  int sd = md->scale_dtype;
  if (token < 0 || token >= md->vocab || pos < 0 || pos >= C) return -1;
  uint16_t* h = (uint16_t*)malloc(sizeof(uint16_t) * H);
  uint16_t* xn = (uint16_t*)malloc(sizeof(uint16_t) * H);
  uint16_t* qkv = (uint16_t*)malloc(sizeof(uint16_t) * (Hq + 2 * Hkv) * D);
  uint16_t* att = (uint16_t*)malloc(sizeof(uint16_t) * Hq * D);
  uint16_t* o = (uint16_t*)malloc(sizeof(uint16_t) * H);
  float cs[128];
  orc_rope_table(md->rope_theta, pos, 1, cs);
  int T = pos + 1;
  int n_super = (T + ATT_BLOCK * ATT_SUPER - 1) / (ATT_BLOCK * ATT_SUPER);
  Partial* supers = (Partial*)malloc(sizeof(Partial) * Hq * n_super);

  embed(&gw->embed, sd, H, token, md->embed_bits == 8 ? 8 : 4, h);
  if (trace) memcpy(trace, h, sizeof(uint16_t) * H);
  for (int li = 0; li < md->n_layers; ++li) {
    const RecLayerWeights* L = &layers[li];
    rmsnorm(h, (const uint16_t*)L->input_norm, H, md->rms_eps, xn);
    gemv(&L->q, sd, 0, Hq * D, H, xn, NULL, qkv);
    gemv(&L->k, sd, 0, Hkv * D, H, xn, NULL, qkv + Hq * D);
    gemv(&L->v, sd, 0, Hkv * D, H, xn, NULL, qkv + (Hq + Hkv) * D);
    uint16_t* q = qkv;
    uint16_t* k = qkv + Hq * D;
    uint16_t* v = qkv + (Hq + Hkv) * D;
    const int rope = !(L->kind & REC_LAYER_NO_ROPE); /* NoPE ("global") layers skip RoPE */
    for (int hh = 0; hh < Hq; ++hh) {
      if ((md->flags & REC_FLAG_QK_NORM) && L->q_norm) head_norm(q + hh * D, (const uint16_t*)L->q_norm, md->rms_eps);
      if (rope) rope_head(q + hh * D, cs);
    }
    for (int g = 0; g < Hkv; ++g) {
      if ((md->flags & REC_FLAG_QK_NORM) && L->k_norm) head_norm(k + g * D, (const uint16_t*)L->k_norm, md->rms_eps);
      if (rope) rope_head(k + g * D, cs);
    }
    const int vbits = md->kv_value_bits ? md->kv_value_bits : md->kv_bits;
    kv_store(&kv[li], Hkv, C, md->kv_bits, vbits, pos, k, v);
    orc_attention_supers_kv(q, &kv[li], Hq, Hkv, C, md->kv_bits, vbits, T,
                                (L->kind & REC_LAYER_SLIDING) ? md->sliding_window : 0, supers, n_super);
    orc_attention_final(supers, Hq, n_super,
                        (md->flags & REC_FLAG_SINKS) ? (const uint16_t*)L->sinks : NULL, att);
    gemv(&L->o, sd, 0, H, Hq * D, att, NULL, o);
    for (int i = 0; i < H; ++i) h[i] = to_bf(bf(h[i]) + bf(o[i]));
    int32_t ids[8];
    float w[8];
    orc_moe(md, L, h, ids, w, NULL, NULL, h);
    if (trace) memcpy(trace + (int64_t)(li + 1) * H, h, sizeof(uint16_t) * H);
  }
  rmsnorm(h, (const uint16_t*)gw->final_norm, H, md->rms_eps, xn);
  gemv(&gw->lm_head, sd, 0, md->vocab, H, xn, NULL, logits);
  free(h);
  free(xn);
  free(qkv);
  free(att);
  free(o);
  free(supers);
  return 0;
}
