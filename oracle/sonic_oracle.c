/*
 * ORACLE -- test infrastructure only. Nothing in the product links, loads or calls this
 * file; it is the CPU checker that tests/, __graft_entry__.smoke() and bench.py's
 * cpu_baseline leg compare the CUDA path against.
 *
 * Plain-C restatement, element by element, of the reference sampler
 * (tachyontrails/sonic-sampler, paths under src/sonic_sampler/). It takes the same
 * argument structs as the C ABI (include/sonic_b200.h) with HOST pointers.
 *
 * Pinning: tests/golden/ holds vectors produced by the reference's own Triton kernels
 * (run through Triton's CPU interpreter in the development container by
 * tests/golden/make_golden.py); tests/test_oracle_golden.py checks this oracle against them.
 *
 * Fixed orders. The reference leaves the association order of its fp32 reductions to the
 * Triton compiler. This restatement fixes one order, and the CUDA kernels use the same one,
 * so the two agree bit for bit:
 *   - sum of 128 terms: lane l (0..31) holds terms 4l..4l+3 summed left to right, then
 *     an xor butterfly over lanes with distances 16, 8, 4, 2, 1;
 *   - inclusive prefix sum of 128 terms: lane-local running sums, a Hillis-Steele scan of
 *     the 32 lane totals (distances 1, 2, 4, 8, 16), and then
 *     ladder[4l+j] = scan[l-1] + local[l][j] (scan[-1] = 0).
 * exp and log are computed by ox_exp / ox_log below: Cody-Waite reduction plus a
 * degree-7 Taylor polynomial, and the atanh series of log. The reference uses the
 * libdevice fast approximations on the GPU, so logprobs agree with it within tolerance,
 * not bit for bit.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#include "../include/sonic_b200.h"

#define MAXK 128

/* ------------------------------------------------------------------------------------ */
/* bf16 helpers (reference ops/encoding.py:31-123)                                        */
/* ------------------------------------------------------------------------------------ */

static inline float bf2f(uint16_t h) {
  uint32_t u = (uint32_t)h << 16;
  float f;
  memcpy(&f, &u, 4);
  return f;
}

static inline uint16_t f2bf(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x0040u);
  u += 0x7fffu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}

/* fp32 op followed by round-to-nearest-even to bf16: exact bf16 arithmetic for these
   operands (products of two bf16 values are exact in fp32; sums and quotients are at
   least 128 fp32 ulps away from a bf16 rounding midpoint, so no double-rounding). */
static inline float rbf(float f) { return bf2f(f2bf(f)); }

static inline uint32_t f2u(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  return u;
}

static inline float u2f(uint32_t u) {
  float f;
  memcpy(&f, &u, 4);
  return f;
}

/* encode_block (ops/encoding.py:31-60): order-preserving u16 of bf16 bits. */
static inline uint32_t enc16(uint16_t h) {
  return (h & 0x8000u) ? (uint32_t)(h ^ 0xffffu) : (uint32_t)(h ^ 0x8000u);
}

static inline uint16_t dec16(uint32_t e) {
  return (uint16_t)((e & 0x8000u) ? (e ^ 0x8000u) : (e ^ 0xffffu));
}

static inline uint32_t enc32(float f) {
  uint32_t u = f2u(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

static inline float dec32(uint32_t e) {
  return u2f((e & 0x80000000u) ? (e & 0x7fffffffu) : ~e);
}

/* ------------------------------------------------------------------------------------ */
/* exp / log (own implementation; see header comment)                                     */
/* ------------------------------------------------------------------------------------ */

#define OX_LOG2E 1.44269502162933349609375f       /* 0x3fb8aa3b */
#define OX_LN2_HI 0.693145751953125f              /* 0x3f317200, 16 significant bits */
#define OX_LN2_LO 1.428606765330187e-06f          /* 0x35bfbe8e = ln2 - OX_LN2_HI */
#define OX_SQRT2 1.41421353816986083984375f       /* 0x3fb504f3 */

float ox_exp(float x) {
  if (x != x) return x;
  if (x > 88.7228317f) return INFINITY;
  if (x < -104.0f) return 0.0f;
  float n = nearbyintf(x * OX_LOG2E);
  float r = fmaf(-n, OX_LN2_HI, x);
  r = fmaf(-n, OX_LN2_LO, r);
  /* e^r = sum r^k / k!, k <= 7, Horner form. */
  float p = 1.0f / 5040.0f;
  p = fmaf(p, r, 1.0f / 720.0f);
  p = fmaf(p, r, 1.0f / 120.0f);
  p = fmaf(p, r, 1.0f / 24.0f);
  p = fmaf(p, r, 1.0f / 6.0f);
  p = fmaf(p, r, 0.5f);
  p = fmaf(p, r, 1.0f);
  p = fmaf(p, r, 1.0f);
  int e = (int)n;
  if (e > 127) return p * u2f((uint32_t)(127 + 127) << 23) * u2f((uint32_t)(e - 127 + 127) << 23);
  if (e < -126) return p * u2f((uint32_t)(e + 64 + 127) << 23) * u2f((uint32_t)(-64 + 127) << 23);
  return p * u2f((uint32_t)(e + 127) << 23);
}

float ox_log(float x) {
  if (x != x) return x;
  if (x < 0.0f) return NAN;
  if (x == 0.0f) return -INFINITY;
  if (x == INFINITY) return x;
  uint32_t u = f2u(x);
  int e = 0;
  if (u < 0x00800000u) { /* subnormal: scale by 2^23 */
    u = f2u(x * 8388608.0f);
    e = -23;
  }
  e += (int)((u >> 23) & 0xffu) - 127;
  float m = u2f((u & 0x007fffffu) | 0x3f800000u);
  if (m > OX_SQRT2) {
    m = m * 0.5f;
    e += 1;
  }
  float f = m - 1.0f;
  float s = f / (2.0f + f);
  float z = s * s;
  /* log(m) = 2 atanh(s) = 2s (1 + z/3 + z^2/5 + ... + z^5/11). */
  float q = 1.0f / 11.0f;
  q = fmaf(q, z, 1.0f / 9.0f);
  q = fmaf(q, z, 1.0f / 7.0f);
  q = fmaf(q, z, 1.0f / 5.0f);
  q = fmaf(q, z, 1.0f / 3.0f);
  q = fmaf(q, z, 1.0f);
  float l = (2.0f * s) * q;
  float fe = (float)e;
  return fmaf(fe, OX_LN2_HI, fmaf(fe, OX_LN2_LO, l));
}

/* ------------------------------------------------------------------------------------ */
/* fixed-order reductions over 128 candidates (mirrored by the CUDA warp code)           */
/* ------------------------------------------------------------------------------------ */

static float sum128(const float* t) {
  float x[32], y[32];
  for (int l = 0; l < 32; ++l) x[l] = ((t[4 * l] + t[4 * l + 1]) + t[4 * l + 2]) + t[4 * l + 3];
  for (int d = 16; d >= 1; d >>= 1) {
    memcpy(y, x, sizeof(x));
    for (int l = 0; l < 32; ++l) x[l] = y[l] + y[l ^ d];
  }
  return x[0];
}

static void ladder128(const float* t, float* out) {
  float p[32][4], S[32], y[32];
  for (int l = 0; l < 32; ++l) {
    p[l][0] = t[4 * l];
    p[l][1] = p[l][0] + t[4 * l + 1];
    p[l][2] = p[l][1] + t[4 * l + 2];
    p[l][3] = p[l][2] + t[4 * l + 3];
    S[l] = p[l][3];
  }
  for (int d = 1; d < 32; d <<= 1) {
    memcpy(y, S, sizeof(S));
    for (int l = d; l < 32; ++l) S[l] = y[l] + y[l - d];
  }
  for (int l = 0; l < 32; ++l) {
    float E = l ? S[l - 1] : 0.0f;
    for (int j = 0; j < 4; ++j) out[4 * l + j] = E + p[l][j];
  }
}

/* argmax with ties to the lowest position (Triton tl.argmax, tie_break_left). */
static int argmax_first(const float* v, int n) {
  int best = 0;
  for (int i = 1; i < n; ++i)
    if (v[i] > v[best]) best = i;
  return best;
}

/* ------------------------------------------------------------------------------------ */
/* Philox4x32-10 (Salmon et al., "Parallel random numbers: as easy as 1, 2, 3", SC'11)   */
/* ------------------------------------------------------------------------------------ */

static void philox4x32_10(uint32_t c[4], uint32_t k0, uint32_t k1) {
  for (int i = 0; i < 10; ++i) {
    uint64_t p0 = (uint64_t)0xD2511F53u * c[0];
    uint64_t p1 = (uint64_t)0xCD9E8D57u * c[2];
    uint32_t n0 = (uint32_t)(p1 >> 32) ^ c[1] ^ k0;
    uint32_t n1 = (uint32_t)p1;
    uint32_t n2 = (uint32_t)(p0 >> 32) ^ c[3] ^ k1;
    uint32_t n3 = (uint32_t)p0;
    c[0] = n0; c[1] = n1; c[2] = n2; c[3] = n3;
    k0 += 0x9E3779B9u;
    k1 += 0xBB67AE85u;
  }
}

/* log(Exp(1)) noise for (slot, token) in the counter-based mode: the same quantity the
   reference keeps in its Gumbel buffer (core/buffer.py:95-120), generated in fp32. */
static float philox_unit(uint64_t seed, uint64_t offset, int64_t slot, uint32_t token) {
  uint32_t c[4] = {token, (uint32_t)slot, (uint32_t)offset, (uint32_t)(offset >> 32)};
  philox4x32_10(c, (uint32_t)seed, (uint32_t)(seed >> 32));
  return ((float)(c[0] >> 9) + 0.5f) * (1.0f / 8388608.0f);
}

float ox_philox_log_exponential(uint64_t seed, uint64_t offset, int64_t slot, int64_t token) {
  float u = philox_unit(seed, offset, slot, (uint32_t)token);
  return ox_log(-ox_log(u));
}

/* Counter-based acceptance uniform of a multistep step (an addition of this library: the
   reference reads its bf16 uniform buffer): token word 0xffffffff, rounded to bf16. */
static float ox_philox_acceptance(uint64_t seed, uint64_t offset, int64_t slot) {
  return rbf(philox_unit(seed, offset, slot, 0xffffffffu));
}

/* ------------------------------------------------------------------------------------ */
/* logit processing (ops/prologue.py:29-114, 340-447)                                    */
/* ------------------------------------------------------------------------------------ */

static inline int64_t load_index(const void* p, int32_t dtype, int64_t i) {
  return dtype == SONIC_DTYPE_I64 ? ((const int64_t*)p)[i] : (int64_t)((const int32_t*)p)[i];
}

/* One logit of kernel row (slot, step); `col` is the aux-buffer column (after the shard
   offset and d2t remap); `extra` is the drafted-token count added to the decode count. */
static float process_logit(const SonicSamplingParams* P, uint16_t ind, int64_t slot, int64_t grow,
                           int64_t col, float v, int32_t extra) {
  if (ind & 0x1F) {
    /* grammar (prologue.py:29-54): keep the logit only when its bit is set. */
    if (P->grammar && (ind & 0x1)) {
      uint32_t w = P->grammar[grow * P->grammar_stride + col / 32];
      if (!((w >> (col % 32)) & 1u)) v = -INFINITY;
    }
    /* repetition (prologue.py:57-102, decode counts 141-195). */
    if (P->decode_counts && (ind & 0xE)) {
      int32_t dec = P->decode_counts[slot * P->counts_stride + col] + extra;
      if (P->context_counts && (ind & 0x2)) {
        int32_t total = dec + P->context_counts[slot * P->counts_stride + col];
        float s = total > 0 ? bf2f(P->repetition[slot]) : 1.0f;
        v = v < 0.0f ? rbf(v * s) : rbf(v / s);
      }
      if (ind & 0x4) v = rbf(v - rbf(rbf((float)dec) * bf2f(P->frequency[slot])));
      if (ind & 0x8) v = rbf(v - rbf((dec > 0 ? 1.0f : 0.0f) * bf2f(P->presence[slot])));
    }
    /* logit bias (prologue.py:105-114). */
    if (P->bias && (ind & 0x10)) v = rbf(v + bf2f(P->bias[slot * P->bias_stride + col]));
  }
  /* temperature (prologue.py:443-447). */
  if (ind & 0x20) v = rbf(v / bf2f(P->temperature[slot]));
  return v;
}

/* Greedy order (prologue.py:117-138 + singular.py:71-131): tile max (ties to the lowest
   in-tile offset), packed (enc16 << 16 | block_n-1-offset), max over tiles (ties to the
   lowest tile). -0.0 is compared as +0.0. */
static inline uint64_t greedy_key(float v, int64_t c, int32_t block_n) {
  uint16_t h = f2bf(v);
  if (h == 0x8000u) h = 0;
  uint64_t e = enc16(h);
  uint64_t loc = (uint64_t)(block_n - 1 - (int32_t)(c & (block_n - 1)));
  uint64_t tile = 0xffffffffu - (uint64_t)(c / block_n);
  return (e << 48) | (loc << 32) | tile;
}

static inline int64_t greedy_col(uint64_t key, int32_t block_n) {
  int64_t tile = (int64_t)(0xffffffffu - (uint32_t)key);
  int64_t loc = block_n - 1 - (int64_t)((key >> 32) & 0xffffu);
  return tile * block_n + loc;
}

/* Exact top-128 (ops/topk/ kernels, merged by ops/topk/unpack.py:26-124) under the key
   (enc16(value) desc, column asc), sorted descending. Keys are unique per row. */
typedef struct { uint64_t key; } Cand;

static int cmp_desc(const void* a, const void* b) {
  uint64_t x = ((const Cand*)a)->key, y = ((const Cand*)b)->key;
  return x < y ? 1 : (x > y ? -1 : 0);
}

/* min-heap of the best n keys seen so far */
static void heap_push(uint64_t* h, int* n, int cap, uint64_t k) {
  if (*n < cap) {
    int i = (*n)++;
    h[i] = k;
    while (i > 0) {
      int p = (i - 1) / 2;
      if (h[p] <= h[i]) break;
      uint64_t t = h[p]; h[p] = h[i]; h[i] = t;
      i = p;
    }
  } else if (k > h[0]) {
    h[0] = k;
    int i = 0;
    for (;;) {
      int l = 2 * i + 1, r = l + 1, m = i;
      if (l < cap && h[l] < h[m]) m = l;
      if (r < cap && h[r] < h[m]) m = r;
      if (m == i) break;
      uint64_t t = h[m]; h[m] = h[i]; h[i] = t;
      i = m;
    }
  }
}

static int top_keys(const uint64_t* keys, int64_t n, int k, uint64_t* out) {
  int cnt = 0;
  for (int64_t i = 0; i < n; ++i) heap_push(out, &cnt, k, keys[i]);
  qsort(out, (size_t)cnt, sizeof(uint64_t), cmp_desc);
  return cnt;
}

/* cumulative_masking (ops/base.py:95-129) on sorted bf16 values (as floats). */
static void cumulative_masking(const SonicSamplingParams* P, int64_t slot, uint16_t ind, float* v,
                               float maximum) {
  if (ind & 0x80) {
    int32_t k = P->top_k[slot];
    for (int i = 0; i < MAXK; ++i)
      if (!(i < k)) v[i] = -INFINITY;
  }
  if (ind & 0x100) {
    float e[MAXK], lad[MAXK];
    for (int i = 0; i < MAXK; ++i) e[i] = ox_exp(v[i] - maximum);
    ladder128(e, lad);
    /* ops/base.py:81-84 scales the prefix sum's last element. The reference's prefix sums of
       these non-negative terms never decrease, so that element is also their maximum; this
       order's scan can end an ulp below an earlier prefix past the last nonzero term (the
       lanes' totals are grouped differently), so the maximum is taken. */
    float total = lad[0];
    for (int i = 1; i < MAXK; ++i)
      if (lad[i] > total) total = lad[i];
    float scale = total * bf2f(P->top_p[slot]);
    for (int i = 0; i < MAXK; ++i)
      if (!(lad[i] <= scale || i == 0)) v[i] = -INFINITY;
  }
  if (ind & 0x200) {
    float pivot = ox_log(bf2f(P->min_p[slot])) + maximum;
    for (int i = 0; i < MAXK; ++i)
      if (!(v[i] >= pivot)) v[i] = -INFINITY;
  }
}

/* log_softmax (ops/base.py:66-72) */
static void log_softmax128(const float* v, float maximum, float* out) {
  float sc[MAXK], e[MAXK];
  for (int i = 0; i < MAXK; ++i) {
    sc[i] = v[i] - maximum;
    e[i] = ox_exp(sc[i]);
  }
  float lse = ox_log(sum128(e));
  for (int i = 0; i < MAXK; ++i) out[i] = sc[i] - lse;
}

static void store_float(void* base, int32_t dtype, int64_t i, float x) {
  if (dtype == SONIC_DTYPE_F32)
    ((float*)base)[i] = x;
  else
    ((uint16_t*)base)[i] = f2bf(x);
}

static float load_float(const void* base, int32_t dtype, int64_t i) {
  return dtype == SONIC_DTYPE_F32 ? ((const float*)base)[i] : bf2f(((const uint16_t*)base)[i]);
}

/* Process one kernel row and rank it. Returns 1 for a greedy row (token in *greedy),
   else fills vals/idx (sorted top-128, raw columns) and returns 0. */
static int rank_row(const SonicSamplingParams* P, uint16_t ind, int64_t slot, int64_t grow,
                    const uint16_t* x, int32_t V, int32_t shard_offset, int32_t block_n,
                    const void* d2t, int32_t d2t_dtype, const int32_t* toks, int ntok,
                    uint64_t* keys, int64_t* greedy, float* vals, int32_t* idx) {
  int processors = (ind & 0x1F) != 0;
  uint64_t best = 0;
  for (int64_t c = 0; c < V; ++c) {
    float v = bf2f(x[c]);
    if (processors || (ind & 0x20)) {
      int64_t col = c + shard_offset;
      if (processors && d2t) col = load_index(d2t, d2t_dtype, col);
      int32_t extra = 0;
      if (processors && toks)
        for (int s = 0; s < ntok; ++s) extra += (toks[s] == col);
      v = process_logit(P, ind, slot, grow, col, v, extra);
    }
    if (ind & 0x40) {
      uint64_t g = greedy_key(v, c, block_n);
      if (c == 0 || g > best) best = g;
    } else {
      keys[c] = ((uint64_t)enc16(f2bf(v)) << 32) | (uint64_t)(0xffffffffu - (uint32_t)c);
    }
  }
  if (ind & 0x40) {
    *greedy = greedy_col(best, block_n);
    return 1;
  }
  uint64_t top[MAXK];
  top_keys(keys, V, MAXK, top);
  for (int i = 0; i < MAXK; ++i) {
    vals[i] = bf2f(dec16((uint32_t)(top[i] >> 32)));
    idx[i] = (int32_t)(0xffffffffu - (uint32_t)top[i]);
  }
  return 0;
}

static int64_t row_slot(const SonicSamplingParams* P, int64_t r) {
  return P->slot_mapping ? load_index(P->slot_mapping, P->slot_dtype, r) : r;
}

/* ------------------------------------------------------------------------------------ */
/* fused singular (interface/functional/singular.py:75-322)                              */
/* ------------------------------------------------------------------------------------ */

/* Stochastic selection of row r from its sorted top-128 (singular.py:259-358): masking,
   Gumbel-max over candidate noise, count update, logprobs, top-Z and candidate probabilities.
   `idx` are the candidates' columns (before d2t). */
static void select_stochastic(const SonicSingularArgs* a, int64_t r, int64_t slot, uint16_t ind, float* vals,
                              const int32_t* idx) {
  const SonicSamplingParams* P = &a->params;
  const int zcap = a->max_top_logprobs;
  float ls[MAXK];
  if (ind & 0x380) cumulative_masking(P, slot, ind, vals, vals[0]);
  int64_t tok[MAXK];
  for (int i = 0; i < MAXK; ++i) tok[i] = a->d2t ? load_index(a->d2t, a->d2t_dtype, idx[i]) : idx[i];
  float diff[MAXK];
  for (int i = 0; i < MAXK; ++i) {
    if (a->flags & SONIC_FLAG_PHILOX)
      diff[i] = vals[i] - ox_philox_log_exponential(a->philox_seed, a->philox_offset, slot, tok[i]);
    else
      diff[i] = rbf(vals[i] - bf2f(a->gumbel[slot * a->gumbel_stride + tok[i]]));
  }
  int sel = argmax_first(diff, MAXK);
  int64_t token = tok[sel];
  if (a->flags & SONIC_FLAG_UPDATE_COUNTS) {
    int32_t* d = &P->decode_counts[slot * P->counts_stride + token];
    *d = (a->flags & SONIC_FLAG_PREFILL) ? 1 : *d + 1;
  }
  if (a->flags & (SONIC_FLAG_LOGPROBS | SONIC_FLAG_PROBABILITIES)) {
    log_softmax128(vals, vals[0], ls);
    if ((a->flags & SONIC_FLAG_LOGPROBS) && a->logprobs) {
      store_float(a->logprobs, a->logprobs_dtype, r * a->logprobs_stride, ls[sel]);
      if (zcap > 0 && (ind & 0x400) && a->top_logprob_values) {
        int32_t z = P->top_logprobs[slot];
        if (z > zcap) z = zcap;
        for (int i = 0; i < z; ++i) {
          store_float(a->top_logprob_values, a->logprobs_dtype, r * a->top_stride + i, ls[i]);
          a->top_logprob_tokens[r * a->top_stride + i] = (int32_t)tok[i];
        }
      }
    }
    if ((a->flags & SONIC_FLAG_PROBABILITIES) && a->probabilities)
      for (int i = 0; i < MAXK; ++i)
        store_float(a->probabilities, a->probabilities_dtype, slot * a->probabilities_stride + tok[i],
                    ox_exp(ls[i]));
  }
  a->tokens[r * a->tokens_stride] = (int32_t)token;
}

static void greedy_update(const SonicSingularArgs* a, int64_t slot, int64_t token) {
  const SonicSamplingParams* P = &a->params;
  if (a->flags & SONIC_FLAG_UPDATE_COUNTS) {
    int32_t* d = &P->decode_counts[slot * P->counts_stride + token];
    *d = (a->flags & SONIC_FLAG_PREFILL) ? 1 : *d + 1;
  }
}

sonic_status oracle_fused_singular(const SonicSingularArgs* a) {
  const SonicSamplingParams* P = &a->params;
  const int32_t V = a->vocab_size;
  uint64_t* keys = (uint64_t*)malloc(sizeof(uint64_t) * (size_t)V);
  if (!keys) return SONIC_ERR_INVALID_ARGUMENT;
  for (int64_t r = 0; r < a->rows; ++r) {
    const int64_t slot = row_slot(P, r);
    const uint16_t ind = P->indicators[slot];
    const uint16_t* x = (const uint16_t*)a->logits + r * a->logits_stride;
    const int32_t* toks = a->drafted_tokens ? a->drafted_tokens + slot * a->drafted_stride : NULL;
    float vals[MAXK];
    int32_t idx[MAXK];
    int64_t token;
    /* singular rows use grammar row `slot` (prologue.py:45 with timesteps = 1) */
    if (rank_row(P, ind, slot, slot, x, V, a->shard_offset, a->block_n, a->d2t, a->d2t_dtype, toks,
                 toks ? a->lookahead : 0, keys, &token, vals, idx)) {
      /* greedy (singular.py:219-257) */
      if (a->d2t) token = load_index(a->d2t, a->d2t_dtype, token);
      greedy_update(a, slot, token);
      a->tokens[r * a->tokens_stride] = (int32_t)token;
      continue;
    }
    select_stochastic(a, r, slot, ind, vals, idx);
  }
  free(keys);
  return SONIC_OK;
}

/* ------------------------------------------------------------------------------------ */
/* vocab-sharded singular (the sharded stage-2 scaffolding of interface/functional/        */
/* singular.py:80-84,129-149 and ops/topk/unpack.py:127-247 sharded_top_k, completed)      */
/* ------------------------------------------------------------------------------------ */

/* Step 1 of one rank: per row, the processed logits of this shard's `vocab_size` columns
   (aux-buffer columns offset by shard_offset, prologue.py:382), and their 128 best keys
   (enc16(value) << 32 | ~global column), sorted descending, zero-padded. Greedy rows take the
   same keys (the merge picks their best). */
sonic_status oracle_shard_candidates(const SonicSingularArgs* a, uint64_t* out) {
  const SonicSamplingParams* P = &a->params;
  const int32_t V = a->vocab_size;
  uint64_t* keys = (uint64_t*)malloc(sizeof(uint64_t) * (size_t)V);
  if (!keys) return SONIC_ERR_INVALID_ARGUMENT;
  for (int64_t r = 0; r < a->rows; ++r) {
    const int64_t slot = row_slot(P, r);
    const uint16_t ind = P->indicators[slot];
    const uint16_t* x = (const uint16_t*)a->logits + r * a->logits_stride;
    const int32_t* toks = a->drafted_tokens ? a->drafted_tokens + slot * a->drafted_stride : NULL;
    const int ntok = toks ? a->lookahead : 0;
    const int processors = (ind & 0x1F) != 0;
    for (int64_t c = 0; c < V; ++c) {
      float v = bf2f(x[c]);
      const int64_t col = c + a->shard_offset;
      if (processors || (ind & 0x20)) {
        int32_t extra = 0;
        if (processors && toks)
          for (int t = 0; t < ntok; ++t) extra += (toks[t] == col);
        v = process_logit(P, ind, slot, slot, col, v, extra);
      }
      keys[c] = ((uint64_t)enc16(f2bf(v)) << 32) | (uint64_t)(0xffffffffu - (uint32_t)col);
    }
    uint64_t top[MAXK];
    const int n = top_keys(keys, V, MAXK, top);
    for (int i = 0; i < MAXK; ++i) out[r * MAXK + i] = i < n ? top[i] : 0;
  }
  free(keys);
  return SONIC_OK;
}

/* Step 3, identical on every rank: merge the `world` lists of every row (gathered
   [world][rows][128]) into the row's top-128 and select as oracle_fused_singular does; a greedy
   row takes the largest value with the lowest global column (the reference's own sharded
   greedy decode, ops/singular.py:61-66, mixes up the shard and block indices and is not
   followed). `a->vocab_size` is the full vocabulary. */
sonic_status oracle_merge_candidates(const SonicSingularArgs* a, const uint64_t* gathered, int32_t world) {
  const SonicSamplingParams* P = &a->params;
  uint64_t* keys = (uint64_t*)malloc(sizeof(uint64_t) * (size_t)world * MAXK);
  if (!keys) return SONIC_ERR_INVALID_ARGUMENT;
  for (int64_t r = 0; r < a->rows; ++r) {
    const int64_t slot = row_slot(P, r);
    const uint16_t ind = P->indicators[slot];
    int64_t n = 0;
    for (int w = 0; w < world; ++w)
      for (int i = 0; i < MAXK; ++i) {
        const uint64_t k = gathered[((int64_t)w * a->rows + r) * MAXK + i];
        if (k) keys[n++] = k;
      }
    uint64_t top[MAXK];
    const int cnt = top_keys(keys, n, MAXK, top);
    for (int i = cnt; i < MAXK; ++i) top[i] = 0;
    if (ind & 0x40) {
      const int64_t token = cnt ? (int64_t)(0xffffffffu - (uint32_t)top[0]) : -1;
      if (token >= 0) greedy_update(a, slot, token);
      a->tokens[r * a->tokens_stride] = (int32_t)token;
      continue;
    }
    float vals[MAXK];
    int32_t idx[MAXK];
    for (int i = 0; i < MAXK; ++i) {
      vals[i] = top[i] ? bf2f(dec16((uint32_t)(top[i] >> 32))) : -INFINITY;
      idx[i] = top[i] ? (int32_t)(0xffffffffu - (uint32_t)top[i]) : 0;
    }
    select_stochastic(a, r, slot, ind, vals, idx);
  }
  free(keys);
  return SONIC_OK;
}

/* ------------------------------------------------------------------------------------ */
/* fused multistep (interface/functional/multistep.py:175-461)                           */
/* ------------------------------------------------------------------------------------ */

sonic_status oracle_fused_multistep(const SonicMultistepArgs* a) {
  const SonicSamplingParams* P = &a->params;
  const int32_t V = a->vocab_size, G = a->lookahead;
  uint64_t* keys = (uint64_t*)malloc(sizeof(uint64_t) * (size_t)V);
  if (!keys) return SONIC_ERR_INVALID_ARGUMENT;
  const int zcap = a->max_top_logprobs;
  float prob[SONIC_MAX_LOOKAHEAD + 1][MAXK];
  int32_t cand[SONIC_MAX_LOOKAHEAD + 1][MAXK];
  int64_t gsel[SONIC_MAX_LOOKAHEAD + 1];
  for (int64_t b = 0; b < a->batch_size; ++b) {
    int64_t margin, T;
    if (a->cu_seqlens) {
      margin = a->cu_seqlens[b];
      T = a->cu_seqlens[b + 1] - margin;
    } else {
      margin = b * (G + 1);
      T = G + 1;
    }
    const int64_t slot = row_slot(P, b);
    const uint16_t ind = P->indicators[slot];
    const int32_t* drafted = a->drafted_tokens + margin;
    /* stages 1+2 for every row of the request (prologue.py:272, multistep.py:76) */
    for (int64_t s = 0; s < T; ++s) {
      const int64_t row = margin + s;
      const uint16_t* x = (const uint16_t*)a->logits + row * a->logits_stride;
      float vals[MAXK], ls[MAXK];
      int32_t idx[MAXK];
      int64_t g;
      /* grammar row slot*(gamma+1)+step (prologue.py:45, timesteps = lookahead+1) */
      if (rank_row(P, ind, slot, slot * (G + 1) + s, x, V, a->shard_offset, a->block_n, NULL, 0,
                   drafted, (int)s, keys, &g, vals, idx)) {
        gsel[s] = g;
        if (a->indices) a->indices[margin * MAXK + s] = (int32_t)g;  /* multistep.py:163-165 */
        continue;
      }
      float maximum = vals[0];
      if (ind & 0x380) cumulative_masking(P, slot, ind, vals, maximum);
      log_softmax128(vals, maximum, ls);
      for (int i = 0; i < MAXK; ++i) {
        prob[s][i] = ox_exp(ls[i]);
        cand[s][i] = idx[i];
        if (a->values) a->values[row * MAXK + i] = prob[s][i];
        if (a->indices) a->indices[row * MAXK + i] = idx[i];
      }
    }
    /* stage 3: chain verification (verify.py:244-434) */
    int64_t dr[SONIC_MAX_LOOKAHEAD + 1];
    for (int s = 0; s <= G; ++s) dr[s] = (s < T - 1) ? drafted[s] : 0;
    int64_t accepted = 0, token;
    int64_t selections[SONIC_MAX_LOOKAHEAD + 1];
    if (ind & 0x40) {
      /* verify_greedy (verify.py:54-72) */
      while (accepted < T - 1 && gsel[accepted] == dr[accepted]) ++accepted;
      token = gsel[accepted];
      for (int s = 0; s < T; ++s) selections[s] = gsel[s];
    } else {
      /* verify_drafted (verify.py:113-154) */
      float targets[SONIC_MAX_LOOKAHEAD + 1];
      for (int s = 0; s <= G; ++s) {
        targets[s] = 0.0f;
        if (s < T)
          for (int i = 0; i < MAXK; ++i) targets[s] += (cand[s][i] == dr[s]) ? prob[s][i] : 0.0f;
      }
      const int stochastic_draft = a->draft_probs && !(ind & 0x800);
      for (accepted = 0; accepted < T - 1; ++accepted) {
        float u = (a->flags & SONIC_FLAG_PHILOX) ? ox_philox_acceptance(a->philox_seed, a->philox_offset + accepted, slot)
                                                 : bf2f(a->uniform[slot * a->uniform_stride + accepted]);
        if (stochastic_draft) {
          int64_t qi = slot * a->draft_stride + accepted * a->draft_step_stride + dr[accepted];
          if (a->draft_dtype == SONIC_DTYPE_F32)
            u = u * ((const float*)a->draft_probs)[qi];
          else
            u = rbf(u * bf2f(((const uint16_t*)a->draft_probs)[qi]));
        }
        if (!(u <= targets[accepted])) break;
      }
      /* rejection_sample (verify.py:157-241) */
      float res[MAXK], score[MAXK];
      for (int i = 0; i < MAXK; ++i) {
        float sc = prob[accepted][i];
        float r;
        if (accepted == T - 1)
          r = sc;
        else if (!stochastic_draft)
          r = (cand[accepted][i] == dr[accepted]) ? 0.0f : sc;
        else {
          float q = load_float(a->draft_probs, a->draft_dtype,
                               slot * a->draft_stride + accepted * a->draft_step_stride + cand[accepted][i]);
          r = sc - q;
          r = r < 0.0f ? 0.0f : (r > 1.0f ? 1.0f : r);
        }
        float g = (a->flags & SONIC_FLAG_PHILOX)
                      ? ox_philox_log_exponential(a->philox_seed, a->philox_offset + accepted, slot, cand[accepted][i])
                      : bf2f(a->gumbel[slot * a->gumbel_stride + accepted * a->gumbel_step_stride + cand[accepted][i]]);
        score[i] = ox_log(r) - g;
        res[i] = r;
      }
      (void)res;
      int sel = argmax_first(score, MAXK);
      token = cand[accepted][sel];
      for (int s = 0; s <= G; ++s) selections[s] = dr[s];
      selections[accepted] = token;
      targets[accepted] = prob[accepted][sel];
      if ((a->flags & SONIC_FLAG_LOGPROBS) && a->logprobs) {
        for (int64_t s = 0; s <= accepted; ++s) {
          store_float(a->logprobs, a->logprobs_dtype, margin + s, ox_log(targets[s]));
          if (zcap > 0 && (ind & 0x400) && a->top_logprob_values) {
            int32_t z = P->top_logprobs[slot];
            if (z > zcap) z = zcap;
            for (int i = 0; i < z; ++i) {
              store_float(a->top_logprob_values, a->logprobs_dtype, (margin + s) * a->top_stride + i, ox_log(prob[s][i]));
              a->top_logprob_tokens[(margin + s) * a->top_stride + i] = cand[s][i];
            }
          }
        }
      }
    }
    if (a->flags & SONIC_FLAG_UPDATE_COUNTS)
      for (int64_t s = 0; s <= accepted; ++s) P->decode_counts[slot * P->counts_stride + selections[s]] += 1;
    a->tokens[margin + accepted] = (int32_t)token;
    a->offsets[b] = (int32_t)accepted;
  }
  free(keys);
  return SONIC_OK;
}

/* ------------------------------------------------------------------------------------ */
/* bounded top-k (interface/topk.py:98-161)                                              */
/* ------------------------------------------------------------------------------------ */

sonic_status oracle_bounded_topk(const SonicTopKArgs* a) {
  const int32_t V = a->vocab_size, k = a->k;
  uint64_t* keys = (uint64_t*)malloc(sizeof(uint64_t) * (size_t)V);
  if (!keys) return SONIC_ERR_INVALID_ARGUMENT;
  uint64_t top[MAXK];
  for (int64_t r = 0; r < a->rows; ++r) {
    if (a->logits_dtype == SONIC_DTYPE_F32) {
      const float* x = (const float*)a->logits + r * a->logits_stride;
      for (int64_t c = 0; c < V; ++c)
        keys[c] = ((uint64_t)enc32(x[c]) << 32) | (uint64_t)(0xffffffffu - (uint32_t)c);
    } else {
      const uint16_t* x = (const uint16_t*)a->logits + r * a->logits_stride;
      for (int64_t c = 0; c < V; ++c)
        keys[c] = ((uint64_t)enc16(x[c]) << 32) | (uint64_t)(0xffffffffu - (uint32_t)c);
    }
    top_keys(keys, V, k, top);
    for (int i = 0; i < k; ++i) {
      uint32_t e = (uint32_t)(top[i] >> 32);
      int64_t col = (int64_t)(0xffffffffu - (uint32_t)top[i]);
      int64_t o = r * k + i;
      if (a->values_dtype == SONIC_DTYPE_F32)
        ((float*)a->values)[o] = a->logits_dtype == SONIC_DTYPE_F32 ? dec32(e) : bf2f(dec16(e));
      else
        ((uint16_t*)a->values)[o] = a->logits_dtype == SONIC_DTYPE_F32 ? f2bf(dec32(e)) : dec16(e);
      if (a->indices_dtype == SONIC_DTYPE_I64)
        ((int64_t*)a->indices)[o] = col;
      else
        ((int32_t*)a->indices)[o] = (int32_t)col;
    }
  }
  free(keys);
  return SONIC_OK;
}
