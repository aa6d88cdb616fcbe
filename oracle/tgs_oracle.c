/*
 * tgs_oracle.c -- CPU restatement of the tinygpt sampling path (TEST INFRASTRUCTURE).
 *
 * This file is the checker, not the product.  Only tests/, __graft_entry__.smoke()
 * and bench.py's cpu_baseline / --impl reference leg may load it.  It is written
 * for clarity: one row at a time, full-vocab arrays, sorts and quickselect.
 *
 * Which reference lines each step restates (paths inside sarthak-fleet/tinygpt):
 *   penalty   native-mac/Sources/TinyGPTApp/ModelController.swift:268-284
 *             (unique history ids; l > 0 ? l / p : l * p; before temperature;
 *              applied only when p > 1)
 *   presence / frequency: not in the reference (build-defined, OpenAI convention)
 *   mask      native-mac/Sources/TinyGPTModel/ConstrainedGen.swift:805-822 and
 *             Serve.swift:1490-1492 (disallowed -> -inf, as a bitmask here)
 *   greedy    python_ref/model.py:215-216, wasm/src/model.cpp:490-493
 *             (first index of the maximum)
 *   /T        python_ref/model.py:218 (fp32 true division)
 *   top-k     python_ref/model.py:219-222 (k-th largest value, ties kept)
 *   softmax   python_ref/model.py:223, here as exact fixed-point masses
 *   top-p / min-p: not in the reference (build-defined)
 *   draw      wasm/src/model.cpp:508-516 (r in [0, sum), subtract in index
 *             order, first crossing wins) fed the caller's uniform
 *   spec      native-mac/Sources/TinyGPT/SpeculativeDecode.swift:121-210
 *             (T = max(T,1e-5); accept iff u <= min(1, pT/max(pD,1e-10));
 *              residual max(0,pT-pD) if its sum > 1e-10 else pT; bonus at K)
 *   greedy spec  SpeculativeDecode.swift:41-98
 *
 * Arithmetic is defined operation by operation so that the CUDA path can match
 * it bit for bit: fp32 with round-to-nearest and no contraction (build with
 * -ffp-contract=off), the exponential below, uint64 masses summed exactly, and
 * IEEE double only for the threshold comparisons.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#include "../include/tgsample.h"

#define MASS_SCALE 17592186044416.0f /* 2^44 */

/* exp(x) by Cody-Waite reduction x = n ln2 + r, |r| <= ln2/2, then the
 * degree-7 Taylor polynomial of e^r in Horner form (remainder < 6e-9), then an
 * exact scaling by 2^n.  Every step is a single correctly rounded IEEE op. */
float tgo_exp(float x) {
  if (!(x > -104.0f)) return 0.0f;
  if (x > 88.0f) return INFINITY;
  const float n = rintf(x * 1.44269504088896341f);
  float r = fmaf(n, -0.693145751953125f, x);
  r = fmaf(n, -1.42860676533018e-06f, r);
  float p = 1.98412698412698e-04f;      /* 1/5040 */
  p = fmaf(p, r, 1.38888888888889e-03f); /* 1/720 */
  p = fmaf(p, r, 8.33333333333333e-03f); /* 1/120 */
  p = fmaf(p, r, 4.16666666666667e-02f); /* 1/24 */
  p = fmaf(p, r, 1.66666666666667e-01f); /* 1/6 */
  p = fmaf(p, r, 0.5f);
  p = fmaf(p, r, 1.0f);
  p = fmaf(p, r, 1.0f);
  int ni = (int)n;
  union { uint32_t u; float f; } sc;
  if (ni >= -126) {
    sc.u = (uint32_t)(ni + 127) << 23;
    return p * sc.f;
  }
  sc.u = 1u << 23; /* 2^-126 */
  p = p * sc.f;
  sc.u = (uint32_t)(ni + 126 + 127) << 23;
  return p * sc.f;
}

uint64_t tgo_qmass(float d) {
  if (!(d >= -32.0f)) return 0;
  return (uint64_t)(tgo_exp(d) * MASS_SCALE);
}

static float load_logit(const void* logits, int32_t dtype, int64_t off) {
  if (dtype == TG_DTYPE_F32) return ((const float*)logits)[off];
  uint16_t h = ((const uint16_t*)logits)[off];
  union { uint32_t u; float f; } c;
  c.u = (uint32_t)h << 16;
  return c.f;
}

static int cmp_i32(const void* a, const void* b) {
  int32_t x = *(const int32_t*)a, y = *(const int32_t*)b;
  return (x > y) - (x < y);
}

/* k-th largest (1-based) of a[0..n) by quickselect on a scratch copy. */
static float kth_largest(float* a, int64_t n, int64_t k) {
  int64_t lo = 0, hi = n - 1, want = k - 1; /* position in descending order */
  while (lo < hi) {
    float pivot = a[lo + (hi - lo) / 2];
    int64_t i = lo, j = hi;
    while (i <= j) {
      while (a[i] > pivot) i++;
      while (a[j] < pivot) j--;
      if (i <= j) { float t = a[i]; a[i] = a[j]; a[j] = t; i++; j--; }
    }
    if (want <= j) hi = j;
    else if (want >= i) lo = i;
    else return a[want];
  }
  return a[want];
}

typedef struct { float s; int32_t id; } sid_t;

static int cmp_sdesc_idasc(const void* a, const void* b) {
  const sid_t* x = (const sid_t*)a;
  const sid_t* y = (const sid_t*)b;
  if (x->s > y->s) return -1;
  if (x->s < y->s) return 1;
  return (x->id > y->id) - (x->id < y->id);
}

/* Inverse-CDF draw over masses q[0..n) listed in index order. */
static int64_t draw_index(const uint64_t* q, int64_t n, uint64_t total, float u) {
  if (!(u >= 0.0f)) u = 0.0f;
  uint64_t r = (uint64_t)((double)u * (double)total);
  if (r >= total) r = total - 1;
  uint64_t c = 0;
  for (int64_t i = 0; i < n; i++) {
    c += q[i];
    if (c > r) return i;
  }
  return n - 1;
}

/* Per-row detail for tests: y after penalties and mask, and the stage flags
 * (bit 0: survives top-k, bit 1: survives top-p/min-p) plus masses. */
typedef struct {
  float* y;        /* [V] */
  uint8_t* stage;  /* [V] */
  uint64_t* q;     /* [V] */
} tgo_detail;

static int32_t sample_row(const void* logits, int32_t dtype, int64_t base, int32_t V,
                          const tg_row_params* p, const int32_t* hist, int32_t hlen,
                          const uint32_t* mask, float u, float* out_prob,
                          tgo_detail* det, float* y, float* tmp, uint64_t* q,
                          sid_t* order, int32_t* hs) {
  for (int32_t v = 0; v < V; v++) y[v] = load_logit(logits, dtype, base + v);

  /* penalties over distinct history ids */
  if (hlen > 0) {
    int32_t n = 0;
    for (int32_t i = 0; i < hlen; i++)
      if (hist[i] >= 0 && hist[i] < V) hs[n++] = hist[i];
    qsort(hs, (size_t)n, sizeof(int32_t), cmp_i32);
    const int rep_on = p->repetition_penalty > 1.0f;
    const int pf_on = p->presence_penalty != 0.0f || p->frequency_penalty != 0.0f;
    for (int32_t i = 0; i < n;) {
      int32_t j = i;
      while (j < n && hs[j] == hs[i]) j++;
      const int32_t t = hs[i];
      const int32_t c = j - i;
      float val = y[t];
      if (rep_on) val = val > 0.0f ? val / p->repetition_penalty : val * p->repetition_penalty;
      if (pf_on) {
        float f = p->frequency_penalty * (float)c;
        f = f + p->presence_penalty;
        val = val - f;
      }
      y[t] = val;
      i = j;
    }
  }
  if (mask) {
    for (int32_t v = 0; v < V; v++)
      if (!((mask[v >> 5] >> (v & 31)) & 1u)) y[v] = -INFINITY;
  }
  if (det) {
    memcpy(det->y, y, sizeof(float) * (size_t)V);
    memset(det->stage, 0, (size_t)V);
    memset(det->q, 0, sizeof(uint64_t) * (size_t)V);
  }

  if (!(p->temperature > 0.0f)) {
    int32_t best = 0;
    for (int32_t v = 1; v < V; v++)
      if (y[v] > y[best]) best = v;
    if (y[best] == -INFINITY) { *out_prob = 0.0f; return -1; }
    *out_prob = 1.0f;
    if (det) { det->stage[best] = 3; det->q[best] = 1; }
    return best;
  }

  const float T = p->temperature;
  for (int32_t v = 0; v < V; v++) y[v] = y[v] / T; /* y now holds s */

  float kth = -INFINITY;
  if (p->top_k > 0 && p->top_k < V) {
    memcpy(tmp, y, sizeof(float) * (size_t)V);
    kth = kth_largest(tmp, V, p->top_k);
  }
  int64_t n = 0;
  float m = -INFINITY;
  for (int32_t v = 0; v < V; v++)
    if (y[v] >= kth && y[v] > -INFINITY) {
      order[n].s = y[v];
      order[n].id = v;
      n++;
      if (y[v] > m) m = y[v];
    }
  if (n == 0) { *out_prob = 0.0f; return -1; }

  uint64_t Q = 0;
  for (int64_t i = 0; i < n; i++) {
    q[order[i].id] = tgo_qmass(order[i].s - m);
    Q += q[order[i].id];
  }
  if (det)
    for (int64_t i = 0; i < n; i++) { det->stage[order[i].id] |= 1; det->q[order[i].id] = q[order[i].id]; }

  qsort(order, (size_t)n, sizeof(sid_t), cmp_sdesc_idasc);
  int64_t keep = n;
  if (p->top_p < 1.0f) {
    const double target = (double)p->top_p * (double)Q;
    uint64_t c = 0;
    for (int64_t j = 0; j < n; j++) {
      c += q[order[j].id];
      if ((double)c >= target) { keep = j + 1; break; }
    }
  }
  /* final set: prefix [0, keep) filtered by min-p (min_p clamped to 1, so the
   * top survivor, whose mass is exactly 2^44, always stays); reuse tmp as flags */
  const int minp_on = p->min_p > 0.0f;
  const double minq = (double)(p->min_p < 1.0f ? p->min_p : 1.0f) * (double)MASS_SCALE;
  uint8_t* keepflag = (uint8_t*)tmp; /* V bytes fit in V floats */
  memset(keepflag, 0, (size_t)V);
  for (int64_t j = 0; j < keep; j++) {
    const int32_t id = order[j].id;
    if (!minp_on || (double)q[id] >= minq) keepflag[id] = 1;
  }
  uint64_t S = 0;
  for (int32_t v = 0; v < V; v++)
    if (keepflag[v]) S += q[v];
  if (det)
    for (int32_t v = 0; v < V; v++)
      if (keepflag[v]) det->stage[v] |= 2;

  float uu = u;
  if (!(uu >= 0.0f)) uu = 0.0f;
  uint64_t r = (uint64_t)((double)uu * (double)S);
  if (r >= S) r = S - 1;
  uint64_t c = 0;
  int32_t last = -1;
  for (int32_t v = 0; v < V; v++) {
    if (!keepflag[v]) continue;
    last = v;
    c += q[v];
    if (c > r) {
      *out_prob = (float)((double)q[v] / (double)S);
      return v;
    }
  }
  *out_prob = (float)((double)q[last] / (double)S);
  return last;
}

static int64_t row_off(int64_t b, int64_t stride) { return b * stride; }

int32_t tgo_sample(const void* logits, int32_t dtype, int64_t row_stride, int32_t batch,
                   int32_t vocab, const tg_row_params* params, const int32_t* history,
                   const int32_t* history_len, int32_t history_stride,
                   const uint32_t* mask_table, int32_t num_states, const int32_t* state_id,
                   const float* uniforms, int32_t* out_ids, float* out_probs) {
  if (!logits || !params || !out_ids || batch < 0 || vocab <= 0 || row_stride < vocab)
    return TG_ERR_INVALID_ARG;
  if (dtype != TG_DTYPE_F32 && dtype != TG_DTYPE_BF16) return TG_ERR_INVALID_ARG;
  const int64_t W = (vocab + 31) / 32;
  int32_t rc = TG_OK;
#pragma omp parallel
  {
    float* y = (float*)malloc(sizeof(float) * (size_t)vocab);
    float* tmp = (float*)malloc(sizeof(float) * (size_t)vocab + 16);
    uint64_t* q = (uint64_t*)malloc(sizeof(uint64_t) * (size_t)vocab);
    sid_t* order = (sid_t*)malloc(sizeof(sid_t) * (size_t)vocab);
    int32_t* hs = (int32_t*)malloc(sizeof(int32_t) * (TG_MAX_HISTORY + 1));
#pragma omp for schedule(dynamic, 1)
    for (int32_t b = 0; b < batch; b++) {
      const tg_row_params* p = &params[b];
      int32_t hlen = history_len ? history_len[b] : 0;
      if (hlen > history_stride) hlen = history_stride;
      if (hlen > TG_MAX_HISTORY) hlen = TG_MAX_HISTORY;
      if (hlen < 0) hlen = 0;
      const int32_t* hist = hlen ? history + (int64_t)b * history_stride : NULL;
      const uint32_t* mask = NULL;
      int bad_state = 0;
      if (mask_table && state_id && state_id[b] >= 0) {
        if (state_id[b] >= num_states) bad_state = 1;
        else mask = mask_table + (int64_t)state_id[b] * W;
      }
      float prob = 0.0f;
      int32_t id;
      if (bad_state) { id = -1; }
      else id = sample_row(logits, dtype, row_off(b, row_stride), vocab, p, hist, hlen, mask,
                           uniforms ? uniforms[b] : 0.0f, &prob, NULL, y, tmp, q, order, hs);
      out_ids[b] = id;
      if (out_probs) out_probs[b] = prob;
    }
    free(y); free(tmp); free(q); free(order); free(hs);
  }
  return rc;
}

/* Single-row variant that also returns the per-token stages and masses. */
int32_t tgo_sample_row_detail(const void* logits, int32_t dtype, int32_t vocab,
                              const tg_row_params* p, const int32_t* hist, int32_t hlen,
                              const uint32_t* mask, float u, float* out_prob,
                              float* det_y, uint8_t* det_stage, uint64_t* det_q) {
  float* y = (float*)malloc(sizeof(float) * (size_t)vocab);
  float* tmp = (float*)malloc(sizeof(float) * (size_t)vocab + 16);
  uint64_t* q = (uint64_t*)malloc(sizeof(uint64_t) * (size_t)vocab);
  sid_t* order = (sid_t*)malloc(sizeof(sid_t) * (size_t)vocab);
  int32_t* hs = (int32_t*)malloc(sizeof(int32_t) * (TG_MAX_HISTORY + 1));
  tgo_detail det = {det_y, det_stage, det_q};
  if (hlen > TG_MAX_HISTORY) hlen = TG_MAX_HISTORY;
  int32_t id = sample_row(logits, dtype, 0, vocab, p, hist, hlen, mask, u, out_prob,
                          det_y ? &det : NULL, y, tmp, q, order, hs);
  free(y); free(tmp); free(q); free(order); free(hs);
  return id;
}

/* ---- speculative verification ------------------------------------------------ */

/* Grammar-masked verification (a build-defined extension; the reference's
 * speculative paths apply no mask, docs/constrained_generation.md:243-246 of the
 * reference).  m: the position's mask row or NULL; a clear bit makes the element
 * -inf in the target and the draft rows of that position. */
static int allowed(const uint32_t* m, int32_t v) { return !m || ((m[v >> 5] >> (v & 31)) & 1u); }

static const uint32_t* pos_mask(const uint32_t* table, int32_t nstates, int32_t words,
                                const int32_t* sids, int64_t idx) {
  if (!table || !sids) return NULL;
  const int32_t sid = sids[idx];
  if (sid < 0 || sid >= nstates) return NULL; /* out of range: unmasked (status bit on the GPU) */
  return table + (int64_t)sid * words;
}

/* Masses of one tempered row: q[v] = qmass(x[v]/T - max), returns the total. */
static uint64_t row_masses(const void* logits, int32_t dtype, int64_t base, int32_t V,
                           float T, float* s, uint64_t* q, const uint32_t* m) {
  float mx = -INFINITY;
  for (int32_t v = 0; v < V; v++) {
    s[v] = allowed(m, v) ? load_logit(logits, dtype, base + v) / T : -INFINITY;
    if (s[v] > mx) mx = s[v];
  }
  uint64_t Z = 0;
  for (int32_t v = 0; v < V; v++) { q[v] = tgo_qmass(s[v] - mx); Z += q[v]; }
  return Z;
}

/* First index of the maximum; with a mask, of the maximum over the allowed
 * elements above -inf (-1 when there is none). */
static int32_t row_argmax(const void* logits, int32_t dtype, int64_t base, int32_t V,
                          const uint32_t* m) {
  if (m) {
    int32_t best = -1;
    float bv = -INFINITY;
    for (int32_t v = 0; v < V; v++) {
      if (!allowed(m, v)) continue;
      float x = load_logit(logits, dtype, base + v);
      if (x > bv) { bv = x; best = v; }
    }
    return best;
  }
  int32_t best = 0;
  float bv = load_logit(logits, dtype, base);
  for (int32_t v = 1; v < V; v++) {
    float x = load_logit(logits, dtype, base + v);
    if (x > bv) { bv = x; best = v; }
  }
  return best;
}

static int32_t spec_verify_impl(const void* target, const void* draft, int32_t dtype, int32_t batch,
                                int32_t K, int32_t vocab, const int32_t* draft_ids,
                                const float* temperature, const float* u_accept, const float* u_draw,
                                const uint32_t* mask_table, int32_t num_states, const int32_t* state_ids,
                                int32_t* out_ids, int32_t* out_n) {
  if (!target || !draft_ids || !temperature || !out_ids || !out_n || K < 0 || vocab <= 0)
    return TG_ERR_INVALID_ARG;
  const int32_t V = vocab;
  const int32_t W = (V + 31) / 32;
#pragma omp parallel
  {
    float* s = (float*)malloc(sizeof(float) * (size_t)V);
    uint64_t* qT = (uint64_t*)malloc(sizeof(uint64_t) * (size_t)V);
    uint64_t* qD = (uint64_t*)malloc(sizeof(uint64_t) * (size_t)V);
#pragma omp for schedule(dynamic, 1)
    for (int32_t b = 0; b < batch; b++) {
      int32_t* out = out_ids + (int64_t)b * (K + 1);
      for (int32_t i = 0; i <= K; i++) out[i] = -1;
      int32_t n = 0;
      const float t0 = temperature[b];
      if (!(t0 > 0.0f)) {
        /* greedy verify: SpeculativeDecode.swift:41-98 */
        int32_t i;
        for (i = 0; i < K; i++) {
          const uint32_t* m = pos_mask(mask_table, num_states, W, state_ids, (int64_t)b * (K + 1) + i);
          const int32_t a = row_argmax(target, dtype, ((int64_t)b * (K + 1) + i) * V, V, m);
          const int32_t tok = draft_ids[(int64_t)b * K + i];
          if (a == tok) { out[n++] = tok; }
          else { out[n++] = a; break; }
        }
        if (i == K) {
          const uint32_t* m = pos_mask(mask_table, num_states, W, state_ids, (int64_t)b * (K + 1) + K);
          out[n++] = row_argmax(target, dtype, ((int64_t)b * (K + 1) + K) * V, V, m);
        }
        out_n[b] = n;
        continue;
      }
      const float T = t0 > 1e-5f ? t0 : 1e-5f;
      int32_t i;
      int rejected = 0;
      for (i = 0; i < K; i++) {
        const uint32_t* m = pos_mask(mask_table, num_states, W, state_ids, (int64_t)b * (K + 1) + i);
        const int64_t tb = ((int64_t)b * (K + 1) + i) * V;
        const int64_t db = ((int64_t)b * K + i) * V;
        const uint64_t ZT = row_masses(target, dtype, tb, V, T, s, qT, m);
        const uint64_t ZD = row_masses(draft, dtype, db, V, T, s, qD, m);
        int32_t tok = draft_ids[(int64_t)b * K + i];
        if (tok < 0 || tok >= V || !allowed(m, tok)) { tok = -1; } /* a disallowed proposal is rejected */
        double pT = tok >= 0 ? (double)qT[tok] / (double)ZT : 0.0;
        double pD = tok >= 0 ? (double)qD[tok] / (double)ZD : 0.0;
        double den = pD > 1e-10 ? pD : 1e-10;
        double ratio = pT / den;
        double lim = ratio < 1.0 ? ratio : 1.0;
        double ua = (double)u_accept[(int64_t)b * K + i];
        if (tok >= 0 && ua <= lim) { out[n++] = tok; continue; }
        /* reject: residual max(0, pT - pD) */
        uint64_t R = 0;
        for (int32_t v = 0; v < V; v++) {
          double d = (double)qT[v] / (double)ZT - (double)qD[v] / (double)ZD;
          uint64_t rq = d > 0.0 ? (uint64_t)(d * 4503599627370496.0) : 0; /* 2^52 */
          qD[v] = rq; /* reuse */
          R += rq;
        }
        const uint64_t* w = qD;
        uint64_t tot = R;
        if (!((double)R * (1.0 / 4503599627370496.0) > 1e-10)) { w = qT; tot = ZT; }
        if (tot > 0) out[n++] = (int32_t)draw_index(w, V, tot, u_draw[b]); /* empty: no token */
        rejected = 1;
        break;
      }
      if (!rejected) {
        const uint32_t* m = pos_mask(mask_table, num_states, W, state_ids, (int64_t)b * (K + 1) + K);
        const int64_t tb = ((int64_t)b * (K + 1) + K) * V;
        const uint64_t ZT = row_masses(target, dtype, tb, V, T, s, qT, m);
        if (ZT > 0) out[n++] = (int32_t)draw_index(qT, V, ZT, u_draw[b]);
      }
      out_n[b] = n;
    }
    free(s); free(qT); free(qD);
  }
  return TG_OK;
}

int32_t tgo_spec_verify(const void* target, const void* draft, int32_t dtype, int32_t batch,
                        int32_t K, int32_t vocab, const int32_t* draft_ids,
                        const float* temperature, const float* u_accept, const float* u_draw,
                        int32_t* out_ids, int32_t* out_n) {
  return spec_verify_impl(target, draft, dtype, batch, K, vocab, draft_ids, temperature, u_accept,
                          u_draw, NULL, 0, NULL, out_ids, out_n);
}

/* state_ids [batch, K+1]: the grammar state before each position's token (-1: unmasked). */
int32_t tgo_spec_verify_masked(const void* target, const void* draft, int32_t dtype, int32_t batch,
                               int32_t K, int32_t vocab, const int32_t* draft_ids,
                               const float* temperature, const float* u_accept, const float* u_draw,
                               const uint32_t* mask_table, int32_t num_states, const int32_t* state_ids,
                               int32_t* out_ids, int32_t* out_n) {
  return spec_verify_impl(target, draft, dtype, batch, K, vocab, draft_ids, temperature, u_accept,
                          u_draw, mask_table, num_states, state_ids, out_ids, out_n);
}
