/*
 * ts_oracle_model.c — CPU restatement of textsift's forward composition.
 *
 * TEST INFRASTRUCTURE ONLY (parity checker + timed CPU baseline).
 * Citations are into packages/textsift/src/browser/ of teamchong/textsift:
 *   inference/model.ts:50-105      modelForward
 *   inference/block.ts:49-197     routerForward / blockForward
 *   inference/attention.ts:45-215 attentionForward
 *   inference/expert.ts:104-212    expertDispatch (single thread)
 *   inference/mt-expert.ts:63-191  expertDispatchParallel (MtPool mode)
 *   inference/rope.ts:27-144       YaRN tables
 *   backends/wasm.ts:328-453       tensor names produced by loadOnnxWeights
 *   backends/wasm.ts:728-805       WasmBackend.forward (mask skip, logits widen)
 */
#include "ts_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#include <stdio.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define TSO_MAX_LAYERS 64

typedef struct {
  const uint8_t* int4;
  const uint16_t* scales;
  const uint8_t* zp;
  const uint16_t* bias;
} i4w;

typedef struct {
  const uint16_t* input_ln;
  const uint16_t* post_ln;
  i4w q, k, v, o;
  const float* sinks;
  i4w router;
  i4w gate_up, down; /* expert tensors: [E, N, ...] */
} layer_w;

struct tso_model {
  tso_config cfg;
  const uint8_t* embed_int4;
  const uint16_t* embed_scales;
  const uint8_t* embed_zp;
  const uint16_t* final_norm;
  i4w score;
  layer_w layers[TSO_MAX_LAYERS];
};

tso_model* tso_model_create(const tso_config* cfg) {
  if (cfg->n_layers > TSO_MAX_LAYERS) return NULL;
  tso_model* m = (tso_model*)calloc(1, sizeof(tso_model));
  if (m) m->cfg = *cfg;
  return m;
}

void tso_model_destroy(tso_model* m) { free(m); }

static int set_i4(i4w* w, const char* field, const void* p) {
  if (!strcmp(field, "int4")) w->int4 = (const uint8_t*)p;
  else if (!strcmp(field, "scales")) w->scales = (const uint16_t*)p;
  else if (!strcmp(field, "zp")) w->zp = (const uint8_t*)p;
  else if (!strcmp(field, "bias")) w->bias = (const uint16_t*)p;
  else return -1;
  return 0;
}

/* Names as produced by loadOnnxWeights (browser/backends/wasm.ts:358-446). */
int tso_model_set(tso_model* m, const char* name, const void* data, size_t nbytes) {
  (void)nbytes;
  if (!strcmp(name, "embed.int4")) { m->embed_int4 = (const uint8_t*)data; return 0; }
  if (!strcmp(name, "embed.scales")) { m->embed_scales = (const uint16_t*)data; return 0; }
  if (!strcmp(name, "embed.zp")) { m->embed_zp = (const uint8_t*)data; return 0; }
  if (!strcmp(name, "final_norm")) { m->final_norm = (const uint16_t*)data; return 0; }
  if (!strncmp(name, "score.", 6)) return set_i4(&m->score, name + 6, data);
  unsigned L;
  int pos = 0;
  if (sscanf(name, "layers.%u.%n", &L, &pos) == 1 && pos > 0 && L < m->cfg.n_layers) {
    layer_w* lw = &m->layers[L];
    const char* rest = name + pos;
    if (!strcmp(rest, "input_layernorm")) { lw->input_ln = (const uint16_t*)data; return 0; }
    if (!strcmp(rest, "post_attention_layernorm")) { lw->post_ln = (const uint16_t*)data; return 0; }
    if (!strcmp(rest, "attn.sinks")) { lw->sinks = (const float*)data; return 0; }
    if (!strncmp(rest, "attn.q_proj.", 12)) return set_i4(&lw->q, rest + 12, data);
    if (!strncmp(rest, "attn.k_proj.", 12)) return set_i4(&lw->k, rest + 12, data);
    if (!strncmp(rest, "attn.v_proj.", 12)) return set_i4(&lw->v, rest + 12, data);
    if (!strncmp(rest, "attn.o_proj.", 12)) return set_i4(&lw->o, rest + 12, data);
    if (!strncmp(rest, "router.", 7)) return set_i4(&lw->router, rest + 7, data);
    if (!strncmp(rest, "experts.gate_up.", 16)) return set_i4(&lw->gate_up, rest + 16, data);
    if (!strncmp(rest, "experts.down.", 13)) return set_i4(&lw->down, rest + 13, data);
  }
  return -1;
}

/* ------------------------------------------------------------------ */
/* YaRN RoPE tables: rope.ts:27-144.  Everything the reference computes in
 * JS doubles is computed in double here; Float32Array stores are (float)
 * casts; fp16 stores use the JS f32->fp16 (±0 -> +0).                 */
/* ------------------------------------------------------------------ */
void tso_build_rope_tables(const tso_rope_cfg* c, uint32_t T, uint16_t* cos_out, uint16_t* sin_out) {
  const uint32_t half = c->head_dim / 2;
  float extrap[256], interp[256], inv_freq[256];
  for (uint32_t i = 0; i < half; i++) {
    double pos_freq = pow(c->theta, (double)(2 * i) / (double)c->head_dim);
    extrap[i] = (float)(1.0 / pos_freq);
    interp[i] = (float)(1.0 / (c->factor * pos_freq));
  }
  const double two_pi = 2.0 * 3.141592653589793;
  double low = ((double)c->head_dim * log(c->original_max_pos / (c->beta_fast * two_pi))) / (2.0 * log(c->theta));
  double high = ((double)c->head_dim * log(c->original_max_pos / (c->beta_slow * two_pi))) / (2.0 * log(c->theta));
  if (c->truncate) { low = floor(low); high = ceil(high); }
  if (low < 0) low = 0;
  if (high > (double)(c->head_dim - 1)) high = (double)(c->head_dim - 1);
  const double ramp_min = low, ramp_max = high == low ? low + 0.001 : high;
  for (uint32_t i = 0; i < half; i++) {
    double linear = ((double)i - ramp_min) / (ramp_max - ramp_min);
    double ramp = linear < 0 ? 0 : (linear > 1 ? 1 : linear);
    double ef = 1.0 - ramp;
    double a = (double)interp[i] * (1.0 - ef);
    double b = (double)extrap[i] * ef;
    inv_freq[i] = (float)(a + b);
  }
  const double att = c->factor <= 1.0 ? 1.0 : 0.1 * log(c->factor) + 1.0;
  for (uint32_t t = 0; t < T; t++)
    for (uint32_t i = 0; i < half; i++) {
      double angle = (double)t * (double)inv_freq[i];
      cos_out[(size_t)t * half + i] = tso_js_f32_to_f16(cos(angle) * att);
      sin_out[(size_t)t * half + i] = tso_js_f32_to_f16(sin(angle) * att);
    }
}

/* ------------------------------------------------------------------ */
/* Composition                                                          */
/* ------------------------------------------------------------------ */

static inline uint32_t part_lo(uint32_t w, uint32_t n, uint32_t N) { return (uint32_t)(((uint64_t)w * n) / N); }

/* T-partitioned int4 matmul (block.ts:63-95, attention.ts:84-146): each
 * worker runs the kernel on its own row slice, which changes which rows
 * take the tile vs tail path exactly as the reference's MtPool does. */
static void matmul_rows(int nt, int x_f32, int o_f32, const void* x, const i4w* w, void* out,
                        uint32_t T, uint32_t N, uint32_t Dk) {
  const size_t xe = x_f32 ? 4 : 2, oe = o_f32 ? 4 : 2;
  if (nt > 1 && T >= (uint32_t)nt * 2) {
#pragma omp parallel num_threads(nt)
    {
#ifdef _OPENMP
      uint32_t wi = (uint32_t)omp_get_thread_num();
#else
      uint32_t wi = 0;
#endif
      uint32_t t0 = part_lo(wi, T, (uint32_t)nt), t1 = part_lo(wi + 1, T, (uint32_t)nt);
      if (t1 > t0)
        tso_matmul_int4(x_f32, o_f32, (const char*)x + (size_t)t0 * Dk * xe, w->int4, w->scales, w->zp,
                        w->bias, (char*)out + (size_t)t0 * N * oe, t1 - t0, N, Dk);
    }
  } else {
    tso_matmul_int4(x_f32, o_f32, x, w->int4, w->scales, w->zp, w->bias, out, T, N, Dk);
  }
}

/* attention.ts:45-215 */
static void attention_forward(const tso_model* m, const layer_w* lw, const float* hf, uint16_t* out,
                              const uint16_t* cos_t, const uint16_t* sin_t, const uint8_t* mask,
                              uint32_t T, int nt) {
  const tso_config* c = &m->cfg;
  const uint32_t D = c->d_model, Hq = c->n_heads, Hkv = c->n_kv_heads, hd = c->head_dim;
  uint16_t* q = (uint16_t*)malloc((size_t)T * Hq * hd * 2);
  uint16_t* k = (uint16_t*)malloc((size_t)T * Hkv * hd * 2);
  uint16_t* v = (uint16_t*)malloc((size_t)T * Hkv * hd * 2);
  uint16_t* ao = (uint16_t*)malloc((size_t)T * Hq * hd * 2);
  float* af = (float*)malloc((size_t)T * Hq * hd * 4);
  if (nt > 1 && T >= (uint32_t)nt * 2) {
#pragma omp parallel num_threads(nt)
    {
#ifdef _OPENMP
      uint32_t wi = (uint32_t)omp_get_thread_num();
#else
      uint32_t wi = 0;
#endif
      uint32_t t0 = part_lo(wi, T, (uint32_t)nt), t1 = part_lo(wi + 1, T, (uint32_t)nt), tc = t1 - t0;
      if (tc > 0) {
        const float* xo = hf + (size_t)t0 * D;
        uint16_t* qo = q + (size_t)t0 * Hq * hd;
        uint16_t* ko = k + (size_t)t0 * Hkv * hd;
        uint16_t* vo = v + (size_t)t0 * Hkv * hd;
        tso_matmul_int4(1, 0, xo, lw->q.int4, lw->q.scales, lw->q.zp, lw->q.bias, qo, tc, Hq * hd, D);
        tso_matmul_int4(1, 0, xo, lw->k.int4, lw->k.scales, lw->k.zp, lw->k.bias, ko, tc, Hkv * hd, D);
        tso_matmul_int4(1, 0, xo, lw->v.int4, lw->v.scales, lw->v.zp, lw->v.bias, vo, tc, Hkv * hd, D);
        tso_rope_apply(qo, cos_t + (size_t)t0 * (hd / 2), sin_t + (size_t)t0 * (hd / 2), tc, Hq, hd);
        tso_rope_apply(ko, cos_t + (size_t)t0 * (hd / 2), sin_t + (size_t)t0 * (hd / 2), tc, Hkv, hd);
      }
    }
  } else {
    tso_matmul_int4(1, 0, hf, lw->q.int4, lw->q.scales, lw->q.zp, lw->q.bias, q, T, Hq * hd, D);
    tso_matmul_int4(1, 0, hf, lw->k.int4, lw->k.scales, lw->k.zp, lw->k.bias, k, T, Hkv * hd, D);
    tso_matmul_int4(1, 0, hf, lw->v.int4, lw->v.scales, lw->v.zp, lw->v.bias, v, T, Hkv * hd, D);
    tso_rope_apply(q, cos_t, sin_t, T, Hq, hd);
    tso_rope_apply(k, cos_t, sin_t, T, Hkv, hd);
  }
  /* attention.ts:150-185: H_q partition when Hq >= 2 * threads */
  if (nt > 1 && Hq >= (uint32_t)nt * 2) {
#pragma omp parallel num_threads(nt)
    {
#ifdef _OPENMP
      uint32_t wi = (uint32_t)omp_get_thread_num();
#else
      uint32_t wi = 0;
#endif
      uint32_t h0 = part_lo(wi, Hq, (uint32_t)nt), h1 = part_lo(wi + 1, Hq, (uint32_t)nt);
      if (h1 > h0) tso_banded_attention(q, k, v, lw->sinks, mask, ao, T, Hq, Hkv, hd, c->window, h0, h1);
    }
  } else {
    tso_banded_attention(q, k, v, lw->sinks, mask, ao, T, Hq, Hkv, hd, c->window, 0, Hq);
  }
  tso_convert_fp16_to_f32(ao, af, T * Hq * hd);
  matmul_rows(nt, 1, 0, af, &lw->o, out, T, D, Hq * hd);
  free(q); free(k); free(v); free(ao); free(af);
}

/* block.ts:49-103: f32 router logits, top-k, softmax over k, x(1/K) in JS doubles */
static void router_forward(const tso_model* m, const layer_w* lw, const float* x, int32_t* idx,
                           float* scores, uint32_t T, int nt, const int32_t* forced) {
  const uint32_t E = m->cfg.n_experts, K = m->cfg.top_k, D = m->cfg.d_model;
  float* logits = (float*)malloc((size_t)T * E * 4);
  float* topv = (float*)malloc((size_t)T * K * 4);
  matmul_rows(nt, 1, 1, x, &lw->router, logits, T, E, D);
  if (forced) {
    /* teacher forcing (parity tooling, not a reference path): take the given
     * experts in the given order, score them with this forward's own logits */
    for (size_t i = 0; i < (size_t)T * K; i++) {
      int32_t e = forced[i];
      idx[i] = e;
      topv[i] = (e >= 0 && (uint32_t)e < E) ? logits[(i / K) * E + (uint32_t)e] : -INFINITY;
    }
  } else {
    tso_topk_partial_f32(logits, idx, topv, T, E, K);
  }
  tso_softmax_f32(topv, scores, T, K);
  const double inv_k = 1.0 / (double)K;
  for (size_t i = 0; i < (size_t)T * K; i++) scores[i] = (float)((double)scores[i] * inv_k);
  free(logits); free(topv);
}

/* One expert-major dispatch over tokens [t0, t1) (expert.ts:127-211;
 * mt-expert.ts:94-181 for the per-worker slice). acc rows t0..t1 must be 0. */
static void expert_slice(const tso_model* m, const layer_w* lw, const float* x, const int32_t* ridx,
                         const float* rsc, float* acc, uint32_t t0, uint32_t t1) {
  const tso_config* c = &m->cfg;
  const uint32_t D = c->d_model, dff = c->d_ff, E = c->n_experts, K = c->top_k;
  const uint32_t cap = (t1 - t0) * K;
  if (cap == 0) return;
  uint32_t* cnt = (uint32_t*)calloc(E + 1, 4);
  int32_t* tok = (int32_t*)malloc((size_t)cap * 4);
  float* wts = (float*)malloc((size_t)cap * 4);
  uint32_t* off = (uint32_t*)calloc(E + 1, 4);
  for (uint32_t t = t0; t < t1; t++)
    for (uint32_t k = 0; k < K; k++) {
      int32_t e = ridx[(size_t)t * K + k];
      if (e < 0 || (uint32_t)e >= E) continue;
      cnt[e]++;
    }
  for (uint32_t e = 0; e < E; e++) off[e + 1] = off[e] + cnt[e];
  memset(cnt, 0, (size_t)(E + 1) * 4);
  for (uint32_t t = t0; t < t1; t++)
    for (uint32_t k = 0; k < K; k++) {
      int32_t e = ridx[(size_t)t * K + k];
      if (e < 0 || (uint32_t)e >= E) continue;
      uint32_t p = off[e] + cnt[e]++;
      tok[p] = (int32_t)t;
      wts[p] = rsc[(size_t)t * K + k];
    }
  uint32_t maxm = 0;
  for (uint32_t e = 0; e < E; e++) if (off[e + 1] - off[e] > maxm) maxm = off[e + 1] - off[e];
  float* xg = (float*)malloc((size_t)maxm * D * 4 + 4);
  float* gu = (float*)malloc((size_t)maxm * 2 * dff * 4 + 4);
  float* gl = (float*)malloc((size_t)maxm * dff * 4 + 4);
  float* of = (float*)malloc((size_t)maxm * D * 4 + 4);
  const uint32_t nbD = D / 32, nbF = dff / 32;
  for (uint32_t e = 0; e < E; e++) {
    uint32_t mm = off[e + 1] - off[e];
    if (mm == 0) continue;
    tso_gather_f32(x, tok + off[e], xg, mm, D);
    /* expert.ts:63-87 slice pointers: [E, N, D/2] int4, [E, N, D/32] scales,
     * [E, N, ceil(D/32/2)] zp, [E, N] bias */
    const uint32_t Ngu = 2 * dff;
    tso_matmul_int4(1, 1, xg, lw->gate_up.int4 + (size_t)e * Ngu * D / 2,
                    lw->gate_up.scales + (size_t)e * Ngu * nbD,
                    lw->gate_up.zp + (size_t)e * Ngu * ((nbD + 1) / 2),
                    lw->gate_up.bias + (size_t)e * Ngu, gu, mm, Ngu, D);
    tso_swiglu_clamp_f32(gu, gl, mm, dff);
    tso_matmul_int4(1, 1, gl, lw->down.int4 + (size_t)e * D * dff / 2,
                    lw->down.scales + (size_t)e * D * nbF,
                    lw->down.zp + (size_t)e * D * ((nbF + 1) / 2),
                    lw->down.bias + (size_t)e * D, of, mm, D, dff);
    tso_scatter_add_weighted_f32(acc, of, tok + off[e], wts + off[e], mm, D);
  }
  free(cnt); free(tok); free(wts); free(off); free(xg); free(gu); free(gl); free(of);
}

static void moe_forward(const tso_model* m, const layer_w* lw, const float* x, uint32_t T,
                        uint16_t* moe_out, int32_t* idx, float* sc, int nt, const int32_t* forced) {
  const uint32_t D = m->cfg.d_model, K = m->cfg.top_k;
  router_forward(m, lw, x, idx, sc, T, nt, forced);
  float* acc = (float*)calloc((size_t)T * D, 4);
  if (nt > 1) {
#pragma omp parallel num_threads(nt)
    {
#ifdef _OPENMP
      uint32_t wi = (uint32_t)omp_get_thread_num();
#else
      uint32_t wi = 0;
#endif
      uint32_t t0 = part_lo(wi, T, (uint32_t)nt), t1 = part_lo(wi + 1, T, (uint32_t)nt);
      if (t1 > t0) {
        expert_slice(m, lw, x, idx, sc, acc, t0, t1);
        tso_cast_f32_to_fp16_scaled(acc + (size_t)t0 * D, moe_out + (size_t)t0 * D, (t1 - t0) * D, (float)K);
      }
    }
  } else {
    expert_slice(m, lw, x, idx, sc, acc, 0, T);
    tso_cast_f32_to_fp16_scaled(acc, moe_out, T * D, (float)K);
  }
  free(acc);
}

int tso_moe_forward(const tso_model* m, uint32_t layer, const float* normed, uint32_t T,
                    uint16_t* moe_out, int32_t* idx_out, float* w_out, int n_threads) {
  if (layer >= m->cfg.n_layers) return -1;
  moe_forward(m, &m->layers[layer], normed, T, moe_out, idx_out, w_out, n_threads, NULL);
  return 0;
}

/* block.ts:108-197 */
static void block_forward(const tso_model* m, const layer_w* lw, const uint16_t* in, uint16_t* out,
                          const uint16_t* cos_t, const uint16_t* sin_t, const uint8_t* mask,
                          uint32_t T, int nt, int32_t* topk_trace, float* normed_trace,
                          const int32_t* forced) {
  const tso_config* c = &m->cfg;
  const uint32_t D = c->d_model, K = c->top_k;
  float* hf = (float*)malloc((size_t)T * D * 4);
  uint16_t* attn = (uint16_t*)malloc((size_t)T * D * 2);
  uint16_t* res2 = (uint16_t*)malloc((size_t)T * D * 2);
  float* n2 = (float*)malloc((size_t)T * D * 4);
  int32_t* idx = (int32_t*)malloc((size_t)T * K * 4);
  float* sc = (float*)malloc((size_t)T * K * 4);
  uint16_t* moe = (uint16_t*)malloc((size_t)T * D * 2);
  tso_rms_norm_fp16_to_f32(in, lw->input_ln, hf, T, D, c->eps);
  attention_forward(m, lw, hf, attn, cos_t, sin_t, mask, T, nt);
  if (nt > 1 && T >= (uint32_t)nt * 2) {
#pragma omp parallel num_threads(nt)
    {
#ifdef _OPENMP
      uint32_t wi = (uint32_t)omp_get_thread_num();
#else
      uint32_t wi = 0;
#endif
      uint32_t t0 = part_lo(wi, T, (uint32_t)nt), t1 = part_lo(wi + 1, T, (uint32_t)nt);
      if (t1 > t0)
        tso_add_rmsnorm_fp16_to_f32(in + (size_t)t0 * D, attn + (size_t)t0 * D, lw->post_ln,
                                    res2 + (size_t)t0 * D, n2 + (size_t)t0 * D, t1 - t0, D, c->eps);
    }
  } else {
    tso_add_rmsnorm_fp16_to_f32(in, attn, lw->post_ln, res2, n2, T, D, c->eps);
  }
  if (normed_trace) memcpy(normed_trace, n2, (size_t)T * D * 4);
  moe_forward(m, lw, n2, T, moe, idx, sc, nt, forced);
  if (topk_trace) memcpy(topk_trace, idx, (size_t)T * K * 4);
  tso_add_fp16(res2, moe, out, T * D);
  free(hf); free(attn); free(res2); free(n2); free(idx); free(sc); free(moe);
}

/* model.ts:50-105 + wasm.ts:728-805 */
int tso_model_forward(const tso_model* m, const int32_t* ids, const uint8_t* mask, uint32_t T,
                      float* logits_out, int n_threads, uint16_t* hidden_trace, int32_t* topk_trace,
                      float* normed_trace) {
  return tso_model_forward_forced(m, ids, mask, T, logits_out, n_threads, hidden_trace, topk_trace,
                                  normed_trace, NULL);
}

int tso_model_forward_forced(const tso_model* m, const int32_t* ids, const uint8_t* mask, uint32_t T,
                             float* logits_out, int n_threads, uint16_t* hidden_trace, int32_t* topk_trace,
                             float* normed_trace, const int32_t* forced_topk) {
  const tso_config* c = &m->cfg;
  const uint32_t D = c->d_model, C = c->n_classes, hd = c->head_dim;
  if (T == 0) return 0;
  if (!m->embed_int4 || !m->embed_scales || !m->embed_zp || !m->final_norm || !m->score.int4) return -2;
  /* wasm.ts:755-764: an all-ones mask is passed as "no mask" */
  const uint8_t* mk = NULL;
  if (mask)
    for (uint32_t i = 0; i < T; i++)
      if (mask[i] != 1) { mk = mask; break; }
  uint16_t* cos_t = (uint16_t*)malloc((size_t)T * (hd / 2) * 2);
  uint16_t* sin_t = (uint16_t*)malloc((size_t)T * (hd / 2) * 2);
  tso_build_rope_tables(&c->rope, T, cos_t, sin_t);
  uint16_t* h0 = (uint16_t*)malloc((size_t)T * D * 2);
  uint16_t* h1 = (uint16_t*)malloc((size_t)T * D * 2);
  tso_embed_lookup_int4(m->embed_int4, m->embed_scales, m->embed_zp, ids, h0, T, c->vocab, D);
  if (hidden_trace) memcpy(hidden_trace, h0, (size_t)T * D * 2);
  uint16_t *src = h0, *dst = h1;
  for (uint32_t L = 0; L < c->n_layers; L++) {
    block_forward(m, &m->layers[L], src, dst, cos_t, sin_t, mk, T, n_threads,
                  topk_trace ? topk_trace + (size_t)L * T * c->top_k : NULL,
                  normed_trace ? normed_trace + (size_t)L * T * D : NULL,
                  forced_topk ? forced_topk + (size_t)L * T * c->top_k : NULL);
    uint16_t* tmp = src; src = dst; dst = tmp;
    if (hidden_trace) memcpy(hidden_trace + (size_t)(L + 1) * T * D, src, (size_t)T * D * 2);
  }
  float* xf = (float*)malloc((size_t)T * D * 4);
  uint16_t* lg = (uint16_t*)malloc((size_t)T * C * 2);
  tso_rms_norm_fp16_to_f32(src, m->final_norm, xf, T, D, c->eps);
  tso_matmul_int4(1, 0, xf, m->score.int4, m->score.scales, m->score.zp, m->score.bias, lg, T, C, D);
  for (size_t i = 0; i < (size_t)T * C; i++) logits_out[i] = tso_js_f16_to_f32(lg[i]);
  free(cos_t); free(sin_t); free(h0); free(h1); free(xf); free(lg);
  return 0;
}
