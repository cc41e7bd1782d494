/*
 * ORACLE — test infrastructure only. A C restatement of the reference's FP32 CPU forward of the
 * Chronos-2 family, the checker for the B200 path (never linked into it).
 *
 * Restates, in src/main/java/ai/beestream/jitcast/chronos2/:
 *   ModelLayout.of / live / members            ModelLayout.java:72-181 (cut + NaN left pad, live keys)
 *   ModelPrep.of / instanceNorm / scaled / finish  ModelPrep.java:37-138
 *   CpuChronos2.forward, inverseFrequencies, rope, timeAttention, groupAttention, softmaxValues
 *                                              cpu/CpuChronos2.java:84-304
 *   Chronos2Weights.qkv (q|k|v concatenated), regToken (shared row 1)  Chronos2Weights.java:131-150
 * with double reductions where the reference uses them. Compiled with -ffp-contract=off.
 */
#include <math.h>
#include <pthread.h>
#include <stdatomic.h>
#include <stdlib.h>
#include <string.h>

#include "oracle.h"
#include "oracle_chronos2.h"

typedef void (*c2_range_fn)(void* ctx, int i);
typedef struct {
  c2_range_fn fn;
  void* ctx;
  int n;
  atomic_int next;
} c2_job;

static void* c2_worker(void* arg) {
  c2_job* j = (c2_job*)arg;
  for (;;) {
    int i = atomic_fetch_add(&j->next, 1);
    if (i >= j->n) break;
    j->fn(j->ctx, i);
  }
  return NULL;
}

static void c2_parallel_for(int n, int threads, c2_range_fn fn, void* ctx) {
  c2_job job = {fn, ctx, n, 0};
  if (threads > n) threads = n;
  if (threads > 256) threads = 256;
  pthread_t tid[256];
  int started = 0;
  for (int t = 1; t < threads; t++)
    if (pthread_create(&tid[started], NULL, c2_worker, &job) == 0) started++;
  c2_worker(&job);
  for (int t = 0; t < started; t++) pthread_join(tid[t], NULL);
}

static float c2_asinh(float v) {
  double a = fabs((double)v);
  double r = log(a + sqrt(a * a + 1.0));
  return (float)(v < 0 ? -r : r);
}

/* ModelPrep.instanceNorm: {loc, scale} over the non-NaN values. */
static void c2_instance_norm(const float* x, int len, float out[2]) {
  double sum = 0;
  int n = 0;
  for (int i = 0; i < len; i++)
    if (!isnan(x[i])) {
      sum += x[i];
      n++;
    }
  if (n == 0) {
    out[0] = 0.0f;
    out[1] = 1.0f;
    return;
  }
  float loc = (float)(sum / n);
  double ss = 0;
  for (int i = 0; i < len; i++)
    if (!isnan(x[i])) {
      float d = x[i] - loc;
      ss += (double)d * d;
    }
  float scale = (float)sqrt(ss / n);
  out[0] = loc;
  out[1] = scale == 0.0f ? 1e-5f : scale;
}

static float c2_scaled(float x, float loc, float scale, int arcsinh) {
  float v = (x - loc) / scale;
  return arcsinh ? c2_asinh(v) : v;
}

int jco_chronos2_prepare(const jco_chronos2* m, const jco_c2_input* in, jco_c2_prepared* p) {
  const int ps = m->patch_size, r = in->rows, h = in->output_patches, t = in->length;
  if (h < 1) return -1;
  const int kept = t < m->context_length ? t : m->context_length;
  const int padded = (kept + ps - 1) / ps * ps;
  const int nc = padded / ps, reg = m->use_reg_token ? 1 : 0, ne = nc + h, n = nc + reg + h;
  p->rows = r;
  p->nc = nc;
  p->reg = reg;
  p->h = h;
  p->n = n;
  p->live = (int*)malloc(sizeof(int) * (size_t)r * n);
  p->tokens = (float*)malloc(sizeof(float) * (size_t)r * ne * 3 * ps);
  p->loc = (float*)malloc(sizeof(float) * r);
  p->scale = (float*)malloc(sizeof(float) * r);
  float* win = (float*)malloc(sizeof(float) * padded);
  float* fut = (float*)malloc(sizeof(float) * h * ps);
  const float ts = (float)m->time_encoding_scale;
  for (int i = 0; i < r; i++) {
    for (int s = 0; s < padded - kept; s++) win[s] = NAN;
    memcpy(win + padded - kept, in->context + (size_t)i * t + (t - kept), sizeof(float) * kept);
    for (int s = 0; s < h * ps; s++) fut[s] = NAN;
    if (in->future && in->future_len > 0)
      memcpy(fut, in->future + (size_t)i * in->future_len, sizeof(float) * in->future_len);
    for (int q = 0; q < nc; q++) {
      int any = 0;
      for (int s = q * ps; s < (q + 1) * ps; s++) any |= !isnan(win[s]);
      p->live[(size_t)i * n + q] = any;
    }
    for (int q = nc; q < n; q++) p->live[(size_t)i * n + q] = 1;
    float ls[2];
    c2_instance_norm(win, padded, ls);
    p->loc[i] = ls[0];
    p->scale[i] = ls[1];
    for (int q = 0; q < nc; q++) {
      float* o = p->tokens + ((size_t)i * ne + q) * 3 * ps;
      for (int s = 0; s < ps; s++) {
        int tt = q * ps + s;
        o[s] = (float)(tt - nc * ps) / ts;
        int obs = !isnan(win[tt]);
        o[ps + s] = obs ? c2_scaled(win[tt], ls[0], ls[1], m->use_arcsinh) : 0.0f;
        o[2 * ps + s] = obs ? 1.0f : 0.0f;
      }
    }
    for (int q = 0; q < h; q++) {
      float* o = p->tokens + ((size_t)i * ne + nc + q) * 3 * ps;
      for (int s = 0; s < ps; s++) {
        int tt = q * ps + s;
        o[s] = (float)tt / ts;
        int obs = !isnan(fut[tt]);
        o[ps + s] = obs ? c2_scaled(fut[tt], ls[0], ls[1], m->use_arcsinh) : 0.0f;
        o[2 * ps + s] = obs ? 1.0f : 0.0f;
      }
    }
  }
  free(win);
  free(fut);
  p->group = (int*)malloc(sizeof(int) * r);
  memcpy(p->group, in->group, sizeof(int) * r);
  return 0;
}

void jco_c2_prepared_free(jco_c2_prepared* p) {
  free(p->live);
  free(p->tokens);
  free(p->loc);
  free(p->scale);
  free(p->group);
  memset(p, 0, sizeof *p);
}

void jco_chronos2_finish(const jco_chronos2* m, const jco_c2_prepared* p, const float* raw, float* out) {
  const int r = p->rows, ps = m->patch_size, q = m->num_quantiles, h = p->h;
  for (int i = 0; i < r; i++)
    for (int pp = 0; pp < h; pp++) {
      size_t o = ((size_t)i * h + pp) * q * ps;
      for (int k = 0; k < q; k++)
        for (int s = 0; s < ps; s++) {
          float v = raw[o + (size_t)k * ps + s];
          if (m->use_arcsinh) v = (float)sinh((double)v);
          out[((size_t)i * q + k) * h * ps + pp * ps + s] = v * p->scale[i] + p->loc[i];
        }
    }
}

/* output(ReLU(hidden(x))) + residual(x) */
static float* c2_residual(const float* x, int rows, int in, int hidden, int out, const float* hw, const float* hb,
                          const float* ow, const float* ob, const float* rw, const float* rb, int threads) {
  float* hdn = (float*)malloc(sizeof(float) * (size_t)rows * hidden);
  jco_linear(x, rows, hw, hb, in, hidden, hdn, threads);
  for (size_t i = 0; i < (size_t)rows * hidden; i++) hdn[i] = hdn[i] > 0.0f ? hdn[i] : 0.0f;
  float* y = (float*)malloc(sizeof(float) * (size_t)rows * out);
  jco_linear(hdn, rows, ow, ob, hidden, out, y, threads);
  free(hdn);
  float* res = (float*)malloc(sizeof(float) * (size_t)rows * out);
  jco_linear(x, rows, rw, rb, in, out, res, threads);
  for (size_t i = 0; i < (size_t)rows * out; i++) y[i] += res[i];
  free(res);
  return y;
}

typedef struct {
  const jco_chronos2* m;
  const jco_c2_prepared* p;
  const float *qkv, *q, *k;
  float* out;
} c2_attn;

/* CpuChronos2.timeAttention for one (row, head): every live key, both directions, unscaled. */
static void c2_time_job(void* vc, int job) {
  c2_attn* c = (c2_attn*)vc;
  const int heads = c->m->num_heads, dh = c->m->d_kv, inner = heads * dh, n = c->p->n;
  const int i = job / heads, hh = job % heads;
  double* pr = (double*)malloc(sizeof(double) * n);
  for (int t = 0; t < n; t++) {
    double mx = -INFINITY;
    size_t qo = ((size_t)i * n + t) * inner + hh * dh;
    for (int s = 0; s < n; s++) {
      if (!c->p->live[(size_t)i * n + s]) {
        pr[s] = -INFINITY;
        continue;
      }
      size_t ko = ((size_t)i * n + s) * inner + hh * dh;
      double dot = 0;
      for (int e = 0; e < dh; e++) dot += (double)c->q[qo + e] * c->k[ko + e];
      pr[s] = dot;
      mx = fmax(mx, dot);
    }
    double sum = 0;
    for (int s = 0; s < n; s++) {
      pr[s] = pr[s] == -INFINITY ? 0 : exp(pr[s] - mx);
      sum += pr[s];
    }
    for (int e = 0; e < dh; e++) {
      double acc = 0;
      for (int s = 0; s < n; s++)
        if (pr[s] != 0) acc += pr[s] * c->qkv[((size_t)i * n + s) * 3 * inner + 2 * inner + hh * dh + e];
      c->out[qo + e] = (float)(acc / sum);
    }
  }
  free(pr);
}

/* CpuChronos2.groupAttention for one token slot: the live rows of the group; zeros if none. */
static void c2_group_job(void* vc, int t) {
  c2_attn* c = (c2_attn*)vc;
  const jco_c2_prepared* p = c->p;
  const int r = p->rows, heads = c->m->num_heads, dh = c->m->d_kv, inner = heads * dh, n = p->n;
  int* mem = (int*)malloc(sizeof(int) * r);
  double* pr = (double*)malloc(sizeof(double) * r);
  for (int i = 0; i < r; i++) {
    int cnt = 0;
    for (int j = 0; j < r; j++)
      if (p->group[j] == p->group[i]) mem[cnt++] = j;
    for (int hh = 0; hh < heads; hh++) {
      size_t qo = ((size_t)i * n + t) * 3 * inner + hh * dh;
      double mx = -INFINITY;
      for (int jj = 0; jj < cnt; jj++) {
        int j = mem[jj];
        if (!p->live[(size_t)j * n + t]) {
          pr[jj] = -INFINITY;
          continue;
        }
        size_t ko = ((size_t)j * n + t) * 3 * inner + inner + hh * dh;
        double dot = 0;
        for (int e = 0; e < dh; e++) dot += (double)c->qkv[qo + e] * c->qkv[ko + e];
        pr[jj] = dot;
        mx = fmax(mx, dot);
      }
      size_t oo = ((size_t)i * n + t) * inner + hh * dh;
      if (mx == -INFINITY) continue; /* out stays zero */
      double sum = 0;
      for (int jj = 0; jj < cnt; jj++) {
        pr[jj] = pr[jj] == -INFINITY ? 0 : exp(pr[jj] - mx);
        sum += pr[jj];
      }
      for (int e = 0; e < dh; e++) {
        double acc = 0;
        for (int jj = 0; jj < cnt; jj++)
          if (pr[jj] != 0) acc += pr[jj] * c->qkv[((size_t)mem[jj] * n + t) * 3 * inner + 2 * inner + hh * dh + e];
        c->out[oo + e] = (float)(acc / sum);
      }
    }
  }
  free(mem);
  free(pr);
}

static void c2_rope(const float* src, float* dst, const float* inv_freq, int dh, int pos) {
  int half = dh / 2;
  for (int e = 0; e < half; e++) {
    float f = (float)pos * inv_freq[e];
    float cs = (float)cos((double)f), sn = (float)sin((double)f);
    float a = src[e], b = src[half + e];
    dst[e] = a * cs + -b * sn;
    dst[half + e] = b * cs + a * sn;
  }
}

void jco_chronos2_inv_freq(const jco_chronos2* m, float* f) {
  int dh = m->d_kv;
  for (int i = 0; i < dh / 2; i++) {
    float e = (float)(2 * i) / (float)dh;
    f[i] = 1.0f / (float)pow((double)m->rope_theta, (double)e);
  }
}

static float* c2_qkv_weight(const jco_chronos2* m, const float* q, const float* k, const float* v) {
  size_t part = (size_t)m->num_heads * m->d_kv * m->d_model;
  float* w = (float*)malloc(sizeof(float) * 3 * part);
  memcpy(w, q, sizeof(float) * part);
  memcpy(w + part, k, sizeof(float) * part);
  memcpy(w + 2 * part, v, sizeof(float) * part);
  return w;
}

void jco_chronos2_model(const jco_chronos2* m, const jco_c2_prepared* p, float* raw, int threads) {
  const int r = p->rows, d = m->d_model, ps = m->patch_size, nc = p->nc, h = p->h, n = p->n, ne = nc + h;
  const int fs = nc + p->reg, inner = m->num_heads * m->d_kv, heads = m->num_heads, dh = m->d_kv, ff = m->d_ff;
  const size_t tokens = (size_t)r * n;
  float* embed = c2_residual(p->tokens, r * ne, 3 * ps, ff, d, m->in_hw, m->in_hb, m->in_ow, m->in_ob, m->in_rw,
                             m->in_rb, threads);
  float* x = (float*)calloc(tokens * d, sizeof(float));
  for (int i = 0; i < r; i++) {
    memcpy(x + (size_t)i * n * d, embed + (size_t)i * ne * d, sizeof(float) * nc * d);
    if (p->reg) memcpy(x + ((size_t)i * n + nc) * d, m->shared + d, sizeof(float) * d);
    memcpy(x + ((size_t)i * n + fs) * d, embed + ((size_t)i * ne + nc) * d, sizeof(float) * h * d);
  }
  free(embed);
  float* inv_freq = (float*)malloc(sizeof(float) * (dh / 2));
  jco_chronos2_inv_freq(m, inv_freq);
  float* hn = (float*)malloc(sizeof(float) * tokens * d);
  float* qkv = (float*)malloc(sizeof(float) * tokens * 3 * inner);
  float* att = (float*)malloc(sizeof(float) * tokens * inner);
  float* qr = (float*)malloc(sizeof(float) * tokens * inner);
  float* kr = (float*)malloc(sizeof(float) * tokens * inner);
  float* y = (float*)malloc(sizeof(float) * tokens * d);
  float* act = (float*)malloc(sizeof(float) * tokens * ff);
  for (int li = 0; li < m->num_layers; li++) {
    /* time attention */
    jco_rmsnorm(x, (int)tokens, d, m->time_norm[li], m->eps, hn);
    float* w = c2_qkv_weight(m, m->time_q[li], m->time_k[li], m->time_v[li]);
    jco_linear(hn, (int)tokens, w, NULL, d, 3 * inner, qkv, threads);
    free(w);
    for (int i = 0; i < r; i++)
      for (int t = 0; t < n; t++) {
        size_t o = ((size_t)i * n + t) * 3 * inner;
        for (int hh = 0; hh < heads; hh++) {
          c2_rope(qkv + o + hh * dh, qr + ((size_t)i * n + t) * inner + hh * dh, inv_freq, dh, t);
          c2_rope(qkv + o + inner + hh * dh, kr + ((size_t)i * n + t) * inner + hh * dh, inv_freq, dh, t);
        }
      }
    c2_attn c = {m, p, qkv, qr, kr, att};
    c2_parallel_for(r * heads, threads, c2_time_job, &c);
    jco_linear(att, (int)tokens, m->time_o[li], NULL, inner, d, y, threads);
    for (size_t i = 0; i < tokens * d; i++) x[i] += y[i];
    /* group attention */
    jco_rmsnorm(x, (int)tokens, d, m->group_norm[li], m->eps, hn);
    w = c2_qkv_weight(m, m->group_q[li], m->group_k[li], m->group_v[li]);
    jco_linear(hn, (int)tokens, w, NULL, d, 3 * inner, qkv, threads);
    free(w);
    memset(att, 0, sizeof(float) * tokens * inner);
    c2_parallel_for(n, threads, c2_group_job, &c);
    jco_linear(att, (int)tokens, m->group_o[li], NULL, inner, d, y, threads);
    for (size_t i = 0; i < tokens * d; i++) x[i] += y[i];
    /* feed-forward */
    jco_rmsnorm(x, (int)tokens, d, m->mlp_norm[li], m->eps, hn);
    jco_linear(hn, (int)tokens, m->wi[li], NULL, d, ff, act, threads);
    for (size_t i = 0; i < tokens * ff; i++) act[i] = act[i] > 0.0f ? act[i] : 0.0f;
    jco_linear(act, (int)tokens, m->wo[li], NULL, ff, d, y, threads);
    for (size_t i = 0; i < tokens * d; i++) x[i] += y[i];
  }
  jco_rmsnorm(x, (int)tokens, d, m->final_norm, m->eps, y);
  float* dec = (float*)malloc(sizeof(float) * (size_t)r * h * d);
  for (int i = 0; i < r; i++) memcpy(dec + (size_t)i * h * d, y + ((size_t)i * n + fs) * d, sizeof(float) * h * d);
  float* out = c2_residual(dec, r * h, d, ff, m->num_quantiles * ps, m->out_hw, m->out_hb, m->out_ow, m->out_ob,
                           m->out_rw, m->out_rb, threads);
  memcpy(raw, out, sizeof(float) * (size_t)r * h * m->num_quantiles * ps);
  free(out);
  free(dec);
  free(inv_freq);
  free(hn);
  free(qkv);
  free(att);
  free(qr);
  free(kr);
  free(y);
  free(act);
  free(x);
}

int jco_chronos2_forward(const jco_chronos2* m, const jco_c2_input* in, float* out, float* raw_out, int threads) {
  jco_c2_prepared p;
  memset(&p, 0, sizeof p);
  int st = jco_chronos2_prepare(m, in, &p);
  if (st) return st;
  size_t nraw = (size_t)p.rows * p.h * m->num_quantiles * m->patch_size;
  float* raw = (float*)malloc(sizeof(float) * nraw);
  jco_chronos2_model(m, &p, raw, threads);
  if (raw_out) memcpy(raw_out, raw, sizeof(float) * nraw);
  jco_chronos2_finish(m, &p, raw, out);
  free(raw);
  jco_c2_prepared_free(&p);
  return 0;
}
