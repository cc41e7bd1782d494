/*
 * ORACLE — test infrastructure only. A C restatement of the reference's FP32 CPU forward of the
 * Timestral family, the checker for the B200 path (never linked into it).
 *
 * Restates, in src/main/java/ai/beestream/jitcast/timestral/:
 *   BlockLayout.of / position / timeAllowed / variateAllowed   BlockLayout.java:77-243
 *   BlockPrep.of / finish                                       BlockPrep.java:40-101
 *   Scaler.causalPatchLocScale / instanceNorm / affine / asinh / invert / clampNonFinite
 *                                                               Scaler.java:36-148
 *   Quantiles (monotone head)                                   Quantiles.java:28-77
 *   CpuTimestral.predictBlock, inverseFrequencies, rope, timeAttention, variateAttention
 *                                                               cpu/CpuTimestral.java:87-314
 *   TimestralWeights.qkv (heads-major rows) and mlpUp (halves swapped)
 *                                                               TimestralWeights.java:150-176
 * with double reductions where the reference uses them. Compiled with -ffp-contract=off.
 */
#include <float.h>
#include <math.h>
#include <pthread.h>
#include <stdatomic.h>
#include <stdlib.h>
#include <string.h>

#include "oracle.h"
#include "oracle_timestral.h"

/* ---- a small parallel-for ------------------------------------------------------------------ */
typedef void (*range_fn)(void* ctx, int i);
typedef struct {
  range_fn fn;
  void* ctx;
  int n;
  atomic_int next;
} pf_job;

static void* pf_worker(void* arg) {
  pf_job* j = (pf_job*)arg;
  for (;;) {
    int i = atomic_fetch_add(&j->next, 1);
    if (i >= j->n) break;
    j->fn(j->ctx, i);
  }
  return NULL;
}

static void parallel_for(int n, int threads, range_fn fn, void* ctx) {
  pf_job job = {fn, ctx, n, 0};
  if (threads > n) threads = n;
  if (threads > 256) threads = 256;
  pthread_t tid[256];
  int started = 0;
  for (int t = 1; t < threads; t++)
    if (pthread_create(&tid[started], NULL, pf_worker, &job) == 0) started++;
  pf_worker(&job);
  for (int t = 0; t < started; t++) pthread_join(tid[t], NULL);
}

/* ---- Scaler -------------------------------------------------------------------------------- */
static const float FLOAT32_EPS = 1.1920928955078125e-07f; /* Math.ulp(1.0f) */

static void causal_patch_loc_scale(const float* x, const unsigned char* obs, int t, int patch, float min_scale,
                                   float* loc, float* scale) {
  double cumW = 0, cumX = 0, m2 = 0, prevMean = 0;
  for (int i = 0; i < t; i++) {
    double w = obs[i] ? 1.0 : 0.0;
    double xi = x[i];
    cumW += w;
    cumX += w * xi;
    double mean = cumX / fmax(cumW, 1.0);
    m2 += (xi - prevMean) * (xi - mean) * w;
    prevMean = mean;
    if (i % patch == patch - 1) {
      double var = m2 / fmax(fmax(cumW, 1.0) - 1.0, 1.0);
      float l = (float)mean;
      float s = (float)fmax(sqrt(var), (double)min_scale);
      for (int j = i - patch + 1; j <= i; j++) {
        loc[j] = l;
        scale[j] = s;
      }
    }
  }
}

static float jasinh(float v) {
  double a = fabs((double)v);
  double r = log(a + sqrt(a * a + 1.0));
  return (float)(v < 0 ? -r : r);
}

static float affine(float x, float loc, float scale, int observed, int use_asinh) {
  if (!observed) return 0.0f;
  float v = (x - loc) / fmaxf(scale, FLOAT32_EPS);
  return use_asinh ? jasinh(v) : v;
}

/* {loc, scale, binary} */
static void instance_norm(const float* x, const unsigned char* obs, int len, float min_scale, float out[3]) {
  double n = 0, sum = 0;
  int zeroOne = 1, any = 0;
  for (int i = 0; i < len; i++) {
    if (obs[i]) {
      n += 1;
      sum += x[i];
      any = 1;
    }
    zeroOne &= x[i] == 0.0f || x[i] == 1.0f || !obs[i];
  }
  n = fmax(n, 1);
  float loc = (float)(sum / n);
  double ss = 0;
  for (int i = 0; i < len; i++) {
    float d = obs[i] ? x[i] - loc : 0.0f;
    ss += (double)d * d;
  }
  float scale = fmaxf((float)sqrt((float)(ss / n)), min_scale);
  if (zeroOne && any) {
    out[0] = 0.0f;
    out[1] = 1.0f;
    out[2] = 1.0f;
  } else {
    out[0] = loc;
    out[1] = scale;
    out[2] = 0.0f;
  }
}

static float invert(float x, float loc, float scale, int use_asinh) {
  float v = use_asinh ? (float)sinh((double)x) : x;
  return v * scale + loc;
}

static void clamp_nonfinite(float* v, int n) {
  float mx = -INFINITY, mn = INFINITY;
  for (int i = 0; i < n; i++)
    if (isfinite(v[i])) {
      mx = fmaxf(mx, v[i]);
      mn = fminf(mn, v[i]);
    }
  for (int i = 0; i < n; i++) {
    float x = v[i] == INFINITY ? mx : v[i] == -INFINITY ? mn : v[i];
    v[i] = isinf(x) ? 0.0f : x;
  }
}

/* ---- Quantiles ------------------------------------------------------------------------------ */
static float softplus(float x) { return x > 20.0f ? x : (float)log1p(exp((double)x)); }

static float clampf_max(float v) { return fmaxf(-FLT_MAX, fminf(FLT_MAX, v)); }

static int median_index(const jco_timestral* m) {
  for (int i = 0; i < m->num_quantiles; i++)
    if (m->quantile_knots[i] == 0.5) return i;
  return -1;
}

static void quantile_scales(const jco_timestral* m, float* scale) {
  int med = median_index(m);
  for (int i = 0; i < m->num_quantiles; i++) {
    const double* L = m->quantile_knots;
    double width = i > med ? L[i] - L[i - 1] : i < med ? L[i + 1] - L[i] : 0.0;
    scale[i] = (float)width;
  }
  for (int i = 0; i < m->num_quantiles; i++) scale[i] = m->quantile_width_factor * scale[i];
}

static void quantiles_apply(const float* scale, int q, int med, float* raw) {
  float mval = raw[med];
  float up = 0;
  for (int i = med + 1; i < q; i++) {
    up += scale[i] * softplus(raw[i]);
    raw[i] = clampf_max(mval + up);
  }
  float down = 0;
  for (int i = med - 1; i >= 0; i--) {
    down += scale[i] * softplus(raw[i]);
    raw[i] = clampf_max(mval - down);
  }
  raw[med] = clampf_max(mval);
}

/* ---- BlockLayout + BlockPrep ------------------------------------------------------------------ */
int jco_timestral_prepare(const jco_timestral* m, const jco_block* b, jco_prepared* p) {
  const int ps = m->patch_size, r = b->rows, t = b->length, h = b->horizon;
  if (t % ps != 0 || h < 1) return -1;
  int cov = 0;
  if (b->role && m->covariate_enabled)
    for (int i = 0; i < r; i++) cov |= b->role[i] != JCO_TARGET;
  if (cov && h > m->block_size) return -2;
  const int ll = t / ps;
  const int wlen = cov ? t + h * ps : t;
  const int enc = wlen / ps;
  p->rows = r;
  p->enc = enc;
  p->horizon = h;
  p->ll = ll;
  p->covariates = cov;
  p->window = (float*)calloc((size_t)r * wlen, sizeof(float));
  p->obs = (unsigned char*)calloc((size_t)r * wlen, 1);
  for (int i = 0; i < r; i++) {
    memcpy(p->window + (size_t)i * wlen, b->inputs + (size_t)i * t, sizeof(float) * t);
    memcpy(p->obs + (size_t)i * wlen, b->observed + (size_t)i * t, t);
    if (cov && b->known_future) {
      memcpy(p->window + (size_t)i * wlen + t, b->known_future + (size_t)i * h * ps, sizeof(float) * h * ps);
      memcpy(p->obs + (size_t)i * wlen + t, b->known_future_mask + (size_t)i * h * ps, h * ps);
    }
  }
  p->key_valid = (int*)calloc((size_t)r * enc, sizeof(int));
  unsigned char* pobs = (unsigned char*)calloc((size_t)r * enc, 1);
  for (int i = 0; i < r; i++) {
    int started = 0;
    for (int q = 0; q < enc; q++) {
      int any = 0;
      for (int s = q * ps; s < (q + 1) * ps; s++) any |= p->obs[(size_t)i * wlen + s];
      pobs[(size_t)i * enc + q] = (unsigned char)any;
      started |= any;
      p->key_valid[(size_t)i * enc + q] = m->attend_missing_patches ? started : any;
    }
  }
  /* the first patch any row of the series observes (0 if none does) */
  int* first_row = (int*)malloc(sizeof(int) * r);
  for (int i = 0; i < r; i++) {
    int f = enc;
    for (int q = 0; q < enc; q++)
      if (pobs[(size_t)i * enc + q]) {
        f = q;
        break;
      }
    first_row[i] = f;
  }
  p->first = (int*)malloc(sizeof(int) * r);
  for (int i = 0; i < r; i++) {
    int f = enc;
    for (int j = 0; j < r; j++)
      if (b->group[j] == b->group[i] && first_row[j] < f) f = first_row[j];
    p->first[i] = f == enc ? 0 : f;
  }
  free(first_row);
  free(pobs);
  p->role = (int*)calloc(r, sizeof(int));
  p->known = (int*)calloc(r, sizeof(int));
  p->group = (int*)malloc(sizeof(int) * r);
  for (int i = 0; i < r; i++) {
    p->group[i] = b->group[i];
    if (cov) p->role[i] = b->role[i];
    p->known[i] = cov && p->role[i] == JCO_KNOWN;
  }
  const int n = enc + h;
  p->pos = (int*)malloc(sizeof(int) * (size_t)r * n);
  for (int i = 0; i < r; i++)
    for (int tok = 0; tok < n; tok++) {
      int q = tok < enc ? tok : ll + tok - enc;
      p->pos[(size_t)i * n + tok] = q - p->first[i];
    }
  /* BlockPrep.of */
  p->loc = (float*)malloc(sizeof(float) * (size_t)r * wlen);
  p->scale = (float*)malloc(sizeof(float) * (size_t)r * wlen);
  p->tokens = (float*)malloc(sizeof(float) * (size_t)r * enc * 2 * ps);
  float* scaled = (float*)malloc(sizeof(float) * (size_t)r * wlen);
  float* l = (float*)malloc(sizeof(float) * wlen);
  float* s = (float*)malloc(sizeof(float) * wlen);
  for (int i = 0; i < r; i++) {
    const float* win = p->window + (size_t)i * wlen;
    const unsigned char* ob = p->obs + (size_t)i * wlen;
    causal_patch_loc_scale(win, ob, wlen, ps, m->minimum_scale, l, s);
    float inst[3] = {0, 0, 0};
    if (p->known[i]) instance_norm(win, ob, wlen, m->minimum_scale, inst);
    for (int tt = 0; tt < wlen; tt++) {
      size_t o = (size_t)i * wlen + tt;
      if (p->known[i]) {
        p->loc[o] = inst[0];
        p->scale[o] = inst[1];
        scaled[o] = affine(win[tt], inst[0], inst[1], ob[tt], m->use_asinh && inst[2] == 0.0f);
      } else {
        p->loc[o] = l[tt];
        p->scale[o] = s[tt];
        scaled[o] = affine(win[tt], l[tt], s[tt], ob[tt], m->use_asinh);
      }
    }
    for (int q = 0; q < enc; q++) {
      float* tok = p->tokens + ((size_t)i * enc + q) * 2 * ps;
      for (int st = 0; st < ps; st++) {
        int tt = q * ps + st;
        tok[st] = scaled[(size_t)i * wlen + tt];
        tok[ps + st] = ob[tt] ? 0.0f : 1.0f;
      }
    }
  }
  free(l);
  free(s);
  free(scaled);
  return 0;
}

void jco_prepared_free(jco_prepared* p) {
  free(p->window);
  free(p->obs);
  free(p->key_valid);
  free(p->first);
  free(p->role);
  free(p->known);
  free(p->group);
  free(p->pos);
  free(p->loc);
  free(p->scale);
  free(p->tokens);
  memset(p, 0, sizeof *p);
}

void jco_timestral_finish(const jco_timestral* m, const jco_prepared* p, float* raw, float* out) {
  const int r = p->rows, ps = m->patch_size, q = m->num_quantiles, h = p->horizon;
  const int w = p->enc * ps, ll = p->ll, med = median_index(m);
  float* sc = (float*)malloc(sizeof(float) * q);
  quantile_scales(m, sc);
  for (int i = 0; i < r; i++) {
    for (int v = i * h * ps; v < (i + 1) * h * ps; v++) quantiles_apply(sc, q, med, raw + (size_t)v * q);
    size_t anchor = (size_t)i * w + (size_t)(ll - 1) * ps;
    for (int t = 0; t < h * ps; t++) {
      float* o = out + ((size_t)i * h * ps + t) * q;
      for (int k = 0; k < q; k++)
        o[k] = invert(raw[((size_t)i * h * ps + t) * q + k], p->loc[anchor], p->scale[anchor], m->use_asinh);
      clamp_nonfinite(o, q);
    }
  }
  free(sc);
}

/* ---- the transformer ---------------------------------------------------------------------------- */
static int time_allowed(const jco_prepared* p, int row, int q, int k) {
  const int enc = p->enc;
  if (q < enc) {
    if (k >= enc) return 0;
    return k == q || (p->key_valid[(size_t)row * enc + k] && (k <= q || p->known[row]));
  }
  if (k < enc) return k < p->ll && p->key_valid[(size_t)row * enc + k];
  return k <= q;
}

static int variate_allowed(const jco_prepared* p, int slot, int q, int k) {
  if (p->group[q] != p->group[k]) return 0;
  if (q == k) return 1;
  if (slot < p->enc && !p->key_valid[(size_t)k * p->enc + slot]) return 0;
  if (p->covariates) {
    if (p->role[q] != JCO_TARGET && p->role[k] == JCO_TARGET) return 0;
    if (p->role[q] == JCO_KNOWN && p->role[k] != JCO_KNOWN) return 0;
  }
  return 1;
}

static int head_dim(const jco_timestral* m) { return m->d_model / m->num_heads; }
static int rope_dim(const jco_timestral* m) { return (int)(head_dim(m) * m->rope_partial_factor); }

void jco_timestral_inv_freq(const jco_timestral* m, float* f) {
  int dh = head_dim(m), rot = rope_dim(m);
  for (int i = 0; i < dh / 2; i++) f[i] = 0.0f;
  for (int i = 0; i < rot / 2; i++) {
    float e = (float)(2 * i) / (float)rot;
    f[i] = 1.0f / (float)pow((double)m->rope_theta, (double)e);
  }
}

typedef struct {
  const jco_timestral* m;
  const jco_prepared* p;
  const float* qkv;
  const float* q;
  const float* k;
  float* out;
  int n;
} attn_ctx;

static void time_attention_job(void* vctx, int job) {
  attn_ctx* c = (attn_ctx*)vctx;
  const int heads = c->m->num_heads, d = c->m->d_model, dh = head_dim(c->m), n = c->n;
  const int i = job / heads, hh = job % heads;
  const double scale = 1.0 / sqrt((double)dh);
  double* pr = (double*)malloc(sizeof(double) * n);
  for (int t = 0; t < n; t++) {
    double mx = -INFINITY;
    size_t qo = ((size_t)i * n + t) * d + hh * dh;
    for (int s = 0; s < n; s++) {
      if (!time_allowed(c->p, i, t, s)) {
        pr[s] = -INFINITY;
        continue;
      }
      size_t ko = ((size_t)i * n + s) * d + hh * dh;
      double dot = 0;
      for (int e = 0; e < dh; e++) dot += (double)c->q[qo + e] * c->k[ko + e];
      pr[s] = dot * scale;
      mx = fmax(mx, pr[s]);
    }
    double sum = 0;
    for (int s = 0; s < n; s++) {
      pr[s] = pr[s] == -INFINITY ? 0 : exp(pr[s] - mx);
      sum += pr[s];
    }
    for (int e = 0; e < dh; e++) {
      double acc = 0;
      for (int s = 0; s < n; s++)
        if (pr[s] != 0) acc += pr[s] * c->qkv[((size_t)i * n + s) * 3 * d + 2 * d + hh * dh + e];
      c->out[qo + e] = (float)(acc / sum);
    }
  }
  free(pr);
}

static void rope_vec(const float* src, float* dst, const float* inv_freq, int dh, int pos) {
  int half = dh / 2;
  for (int e = 0; e < half; e++) {
    float f = (float)pos * inv_freq[e];
    float cs = (float)cos((double)f), sn = (float)sin((double)f);
    float a = src[e], b = src[half + e];
    dst[e] = a * cs + -b * sn;
    dst[half + e] = b * cs + a * sn;
  }
}

static void variate_attention_job(void* vctx, int t) {
  attn_ctx* c = (attn_ctx*)vctx;
  const jco_prepared* p = c->p;
  const int r = p->rows, heads = c->m->num_heads, d = c->m->d_model, dh = head_dim(c->m), n = c->n;
  const double scale = 1.0 / sqrt((double)dh);
  int* mem = (int*)malloc(sizeof(int) * r);
  double* pr = (double*)malloc(sizeof(double) * r);
  for (int i = 0; i < r; i++) {
    int cnt = 0;
    for (int j = 0; j < r; j++)
      if (p->group[j] == p->group[i]) mem[cnt++] = j;
    for (int hh = 0; hh < heads; hh++) {
      size_t qo = ((size_t)i * n + t) * 3 * d + hh * dh;
      double mx = -INFINITY;
      for (int jj = 0; jj < cnt; jj++) {
        int j = mem[jj];
        if (!variate_allowed(p, t, i, j)) {
          pr[jj] = -INFINITY;
          continue;
        }
        size_t ko = ((size_t)j * n + t) * 3 * d + d + hh * dh;
        double dot = 0;
        for (int e = 0; e < dh; e++) dot += (double)c->qkv[qo + e] * c->qkv[ko + e];
        pr[jj] = dot * scale;
        mx = fmax(mx, pr[jj]);
      }
      double sum = 0;
      for (int jj = 0; jj < cnt; jj++) {
        pr[jj] = pr[jj] == -INFINITY ? 0 : exp(pr[jj] - mx);
        sum += pr[jj];
      }
      for (int e = 0; e < dh; e++) {
        double acc = 0;
        for (int jj = 0; jj < cnt; jj++)
          if (pr[jj] != 0) acc += pr[jj] * c->qkv[((size_t)mem[jj] * n + t) * 3 * d + 2 * d + hh * dh + e];
        c->out[((size_t)i * n + t) * d + hh * dh + e] = (float)(acc / sum);
      }
    }
  }
  free(mem);
  free(pr);
}

/* TimestralWeights.qkv: row (s·heads + h)·dh + e ← stored row s·D + e·heads + h. */
static float* qkv_heads_major(const jco_timestral* m, const float* src) {
  int d = m->d_model, heads = m->num_heads, dh = head_dim(m);
  float* dst = (float*)malloc(sizeof(float) * 3 * (size_t)d * d);
  for (int s = 0; s < 3; s++)
    for (int h = 0; h < heads; h++)
      for (int e = 0; e < dh; e++)
        memcpy(dst + ((size_t)s * d + h * dh + e) * d, src + ((size_t)s * d + e * heads + h) * d, sizeof(float) * d);
  return dst;
}

/* output(SiLU(hidden(x))) + residual(x) */
static float* residual_block(const float* x, int rows, int in, int hidden, int out, const float* hw, const float* hb,
                             const float* ow, const float* ob, const float* rw, const float* rb, int threads) {
  float* hdn = (float*)malloc(sizeof(float) * (size_t)rows * hidden);
  jco_linear(x, rows, hw, hb, in, hidden, hdn, threads);
  for (size_t i = 0; i < (size_t)rows * hidden; i++) hdn[i] = jco_silu(hdn[i]);
  float* y = (float*)malloc(sizeof(float) * (size_t)rows * out);
  jco_linear(hdn, rows, ow, ob, hidden, out, y, threads);
  free(hdn);
  float* res = (float*)malloc(sizeof(float) * (size_t)rows * out);
  jco_linear(x, rows, rw, rb, in, out, res, threads);
  for (size_t i = 0; i < (size_t)rows * out; i++) y[i] += res[i];
  free(res);
  return y;
}

void jco_timestral_model(const jco_timestral* m, const jco_prepared* p, float* raw, int threads) {
  const int r = p->rows, d = m->d_model, ps = m->patch_size, enc = p->enc, h = p->horizon, n = enc + h;
  const int f = m->mlp_hidden_dim, heads = m->num_heads, dh = head_dim(m), q = m->num_quantiles;
  const size_t tokens = (size_t)r * n;
  float* embed = residual_block(p->tokens, r * enc, 2 * ps, 4 * d, d, m->emb_hidden_w, m->emb_hidden_b,
                                m->emb_output_w, m->emb_output_b, m->emb_residual_w, m->emb_residual_b, threads);
  float* x = (float*)malloc(sizeof(float) * tokens * d);
  for (int i = 0; i < r; i++) {
    memcpy(x + (size_t)i * n * d, embed + (size_t)i * enc * d, sizeof(float) * enc * d);
    for (int t = enc; t < n; t++) memcpy(x + ((size_t)i * n + t) * d, m->forecast_query, sizeof(float) * d);
  }
  free(embed);
  float* inv_freq = (float*)malloc(sizeof(float) * (dh / 2));
  jco_timestral_inv_freq(m, inv_freq);
  float* hn = (float*)malloc(sizeof(float) * tokens * d);
  float* qkv = (float*)malloc(sizeof(float) * tokens * 3 * d);
  float* att = (float*)malloc(sizeof(float) * tokens * d);
  float* g = (float*)malloc(sizeof(float) * tokens * d);
  float* y = (float*)malloc(sizeof(float) * tokens * d);
  float* qr = (float*)malloc(sizeof(float) * tokens * d);
  float* kr = (float*)malloc(sizeof(float) * tokens * d);
  float* up = (float*)malloc(sizeof(float) * tokens * 2 * f);
  float* act = (float*)malloc(sizeof(float) * tokens * f);
  int a_idx = 0;
  for (int li = 0; li < m->num_layers; li++) {
    for (int ai = 0; ai < m->attn_per_layer[li]; ai++, a_idx++) {
      const int is_time = m->attn_is_time[a_idx];
      jco_rmsnorm(x, (int)tokens, d, m->attn_norm[a_idx], m->norm_eps, hn);
      float* wq = qkv_heads_major(m, m->wqkv[a_idx]);
      jco_linear(hn, (int)tokens, wq, NULL, d, 3 * d, qkv, threads);
      free(wq);
      attn_ctx c = {m, p, qkv, NULL, NULL, att, n};
      if (is_time) {
        for (int i = 0; i < r; i++)
          for (int t = 0; t < n; t++) {
            int pos = p->pos[(size_t)i * n + t];
            size_t o = ((size_t)i * n + t) * 3 * d;
            for (int hh = 0; hh < heads; hh++) {
              rope_vec(qkv + o + hh * dh, qr + ((size_t)i * n + t) * d + hh * dh, inv_freq, dh, pos);
              rope_vec(qkv + o + d + hh * dh, kr + ((size_t)i * n + t) * d + hh * dh, inv_freq, dh, pos);
            }
          }
        c.q = qr;
        c.k = kr;
        parallel_for(r * heads, threads, time_attention_job, &c);
      } else {
        parallel_for(n, threads, variate_attention_job, &c);
      }
      if (m->attn_gate[a_idx]) {
        jco_linear(hn, (int)tokens, m->gate_w[a_idx], NULL, d, d, g, threads);
        for (size_t i = 0; i < tokens * d; i++) att[i] = att[i] * (float)jco_sigmoid(g[i]);
      }
      jco_linear(att, (int)tokens, m->wo[a_idx], NULL, d, d, y, threads);
      for (size_t i = 0; i < tokens * d; i++) x[i] += y[i];
    }
    jco_rmsnorm(x, (int)tokens, d, m->mlp_norm[li], m->norm_eps, hn);
    /* mlpUp: the SiLU half (stored second) first */
    float* wu = (float*)malloc(sizeof(float) * 2 * (size_t)f * d);
    memcpy(wu, m->w12[li] + (size_t)f * d, sizeof(float) * (size_t)f * d);
    memcpy(wu + (size_t)f * d, m->w12[li], sizeof(float) * (size_t)f * d);
    jco_linear(hn, (int)tokens, wu, NULL, d, 2 * f, up, threads);
    free(wu);
    for (size_t t = 0; t < tokens; t++)
      for (int j = 0; j < f; j++) act[t * f + j] = jco_silu(up[t * 2 * f + j]) * up[t * 2 * f + f + j];
    jco_linear(act, (int)tokens, m->w3[li], NULL, f, d, y, threads);
    for (size_t i = 0; i < tokens * d; i++) x[i] += y[i];
  }
  jco_rmsnorm(x, (int)tokens, d, m->out_norm, m->norm_eps, y);
  float* dec = (float*)malloc(sizeof(float) * (size_t)r * h * d);
  for (int i = 0; i < r; i++) memcpy(dec + (size_t)i * h * d, y + ((size_t)i * n + enc) * d, sizeof(float) * h * d);
  float* out = residual_block(dec, r * h, d, 4 * d, ps * q, m->head_hidden_w, NULL, m->head_output_w, NULL,
                              m->head_residual_w, NULL, threads);
  memcpy(raw, out, sizeof(float) * (size_t)r * h * ps * q);
  free(out);
  free(dec);
  free(inv_freq);
  free(hn);
  free(qkv);
  free(att);
  free(g);
  free(y);
  free(qr);
  free(kr);
  free(up);
  free(act);
  free(x);
}

int jco_timestral_predict_block(const jco_timestral* m, const jco_block* b, float* out, float* raw_out,
                                int threads) {
  jco_prepared p;
  memset(&p, 0, sizeof p);
  int st = jco_timestral_prepare(m, b, &p);
  if (st) return st;
  size_t nraw = (size_t)p.rows * p.horizon * m->patch_size * m->num_quantiles;
  float* raw = (float*)malloc(sizeof(float) * nraw);
  jco_timestral_model(m, &p, raw, threads);
  if (raw_out) memcpy(raw_out, raw, sizeof(float) * nraw);
  jco_timestral_finish(m, &p, raw, out);
  free(raw);
  jco_prepared_free(&p);
  return 0;
}
