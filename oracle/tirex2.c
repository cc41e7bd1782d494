/*
 * ORACLE — test infrastructure only (see ops.c). A plain-C restatement of the reference's FP32
 * TiRex-2 CPU forward, the checker for jc_forward_tirex2. Paths are in the jitCast tree,
 * src/main/java/ai/beestream/jitcast/tirex2/:
 *
 *   forward              cpu/CpuReference.java:67-90     input stage, blocks, out norm, output embedding, unpatch
 *   knownCovariates      cpu/CpuReference.java:92-108    covariate rows observed in the last future_len steps
 *   timeMixer            cpu/CpuReference.java:110-145   RMSNorm, cell, reverse pass + combination, SwiGLU FFN
 *   variateMixer         cpu/CpuReference.java:156-236   attention across a group's rows per patch, SiLU MLP
 *   unpatch              cpu/CpuReference.java:238-266   sinh(clamp(y, ±20))·scale + loc
 *   InputStage.apply     cpu/InputStage.java:37-93       scaler (nanmean / nanstd, binary-aware), arcsinh, patches
 *   Cells.mlstm          cpu/Cells.java:44-72            fused q|k|v|o|i|f projection, core, head norm, σ(o), out_proj
 *   Cells.mlstmCore      cpu/Cells.java:74-118           stabilised parallel mLSTM
 *   Cells.slstm          cpu/Cells.java:135-141          headwise gates, recurrence, head norm
 *   Cells.headwiseGates  cpu/Cells.java:143-168
 *   Cells.slstmRecurrence cpu/Cells.java:170-218
 *   TiRexOps             cpu/TiRexOps.java:30-82         headLayerNorm, logSigmoid, softCap, residualBlock, swiGlu
 *
 * Arithmetic follows the Java statement by statement: float where Java computes in float, double
 * where it widens (Java does not contract a*b+c, so this file is built with -ffp-contract=off).
 */
#include <math.h>
#include <stdlib.h>
#include <string.h>

#include "oracle.h"
#include "oracle_tirex2.h"

#define NORM_EPS 1e-6f
#define MLSTM_EPS 1e-6f
#define GATE_SOFT_CAP 15.0f
#define SCALER_EPS 1e-8f
#define SINH_CLAMP 20.0f
#define FLOAT32_EPS 1.1920928955078125e-07f /* Math.ulp(1.0f) */

static float* fa(size_t n) { return (float*)calloc(n ? n : 1, sizeof(float)); }

static double log_sigmoid(double z) { return fmin(z, 0.0) - log1p(exp(-fabs(z))); }

static float soft_cap(float z, float cap) { return (float)((double)cap * tanh((double)(z / cap))); }

static void add_in_place(float* acc, const float* x, size_t n) {
  for (size_t i = 0; i < n; i++) acc[i] += x[i];
}

static void silu_in_place(float* x, size_t n) {
  for (size_t i = 0; i < n; i++) x[i] = jco_silu(x[i]);
}

/* TiRexOps.headLayerNorm (TiRexOps.java:30-52) */
static void head_layer_norm(const float* x, int rows, int heads, int hd, const float* w, float eps, float* y) {
  for (int r = 0; r < rows; r++)
    for (int h = 0; h < heads; h++) {
      size_t o = ((size_t)r * heads + h) * hd;
      double mean = 0;
      for (int i = 0; i < hd; i++) mean += x[o + i];
      mean /= hd;
      double var = 0;
      for (int i = 0; i < hd; i++) {
        double dv = x[o + i] - mean;
        var += dv * dv;
      }
      var /= hd;
      double inv = 1.0 / sqrt(var + (double)eps);
      for (int i = 0; i < hd; i++) y[o + i] = (float)((x[o + i] - mean) * inv) * w[h * hd + i];
    }
}

/* TiRexOps.residualBlock: output(SiLU(hidden(x))) + residual(x) */
static float* residual_block(const float* x, int rows, int in, int hid, int out, const float* hw, const float* hb,
                             const float* ow, const float* ob, const float* rw, const float* rb, int th) {
  float* h = fa((size_t)rows * hid);
  jco_linear(x, rows, hw, hb, in, hid, h, th);
  silu_in_place(h, (size_t)rows * hid);
  float* y = fa((size_t)rows * out);
  jco_linear(h, rows, ow, ob, hid, out, y, th);
  float* r = fa((size_t)rows * out);
  jco_linear(x, rows, rw, rb, in, out, r, th);
  add_in_place(y, r, (size_t)rows * out);
  free(h);
  free(r);
  return y;
}

/* TiRexOps.swiGlu: down(SiLU(upGate(x)) · up(x)) */
static float* swiglu(const float* x, int rows, int d, int ff, const float* ug, const float* u, const float* dn,
                     int th) {
  float* g = fa((size_t)rows * ff);
  float* v = fa((size_t)rows * ff);
  jco_linear(x, rows, ug, NULL, d, ff, g, th);
  jco_linear(x, rows, u, NULL, d, ff, v, th);
  for (size_t i = 0; i < (size_t)rows * ff; i++) g[i] = jco_silu(g[i]) * v[i];
  float* y = fa((size_t)rows * d);
  jco_linear(g, rows, dn, NULL, ff, d, y, th);
  free(g);
  free(v);
  return y;
}

void jco_tirex2_mlstm_core(const float* p, int rows, int seq, int heads, int stride, float* h) {
  const int dqk = 64, dv = 128;
  const int k_off = heads * dqk, v_off = 2 * heads * dqk, i_off = v_off + 2 * heads * dv, f_off = i_off + heads;
  const double scale = 1.0 / sqrt((double)dqk);
  double* cum_f = (double*)malloc(sizeof(double) * seq);
  double* in = (double*)malloc(sizeof(double) * seq);
  double num[128];
  for (int rh = 0; rh < rows * heads; rh++) {
    const int r = rh / heads, hd = rh % heads;
    double acc = 0;
    for (int t = 0; t < seq; t++) {
      size_t base = ((size_t)r * seq + t) * stride;
      acc += log_sigmoid(soft_cap(p[base + f_off + hd], GATE_SOFT_CAP));
      cum_f[t] = acc;
      in[t] = soft_cap(p[base + i_off + hd], GATE_SOFT_CAP);
    }
    for (int t = 0; t < seq; t++) {
      double m = cum_f[t];
      for (int s = 0; s <= t; s++) m = fmax(m, cum_f[t] - cum_f[s] + in[s]);
      size_t qo = ((size_t)r * seq + t) * stride + (size_t)hd * dqk;
      double den = 0;
      memset(num, 0, sizeof num);
      for (int s = 0; s <= t; s++) {
        size_t so = ((size_t)r * seq + s) * stride;
        double dot = 0;
        for (int j = 0; j < dqk; j++) dot += (double)p[qo + j] * p[so + k_off + (size_t)hd * dqk + j];
        double cts = dot * scale * exp(cum_f[t] - cum_f[s] + in[s] - m);
        den += cts;
        for (int j = 0; j < dv; j++) num[j] += cts * p[so + v_off + (size_t)hd * dv + j];
      }
      double norm = fmax(fabs(den), exp(-m)) + (double)MLSTM_EPS;
      size_t ho = ((size_t)r * seq + t) * heads * dv + (size_t)hd * dv;
      for (int j = 0; j < dv; j++) h[ho + j] = (float)(num[j] / norm);
    }
  }
  free(cum_f);
  free(in);
}

void jco_tirex2_slstm_recurrence(const float* wx, int rows, int seq, int d, int heads, const float* r,
                                 const float* b, float* out) {
  const int dh = d / heads;
  double* y = (double*)malloc(sizeof(double) * d);
  double* c = (double*)malloc(sizeof(double) * d);
  double* nn = (double*)malloc(sizeof(double) * d);
  double* m = (double*)malloc(sizeof(double) * d);
  double* raw = (double*)malloc(sizeof(double) * 4 * d);
  for (int row = 0; row < rows; row++) {
    for (int j = 0; j < d; j++) y[j] = c[j] = nn[j] = m[j] = 0;
    for (int t = 0; t < seq; t++) {
      size_t base = ((size_t)row * seq + t) * d;
      size_t wx_base = ((size_t)row * seq + t) * 4 * d;
      for (int h = 0; h < heads; h++) {
        for (int g = 0; g < 4; g++)
          for (int e = 0; e < dh; e++)
            raw[g * d + h * dh + e] = wx[wx_base + g * d + h * dh + e] + b[(h * 4 + g) * dh + e]; /* float add */
        for (int q = 0; q < dh; q++) {
          double yp = y[h * dh + q];
          if (yp == 0) continue;
          size_t ro = ((size_t)h * dh + q) * 4 * dh;
          for (int g = 0; g < 4; g++)
            for (int e = 0; e < dh; e++) raw[g * d + h * dh + e] += yp * r[ro + g * dh + e];
        }
      }
      for (int j = 0; j < d; j++) {
        double i_raw = raw[j], f_raw = raw[d + j], z_raw = raw[2 * d + j], o_raw = raw[3 * d + j];
        double logf = log_sigmoid(f_raw) + m[j];
        double m_new = t == 0 ? i_raw : fmax(i_raw, logf);
        double ig = exp(i_raw - m_new);
        double fg = exp(logf - m_new);
        c[j] = fg * c[j] + ig * tanh(z_raw);
        nn[j] = fmax(fg * nn[j] + ig, 1.0);
        y[j] = jco_sigmoid(o_raw) * c[j] / nn[j];
        m[j] = m_new;
        out[base + j] = (float)y[j];
      }
    }
  }
  free(y);
  free(c);
  free(nn);
  free(m);
  free(raw);
}

/* Cells.headwiseGates (Cells.java:143-168): wx[rt·4d + g·d + h·dh + o]. Under a reduced-precision operand
 * format (jco_set_operand_format) its operands are rounded like every other GEMM's. */
static void headwise_gates(const float* x, int n, int d, int heads, const float* const gates[4], float* wx) {
  const int dh = d / heads;
  const int fmt = jco_operand_format();
  float* xr = NULL;
  const float* gr[4] = {gates[0], gates[1], gates[2], gates[3]};
  float* gown[4] = {NULL, NULL, NULL, NULL};
  if (fmt != JCO_OPERANDS_FP32) {
    xr = fa((size_t)n * d);
    for (size_t i = 0; i < (size_t)n * d; i++) xr[i] = jco_round_operand(x[i], fmt);
    x = xr;
    for (int g = 0; g < 4; g++) {
      gown[g] = fa((size_t)d * dh);
      for (size_t i = 0; i < (size_t)d * dh; i++) gown[g][i] = jco_round_operand(gates[g][i], fmt);
      gr[g] = gown[g];
    }
    gates = gr;
  }
  for (int rt = 0; rt < n; rt++) {
    size_t xo = (size_t)rt * d;
    for (int g = 0; g < 4; g++)
      for (int h = 0; h < heads; h++)
        for (int o = 0; o < dh; o++) {
          size_t wo = ((size_t)h * dh + o) * dh;
          double acc = 0;
          for (int j = 0; j < dh; j++) acc += (double)x[xo + h * dh + j] * gates[g][wo + j];
          wx[(size_t)rt * 4 * d + g * d + h * dh + o] = (float)acc;
        }
  }
  free(xr);
  for (int g = 0; g < 4; g++) free(gown[g]);
}

/* Cells.mlstm / Cells.slstm on x [rows·seq·d]; returns [rows·seq·d]. */
static float* cell(const JcoTirex2* m, int blk, const float* x, int rows, int th) {
  const int seq = (m->context_len + m->future_len) / m->patch, d = m->d, n = rows * seq;
  float* out = fa((size_t)n * d);
  if (m->block_types[blk] == JCO_TIREX_MLSTM) {
    const int heads = m->tm_heads, qk = d / 2;
    const float* ws[6] = {m->mq[blk], m->mk[blk], m->mv[blk], m->mo[blk], m->ig_w[blk], m->fg_w[blk]};
    const float* bs[6] = {NULL, NULL, NULL, NULL, m->ig_b[blk], m->fg_b[blk]};
    const int outs[6] = {qk, qk, d, d, heads, heads};
    int stride = 0;
    for (int i = 0; i < 6; i++) stride += outs[i];
    float* p = fa((size_t)n * stride);
    int col = 0;
    for (int i = 0; i < 6; i++) {
      float* y = fa((size_t)n * outs[i]);
      jco_linear(x, n, ws[i], bs[i], d, outs[i], y, th);
      for (int t = 0; t < n; t++) memcpy(p + (size_t)t * stride + col, y + (size_t)t * outs[i], sizeof(float) * outs[i]);
      col += outs[i];
      free(y);
    }
    float* h = fa((size_t)n * heads * 128);
    jco_tirex2_mlstm_core(p, rows, seq, heads, stride, h);
    const int dv = d / heads;
    float* hn = fa((size_t)n * d);
    head_layer_norm(h, n, heads, dv, m->head_norm[blk], NORM_EPS, hn);
    const int o_off = 2 * qk + d;
    for (int t = 0; t < n; t++)
      for (int j = 0; j < d; j++)
        hn[(size_t)t * d + j] = (float)(jco_sigmoid(p[(size_t)t * stride + o_off + j]) * hn[(size_t)t * d + j]);
    jco_linear(hn, n, m->out_proj[blk], NULL, d, d, out, th);
    free(p);
    free(h);
    free(hn);
  } else {
    const int heads = m->slstm_heads;
    const float* gates[4] = {m->sg0[blk], m->sg1[blk], m->sg2[blk], m->sg3[blk]};
    float* wx = fa((size_t)n * 4 * d);
    headwise_gates(x, n, d, heads, gates, wx);
    float* y = fa((size_t)n * d);
    jco_tirex2_slstm_recurrence(wx, rows, seq, d, heads, m->srec[blk], m->sbias[blk], y);
    head_layer_norm(y, n, heads, d / heads, m->group_norm[blk], NORM_EPS, out);
    free(wx);
    free(y);
  }
  return out;
}

/* CpuReference.timeMixer (CpuReference.java:110-145); returns the new residual stream. */
static float* time_mixer(const JcoTirex2* m, int blk, const float* x, int rows, const int* known, int nk, int th) {
  const int seq = (m->context_len + m->future_len) / m->patch, d = m->d, n = rows * seq;
  float* xn = fa((size_t)n * d);
  jco_rmsnorm(x, n, d, m->norm_lstm[blk], NORM_EPS, xn);
  float* y = cell(m, blk, xn, rows, th);
  if (nk > 0) {
    float* rev = fa((size_t)nk * seq * d);
    for (int k = 0; k < nk; k++)
      for (int t = 0; t < seq; t++)
        memcpy(rev + ((size_t)k * seq + t) * d, xn + ((size_t)known[k] * seq + (seq - 1 - t)) * d, sizeof(float) * d);
    float* rev_out = cell(m, blk, rev, nk, th);
    float* cat = fa((size_t)nk * seq * 2 * d);
    for (int k = 0; k < nk; k++)
      for (int t = 0; t < seq; t++) {
        size_t dst = ((size_t)k * seq + t) * 2 * d;
        memcpy(cat + dst, y + ((size_t)known[k] * seq + t) * d, sizeof(float) * d);
        memcpy(cat + dst + d, rev_out + ((size_t)k * seq + (seq - 1 - t)) * d, sizeof(float) * d);
      }
    float* combined = fa((size_t)nk * seq * d);
    jco_linear(cat, nk * seq, m->comb[blk], NULL, 2 * d, d, combined, th);
    for (int k = 0; k < nk; k++)
      memcpy(y + (size_t)known[k] * seq * d, combined + (size_t)k * seq * d, sizeof(float) * seq * d);
    free(rev);
    free(rev_out);
    free(cat);
    free(combined);
  }
  add_in_place(y, x, (size_t)n * d);
  const int ff = ((int)(d * 2.6667f) + 63) / 64 * 64;
  jco_rmsnorm(y, n, d, m->norm_ffn[blk], NORM_EPS, xn);
  float* ffn = swiglu(xn, n, d, ff, m->up_gate[blk], m->up[blk], m->down[blk], th);
  add_in_place(ffn, y, (size_t)n * d);
  free(xn);
  free(y);
  return ffn;
}

/* CpuReference.variateMixer (CpuReference.java:156-236); x is updated in place. */
static void variate_mixer(const JcoTirex2* m, int blk, float* x, int rows, const float* group, const int* target,
                          int th) {
  int* kept = (int*)malloc(sizeof(int) * (rows ? rows : 1));
  int nk = 0;
  for (int r = 0; r < rows; r++)
    for (int o = 0; o < rows; o++)
      if (o != r && group[o] == group[r]) {
        kept[nk++] = r;
        break;
      }
  if (nk == 0) {
    free(kept);
    return;
  }
  const int seq = (m->context_len + m->future_len) / m->patch, d = m->d, heads = m->var_heads, dh = d / heads;
  const int n = nk * seq;
  float* xk = fa((size_t)n * d);
  for (int k = 0; k < nk; k++) memcpy(xk + (size_t)k * seq * d, x + (size_t)kept[k] * seq * d, sizeof(float) * seq * d);
  float* nrm = fa((size_t)n * d);
  jco_rmsnorm(xk, n, d, m->norm_attn[blk], NORM_EPS, nrm);
  float* q_raw = fa((size_t)n * d);
  float* k_raw = fa((size_t)n * d);
  float* v = fa((size_t)n * d);
  jco_linear(nrm, n, m->wq[blk], NULL, d, d, q_raw, th);
  jco_linear(nrm, n, m->wk[blk], NULL, d, d, k_raw, th);
  float* q = q_raw;
  float* kk = k_raw;
  float *qn = NULL, *kn = NULL;
  if (m->use_qk_norm) {
    qn = fa((size_t)n * d);
    kn = fa((size_t)n * d);
    jco_rmsnorm(q_raw, n * heads, dh, NULL, FLOAT32_EPS, qn);
    jco_rmsnorm(k_raw, n * heads, dh, NULL, FLOAT32_EPS, kn);
    q = qn;
    kk = kn;
  }
  jco_linear(nrm, n, m->wv[blk], NULL, d, d, v, th);
  const double scale = 1.0 / sqrt((double)dh);
  float* attn = fa((size_t)n * d);
  double* s = (double*)malloc(sizeof(double) * nk);
  for (int th_ = 0; th_ < seq * heads; th_++) {
    const int t = th_ / heads, h = th_ % heads;
    for (int qi = 0; qi < nk; qi++) {
      size_t qo = ((size_t)qi * seq + t) * d + (size_t)h * dh;
      double mx = -INFINITY;
      for (int ki = 0; ki < nk; ki++) {
        int allowed = group[kept[qi]] == group[kept[ki]] && !(!target[kept[qi]] && target[kept[ki]]);
        if (!allowed) {
          s[ki] = -INFINITY;
          continue;
        }
        size_t ko = ((size_t)ki * seq + t) * d + (size_t)h * dh;
        double dot = 0;
        for (int j = 0; j < dh; j++) dot += (double)q[qo + j] * kk[ko + j];
        s[ki] = dot * scale;
        mx = fmax(mx, s[ki]);
      }
      double sum = 0;
      for (int ki = 0; ki < nk; ki++) {
        s[ki] = s[ki] == -INFINITY ? 0 : exp(s[ki] - mx);
        sum += s[ki];
      }
      for (int j = 0; j < dh; j++) {
        double acc = 0;
        for (int ki = 0; ki < nk; ki++) acc += s[ki] * v[((size_t)ki * seq + t) * d + (size_t)h * dh + j];
        attn[qo + j] = (float)(acc / sum);
      }
    }
  }
  float* out = fa((size_t)n * d);
  jco_linear(attn, n, m->wo[blk], NULL, d, d, out, th);
  add_in_place(out, xk, (size_t)n * d);
  const int hidden = 4 * d;
  jco_rmsnorm(out, n, d, m->norm_ffn_attn[blk], NORM_EPS, nrm);
  float* hid = fa((size_t)n * hidden);
  jco_linear(nrm, n, m->ffn_in[blk], NULL, d, hidden, hid, th);
  silu_in_place(hid, (size_t)n * hidden);
  float* mlp = fa((size_t)n * d);
  jco_linear(hid, n, m->ffn_out[blk], NULL, hidden, d, mlp, th);
  add_in_place(mlp, out, (size_t)n * d);
  for (int k = 0; k < nk; k++) memcpy(x + (size_t)kept[k] * seq * d, mlp + (size_t)k * seq * d, sizeof(float) * seq * d);
  free(kept);
  free(xk);
  free(nrm);
  free(q_raw);
  free(k_raw);
  free(qn);
  free(kn);
  free(v);
  free(attn);
  free(s);
  free(out);
  free(hid);
  free(mlp);
}

/* InputStage.asinh (InputStage.java:96-101) */
static double asinh_ref(double z) {
  double a = fabs(z);
  double r = log(a + sqrt(a * a + 1.0));
  return z < 0 ? -r : r;
}

int jco_tirex2_forward(const JcoTirex2* m, int rows, const float* x, const float* group, const int* target,
                       float* out, int th) {
  if (!m || rows < 1 || !x || !group || !target || !out) return -1;
  const int len = m->context_len + m->future_len, p = m->patch, seq = len / p, d = m->d, nq = m->num_q;
  const int n = rows * seq;
  /* InputStage.apply */
  float* loc = fa(rows);
  float* scl = fa(rows);
  int* binary = (int*)calloc(rows, sizeof(int));
  float* tokens = fa((size_t)n * 2 * p);
  for (int r = 0; r < rows; r++) {
    const float* row = x + (size_t)r * len;
    double sum = 0;
    int cnt = 0, is_binary = 1;
    for (int t = 0; t < len; t++) {
      float v = row[t];
      if (!isnan(v)) {
        sum += v;
        cnt++;
        is_binary &= v == 0.0f || v == 1.0f;
      }
    }
    float l = cnt == 0 ? 0.0f : (float)(sum / cnt);
    double ss = 0;
    for (int t = 0; t < len; t++) {
      float v = row[t];
      if (!isnan(v)) {
        double dv = v - l;
        ss += dv * dv;
      }
    }
    float s = cnt == 0 ? 1.0f : (float)sqrt(ss / cnt);
    s = fmaxf(s, SCALER_EPS);
    if (m->binary_aware && is_binary) {
      l = 0.0f;
      s = 1.0f;
    }
    loc[r] = l;
    scl[r] = s;
    binary[r] = m->binary_aware && is_binary;
    const int arcsinh = m->use_arcsinh && !binary[r];
    for (int t = 0; t < seq; t++) {
      size_t base = ((size_t)r * seq + t) * 2 * p;
      for (int i = 0; i < p; i++) {
        float v = row[t * p + i];
        int present = !isnan(v);
        float z = (v - l) / s;
        if (arcsinh) z = (float)asinh_ref(z);
        tokens[base + i] = present ? z : 0.0f;
        tokens[base + p + i] = present ? 1.0f : 0.0f;
      }
    }
  }
  /* knownCovariates */
  int* known = (int*)malloc(sizeof(int) * rows);
  int nk = 0;
  for (int r = 0; r < rows; r++) {
    if (target[r]) continue;
    for (int t = len - m->future_len; t < len; t++)
      if (!isnan(x[(size_t)r * len + t])) {
        known[nk++] = r;
        break;
      }
  }
  float* h = residual_block(tokens, n, 2 * p, m->in_ff, d, m->in_hw, m->in_hb, m->in_ow, m->in_ob, m->in_rw, m->in_rb,
                            th);
  for (int b = 0; b < m->blocks; b++) {
    float* h2 = time_mixer(m, b, h, rows, known, nk, th);
    free(h);
    h = h2;
    variate_mixer(m, b, h, rows, group, target, th);
  }
  float* hn = fa((size_t)n * d);
  jco_rmsnorm(h, n, d, m->out_norm, m->out_norm_eps, hn);
  float* y = residual_block(hn, n, d, m->out_ff, nq * p, m->out_hw, m->out_hb, m->out_ow, m->out_ob, m->out_rw,
                            m->out_rb, th);
  /* unpatch */
  for (int r = 0; r < rows; r++) {
    const int sinh_on = m->use_arcsinh && !binary[r];
    for (int t = 0; t < seq; t++) {
      size_t base = ((size_t)r * seq + t) * nq * p;
      for (int q = 0; q < nq; q++)
        for (int i = 0; i < p; i++) {
          float v = y[base + (size_t)q * p + i];
          if (sinh_on) {
            float c = fmaxf(-SINH_CLAMP, fminf(SINH_CLAMP, v));
            v = (float)sinh(c);
          }
          out[((size_t)r * nq + q) * len + (size_t)t * p + i] = v * scl[r] + loc[r];
        }
    }
  }
  free(loc);
  free(scl);
  free(binary);
  free(tokens);
  free(known);
  free(h);
  free(hn);
  free(y);
  return 0;
}
