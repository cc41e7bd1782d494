// The Chronos-2 encoder on B200: weights bound by checkpoint name and converted once per GPU; one
// plan (activation buffers + CUDA graph) per (rows, context patches, output patches); every linear
// layer a tcgen05 GEMM with its elementwise work fused into the epilogue:
//
//   input embedding  hidden (bias, ReLU) → output (bias, written around the [REG] token of x)
//                    → residual (bias, += x); the [REG] row filled from the token table
//   per block        RMSNorm → q|k|v GEMM (RoPE at the token index) → time attention over live keys
//                    (unscaled, both directions) → o GEMM (+= x);
//                    RMSNorm → q|k|v GEMM → group attention over the group's live rows → o (+= x);
//                    RMSNorm → wi GEMM (ReLU) → wo GEMM (+= x)
//   output           RMSNorm of the future tokens → hidden (bias, ReLU) → output (bias) → residual (+=)
//
// This replaces Chronos2Forward's task graph (chronos2/tornado/Chronos2Forward.java:225-304), its
// cuBLAS dispatch with a separate ReLU pass (:314-409) and Chronos2Kernels; the arithmetic is
// CpuChronos2.forward's (chronos2/cpu/CpuChronos2.java:122-173).
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <thread>

#include "attention.cuh"
#include "engine.h"
#include "kernels.cuh"
#include "runtime.h"

namespace jc {
namespace {

struct C2Attn {
  float* norm = nullptr;
  DevLinear qkv;  // [3·inner, d]: q | k | v, each heads-major (as Chronos2Weights.qkv concatenates them)
  DevLinear o;
};

struct C2Layer {
  C2Attn time, group;
  float* mlp_norm = nullptr;
  DevLinear wi, wo;
};

struct C2Weights {
  DevLinear in_h, in_o, in_r;
  float* reg = nullptr;  // the [REG] token's embedding (row 1 of the token table), or null
  std::vector<C2Layer> layers;
  float* final_norm = nullptr;
  DevLinear out_h, out_o, out_r;
};

struct C2Plan {
  int rows = 0, nc = 0, h = 0;
  DeviceMem mem;
  float* tok_f32 = nullptr;
  OpBuf tok, emb_h, hn, att, act, dec, head_h;
  float* x = nullptr;
  void* qkv = nullptr;
  float* raw = nullptr;
  float* rowsq = nullptr;  // the folded norms' Σx² per row and 64-column unit [T, d / 64]
  int *pos = nullptr, *live = nullptr, *gs = nullptr, *ge = nullptr;
  float* table = nullptr;
  GraphRunner graph;
  std::vector<int> h_gs, h_ge;
  // the host ends on the device (jc_forecast_chronos2), allocated on first use: per-row (loc, scale), and for
  // host calls the window, the future covariates and the finished quantiles staged in HBM
  DeviceMem ends_mem, stage_mem;
  float2* norm = nullptr;
  float *win = nullptr, *fut = nullptr, *qout = nullptr;
};

struct C2Device : DeviceSlot {
  C2Weights w;
  std::list<std::unique_ptr<C2Plan>> plans;
  Profiler prof;
  cudaEvent_t ev_in = nullptr, ev_out = nullptr;
  ~C2Device() {
    if (ev_in) cudaEventDestroy(ev_in);
    if (ev_out) cudaEventDestroy(ev_out);
  }
};

struct Chronos2Engine : jc_engine {
  int d = 0, dkv = 0, ff = 0, layers = 0, heads = 0, inner = 0, P = 0, Q = 0, reg = 0;
  float eps = 0, theta = 0;
  int op = kOpBF16;
  // The 16-bit modes fold the attention and MLP norms into the GEMMs around them, as the Timestral engine does:
  // the GEMM that writes x also writes its 16-bit copy and Σx² per 64-column unit, the next GEMM (whose W carries
  // the norm's weights) scales its rows by the norm. JC_FOLD_NORM=0 in the environment keeps the norm kernel.
  bool fold_norms = false;
  std::vector<float> inv_freq;
  std::vector<std::unique_ptr<C2Device>> devs;

  int slots() const override { return static_cast<int>(devs.size()); }
  DeviceSlot* slot(int i) override { return devs[i].get(); }
  Profiler* profiler(int i) override { return &devs[i]->prof; }
  void drop_plans() override {
    for (auto& dv : devs) {
      cudaSetDevice(dv->device);
      cudaStreamSynchronize(dv->stream);
      dv->plans.clear();
    }
  }
  int qkv_kind() const { return op == kOpBF16 ? kOutBF16 : op == kOpF16 ? kOutF16 : kOutF32; }
  size_t qkv_esize() const { return op_is_16bit(op) ? 2 : 4; }
};

struct HostC2 {
  const float* shared;
  const float *in_hw, *in_hb, *in_ow, *in_ob, *in_rw, *in_rb;
  struct A {
    const float *norm, *q, *k, *v, *o;
  };
  struct L {
    A time, group;
    const float *mlp_norm, *wi, *wo;
  };
  std::vector<L> layers;
  const float* final_norm;
  const float *out_hw, *out_hb, *out_ow, *out_ob, *out_rw, *out_rb;
};

bool bind(const Chronos2Engine& e, Binder& b, HostC2* hw) {
  const long long d = e.d, inner = e.inner, ff = e.ff, p = e.P, q = e.Q;
  hw->shared = b.take("shared.weight", {e.reg ? 2 : 1, d});
  auto residual = [&](const std::string& pre, long long in, long long hid, long long out, const float** w) {
    w[0] = b.take(pre + ".hidden_layer.weight", {hid, in});
    w[1] = b.take(pre + ".hidden_layer.bias", {hid});
    w[2] = b.take(pre + ".output_layer.weight", {out, hid});
    w[3] = b.take(pre + ".output_layer.bias", {out});
    w[4] = b.take(pre + ".residual_layer.weight", {out, in});
    w[5] = b.take(pre + ".residual_layer.bias", {out});
  };
  const float* in[6];
  residual("input_patch_embedding", 3 * p, ff, d, in);
  hw->in_hw = in[0], hw->in_hb = in[1], hw->in_ow = in[2], hw->in_ob = in[3], hw->in_rw = in[4], hw->in_rb = in[5];
  for (int i = 0; i < e.layers; ++i) {
    const std::string s = "encoder.block." + std::to_string(i) + ".layer.";
    HostC2::L L;
    auto attn = [&](const std::string& pre, HostC2::A* a) {
      a->norm = b.take(pre + ".layer_norm.weight", {d});
      a->q = b.take(pre + ".self_attention.q.weight", {inner, d});
      a->k = b.take(pre + ".self_attention.k.weight", {inner, d});
      a->v = b.take(pre + ".self_attention.v.weight", {inner, d});
      a->o = b.take(pre + ".self_attention.o.weight", {d, inner});
    };
    attn(s + "0", &L.time);
    attn(s + "1", &L.group);
    L.mlp_norm = b.take(s + "2.layer_norm.weight", {d});
    L.wi = b.take(s + "2.mlp.wi.weight", {ff, d});
    L.wo = b.take(s + "2.mlp.wo.weight", {d, ff});
    hw->layers.push_back(L);
  }
  hw->final_norm = b.take("encoder.final_layer_norm.weight", {d});
  const float* out[6];
  residual("output_patch_embedding", d, ff, q * p, out);
  hw->out_hw = out[0], hw->out_hb = out[1], hw->out_ow = out[2], hw->out_ob = out[3], hw->out_rw = out[4],
  hw->out_rb = out[5];
  return b.require_all_bound();
}

bool upload(Chronos2Engine& e, const HostC2& hw, C2Device& dv, std::string* err) {
  const int d = e.d, inner = e.inner, ff = e.ff, p = e.P, q = e.Q, op = e.op;
  DeviceMem& m = dv.weights;
  C2Weights& w = dv.w;
  if (!upload_linear(m, op, hw.in_hw, hw.in_hb, 3 * p, ff, &w.in_h, err) ||
      !upload_linear(m, op, hw.in_ow, hw.in_ob, ff, d, &w.in_o, err) ||
      !upload_linear(m, op, hw.in_rw, hw.in_rb, 3 * p, d, &w.in_r, err))
    return false;
  if (e.reg && !(w.reg = upload_f32(m, hw.shared + d, d, err))) return false;
  auto attn = [&](const HostC2::A& a, C2Attn* t) {
    if (!(t->norm = upload_f32(m, a.norm, d, err))) return false;
    std::vector<float> qkv(static_cast<size_t>(3) * inner * d);
    const size_t part = static_cast<size_t>(inner) * d;
    std::memcpy(qkv.data(), a.q, sizeof(float) * part);
    std::memcpy(qkv.data() + part, a.k, sizeof(float) * part);
    std::memcpy(qkv.data() + 2 * part, a.v, sizeof(float) * part);
    if (e.fold_norms)
      for (size_t i = 0; i < qkv.size(); ++i) qkv[i] *= a.norm[i % d];
    return upload_linear(m, op, qkv.data(), nullptr, d, 3 * inner, &t->qkv, err) &&
           upload_linear(m, op, a.o, nullptr, inner, d, &t->o, err);
  };
  for (const auto& L : hw.layers) {
    C2Layer cl;
    if (!attn(L.time, &cl.time) || !attn(L.group, &cl.group)) return false;
    if (!(cl.mlp_norm = upload_f32(m, L.mlp_norm, d, err))) return false;
    std::vector<float> wi(L.wi, L.wi + static_cast<size_t>(ff) * d);
    if (e.fold_norms)
      for (size_t i = 0; i < wi.size(); ++i) wi[i] *= L.mlp_norm[i % d];
    if (!upload_linear(m, op, wi.data(), nullptr, d, ff, &cl.wi, err) ||
        !upload_linear(m, op, L.wo, nullptr, ff, d, &cl.wo, err))
      return false;
    w.layers.push_back(std::move(cl));
  }
  if (!(w.final_norm = upload_f32(m, hw.final_norm, d, err))) return false;
  return upload_linear(m, op, hw.out_hw, hw.out_hb, d, ff, &w.out_h, err) &&
         upload_linear(m, op, hw.out_ow, hw.out_ob, ff, q * p, &w.out_o, err) &&
         upload_linear(m, op, hw.out_rw, hw.out_rb, d, q * p, &w.out_r, err);
}

std::unique_ptr<C2Plan> make_plan(const Chronos2Engine& e, int rows, int nc, int h) {
  auto p = std::make_unique<C2Plan>();
  p->rows = rows;
  p->nc = nc;
  p->h = h;
  const int n = nc + e.reg + h, ne = nc + h, d = e.d, op = e.op;
  const long long T = static_cast<long long>(rows) * n, EN = static_cast<long long>(rows) * ne,
                  decT = static_cast<long long>(rows) * h;
  DeviceMem& m = p->mem;
  bool ok = (p->tok_f32 = static_cast<float*>(m.alloc(sizeof(float) * EN * 3 * e.P))) &&
            alloc_op(m, op, EN, 3 * e.P, &p->tok) && alloc_op(m, op, EN, e.ff, &p->emb_h) &&
            (p->x = static_cast<float*>(m.alloc(sizeof(float) * T * d))) && alloc_op(m, op, T, d, &p->hn) &&
            (!e.fold_norms || (p->rowsq = static_cast<float*>(m.alloc(sizeof(float) * T * (d / 64))))) &&
            (p->qkv = m.alloc(e.qkv_esize() * T * 3 * e.inner)) && alloc_op(m, op, T, e.inner, &p->att) &&
            alloc_op(m, op, T, e.ff, &p->act) && alloc_op(m, op, decT, d, &p->dec) &&
            alloc_op(m, op, decT, e.ff, &p->head_h) &&
            (p->raw = static_cast<float*>(m.alloc(sizeof(float) * decT * e.P * e.Q))) &&
            (p->pos = static_cast<int*>(m.alloc(sizeof(int) * T))) &&
            (p->live = static_cast<int*>(m.alloc(sizeof(int) * T))) &&
            (p->gs = static_cast<int*>(m.alloc(sizeof(int) * rows))) &&
            (p->ge = static_cast<int*>(m.alloc(sizeof(int) * rows))) &&
            (p->table = static_cast<float*>(m.alloc(sizeof(float) * n * e.dkv)));
  if (!ok) {
    cudaGetLastError();
    return nullptr;
  }
  // a token's position is its index in the row (CpuChronos2.timeAttention, CpuChronos2.java:176-186)
  const int half = e.dkv / 2;
  std::vector<float> table(static_cast<size_t>(n) * e.dkv);
  for (int t = 0; t < n; ++t)
    for (int k = 0; k < half; ++k) {
      const float a = static_cast<float>(t) * e.inv_freq[k];
      table[static_cast<size_t>(t) * e.dkv + k] = static_cast<float>(std::cos(static_cast<double>(a)));
      table[static_cast<size_t>(t) * e.dkv + half + k] = static_cast<float>(std::sin(static_cast<double>(a)));
    }
  std::vector<int> pos(T);
  for (long long i = 0; i < T; ++i) pos[i] = static_cast<int>(i % n);
  // every row starts as a valid, independent dummy series (zero tokens, every token live, its own group), so
  // rows past a call's own (bucket padding) compute harmlessly and never reach a real row
  std::vector<int> live(T, 1), gs(rows), ge(rows);
  for (int i = 0; i < rows; ++i) gs[i] = i, ge[i] = i + 1;
  if (cudaMemcpy(p->table, table.data(), sizeof(float) * table.size(), cudaMemcpyHostToDevice) != cudaSuccess ||
      cudaMemcpy(p->pos, pos.data(), sizeof(int) * T, cudaMemcpyHostToDevice) != cudaSuccess ||
      cudaMemset(p->tok_f32, 0, sizeof(float) * EN * 3 * e.P) != cudaSuccess ||
      cudaMemcpy(p->live, live.data(), sizeof(int) * T, cudaMemcpyHostToDevice) != cudaSuccess ||
      cudaMemcpy(p->gs, gs.data(), sizeof(int) * rows, cudaMemcpyHostToDevice) != cudaSuccess ||
      cudaMemcpy(p->ge, ge.data(), sizeof(int) * rows, cudaMemcpyHostToDevice) != cudaSuccess)
    return nullptr;
  p->h_gs.resize(rows);
  p->h_ge.resize(rows);
  return p;
}

C2Plan* get_plan(Chronos2Engine& e, C2Device& dv, int rows, int nc, int h, std::string* err) {
  for (auto it = dv.plans.begin(); it != dv.plans.end(); ++it) {
    C2Plan* p = it->get();
    if (p->rows == rows && p->nc == nc && p->h == h) {
      dv.plans.splice(dv.plans.begin(), dv.plans, it);
      return p;
    }
  }
  while (static_cast<int>(dv.plans.size()) >= std::max(1, e.max_plans)) dv.plans.pop_back();
  auto p = e.take_plan_failure() ? nullptr : make_plan(e, rows, nc, h);
  if (!p && !dv.plans.empty()) {
    cudaStreamSynchronize(dv.stream);
    dv.plans.clear();
    p = e.take_plan_failure() ? nullptr : make_plan(e, rows, nc, h);
  }
  if (!p) {
    *err = "out of device memory for a plan of " + std::to_string(rows) + " rows";
    return nullptr;
  }
  dv.plans.push_front(std::move(p));
  return dv.plans.front().get();
}

cudaError_t gemm(C2Device& dv, GemmArgs& g, cudaStream_t s, const char* name) {
  dv.prof.begin(s, name, 2.0 * g.M * g.N * g.K);
  cudaError_t r = launch_gemm(g, s, dv.err);
  dv.prof.end(s);
  return r;
}

// Independent GEMMs as one grouped launch (launch_gemm_group), timed as one launch under `name`.
cudaError_t gemm_group(C2Device& dv, GemmArgs* g, int count, cudaStream_t s, const char* name) {
  double flops = 0.0;
  for (int i = 0; i < count; ++i) flops += 2.0 * g[i].M * g[i].N * g[i].K;
  dv.prof.begin(s, name, flops);
  cudaError_t r = launch_gemm_group(g, count, s, dv.err);
  dv.prof.end(s);
  return r;
}

void set_out(EpiParams& ep, int op, const OpBuf& o) {
  ep.o_kind = out_of_op(op);
  ep.o_hi = o.hi;
  ep.o_lo = o.lo;
  ep.ldo = o.ld;
}

void residual_into(GemmArgs& g, float* x, int d) {
  g.ep.c = x;
  g.ep.ldc = d;
  g.ep.cin = x;
  g.ep.ldcin = d;
  g.ep.accumulate = 1;
}

cudaError_t enqueue_forward(const Chronos2Engine& e, C2Device& dv, C2Plan& p, cudaStream_t s) {
  const int R = p.rows, nc = p.nc, h = p.h, reg = e.reg, n = nc + reg + h, ne = nc + h, fs = nc + reg;
  const int d = e.d, op = e.op, P3 = 3 * e.P, inner = e.inner;
  const long long T = static_cast<long long>(R) * n, EN = static_cast<long long>(R) * ne,
                  decT = static_cast<long long>(R) * h;
  const C2Weights& w = dv.w;
  Profiler& prof = dv.prof;
  const int out_kind = out_of_op(op);
  // the folded norms (fold_norms): a GEMM that writes x also writes its 16-bit copy into hn and Σx² per unit; the
  // GEMM that reads hn scales its rows by the norm
  const bool fold = e.fold_norms;
  auto produce = [&](GemmArgs& g) {
    if (!fold) return;
    set_out(g.ep, op, p.hn);
    g.ep.rowsq = p.rowsq;
    g.ep.rowsq_units = d / 64;
  };
  auto consume = [&](GemmArgs& g) {
    if (!fold) return;
    g.ep.norm_sq = p.rowsq;
    g.ep.norm_units = d / 64;
    g.ep.norm_inv_d = 1.0f / static_cast<float>(d);
    g.ep.norm_eps = e.eps;
  };
  cudaError_t r;
#define JC_TRY(x)                   \
  do {                              \
    if ((r = (x)) != cudaSuccess) { \
      return r;                     \
    }                               \
  } while (0)
  prof.begin(s, "convert", 0);
  launch_convert(op, p.tok_f32, P3, p.tok.hi, p.tok.lo, p.tok.ld, EN, P3, s);
  prof.end(s);
  // input embedding: output(ReLU(hidden(tok))) + residual(tok), around the [REG] token. The two GEMMs of tok
  // (hidden, and residual stored into x) run as one grouped launch; output then adds into x, the same float
  // sum as the reference's output + residual
  GemmArgs ge[2] = {gemm_args(op, p.tok, EN, w.in_h), gemm_args(op, p.tok, EN, w.in_r)};
  ge[0].ep.act = kActRelu;
  set_out(ge[0].ep, op, p.emb_h);
  ge[1].ep.c = p.x;
  ge[1].ep.ldc = d;
  ge[1].ep.rg = ne;
  ge[1].ep.rg_stride = n;
  ge[1].ep.rg_split = nc;
  ge[1].ep.rg_shift = reg;
  JC_TRY(gemm_group(dv, ge, 2, s, "gemm.embed"));
  GemmArgs g = gemm_args(op, p.emb_h, EN, w.in_o);
  residual_into(g, p.x, d);
  g.ep.rg = ne;
  g.ep.rg_stride = n;
  g.ep.rg_split = nc;
  g.ep.rg_shift = reg;
  produce(g);
  JC_TRY(gemm(dv, g, s, "gemm.embed"));
  if (reg) {
    prof.begin(s, "fill", 0);
    launch_fill_rows(p.x, d, w.reg, d, R, nc, nc + 1, n, s);
    if (fold) launch_norm_copy_rows(p.x, d, d, out_kind, p.hn.hi, p.hn.ld, p.rowsq, R, nc, nc + 1, n, s);
    prof.end(s);
  }
  AttnArgs a{};
  a.qkv = p.qkv;
  a.qkv_kind = e.qkv_kind();
  a.ld_qkv = 3LL * inner;
  a.out_hi = p.att.hi;
  a.out_lo = p.att.lo;
  a.ld_out = p.att.ld;
  a.out_kind = out_kind;
  a.rows = R;
  a.n = n;
  a.enc = n;
  a.ll = n;
  a.heads = e.heads;
  a.head_dim = e.dkv;
  a.d = inner;
  a.scale = 1.0f;  // T5-style attention: no 1/√d_kv
  a.group_start = p.gs;
  a.group_end = p.ge;
  a.mask_mode = 1;
  a.live = p.live;
  a.err = dv.err;
  for (size_t li = 0; li < w.layers.size(); ++li) {
    const C2Layer& L = w.layers[li];
    for (int which = 0; which < 2; ++which) {
      const C2Attn& A = which == 0 ? L.time : L.group;
      if (!fold) {
        prof.begin(s, "rmsnorm", 0);
        launch_rmsnorm(p.x, d, A.norm, d, e.eps, out_kind, p.hn.hi, p.hn.lo, p.hn.ld, T, 0, 0, 0, s);
        prof.end(s);
      }
      g = gemm_args(op, p.hn, T, A.qkv);
      consume(g);
      g.ep.mode = kEpiQKV;
      g.ep.o_kind = e.qkv_kind();
      g.ep.o_hi = p.qkv;
      g.ep.ldo = 3LL * inner;
      g.ep.rope_cols = which == 0 ? 2 * inner : 0;
      g.ep.head_dim = e.dkv;
      g.ep.pos = p.pos;
      g.ep.rope_table = p.table;
      g.ep.n_split = 3 * inner;
      JC_TRY(gemm(dv, g, s, which == 0 ? "gemm.time_qkv" : "gemm.group_qkv"));
      prof.begin(s, which == 0 ? "attention" : "attention.group", 4.0 * T * n * inner);
      JC_TRY(which == 0 ? launch_time_attention(a, s) : launch_variate_attention(a, s));
      prof.end(s);
      g = gemm_args(op, p.att, T, A.o);
      residual_into(g, p.x, d);
      produce(g);
      JC_TRY(gemm(dv, g, s, "gemm.o"));
    }
    if (!fold) {
      prof.begin(s, "rmsnorm", 0);
      launch_rmsnorm(p.x, d, L.mlp_norm, d, e.eps, out_kind, p.hn.hi, p.hn.lo, p.hn.ld, T, 0, 0, 0, s);
      prof.end(s);
    }
    g = gemm_args(op, p.hn, T, L.wi);
    consume(g);
    g.ep.act = kActRelu;
    set_out(g.ep, op, p.act);
    JC_TRY(gemm(dv, g, s, "gemm.wi"));
    g = gemm_args(op, p.act, T, L.wo);
    residual_into(g, p.x, d);
    if (li + 1 < w.layers.size()) produce(g);  // the last x goes to final_norm, which reads it directly
    JC_TRY(gemm(dv, g, s, "gemm.wo"));
  }
  prof.begin(s, "rmsnorm", 0);
  launch_rmsnorm(p.x, d, w.final_norm, d, e.eps, out_kind, p.dec.hi, p.dec.lo, p.dec.ld, decT, h, n, fs, s);
  prof.end(s);
  // the output embedding: output(ReLU(hidden(dec))) + residual(dec); hidden and residual (stored into raw) as
  // one grouped launch, then output adds into raw
  const int qp = e.Q * e.P;
  GemmArgs gh[2] = {gemm_args(op, p.dec, decT, w.out_h), gemm_args(op, p.dec, decT, w.out_r)};
  gh[0].ep.act = kActRelu;
  set_out(gh[0].ep, op, p.head_h);
  gh[1].ep.c = p.raw;
  gh[1].ep.ldc = qp;
  JC_TRY(gemm_group(dv, gh, 2, s, "gemm.head"));
  g = gemm_args(op, p.head_h, decT, w.out_o);
  g.ep.c = p.raw;
  g.ep.ldc = qp;
  g.ep.cin = p.raw;
  g.ep.ldcin = qp;
  g.ep.accumulate = 1;
  JC_TRY(gemm(dv, g, s, "gemm.head"));
#undef JC_TRY
  return cudaGetLastError();
}

jc_status check_block(const jc_chronos2_block* b, bool host, bool tokens = true) {
  if (!b) return fail(JC_ERR_INVALID_ARG, "null block");
  if (b->rows < 1) return fail(JC_ERR_INVALID_ARG, "rows must be >= 1");
  if (b->context_patches < 1) return fail(JC_ERR_INVALID_ARG, "context patches must be >= 1");
  if (b->output_patches < 1)
    return fail(JC_ERR_INVALID_ARG, "output patches must be >= 1, got " + std::to_string(b->output_patches));
  if ((tokens && !b->tokens) || !b->live || !b->group_start || !b->group_end)
    return fail(JC_ERR_INVALID_ARG, "null block field");
  if (host)
    for (int i = 0; i < b->rows; ++i) {
      const int s = b->group_start[i], t = b->group_end[i];
      if (s < 0 || s > i || t <= i || t > b->rows || b->group_start[s] != s || b->group_end[s] != t)
        return fail(JC_ERR_INVALID_ARG, "rows of a group are not contiguous (row " + std::to_string(i) + ")");
    }
  return JC_OK;
}

// The host ends' buffers of a plan, sized for its rows: the row statistics always, the staged window,
// future covariates and quantiles only for host calls. False when device memory runs out.
bool ensure_ends(C2Plan& p, int P, int Q, bool host) {
  if (!p.norm) {
    if (!(p.norm = static_cast<float2*>(p.ends_mem.alloc(sizeof(float2) * p.rows)))) {
      cudaGetLastError();
      return false;
    }
  }
  if (host && !p.win) {
    const long long r = p.rows;
    if (!(p.win = static_cast<float*>(p.stage_mem.alloc(sizeof(float) * r * p.nc * P))) ||
        !(p.fut = static_cast<float*>(p.stage_mem.alloc(sizeof(float) * r * p.h * P))) ||
        !(p.qout = static_cast<float*>(p.stage_mem.alloc(sizeof(float) * r * Q * p.h * P)))) {
      cudaGetLastError();
      p.stage_mem.release();
      p.win = p.fut = p.qout = nullptr;
      return false;
    }
  }
  return true;
}

// Runs rows [r0, r1) of `b` on one GPU; raw_out points at the block's first row's outputs. With `ends`
// (whose layout is `b`) the window and future covariates replace the tokens and raw_out receives
// ModelPrep.finish's quantiles [rows · Q · h·P].
jc_status run_shard(Chronos2Engine& e, C2Device& dv, const jc_chronos2_block* b, int r0, int r1, float* raw_out,
                    bool host, cudaStream_t stream, std::string* err, const jc_chronos2_window* ends = nullptr) {
  if (e.take_slot_failure(dv.slot)) {  // injected (engine option fail_slot), before any device work
    *err = "injected shard failure (engine option fail_slot)";
    return JC_ERR_CUDA;
  }
  if (cudaSetDevice(dv.device) != cudaSuccess) {
    *err = "cannot select device " + std::to_string(dv.device);
    return JC_ERR_CUDA;
  }
  cudaStream_t s = dv.stream;
  if (!host && (cudaEventRecord(dv.ev_in, stream) != cudaSuccess || cudaStreamWaitEvent(s, dv.ev_in, 0) != cudaSuccess)) {
    *err = "cannot order the caller's stream before the forward";
    return JC_ERR_CUDA;
  }
  const int rows = r1 - r0, nc = b->context_patches, h = b->output_patches, n = nc + e.reg + h, ne = nc + h;
  const int prows = e.buckets ? bucket_rows(rows) : rows;  // the plan's rows ≥ this shard's
  C2Plan* p = get_plan(e, dv, prows, nc, h, err);
  if (!p) return JC_ERR_OOM;
  const cudaMemcpyKind kind = host ? cudaMemcpyHostToDevice : cudaMemcpyDeviceToDevice;
  cudaError_t ce = cudaSuccess;
  if (!ends)
    ce = cudaMemcpyAsync(p->tok_f32, b->tokens + static_cast<long long>(r0) * ne * 3 * e.P,
                         sizeof(float) * rows * ne * 3 * e.P, kind, s);
  if (ce == cudaSuccess)
    ce = cudaMemcpyAsync(p->live, b->live + static_cast<long long>(r0) * n, sizeof(int) * rows * n, kind, s);
  if (ce == cudaSuccess) {
    if (host) {
      for (int i = 0; i < rows; ++i) {
        p->h_gs[i] = b->group_start[r0 + i] - r0;
        p->h_ge[i] = b->group_end[r0 + i] - r0;
      }
      ce = cudaMemcpyAsync(p->gs, p->h_gs.data(), sizeof(int) * rows, cudaMemcpyHostToDevice, s);
      if (ce == cudaSuccess) ce = cudaMemcpyAsync(p->ge, p->h_ge.data(), sizeof(int) * rows, cudaMemcpyHostToDevice, s);
    } else {
      launch_add_i32(b->group_start + r0, p->gs, rows, -r0, s);
      launch_add_i32(b->group_end + r0, p->ge, rows, -r0, s);
      ce = cudaGetLastError();
    }
  }
  if (ce != cudaSuccess) {
    *err = std::string("upload: ") + cudaGetErrorString(ce);
    return JC_ERR_CUDA;
  }
  dv.prof.on = e.profile;
  C2Ends ep;
  if (ends) {
    // ModelPrep.of on the GPU: the rows' instance norm, then the tokens, into the plan's token rows
    if (!ensure_ends(*p, e.P, e.Q, host)) {
      *err = "out of device memory for the host ends of a plan of " + std::to_string(p->rows) + " rows";
      return JC_ERR_OOM;
    }
    const float* win = ends->window + static_cast<long long>(r0) * nc * e.P;
    const float* fut = ends->future + static_cast<long long>(r0) * h * e.P;
    if (host) {
      ce = cudaMemcpyAsync(p->win, win, sizeof(float) * rows * nc * e.P, cudaMemcpyHostToDevice, s);
      if (ce == cudaSuccess) ce = cudaMemcpyAsync(p->fut, fut, sizeof(float) * rows * h * e.P, cudaMemcpyHostToDevice, s);
      if (ce != cudaSuccess) {
        *err = std::string("upload: ") + cudaGetErrorString(ce);
        return JC_ERR_CUDA;
      }
      win = p->win;
      fut = p->fut;
    }
    ep.rows = rows;
    ep.nc = nc;
    ep.h = h;
    ep.P = e.P;
    ep.Q = e.Q;
    ep.use_arcsinh = ends->use_arcsinh ? 1 : 0;
    ep.time_scale = ends->time_encoding_scale;
    dv.prof.begin(s, "prep.norm", 0);
    launch_c2_norm(win, ep, p->norm, s);
    dv.prof.end(s);
    dv.prof.begin(s, "prep.tokens", 0);
    launch_c2_tokens(win, fut, p->norm, ep, p->tok_f32, s);
    dv.prof.end(s);
    ce = cudaGetLastError();
    if (ce != cudaSuccess) {
      *err = std::string("prep: ") + cudaGetErrorString(ce);
      return JC_ERR_CUDA;
    }
  }
  Chronos2Engine& ec = e;
  C2Device& dvc = dv;
  ce = p->graph.run(s, [&](cudaStream_t st) { return enqueue_forward(ec, dvc, *p, st); }, e.use_graph && !e.profile);
  if (ce != cudaSuccess) {
    *err = std::string("forward: ") + cudaGetErrorString(ce);
    return JC_ERR_CUDA;
  }
  const size_t per_row = static_cast<size_t>(h) * e.Q * e.P;
  const float* result = p->raw;
  if (ends) {
    // ModelPrep.finish on the GPU: straight into a device caller's output, else into the staged quantiles
    float* q = host ? p->qout : raw_out + static_cast<size_t>(r0) * per_row;
    dv.prof.begin(s, "finish", 0);
    launch_c2_finish(p->raw, p->norm, ep, q, s);
    dv.prof.end(s);
    ce = cudaGetLastError();
    if (ce != cudaSuccess) {
      *err = std::string("finish: ") + cudaGetErrorString(ce);
      return JC_ERR_CUDA;
    }
    result = q;
  }
  if (result != raw_out + static_cast<size_t>(r0) * per_row)
    ce = cudaMemcpyAsync(raw_out + static_cast<size_t>(r0) * per_row, result, sizeof(float) * rows * per_row,
                         host ? cudaMemcpyDeviceToHost : cudaMemcpyDeviceToDevice, s);
  if (ce != cudaSuccess) {
    *err = std::string("download: ") + cudaGetErrorString(ce);
    return JC_ERR_CUDA;
  }
  if (!host) {
    if (cudaEventRecord(dv.ev_out, s) != cudaSuccess || cudaStreamWaitEvent(stream, dv.ev_out, 0) != cudaSuccess) {
      *err = "cannot order the caller's stream after the forward";
      return JC_ERR_CUDA;
    }
    return JC_OK;
  }
  ce = cudaStreamSynchronize(s);
  if (ce != cudaSuccess) {
    *err = std::string("forward: ") + cudaGetErrorString(ce);
    return JC_ERR_CUDA;
  }
  if (e.profile) dv.prof.collect();
  uint32_t word = 0;
  cudaMemcpy(&word, dv.err, sizeof word, cudaMemcpyDeviceToHost);
  if (word) {
    cudaMemset(dv.err, 0, sizeof word);
    *err = "a device wait gave up (error bits " + std::to_string(word) + ")";
    return JC_ERR_TIMEOUT;
  }
  return JC_OK;
}

jc_status check_window(const jc_chronos2_window* w, bool host) {
  if (!w) return fail(JC_ERR_INVALID_ARG, "null block");
  if (!w->window || !w->future) return fail(JC_ERR_INVALID_ARG, "null window field");
  if (!(w->time_encoding_scale > 0.0f)) return fail(JC_ERR_INVALID_ARG, "time encoding scale must be > 0");
  return check_block(&w->layout, host, false);
}

}  // namespace
}  // namespace jc

using namespace jc;

extern "C" {

jc_status jc_engine_create_chronos2(const jc_chronos2_desc* desc, const jc_tensor_view* weights, int n_weights,
                                    const int* devices, int n_devices, jc_precision precision, jc_engine** out) {
  clear_error();
  if (!out) return fail(JC_ERR_INVALID_ARG, "null engine out-pointer");
  *out = nullptr;
  if (!desc || !weights || n_weights < 1) return fail(JC_ERR_INVALID_ARG, "null description or weights");
  if (!valid_precision_code(precision)) return fail(JC_ERR_INVALID_ARG, "unknown precision");
  const jc_chronos2_desc& c = *desc;
  if (c.d_model < 1 || c.d_kv < 1 || c.d_ff < 1 || c.num_layers < 1 || c.num_heads < 1 || c.patch_size < 1 ||
      c.num_quantiles < 1)
    return fail(JC_ERR_INVALID_ARG, "non-positive model dimensions");
  if (c.d_kv % 2 != 0) return fail(JC_ERR_INVALID_ARG, "d_kv must be even for RoPE, got " + std::to_string(c.d_kv));
  if (c.d_kv != 64)
    return fail(JC_ERR_UNSUPPORTED_SHAPE,
                "unsupported attention head width " + std::to_string(c.d_kv) + " (this engine supports 64)");
  auto e = std::make_unique<Chronos2Engine>();
  e->family = 2;
  e->d = c.d_model;
  e->dkv = c.d_kv;
  e->ff = c.d_ff;
  e->layers = c.num_layers;
  e->heads = c.num_heads;
  e->inner = c.num_heads * c.d_kv;
  e->P = c.patch_size;
  e->Q = c.num_quantiles;
  e->reg = c.use_reg_token ? 1 : 0;
  e->eps = c.layer_norm_eps;
  e->theta = c.rope_theta;
  e->op = op_of_precision(precision);
  {
    const char* v = std::getenv("JC_FOLD_NORM");
    // the producing epilogues sum x² per 64-column unit of x: a d_model that is not a multiple of 64 keeps
    // the norm kernels
    e->fold_norms = op_is_16bit(e->op) && !(v && v[0] == '0') && e->d % 64 == 0;
  }
  // CpuChronos2.inverseFrequencies (chronos2/cpu/CpuChronos2.java:101-109), in float
  e->inv_freq.resize(e->dkv / 2);
  for (int i = 0; i < e->dkv / 2; ++i) {
    const float ex = static_cast<float>(2 * i) / static_cast<float>(e->dkv);
    e->inv_freq[i] = 1.0f / static_cast<float>(std::pow(static_cast<double>(c.rope_theta), static_cast<double>(ex)));
  }
  Binder binder(weights, n_weights);
  HostC2 hw;
  if (!bind(*e, binder, &hw)) return fail(JC_ERR_INVALID_ARG, binder.error());
  std::vector<int> devs = (n_devices <= 0 || !devices) ? std::vector<int>{0}
                                                       : std::vector<int>(devices, devices + n_devices);
  for (int dev : devs) {
    std::string why;
    if (!device_rt(dev, &why)) return fail(JC_ERR_NO_DEVICE, why);
    auto dv = std::make_unique<C2Device>();
    dv->device = dev;
    cudaSetDevice(dev);
    if (cudaStreamCreateWithFlags(&dv->stream, cudaStreamNonBlocking) != cudaSuccess ||
        cudaMalloc(&dv->err, sizeof(uint32_t)) != cudaSuccess || cudaMemset(dv->err, 0, sizeof(uint32_t)) != cudaSuccess ||
        cudaEventCreateWithFlags(&dv->ev_in, cudaEventDisableTiming) != cudaSuccess ||
        cudaEventCreateWithFlags(&dv->ev_out, cudaEventDisableTiming) != cudaSuccess)
      return fail_cuda(cudaGetLastError(), "engine device setup");
    std::string err;
    if (!upload(*e, hw, *dv, &err)) return fail(JC_ERR_OOM, err);
    dv->slot = static_cast<int>(e->devs.size());
    e->devs.push_back(std::move(dv));
  }
  *out = e.release();
  return JC_OK;
}

jc_status jc_forward_chronos2(jc_engine* engine, const jc_chronos2_block* block, float* raw_out) {
  clear_error();
  if (!engine || engine->family != 2) return fail(JC_ERR_INVALID_ARG, "not a Chronos-2 engine");
  auto* e = static_cast<Chronos2Engine*>(engine);
  if (!raw_out) return fail(JC_ERR_INVALID_ARG, "null output");
  jc_status st = check_block(block, true);
  if (st != JC_OK) return st;
  std::lock_guard<std::mutex> lk(e->mu);
  const int parts = std::min<int>(static_cast<int>(e->devs.size()), block->rows);
  std::vector<int> cuts = shard_rows(block->rows, block->group_start, block->group_end, parts);
  std::vector<jc_status> status(parts, JC_OK);
  std::vector<std::string> errs(parts);
  auto work = [&](int i) {
    if (cuts[i + 1] > cuts[i])
      status[i] = run_shard(*e, *e->devs[i], block, cuts[i], cuts[i + 1], raw_out, true, nullptr, &errs[i]);
  };
  if (parts == 1) {
    work(0);
  } else {
    std::vector<std::thread> th;
    for (int i = 0; i < parts; ++i) th.emplace_back(work, i);
    for (auto& t : th) t.join();
  }
  for (int i = 0; i < parts; ++i)
    if (status[i] != JC_OK) return fail(status[i], "slot " + std::to_string(i) + " (GPU " + std::to_string(e->devs[i]->device) + "): " + errs[i]);
  return JC_OK;
}

jc_status jc_forward_chronos2_device(jc_engine* engine, int slot, const jc_chronos2_block* block, float* raw_out,
                                     void* stream) {
  clear_error();
  if (!engine || engine->family != 2) return fail(JC_ERR_INVALID_ARG, "not a Chronos-2 engine");
  auto* e = static_cast<Chronos2Engine*>(engine);
  if (slot < 0 || slot >= static_cast<int>(e->devs.size())) return fail(JC_ERR_INVALID_ARG, "slot out of range");
  if (!raw_out) return fail(JC_ERR_INVALID_ARG, "null output");
  jc_status st = check_block(block, false);
  if (st != JC_OK) return st;
  std::lock_guard<std::mutex> lk(e->mu);
  std::string err;
  st = run_shard(*e, *e->devs[slot], block, 0, block->rows, raw_out, false, static_cast<cudaStream_t>(stream), &err);
  return st == JC_OK ? JC_OK : fail(st, err);
}

jc_status jc_forecast_chronos2(jc_engine* engine, const jc_chronos2_window* block, float* quantiles_out) {
  clear_error();
  if (!engine || engine->family != 2) return fail(JC_ERR_INVALID_ARG, "not a Chronos-2 engine");
  auto* e = static_cast<Chronos2Engine*>(engine);
  if (!quantiles_out) return fail(JC_ERR_INVALID_ARG, "null output");
  jc_status st = check_window(block, true);
  if (st != JC_OK) return st;
  const jc_chronos2_block* lay = &block->layout;
  std::lock_guard<std::mutex> lk(e->mu);
  const int parts = std::min<int>(static_cast<int>(e->devs.size()), lay->rows);
  std::vector<int> cuts = shard_rows(lay->rows, lay->group_start, lay->group_end, parts);
  std::vector<jc_status> status(parts, JC_OK);
  std::vector<std::string> errs(parts);
  auto work = [&](int i) {
    if (cuts[i + 1] > cuts[i])
      status[i] = run_shard(*e, *e->devs[i], lay, cuts[i], cuts[i + 1], quantiles_out, true, nullptr, &errs[i], block);
  };
  if (parts == 1) {
    work(0);
  } else {
    std::vector<std::thread> th;
    for (int i = 0; i < parts; ++i) th.emplace_back(work, i);
    for (auto& t : th) t.join();
  }
  for (int i = 0; i < parts; ++i)
    if (status[i] != JC_OK) return fail(status[i], "slot " + std::to_string(i) + " (GPU " + std::to_string(e->devs[i]->device) + "): " + errs[i]);
  return JC_OK;
}

jc_status jc_forecast_chronos2_device(jc_engine* engine, int slot, const jc_chronos2_window* block,
                                      float* quantiles_out, void* stream) {
  clear_error();
  if (!engine || engine->family != 2) return fail(JC_ERR_INVALID_ARG, "not a Chronos-2 engine");
  auto* e = static_cast<Chronos2Engine*>(engine);
  if (slot < 0 || slot >= static_cast<int>(e->devs.size())) return fail(JC_ERR_INVALID_ARG, "slot out of range");
  if (!quantiles_out) return fail(JC_ERR_INVALID_ARG, "null output");
  jc_status st = check_window(block, false);
  if (st != JC_OK) return st;
  std::lock_guard<std::mutex> lk(e->mu);
  std::string err;
  st = run_shard(*e, *e->devs[slot], &block->layout, 0, block->layout.rows, quantiles_out, false,
                 static_cast<cudaStream_t>(stream), &err, block);
  return st == JC_OK ? JC_OK : fail(st, err);
}

}  // extern "C"
