// The Timestral forward on B200: weights bound by checkpoint name, rearranged and converted once
// per GPU; one plan (activation buffers + CUDA graph) per block shape; every linear layer a
// tcgen05 GEMM with its elementwise work fused into the epilogue:
//
//   patch embedding   hidden (bias, SiLU) → output (bias, written into the token rows of x)
//                     → residual (bias, += x)
//   per attention     RMSNorm → q|k|v|gate GEMM (RoPE on q and k, sigmoid on the gate)
//                     → attention (gate multiplied in) → output GEMM (+= x)
//   per MLP           RMSNorm → w12 GEMM (SwiGLU pairs) → w3 GEMM (+= x)
//   head              RMSNorm of the decoder tokens → hidden (SiLU) → output → residual (+=)
//
// This replaces TimestralForward's task graph (timestral/tornado/TimestralForward.java:298-394),
// its cuBLAS dispatch with separate bias/activation passes (:404-499) and the companion kernels of
// TimestralKernels; the arithmetic is CpuTimestral.predictBlock's (timestral/cpu/CpuTimestral.java:
// 127-188) between BlockPrep.of and BlockPrep.finish.
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

struct TsAttn {
  bool time = true, gated = true;
  float* norm = nullptr;
  DevLinear qkvg;  // [3d (+ d gate), d]: q|k|v heads-major, then the gate rows
  DevLinear wo;
};

struct TsLayer {
  std::vector<TsAttn> attns;
  float* mlp_norm = nullptr;
  DevLinear w12;  // [2F, d], SiLU and linear halves interleaved in 32-row groups
  DevLinear w3;
};

struct TsWeights {
  // the patch embedding: hidden [4d, 2P]; output and residual as one linear over [SiLU(hidden) | tokens]:
  // [d, 4d + 2P] = [W_out | W_res], bias b_out + b_res
  DevLinear emb_h, emb_or;
  float* forecast_query = nullptr;
  std::vector<TsLayer> layers;
  float* out_norm = nullptr;
  DevLinear head_h, head_o, head_r;
};

struct TsPlan {
  int rows = 0, enc = 0, h = 0, ll = 0, cov = 0;
  DeviceMem mem;
  float* tok_f32 = nullptr;
  OpBuf tok, emb_h, hn, att, act, dec, head_h;
  float* x = nullptr;
  void* qkv = nullptr;
  void* gate = nullptr;
  float* raw = nullptr;
  float* rowsq = nullptr;  // the folded norms' Σx² per row and 64-column unit [T, d / 64]
  int *pos = nullptr, *key_valid = nullptr, *known = nullptr, *role = nullptr, *gs = nullptr, *ge = nullptr;
  float* table = nullptr;
  float* rope_pack = nullptr;  // the table's rotating pairs packed per position (rope_dim / 2 ≤ 16), or null
  GraphRunner graph;
  std::vector<int> h_pos, h_gs, h_ge;  // host staging of the transformed integer inputs
  // the host ends on the device (jc_forecast_timestral), allocated on first use: per-patch frames and
  // asinh flags, and for host calls the window and its flags staged in HBM
  DeviceMem ends_mem, stage_mem;
  float2* frame = nullptr;
  uint8_t* row_asinh = nullptr;
  float* win = nullptr;
  uint8_t* obs = nullptr;
};

struct TsDevice : DeviceSlot {
  TsWeights w;
  std::list<std::unique_ptr<TsPlan>> plans;  // most recently used first
  Profiler prof;
  cudaEvent_t ev_in = nullptr, ev_out = nullptr;  // chain a caller's stream to the engine stream
  ~TsDevice() {
    if (ev_in) cudaEventDestroy(ev_in);
    if (ev_out) cudaEventDestroy(ev_out);
  }
};

struct TimestralEngine : jc_engine {
  int P = 0, d = 0, heads = 0, dh = 0, F = 0, Q = 0, rope_dim = 0;
  float theta = 0, partial = 0, eps = 0;
  int op = kOpBF16;
  // The 16-bit modes fold the attention and MLP RMSNorms into the GEMMs around them: the GEMM that writes the
  // residual stream x also writes x's 16-bit copy and its Σx² per 64-column unit, and the next GEMM, whose W
  // carries the norm's weights, scales each output row by 1 / sqrt(Σx² / d + eps). JC_FOLD_NORM=0 in the
  // environment keeps the standalone RMSNorm kernel (for comparisons).
  bool fold_norms = false;
  std::vector<int> kinds;
  std::vector<float> inv_freq;
  std::vector<std::unique_ptr<TsDevice>> devs;

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

  // q|k|v and the gate: 16-bit in the 16-bit modes, FP32 otherwise (attention then runs on FP32 inputs)
  int qkv_out_kind() const { return op == kOpBF16 ? kOutBF16 : op == kOpF16 ? kOutF16 : kOutF32; }
  size_t qkv_esize() const { return op_is_16bit(op) ? 2 : 4; }
};

// ---- weight binding and packing ---------------------------------------------------------------

// TimestralWeights.qkv: row (s·heads + h)·dh + e of the result is stored row s·D + e·heads + h.
std::vector<float> qkv_heads_major(const float* src, int d, int heads, int dh) {
  std::vector<float> dst(static_cast<size_t>(3) * d * d);
  for (int s = 0; s < 3; ++s)
    for (int h = 0; h < heads; ++h)
      for (int e = 0; e < dh; ++e)
        std::memcpy(&dst[(static_cast<size_t>(s) * d + h * dh + e) * d],
                    src + (static_cast<size_t>(s) * d + e * heads + h) * d, sizeof(float) * d);
  return dst;
}

// w12 [2F, d] stored gate half first (TimestralWeights.mlpUp swaps the halves so SiLU applies to
// stored rows F..2F). Packed for the SwiGLU epilogue: rows 64u..64u+31 are SiLU rows F+32u.., rows
// 64u+32.. are linear rows 32u..
std::vector<float> swiglu_interleave(const float* src, int F, int d) {
  std::vector<float> dst(static_cast<size_t>(2) * F * d);
  for (int u = 0; u < F / 32; ++u)
    for (int i = 0; i < 32; ++i) {
      std::memcpy(&dst[(static_cast<size_t>(64) * u + i) * d], src + (static_cast<size_t>(F) + 32 * u + i) * d,
                  sizeof(float) * d);
      std::memcpy(&dst[(static_cast<size_t>(64) * u + 32 + i) * d], src + (static_cast<size_t>(32) * u + i) * d,
                  sizeof(float) * d);
    }
  return dst;
}

struct HostTs {
  const float *emb_hw, *emb_hb, *emb_ow, *emb_ob, *emb_rw, *emb_rb, *fq, *out_norm, *head_hw, *head_ow, *head_rw;
  struct A {
    bool time, gated;
    const float *norm, *wqkv, *gate, *wo;
  };
  struct L {
    std::vector<A> attns;
    const float *mlp_norm, *w12, *w3;
  };
  std::vector<L> layers;
};

bool bind_weights(const TimestralEngine& e, const jc_timestral_desc& desc, Binder& b, HostTs* hw) {
  const int d = e.d, p = e.P, F = e.F, Q = e.Q;
  const std::string pe = "representation.patch_proj.";
  hw->emb_hw = b.take(pe + "hidden_layer.weight", {4LL * d, 2LL * p});
  hw->emb_hb = b.take(pe + "hidden_layer.bias", {4LL * d});
  hw->emb_ow = b.take(pe + "output_layer.weight", {d, 4LL * d});
  hw->emb_ob = b.take(pe + "output_layer.bias", {d});
  hw->emb_rw = b.take(pe + "residual_layer.weight", {d, 2LL * p});
  hw->emb_rb = b.take(pe + "residual_layer.bias", {d});
  hw->fq = b.take("representation.forecast_query", {d});
  for (int i = 0; i < desc.num_layers; ++i) {
    const std::string s = "transformer.layers." + std::to_string(i);
    HostTs::L L;
    const int kind = desc.layer_kinds[i];
    std::vector<bool> axes;
    if (kind == JC_LAYER_TIME) axes = {true};
    if (kind == JC_LAYER_VARIATE) axes = {false};
    if (kind == JC_LAYER_TIME_VARIATE) axes = {true, false};
    if (kind == JC_LAYER_VARIATE_TIME) axes = {false, true};
    for (size_t a = 0; a < axes.size(); ++a) {
      HostTs::A A;
      A.time = axes[a];
      A.gated = axes[a] ? desc.time_attn_gate : desc.variate_attn_gate;
      const std::string pa = s + ".attns." + std::to_string(a);
      A.norm = b.take(s + ".attn_norms." + std::to_string(a) + ".scale", {d});
      A.wqkv = b.take(pa + ".wQKV.weight", {3LL * d, d});
      A.gate = A.gated ? b.take(pa + "._gate.weight", {d, d}) : nullptr;
      A.wo = b.take(pa + ".wO.weight", {d, d});
      L.attns.push_back(A);
    }
    L.mlp_norm = b.take(s + ".mlp_norm.scale", {d});
    L.w12 = b.take(s + ".mlp.w12.weight", {2LL * F, d});
    L.w3 = b.take(s + ".mlp.w3.weight", {d, F});
    hw->layers.push_back(L);
  }
  hw->out_norm = b.take("transformer.out_norm.scale", {d});
  const std::string hp = "head.projection.";
  hw->head_hw = b.take(hp + "hidden_layer.weight", {4LL * d, d});
  hw->head_ow = b.take(hp + "output_layer.weight", {static_cast<long long>(p) * Q, 4LL * d});
  hw->head_rw = b.take(hp + "residual_layer.weight", {static_cast<long long>(p) * Q, d});
  return b.require_all_bound();
}

// W[:, k] *= g[k]: a folded RMSNorm's weights g moved into the next GEMM's W [rows, cols].
void scale_columns(std::vector<float>& w, int cols, const float* g) {
  for (size_t i = 0; i < w.size(); ++i) w[i] *= g[i % cols];
}

bool upload_weights(TimestralEngine& e, const HostTs& hw, TsDevice& dv, std::string* err) {
  const int d = e.d, p = e.P, F = e.F, Q = e.Q, op = e.op;
  DeviceMem& m = dv.weights;
  TsWeights& w = dv.w;
  if (!upload_linear(m, op, hw.emb_hw, hw.emb_hb, 2 * p, 4 * d, &w.emb_h, err)) return false;
  {
    // output(SiLU(hidden)) + residual(tokens) as one GEMM over the concatenated K
    const int K = 4 * d + 2 * p;
    std::vector<float> wor(static_cast<size_t>(d) * K), bor(d);
    for (int o = 0; o < d; ++o) {
      std::memcpy(wor.data() + static_cast<size_t>(o) * K, hw.emb_ow + static_cast<size_t>(o) * 4 * d,
                  sizeof(float) * 4 * d);
      std::memcpy(wor.data() + static_cast<size_t>(o) * K + 4 * d, hw.emb_rw + static_cast<size_t>(o) * 2 * p,
                  sizeof(float) * 2 * p);
      bor[o] = hw.emb_ob[o] + hw.emb_rb[o];
    }
    if (!upload_linear(m, op, wor.data(), bor.data(), K, d, &w.emb_or, err)) return false;
  }
  if (!(w.forecast_query = upload_f32(m, hw.fq, d, err))) return false;
  for (const auto& L : hw.layers) {
    TsLayer tl;
    for (const auto& A : L.attns) {
      TsAttn ta;
      ta.time = A.time;
      ta.gated = A.gated;
      if (!(ta.norm = upload_f32(m, A.norm, d, err))) return false;
      std::vector<float> q = qkv_heads_major(A.wqkv, d, e.heads, e.dh);
      if (A.gated) q.insert(q.end(), A.gate, A.gate + static_cast<size_t>(d) * d);
      if (e.fold_norms) scale_columns(q, d, A.norm);
      if (!upload_linear(m, op, q.data(), nullptr, d, A.gated ? 4 * d : 3 * d, &ta.qkvg, err) ||
          !upload_linear(m, op, A.wo, nullptr, d, d, &ta.wo, err))
        return false;
      tl.attns.push_back(std::move(ta));
    }
    if (!(tl.mlp_norm = upload_f32(m, L.mlp_norm, d, err))) return false;
    std::vector<float> up = swiglu_interleave(L.w12, F, d);
    if (e.fold_norms) scale_columns(up, d, L.mlp_norm);
    if (!upload_linear(m, op, up.data(), nullptr, d, 2 * F, &tl.w12, err) ||
        !upload_linear(m, op, L.w3, nullptr, F, d, &tl.w3, err))
      return false;
    w.layers.push_back(std::move(tl));
  }
  if (!(w.out_norm = upload_f32(m, hw.out_norm, d, err))) return false;
  return upload_linear(m, op, hw.head_hw, nullptr, d, 4 * d, &w.head_h, err) &&
         upload_linear(m, op, hw.head_ow, nullptr, 4 * d, p * Q, &w.head_o, err) &&
         upload_linear(m, op, hw.head_rw, nullptr, d, p * Q, &w.head_r, err);
}

// ---- plans --------------------------------------------------------------------------------------

std::unique_ptr<TsPlan> make_plan(const TimestralEngine& e, int rows, int enc, int h, int ll, int cov) {
  auto p = std::make_unique<TsPlan>();
  p->rows = rows;
  p->enc = enc;
  p->h = h;
  p->ll = ll;
  p->cov = cov;
  const int n = enc + h, d = e.d, op = e.op;
  const long long T = static_cast<long long>(rows) * n, encT = static_cast<long long>(rows) * enc,
                  decT = static_cast<long long>(rows) * h;
  DeviceMem& m = p->mem;
  bool ok = (p->tok_f32 = static_cast<float*>(m.alloc(sizeof(float) * encT * 2 * e.P))) &&
            alloc_op(m, op, encT, 2 * e.P, &p->tok) && alloc_op(m, op, encT, 4 * d + 2 * e.P, &p->emb_h) &&
            (p->x = static_cast<float*>(m.alloc(sizeof(float) * T * d))) && alloc_op(m, op, T, d, &p->hn) &&
            (p->qkv = m.alloc(e.qkv_esize() * T * 3 * d)) && (p->gate = m.alloc(e.qkv_esize() * T * d)) &&
            alloc_op(m, op, T, d, &p->att) && alloc_op(m, op, T, e.F, &p->act) && alloc_op(m, op, decT, d, &p->dec) &&
            alloc_op(m, op, decT, 4 * d, &p->head_h) &&
            (p->raw = static_cast<float*>(m.alloc(sizeof(float) * decT * e.P * e.Q))) &&
            (!e.fold_norms || (p->rowsq = static_cast<float*>(m.alloc(sizeof(float) * T * (d / 64))))) &&
            (p->pos = static_cast<int*>(m.alloc(sizeof(int) * T))) &&
            (p->key_valid = static_cast<int*>(m.alloc(sizeof(int) * encT))) &&
            (p->known = static_cast<int*>(m.alloc(sizeof(int) * rows))) &&
            (p->role = static_cast<int*>(m.alloc(sizeof(int) * rows))) &&
            (p->gs = static_cast<int*>(m.alloc(sizeof(int) * rows))) &&
            (p->ge = static_cast<int*>(m.alloc(sizeof(int) * rows))) &&
            (p->table = static_cast<float*>(m.alloc(sizeof(float) * (2 * enc + h) * e.dh))) &&
            (e.rope_dim / 2 > 16 || (p->rope_pack = static_cast<float*>(m.alloc(sizeof(float) * (2 * enc + h) * 32))));
  if (!ok) {
    cudaGetLastError();
    return nullptr;
  }
  // RoPE table over every position a token can have, (−enc, enc + h), row p ↔ position p − enc,
  // as TimestralForward.Plan.run builds it (TimestralForward.java:600-608)
  const int half = e.dh / 2;
  std::vector<float> table(static_cast<size_t>(2 * enc + h) * e.dh, 0.0f);
  for (int q = 0; q < 2 * enc + h; ++q) {
    const float position = static_cast<float>(q - enc);
    for (int k = 0; k < half; ++k) {
      const float a = position * e.inv_freq[k];
      table[static_cast<size_t>(q) * e.dh + k] = static_cast<float>(std::cos(static_cast<double>(a)));
      table[static_cast<size_t>(q) * e.dh + half + k] = static_cast<float>(std::sin(static_cast<double>(a)));
    }
  }
  if (cudaMemcpy(p->table, table.data(), sizeof(float) * table.size(), cudaMemcpyHostToDevice) != cudaSuccess)
    return nullptr;
  if (p->rope_pack) {
    // per position: cos of the rotating pairs 0 .. rope_dim / 2 − 1 at 0 .., their sin at 16 .. (zeros elsewhere)
    const int rp = e.rope_dim / 2;
    std::vector<float> pack(static_cast<size_t>(2 * enc + h) * 32, 0.0f);
    for (int q = 0; q < 2 * enc + h; ++q)
      for (int k = 0; k < rp; ++k) {
        pack[static_cast<size_t>(q) * 32 + k] = table[static_cast<size_t>(q) * e.dh + k];
        pack[static_cast<size_t>(q) * 32 + 16 + k] = table[static_cast<size_t>(q) * e.dh + half + k];
      }
    if (cudaMemcpy(p->rope_pack, pack.data(), sizeof(float) * pack.size(), cudaMemcpyHostToDevice) != cudaSuccess)
      return nullptr;
  }
  // every row starts as a valid, independent dummy series (zero tokens, positions 0 .., all keys valid, its
  // own group), so rows past a call's own (bucket padding) compute harmlessly and never reach a real row
  {
    std::vector<int> pos(static_cast<size_t>(T)), ones(static_cast<size_t>(encT), 1), gs(rows), ge(rows);
    for (long long i = 0; i < T; ++i) pos[static_cast<size_t>(i)] = static_cast<int>(i % n) + enc;
    for (int i = 0; i < rows; ++i) gs[i] = i, ge[i] = i + 1;
    if (cudaMemset(p->tok_f32, 0, sizeof(float) * encT * 2 * e.P) != cudaSuccess ||
        cudaMemcpy(p->pos, pos.data(), sizeof(int) * T, cudaMemcpyHostToDevice) != cudaSuccess ||
        cudaMemcpy(p->key_valid, ones.data(), sizeof(int) * encT, cudaMemcpyHostToDevice) != cudaSuccess ||
        cudaMemset(p->known, 0, sizeof(int) * rows) != cudaSuccess ||
        cudaMemset(p->role, 0, sizeof(int) * rows) != cudaSuccess ||
        cudaMemcpy(p->gs, gs.data(), sizeof(int) * rows, cudaMemcpyHostToDevice) != cudaSuccess ||
        cudaMemcpy(p->ge, ge.data(), sizeof(int) * rows, cudaMemcpyHostToDevice) != cudaSuccess)
      return nullptr;
  }
  p->h_pos.resize(T);
  p->h_gs.resize(rows);
  p->h_ge.resize(rows);
  return p;
}

TsPlan* get_plan(TimestralEngine& e, TsDevice& dv, int rows, int enc, int h, int ll, int cov, std::string* err) {
  for (auto it = dv.plans.begin(); it != dv.plans.end(); ++it) {
    TsPlan* p = it->get();
    if (p->rows == rows && p->enc == enc && p->h == h && p->ll == ll && p->cov == cov) {
      dv.plans.splice(dv.plans.begin(), dv.plans, it);
      return p;
    }
  }
  while (static_cast<int>(dv.plans.size()) >= std::max(1, e.max_plans)) dv.plans.pop_back();
  auto p = e.take_plan_failure() ? nullptr : make_plan(e, rows, enc, h, ll, cov);
  if (!p && !dv.plans.empty()) {
    // out of memory: drop the cached plans and retry once (PlanCache.run, PlanCache.java:70-100)
    cudaStreamSynchronize(dv.stream);
    dv.plans.clear();
    p = e.take_plan_failure() ? nullptr : make_plan(e, rows, enc, h, ll, cov);
  }
  if (!p) {
    *err = "out of device memory for a plan of " + std::to_string(rows) + " rows";
    return nullptr;
  }
  dv.plans.push_front(std::move(p));
  return dv.plans.front().get();
}

// ---- the forward ----------------------------------------------------------------------------------

// One GEMM launch, timed under `name` ("gemm.<layer>") when profiling.
cudaError_t gemm(TsDevice& dv, GemmArgs& g, cudaStream_t s, const char* name) {
  dv.prof.begin(s, name, 2.0 * g.M * g.N * g.K);  // algorithmic FLOPs (the split mode runs 4 MMAs each)
  cudaError_t r = launch_gemm(g, s, dv.err);
  dv.prof.end(s);
  return r;
}

// Independent GEMMs as one grouped launch (launch_gemm_group), timed as one launch under `name`.
cudaError_t gemm_group(TsDevice& dv, GemmArgs* g, int count, cudaStream_t s, const char* name) {
  double flops = 0.0;
  for (int i = 0; i < count; ++i) flops += 2.0 * g[i].M * g[i].N * g[i].K;
  dv.prof.begin(s, name, flops);
  cudaError_t r = launch_gemm_group(g, count, s, dv.err);
  dv.prof.end(s);
  return r;
}

void set_op_out(EpiParams& ep, int op, const OpBuf& o) {
  ep.o_kind = out_of_op(op);
  ep.o_hi = o.hi;
  ep.o_lo = o.lo;
  ep.ldo = o.ld;
}

cudaError_t enqueue_forward(const TimestralEngine& e, TsDevice& dv, TsPlan& p, cudaStream_t s) {
  const int R = p.rows, E = p.enc, H = p.h, n = E + H, d = e.d, op = e.op, P2 = 2 * e.P;
  const long long T = static_cast<long long>(R) * n, encT = static_cast<long long>(R) * E,
                  decT = static_cast<long long>(R) * H;
  const TsWeights& w = dv.w;
  Profiler& prof = dv.prof;
  cudaError_t r;
#define JC_TRY(x)                   \
  do {                              \
    if ((r = (x)) != cudaSuccess) { \
      return r;                     \
    }                               \
  } while (0)

  const int out_kind = out_of_op(op);
  // the folded norms (fold_norms): a GEMM that writes x also writes its 16-bit copy into hn and Σx² per unit;
  // the GEMM that reads hn scales its rows by the norm
  const bool fold = e.fold_norms;
  auto produce = [&](GemmArgs& g) {
    if (!fold) return;
    set_op_out(g.ep, op, p.hn);
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
  // the tokens, in the operand format, for the hidden GEMM and as the last 2P columns of its output buffer
  const size_t esz = op_esize(op);
  prof.begin(s, "convert", 0);
  launch_convert(op, p.tok_f32, P2, p.tok.hi, p.tok.lo, p.tok.ld, encT, P2, s);
  launch_convert_cols(op, p.tok_f32, P2, static_cast<uint8_t*>(p.emb_h.hi) + 4 * d * esz,
                      p.emb_h.lo ? static_cast<uint8_t*>(p.emb_h.lo) + 4 * d * esz : nullptr, p.emb_h.ld, encT, P2, s);
  prof.end(s);
  // patch embedding: output(SiLU(hidden(tok))) + residual(tok), into the encoder rows of x: hidden into the first
  // 4d columns of emb_h, then one GEMM over [SiLU(hidden) | tok] with [W_out | W_res] and b_out + b_res
  GemmArgs g = gemm_args(op, p.tok, encT, w.emb_h);
  g.ep.act = kActSilu;
  set_op_out(g.ep, op, p.emb_h);
  JC_TRY(gemm(dv, g, s, "gemm.embed"));
  g = gemm_args(op, p.emb_h, encT, w.emb_or);
  g.ep.c = p.x;
  g.ep.ldc = d;
  g.ep.rg = E;
  g.ep.rg_stride = n;
  produce(g);
  JC_TRY(gemm(dv, g, s, "gemm.embed"));
  prof.begin(s, "fill", 0);
  launch_fill_rows(p.x, d, w.forecast_query, d, R, E, n, n, s);
  if (fold) launch_norm_copy_rows(p.x, d, d, out_kind, p.hn.hi, p.hn.ld, p.rowsq, R, E, n, n, s);
  prof.end(s);

  for (size_t li = 0; li < w.layers.size(); ++li) {
    const TsLayer& L = w.layers[li];
    for (const TsAttn& A : L.attns) {
      if (!fold) {
        prof.begin(s, "rmsnorm", 0);
        launch_rmsnorm(p.x, d, A.norm, d, e.eps, out_kind, p.hn.hi, p.hn.lo, p.hn.ld, T, 0, 0, 0, s);
        prof.end(s);
      }
      g = gemm_args(op, p.hn, T, A.qkvg);
      consume(g);
      g.ep.mode = kEpiQKV;
      g.ep.o_kind = e.qkv_out_kind();
      g.ep.o_hi = p.qkv;
      g.ep.ldo = 3LL * d;
      g.ep.rope_cols = A.time ? 2 * d : 0;
      g.ep.head_dim = e.dh;
      g.ep.rope_pairs = e.rope_dim / 2;  // partial rotary: the pairs past rope_dim/2 keep cos 1, sin 0
      g.ep.pos = p.pos;
      g.ep.rope_table = p.table;
      g.ep.rope_pack = p.rope_pack;
      g.ep.n_split = 3 * d;
      g.ep.g_out = p.gate;
      g.ep.ldg = d;
      g.ep.g_kind = e.qkv_out_kind();
      JC_TRY(gemm(dv, g, s, "gemm.qkvg"));
      AttnArgs a{};
      a.qkv = p.qkv;
      a.qkv_kind = e.qkv_out_kind();
      a.ld_qkv = 3LL * d;
      a.gate = A.gated ? p.gate : nullptr;
      a.gate_kind = e.qkv_out_kind();
      a.ld_gate = d;
      a.out_hi = p.att.hi;
      a.out_lo = p.att.lo;
      a.ld_out = p.att.ld;
      a.out_kind = out_kind;
      a.rows = R;
      a.n = n;
      a.enc = E;
      a.ll = p.ll;
      a.heads = e.heads;
      a.head_dim = e.dh;
      a.d = d;
      a.scale = 1.0f / std::sqrt(static_cast<float>(e.dh));
      a.key_valid = p.key_valid;
      a.known = p.known;
      a.role = p.role;
      a.group_start = p.gs;
      a.group_end = p.ge;
      a.covariates = p.cov;
      a.err = dv.err;
      prof.begin(s, "attention", 4.0 * T * n * d);
      JC_TRY(A.time ? launch_time_attention(a, s) : launch_variate_attention(a, s));
      prof.end(s);
      g = gemm_args(op, p.att, T, A.wo);
      g.ep.c = p.x;
      g.ep.ldc = d;
      g.ep.cin = p.x;
      g.ep.ldcin = d;
      g.ep.accumulate = 1;
      produce(g);
      JC_TRY(gemm(dv, g, s, "gemm.wo"));
    }
    if (!fold) {
      prof.begin(s, "rmsnorm", 0);
      launch_rmsnorm(p.x, d, L.mlp_norm, d, e.eps, out_kind, p.hn.hi, p.hn.lo, p.hn.ld, T, 0, 0, 0, s);
      prof.end(s);
    }
    g = gemm_args(op, p.hn, T, L.w12);
    consume(g);
    g.ep.mode = kEpiSwiGLU;
    set_op_out(g.ep, op, p.act);
    JC_TRY(gemm(dv, g, s, "gemm.w12"));
    g = gemm_args(op, p.act, T, L.w3);
    g.ep.c = p.x;
    g.ep.ldc = d;
    g.ep.cin = p.x;
    g.ep.ldcin = d;
    g.ep.accumulate = 1;
    if (li + 1 < w.layers.size()) produce(g);  // the last x goes to out_norm, which reads it directly
    JC_TRY(gemm(dv, g, s, "gemm.w3"));
  }
  // out_norm on the decoder tokens only (the head reads nothing else), gathered per row
  prof.begin(s, "rmsnorm", 0);
  launch_rmsnorm(p.x, d, w.out_norm, d, e.eps, out_kind, p.dec.hi, p.dec.lo, p.dec.ld, decT, H, n, E, s);
  prof.end(s);
  // the head: output(SiLU(hidden(dec))) + residual(dec); hidden and residual (stored into raw) as one grouped
  // launch, then output adds into raw
  const int pq = e.P * e.Q;
  GemmArgs gh[2] = {gemm_args(op, p.dec, decT, w.head_h), gemm_args(op, p.dec, decT, w.head_r)};
  gh[0].ep.act = kActSilu;
  set_op_out(gh[0].ep, op, p.head_h);
  gh[1].ep.c = p.raw;
  gh[1].ep.ldc = pq;
  JC_TRY(gemm_group(dv, gh, 2, s, "gemm.head"));
  g = gemm_args(op, p.head_h, decT, w.head_o);
  g.ep.c = p.raw;
  g.ep.ldc = pq;
  g.ep.cin = p.raw;
  g.ep.ldcin = pq;
  g.ep.accumulate = 1;
  JC_TRY(gemm(dv, g, s, "gemm.head"));
#undef JC_TRY
  return cudaGetLastError();
}

// Validates one block's host or device-independent fields.
jc_status check_block(const TimestralEngine& e, const jc_timestral_block* b, bool host, bool tokens = true) {
  if (!b) return fail(JC_ERR_INVALID_ARG, "null block");
  if (b->rows < 1) return fail(JC_ERR_INVALID_ARG, "rows must be >= 1");
  if (b->encoder < 1) return fail(JC_ERR_INVALID_ARG, "encoder tokens must be >= 1");
  if (b->horizon < 1) return fail(JC_ERR_INVALID_ARG, "horizon patches must be >= 1, got " + std::to_string(b->horizon));
  if (b->context_patches < 1 || b->context_patches > b->encoder)
    return fail(JC_ERR_INVALID_ARG, "context patches must be in [1, encoder]");
  if ((tokens && !b->tokens) || !b->positions || !b->key_valid || !b->known || !b->role || !b->group_start ||
      !b->group_end)
    return fail(JC_ERR_INVALID_ARG, "null block field");
  if (host) {
    for (int i = 0; i < b->rows; ++i) {
      const int s = b->group_start[i], t = b->group_end[i];
      if (s < 0 || s > i || t <= i || t > b->rows || b->group_start[s] != s || b->group_end[s] != t)
        return fail(JC_ERR_INVALID_ARG, "rows of a series are not contiguous (row " + std::to_string(i) + ")");
    }
  }
  (void)e;
  return JC_OK;
}

// Copies rows [r0, r1) of a block into the plan's device inputs. Positions become RoPE table
// rows (position + encoder) and series ranges become shard-relative. `kind` is HostToDevice for
// host blocks and DeviceToDevice for device blocks (then the integer transforms run on the GPU).
cudaError_t upload_shard(const jc_timestral_block* b, int r0, int r1, TsPlan& p, int two_p, cudaStream_t s,
                         bool host, bool tokens) {
  const int rows = r1 - r0, E = b->encoder, n = E + b->horizon;
  const long long T = static_cast<long long>(rows) * n;
  const cudaMemcpyKind kind = host ? cudaMemcpyHostToDevice : cudaMemcpyDeviceToDevice;
  cudaError_t e = cudaSuccess;
  if (tokens)
    e = cudaMemcpyAsync(p.tok_f32, b->tokens + static_cast<long long>(r0) * E * two_p,
                        sizeof(float) * rows * E * two_p, kind, s);
  if (e == cudaSuccess)
    e = cudaMemcpyAsync(p.key_valid, b->key_valid + static_cast<long long>(r0) * E, sizeof(int) * rows * E, kind, s);
  if (e == cudaSuccess) e = cudaMemcpyAsync(p.known, b->known + r0, sizeof(int) * rows, kind, s);
  if (e == cudaSuccess) e = cudaMemcpyAsync(p.role, b->role + r0, sizeof(int) * rows, kind, s);
  if (e != cudaSuccess) return e;
  if (host) {
    for (long long i = 0; i < T; ++i) p.h_pos[i] = b->positions[static_cast<long long>(r0) * n + i] + E;
    for (int i = 0; i < rows; ++i) {
      p.h_gs[i] = b->group_start[r0 + i] - r0;
      p.h_ge[i] = b->group_end[r0 + i] - r0;
    }
    e = cudaMemcpyAsync(p.pos, p.h_pos.data(), sizeof(int) * T, cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess) e = cudaMemcpyAsync(p.gs, p.h_gs.data(), sizeof(int) * rows, cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess) e = cudaMemcpyAsync(p.ge, p.h_ge.data(), sizeof(int) * rows, cudaMemcpyHostToDevice, s);
    return e;
  }
  launch_add_i32(b->positions + static_cast<long long>(r0) * n, p.pos, T, E, s);
  launch_add_i32(b->group_start + r0, p.gs, rows, -r0, s);
  launch_add_i32(b->group_end + r0, p.ge, rows, -r0, s);
  return cudaGetLastError();
}

// The host ends' buffers of a plan, sized for its rows: frames and asinh flags always, the
// staged window and flags only for host calls. False when device memory runs out.
bool ensure_ends(TsPlan& p, int P, bool host) {
  if (!p.frame) {
    if (!(p.frame = static_cast<float2*>(p.ends_mem.alloc(sizeof(float2) * p.rows * p.enc))) ||
        !(p.row_asinh = static_cast<uint8_t*>(p.ends_mem.alloc(p.rows)))) {
      cudaGetLastError();
      p.ends_mem.release();
      p.frame = nullptr;
      p.row_asinh = nullptr;
      return false;
    }
  }
  if (host && !p.win) {
    const long long n = static_cast<long long>(p.rows) * p.enc * P;
    if (!(p.win = static_cast<float*>(p.stage_mem.alloc(sizeof(float) * n))) ||
        !(p.obs = static_cast<uint8_t*>(p.stage_mem.alloc(n)))) {
      cudaGetLastError();
      p.stage_mem.release();
      p.win = nullptr;
      p.obs = nullptr;
      return false;
    }
  }
  return true;
}

TsEnds ends_params(const TimestralEngine& e, const jc_timestral_window* w, int rows) {
  TsEnds ep;
  ep.rows = rows;
  ep.enc = w->layout.encoder;
  ep.P = e.P;
  ep.ll = w->layout.context_patches;
  ep.Q = e.Q;
  ep.median = w->median;
  ep.use_asinh = w->use_asinh ? 1 : 0;
  ep.min_scale = w->minimum_scale;
  for (int i = 0; i < e.Q; ++i) ep.qscale[i] = w->quantile_scale[i];
  return ep;
}

// Runs rows [r0, r1) of `b` on one GPU; raw_out points at the block's first row's outputs. With
// `ends` (whose layout is `b`) the window replaces the tokens and raw_out receives the finished
// quantiles.
jc_status run_shard(TimestralEngine& e, TsDevice& dv, const jc_timestral_block* b, int r0, int r1, float* raw_out,
                    bool host, cudaStream_t stream, std::string* err, const jc_timestral_window* ends = nullptr) {
  if (e.take_slot_failure(dv.slot)) {  // injected (engine option fail_slot), before any device work
    *err = "injected shard failure (engine option fail_slot)";
    return JC_ERR_CUDA;
  }
  if (cudaSetDevice(dv.device) != cudaSuccess) {
    *err = "cannot select device " + std::to_string(dv.device);
    return JC_ERR_CUDA;
  }
  // always run on the engine's own stream (graph capture needs a non-legacy stream); a device
  // caller's stream is chained in and out with events
  cudaStream_t s = dv.stream;
  if (!host) {
    if (cudaEventRecord(dv.ev_in, stream) != cudaSuccess || cudaStreamWaitEvent(s, dv.ev_in, 0) != cudaSuccess) {
      *err = "cannot order the caller's stream before the forward";
      return JC_ERR_CUDA;
    }
  }
  const int prows = e.buckets ? bucket_rows(r1 - r0) : r1 - r0;  // the plan's rows ≥ this shard's
  TsPlan* p = get_plan(e, dv, prows, b->encoder, b->horizon, b->context_patches, b->covariates, err);
  if (!p) return JC_ERR_OOM;
  cudaError_t ce = upload_shard(b, r0, r1, *p, 2 * e.P, s, host, ends == nullptr);
  if (ce != cudaSuccess) {
    *err = std::string("upload: ") + cudaGetErrorString(ce);
    return JC_ERR_CUDA;
  }
  dv.prof.on = e.profile;
  TsEnds ep;
  if (ends) {
    // BlockPrep.of on the GPU: the scaler's frames, then the tokens, into the plan's token rows
    if (!ensure_ends(*p, e.P, host)) {
      *err = "out of device memory for the host ends of a plan of " + std::to_string(p->rows) + " rows";
      return JC_ERR_OOM;
    }
    const long long W = static_cast<long long>(b->encoder) * e.P, n = static_cast<long long>(r1 - r0) * W;
    const float* win = ends->window + r0 * W;
    const uint8_t* obs = ends->observed + r0 * W;
    if (host) {
      ce = cudaMemcpyAsync(p->win, win, sizeof(float) * n, cudaMemcpyHostToDevice, s);
      if (ce == cudaSuccess) ce = cudaMemcpyAsync(p->obs, obs, n, cudaMemcpyHostToDevice, s);
      if (ce != cudaSuccess) {
        *err = std::string("upload: ") + cudaGetErrorString(ce);
        return JC_ERR_CUDA;
      }
      win = p->win;
      obs = p->obs;
    }
    ep = ends_params(e, ends, r1 - r0);
    dv.prof.begin(s, "prep.scaler", 0);
    launch_ts_scaler(win, obs, p->known, ep, p->frame, p->row_asinh, s);
    dv.prof.end(s);
    dv.prof.begin(s, "prep.tokens", 0);
    launch_ts_tokens(win, obs, p->frame, p->row_asinh, ep, p->tok_f32, s);
    dv.prof.end(s);
    ce = cudaGetLastError();
    if (ce != cudaSuccess) {
      *err = std::string("prep: ") + cudaGetErrorString(ce);
      return JC_ERR_CUDA;
    }
  }
  TimestralEngine& ec = e;
  TsDevice& dvc = dv;
  ce = p->graph.run(s, [&](cudaStream_t st) { return enqueue_forward(ec, dvc, *p, st); }, e.use_graph && !e.profile);
  if (ce != cudaSuccess) {
    *err = std::string("forward: ") + cudaGetErrorString(ce);
    return JC_ERR_CUDA;
  }
  if (ends) {
    // BlockPrep.finish on the GPU, in place on the shard's raw outputs
    dv.prof.begin(s, "finish", 0);
    launch_ts_finish(p->raw, p->frame, ep, b->horizon * e.P, s);
    dv.prof.end(s);
    ce = cudaGetLastError();
    if (ce != cudaSuccess) {
      *err = std::string("finish: ") + cudaGetErrorString(ce);
      return JC_ERR_CUDA;
    }
  }
  const size_t nraw = static_cast<size_t>(r1 - r0) * b->horizon * e.P * e.Q;
  ce = cudaMemcpyAsync(raw_out + static_cast<size_t>(r0) * b->horizon * e.P * e.Q, p->raw, sizeof(float) * nraw,
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

jc_status check_window(const TimestralEngine& e, const jc_timestral_window* w, bool host) {
  if (!w) return fail(JC_ERR_INVALID_ARG, "null block");
  if (!w->window || !w->observed || !w->quantile_scale) return fail(JC_ERR_INVALID_ARG, "null window field");
  if (e.Q > kMaxQuantiles)
    return fail(JC_ERR_UNSUPPORTED_SHAPE, "the host ends on the device support at most " +
                                              std::to_string(kMaxQuantiles) + " quantiles");
  if (w->median < 0 || w->median >= e.Q) return fail(JC_ERR_INVALID_ARG, "median index out of range");
  return check_block(e, &w->layout, host, false);
}

}  // namespace
}  // namespace jc

using namespace jc;

extern "C" {

jc_status jc_engine_create_timestral(const jc_timestral_desc* desc, const jc_tensor_view* weights, int n_weights,
                                     const int* devices, int n_devices, jc_precision precision, jc_engine** out) {
  clear_error();
  if (!out) return fail(JC_ERR_INVALID_ARG, "null engine out-pointer");
  *out = nullptr;
  if (!desc || !weights || n_weights < 1) return fail(JC_ERR_INVALID_ARG, "null description or weights");
  if (!valid_precision_code(precision)) return fail(JC_ERR_INVALID_ARG, "unknown precision");
  const jc_timestral_desc& c = *desc;
  if (c.patch_size < 1 || c.d_model < 1 || c.num_heads < 1 || c.d_model % c.num_heads != 0)
    return fail(JC_ERR_INVALID_ARG, "d_model " + std::to_string(c.d_model) + " is not divisible by num_heads " +
                                        std::to_string(c.num_heads));
  if (c.num_layers < 0 || (c.num_layers > 0 && !c.layer_kinds)) return fail(JC_ERR_INVALID_ARG, "layer kinds");
  for (int i = 0; i < c.num_layers; ++i)
    if (c.layer_kinds[i] < JC_LAYER_TIME || c.layer_kinds[i] > JC_LAYER_VARIATE_TIME)
      return fail(JC_ERR_INVALID_ARG, "unknown layer kind " + std::to_string(c.layer_kinds[i]));
  if (c.num_quantiles < 1 || c.mlp_hidden_dim < 1) return fail(JC_ERR_INVALID_ARG, "quantiles / mlp width");
  auto e = std::make_unique<TimestralEngine>();
  e->family = 1;
  e->P = c.patch_size;
  e->d = c.d_model;
  e->heads = c.num_heads;
  e->dh = c.d_model / c.num_heads;
  e->F = c.mlp_hidden_dim;
  e->Q = c.num_quantiles;
  e->theta = c.rope_theta;
  e->partial = c.rope_partial_factor;
  e->eps = c.norm_eps;
  e->rope_dim = static_cast<int>(e->dh * c.rope_partial_factor);
  e->op = op_of_precision(precision);
  {
    const char* v = std::getenv("JC_FOLD_NORM");
    e->fold_norms = op_is_16bit(e->op) && !(v && v[0] == '0');
  }
  if (e->rope_dim <= 0 || e->rope_dim % 2 != 0)
    return fail(JC_ERR_INVALID_ARG, "rope_partial_factor gives rope_dim " + std::to_string(e->rope_dim));
  if (e->dh != 64)
    return fail(JC_ERR_UNSUPPORTED_SHAPE, "unsupported attention head width " + std::to_string(e->dh) +
                                              " (this engine supports 64)");
  if (e->F % 32 != 0) return fail(JC_ERR_UNSUPPORTED_SHAPE, "mlp_hidden_dim must be a multiple of 32");
  // CpuTimestral.inverseFrequencies (timestral/cpu/CpuTimestral.java:108-116), in float
  e->inv_freq.assign(e->dh / 2, 0.0f);
  for (int i = 0; i < e->rope_dim / 2; ++i) {
    const float ex = static_cast<float>(2 * i) / static_cast<float>(e->rope_dim);
    e->inv_freq[i] = 1.0f / static_cast<float>(std::pow(static_cast<double>(c.rope_theta), static_cast<double>(ex)));
  }
  Binder binder(weights, n_weights);
  HostTs hw;
  if (!bind_weights(*e, c, binder, &hw)) return fail(JC_ERR_INVALID_ARG, binder.error());
  std::vector<int> devs;
  if (n_devices <= 0 || !devices) {
    devs.push_back(0);
  } else {
    devs.assign(devices, devices + n_devices);
  }
  for (int dev : devs) {
    std::string why;
    if (!device_rt(dev, &why)) return fail(JC_ERR_NO_DEVICE, why);
    auto dv = std::make_unique<TsDevice>();
    dv->device = dev;
    cudaSetDevice(dev);
    if (cudaStreamCreateWithFlags(&dv->stream, cudaStreamNonBlocking) != cudaSuccess ||
        cudaMalloc(&dv->err, sizeof(uint32_t)) != cudaSuccess || cudaMemset(dv->err, 0, sizeof(uint32_t)) != cudaSuccess ||
        cudaEventCreateWithFlags(&dv->ev_in, cudaEventDisableTiming) != cudaSuccess ||
        cudaEventCreateWithFlags(&dv->ev_out, cudaEventDisableTiming) != cudaSuccess)
      return fail_cuda(cudaGetLastError(), "engine device setup");
    std::string err;
    if (!upload_weights(*e, hw, *dv, &err)) return fail(JC_ERR_OOM, err);
    dv->slot = static_cast<int>(e->devs.size());
    e->devs.push_back(std::move(dv));
  }
  *out = e.release();
  return JC_OK;
}

jc_status jc_forward_timestral(jc_engine* engine, const jc_timestral_block* block, float* raw_out) {
  clear_error();
  if (!engine || engine->family != 1) return fail(JC_ERR_INVALID_ARG, "not a Timestral engine");
  auto* e = static_cast<TimestralEngine*>(engine);
  if (!raw_out) return fail(JC_ERR_INVALID_ARG, "null output");
  jc_status st = check_block(*e, block, true);
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
    if (status[i] != JC_OK)
      return fail(status[i], "slot " + std::to_string(i) + " (GPU " + std::to_string(e->devs[i]->device) + "): " + errs[i]);
  return JC_OK;
}

jc_status jc_forward_timestral_device(jc_engine* engine, int slot, const jc_timestral_block* block, float* raw_out,
                                      void* stream) {
  clear_error();
  if (!engine || engine->family != 1) return fail(JC_ERR_INVALID_ARG, "not a Timestral engine");
  auto* e = static_cast<TimestralEngine*>(engine);
  if (slot < 0 || slot >= static_cast<int>(e->devs.size())) return fail(JC_ERR_INVALID_ARG, "slot out of range");
  if (!raw_out) return fail(JC_ERR_INVALID_ARG, "null output");
  jc_status st = check_block(*e, block, false);
  if (st != JC_OK) return st;
  std::lock_guard<std::mutex> lk(e->mu);
  std::string err;
  st = run_shard(*e, *e->devs[slot], block, 0, block->rows, raw_out, false, static_cast<cudaStream_t>(stream), &err);
  return st == JC_OK ? JC_OK : fail(st, err);
}

jc_status jc_forecast_timestral(jc_engine* engine, const jc_timestral_window* block, float* quantiles_out) {
  clear_error();
  if (!engine || engine->family != 1) return fail(JC_ERR_INVALID_ARG, "not a Timestral engine");
  auto* e = static_cast<TimestralEngine*>(engine);
  if (!quantiles_out) return fail(JC_ERR_INVALID_ARG, "null output");
  jc_status st = check_window(*e, block, true);
  if (st != JC_OK) return st;
  const jc_timestral_block* lay = &block->layout;
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
    if (status[i] != JC_OK)
      return fail(status[i], "slot " + std::to_string(i) + " (GPU " + std::to_string(e->devs[i]->device) + "): " + errs[i]);
  return JC_OK;
}

jc_status jc_forecast_timestral_device(jc_engine* engine, int slot, const jc_timestral_window* block,
                                       float* quantiles_out, void* stream) {
  clear_error();
  if (!engine || engine->family != 1) return fail(JC_ERR_INVALID_ARG, "not a Timestral engine");
  auto* e = static_cast<TimestralEngine*>(engine);
  if (slot < 0 || slot >= static_cast<int>(e->devs.size())) return fail(JC_ERR_INVALID_ARG, "slot out of range");
  if (!quantiles_out) return fail(JC_ERR_INVALID_ARG, "null output");
  jc_status st = check_window(*e, block, false);
  if (st != JC_OK) return st;
  std::lock_guard<std::mutex> lk(e->mu);
  std::string err;
  st = run_shard(*e, *e->devs[slot], &block->layout, 0, block->layout.rows, quantiles_out, false,
                 static_cast<cudaStream_t>(stream), &err, block);
  return st == JC_OK ? JC_OK : fail(st, err);
}

}  // extern "C"
