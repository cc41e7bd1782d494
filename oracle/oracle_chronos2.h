/*
 * ORACLE — test infrastructure only: the Chronos-2 CPU forward restated in C (see chronos2.c).
 */
#ifndef JC_ORACLE_CHRONOS2_H
#define JC_ORACLE_CHRONOS2_H

#ifdef __cplusplus
extern "C" {
#endif

/* Chronos2Config (chronos2/Chronos2Config.java:45-60) and the checkpoint tensors
 * (Chronos2Weights.load, Chronos2Weights.java:80-100), per-layer arrays indexed by layer. */
typedef struct jco_chronos2 {
  int d_model, d_kv, d_ff, num_layers, num_heads, context_length, patch_size, num_quantiles;
  int use_reg_token, use_arcsinh, time_encoding_scale;
  float eps, rope_theta;
  const float* shared; /* [vocab, d]; row 1 is [REG] */
  const float *in_hw, *in_hb, *in_ow, *in_ob, *in_rw, *in_rb;
  const float* const* time_norm;
  const float* const* time_q;
  const float* const* time_k;
  const float* const* time_v;
  const float* const* time_o;
  const float* const* group_norm;
  const float* const* group_q;
  const float* const* group_k;
  const float* const* group_v;
  const float* const* group_o;
  const float* const* mlp_norm;
  const float* const* wi;
  const float* const* wo;
  const float* final_norm;
  const float *out_hw, *out_hb, *out_ow, *out_ob, *out_rw, *out_rb;
} jco_chronos2;

/* ModelInput (ModelInput.java:28): context [rows, length] with NaN where missing. */
typedef struct jco_c2_input {
  int rows, length, output_patches;
  const float* context;
  const int* group;
  const float* future; /* [rows, future_len] or NULL */
  int future_len;
} jco_c2_input;

typedef struct jco_c2_prepared {
  int rows, nc, reg, h, n;
  int* live;     /* [rows, n] */
  float* tokens; /* [rows, nc + h, 3P] */
  float* loc;
  float* scale;
  int* group;
} jco_c2_prepared;

int jco_chronos2_prepare(const jco_chronos2* m, const jco_c2_input* in, jco_c2_prepared* p);
void jco_c2_prepared_free(jco_c2_prepared* p);
void jco_chronos2_inv_freq(const jco_chronos2* m, float* f);
void jco_chronos2_model(const jco_chronos2* m, const jco_c2_prepared* p, float* raw, int threads);
void jco_chronos2_finish(const jco_chronos2* m, const jco_c2_prepared* p, const float* raw, float* out);
/* CpuChronos2.forward: out [rows, Q, h·P]; raw_out (optional) [rows·h, Q·P]. */
int jco_chronos2_forward(const jco_chronos2* m, const jco_c2_input* in, float* out, float* raw_out, int threads);

#ifdef __cplusplus
}
#endif

#endif
