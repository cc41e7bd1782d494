/*
 * ORACLE — test infrastructure only: the Timestral CPU forward restated in C (see timestral.c).
 */
#ifndef JC_ORACLE_TIMESTRAL_H
#define JC_ORACLE_TIMESTRAL_H

#ifdef __cplusplus
extern "C" {
#endif

#define JCO_TARGET 0
#define JCO_PAST 1
#define JCO_KNOWN 2

/* A Timestral checkpoint: the TimestralConfig fields the forward uses (TimestralConfig.java:53-71)
 * and the checkpoint tensors in their stored layouts (TimestralWeights.java:83-115). Per-attention
 * arrays are flattened over layers, then each layer's attention sublayers in order. */
typedef struct jco_timestral {
  int patch_size, d_model, num_heads, mlp_hidden_dim, num_layers, num_quantiles, block_size;
  const int* attn_per_layer; /* [num_layers] */
  const int* attn_is_time;   /* [total attentions] */
  const int* attn_gate;      /* [total attentions] */
  const double* quantile_knots;
  float rope_theta, rope_partial_factor, norm_eps, minimum_scale, quantile_width_factor;
  int use_asinh, covariate_enabled, attend_missing_patches;
  const float *emb_hidden_w, *emb_hidden_b, *emb_output_w, *emb_output_b, *emb_residual_w, *emb_residual_b;
  const float* forecast_query;
  const float* const* attn_norm; /* [total] [d] */
  const float* const* wqkv;      /* [total] [3d, d], stored head-dim-major */
  const float* const* gate_w;    /* [total] [d, d] or NULL */
  const float* const* wo;        /* [total] [d, d] */
  const float* const* mlp_norm;  /* [layers] [d] */
  const float* const* w12;       /* [layers] [2F, d], stored gate half first */
  const float* const* w3;        /* [layers] [d, F] */
  const float* out_norm;
  const float *head_hidden_w, *head_output_w, *head_residual_w;
} jco_timestral;

/* BlockInput (BlockInput.java:32-46), flattened: inputs/observed [rows, length]. */
typedef struct jco_block {
  int rows, length, horizon;
  const float* inputs;
  const unsigned char* observed;
  const int* group;
  const int* role;                       /* NULL = all targets */
  const float* known_future;             /* [rows, horizon·P] or NULL */
  const unsigned char* known_future_mask;
} jco_block;

/* BlockLayout + BlockPrep results. */
typedef struct jco_prepared {
  int rows, enc, horizon, ll, covariates;
  float* window;
  unsigned char* obs;
  int* key_valid; /* [rows, enc] */
  int* first;     /* [rows] */
  int* role;
  int* known;
  int* group;
  int* pos;       /* [rows, enc + horizon]: BlockLayout.position */
  float* loc;     /* [rows, window] */
  float* scale;
  float* tokens;  /* [rows, enc, 2P] */
} jco_prepared;

int jco_timestral_prepare(const jco_timestral* m, const jco_block* b, jco_prepared* p);
void jco_prepared_free(jco_prepared* p);
void jco_timestral_inv_freq(const jco_timestral* m, float* f);
/* raw [rows·h·P·Q] = the model between BlockPrep.of and BlockPrep.finish. */
void jco_timestral_model(const jco_timestral* m, const jco_prepared* p, float* raw, int threads);
/* raw is made monotone in place; out [rows, h·P, Q]. */
void jco_timestral_finish(const jco_timestral* m, const jco_prepared* p, float* raw, float* out);
/* CpuTimestral.predictBlock: out [rows, h·P, Q]; raw_out (optional) the head's raw outputs. */
int jco_timestral_predict_block(const jco_timestral* m, const jco_block* b, float* out, float* raw_out, int threads);

#ifdef __cplusplus
}
#endif

#endif
