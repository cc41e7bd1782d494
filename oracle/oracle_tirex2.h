/*
 * ORACLE — test infrastructure only (see ops.c). The C restatement of the reference's FP32
 * TiRex-2 CPU forward (tirex2/cpu/CpuReference.java); the checker for jc_forward_tirex2.
 */
#ifndef JC_ORACLE_TIREX2_H
#define JC_ORACLE_TIREX2_H

#ifdef __cplusplus
extern "C" {
#endif

#define JCO_TIREX_MLSTM 0
#define JCO_TIREX_SLSTM 1

/* The TiRex2Config fields the forward reads (tirex2/TiRex2Config.java:48-66) and the weights,
 * FP32 row-major in the checkpoint's layouts (tirex2/TiRex2Weights.java:169-247). Per-block
 * arrays hold one pointer per block; a block's unused cell pointers are NULL. */
typedef struct {
  int d, blocks, patch, in_ff, out_ff, context_len, future_len, num_q;
  int use_arcsinh, binary_aware, use_qk_norm;
  int tm_heads, slstm_heads, var_heads;
  float out_norm_eps;
  const int* block_types; /* [blocks] JCO_TIREX_MLSTM / JCO_TIREX_SLSTM */
  const float *in_hw, *in_hb, *in_ow, *in_ob, *in_rw, *in_rb;
  const float** norm_lstm;
  /* mLSTM: q, k [qk, d]; v, o [d, d]; igate, fgate [heads, d] + bias; head_norm [d]; out_proj [d, d] */
  const float **mq, **mk, **mv, **mo, **ig_w, **ig_b, **fg_w, **fg_b, **head_norm, **out_proj;
  /* sLSTM: gate slot g (i, f, z, o order) [H, dh, dh]; recurrent [H, dh, 4, dh]; bias [H, 4, dh]; group_norm [d] */
  const float **sg0, **sg1, **sg2, **sg3, **srec, **sbias, **group_norm;
  const float **comb, **norm_ffn, **up_gate, **up, **down;
  const float **norm_attn, **wq, **wk, **wv, **wo, **norm_ffn_attn, **ffn_in, **ffn_out;
  const float* out_norm;
  const float *out_hw, *out_hb, *out_ow, *out_ob, *out_rw, *out_rb;
} JcoTirex2;

/*
 * CpuReference.forward (CpuReference.java:67-90): x [rows · (context_len + future_len)] with NaN where
 * there is no observation, group [rows], target [rows] (0/1); out [rows · Q · len] in data units.
 * Returns 0, or -1 on a bad argument.
 */
int jco_tirex2_forward(const JcoTirex2* m, int rows, const float* x, const float* group, const int* target,
                       float* out, int threads);

/* Cells.mlstmCore (Cells.java:74-118) on the fused projection p [(r·seq + t)·stride]; h [rows·seq·heads·128]. */
void jco_tirex2_mlstm_core(const float* p, int rows, int seq, int heads, int stride, float* h);

/* Cells.slstmRecurrence (Cells.java:170-218) on wx [(r·seq + t)·4d]; y [rows·seq·d]. */
void jco_tirex2_slstm_recurrence(const float* wx, int rows, int seq, int d, int heads, const float* r,
                                 const float* b, float* y);

#ifdef __cplusplus
}
#endif

#endif
