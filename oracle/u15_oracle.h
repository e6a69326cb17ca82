/*
 * TEST INFRASTRUCTURE ONLY -- the CPU checker for the CUDA path.
 *
 * A plain-C restatement of the reference's CPU algorithm for the MoT
 * backbone layer (src/u15-ref.cc, src/u15-metal-ops.cc:547-605 and the
 * operation order of src/u15-backbone.cc:173-257 in the reference tree),
 * widened with the pieces the reference does not carry on the CPU: the
 * joint two-expert layer, the frozen-prefix KV form, the W8A8 integer
 * product and the Sage int8-QK attention.
 *
 * Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg load
 * this library, and only as the checker. The product never links it.
 *
 * Conventions (as the reference's):
 *   activations   [tokens][dim]                 token-major
 *   linear weight [out][in]
 *   q             [head][tokens][head_dim]       head-major
 *   k / v cache   [kv_head][kv_stride][head_dim] stride = capacity in tokens
 * Every float routine reads and writes fp32 and accumulates in double.
 */
#ifndef U15_ORACLE_H
#define U15_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* attention masks, as the three rules of src/u15-backbone.h:48-57 */
enum { ORC_BIDIR = 0, ORC_CAUSAL = 1, ORC_BLOCK_CAUSAL = 2 };

void orc_rms_norm(const float* x, const float* w, float eps, long rows,
                  long dim, float* out);
void orc_linear(const float* x, const float* w, const float* b, long rows,
                long in_dim, long out_dim, float* out);
void orc_silu(float* x, long n);
void orc_swiglu(const float* g, const float* u, float* y, long n);

void orc_rope_tables(const int* pos_t, const int* pos_h, const int* pos_w,
                     long tokens, int head_dim, int d_t, int d_h,
                     double theta_t, double theta_hw, int inv_freq_f32,
                     float* cos_tab, float* sin_tab);
void orc_split_qk_norm(float* x, const float* w_t, const float* w_hw,
                       long heads, long tokens, long head_dim, float eps);
void orc_split_rope(float* x, const float* cos_tab, const float* sin_tab,
                    long heads, long tokens, long head_dim, int d_t,
                    int d_h);

void orc_attention(const float* q, const float* k, const float* v,
                   long hq, long hkv, long tq, long tk, long d,
                   long kv_stride, int mode, long q_offset,
                   const int* t_index, float* out);

/* One expert-layer's 13 tensors, in the reference's LayerWeights order
 * (src/u15-ref.h:113-127). */
typedef struct {
  const float* input_layernorm;
  const float* post_attention_layernorm;
  const float* q_proj;
  const float* k_proj;
  const float* v_proj;
  const float* o_proj;
  const float* q_norm;
  const float* k_norm;
  const float* q_norm_hw;
  const float* k_norm_hw;
  const float* gate_proj;
  const float* up_proj;
  const float* down_proj;
} orc_expert;

typedef struct {
  long hidden, heads, kv_heads, head_dim, inter;
  double eps, theta_t, theta_hw;
} orc_dims;

void orc_mot_layer(const float* x, long tokens, int nseg, const int* seg_off,
                   const int* seg_expert, const orc_expert* experts,
                   const orc_dims* d, const int* pos_t, const int* pos_h,
                   const int* pos_w, long n_prefix, const float* k_prefix,
                   const float* v_prefix, int mode, const int* t_index,
                   float* out, float* k_new, float* v_new);

/* The same layer under the two lossy tiers (flags may combine):
 * ORC_LAYER_W8A8  every projection through the W8A8 rule (per-token int8
 *                 activations, per-output-channel int8 weights, exact int32
 *                 accumulators, the fp32 dequant) -- the i8_gemm tier;
 * ORC_LAYER_SAGE  the bidirectional attention through orc_sage_attention
 *                 with the reference's Sage tiles (64 query rows, 32 keys)
 *                 -- the sage_attn tier; the masked rules stay exact;
 * ORC_LAYER_BF16  every activation buffer of the reference's layer_step_
 *                 (src/u15-backbone.cc:173-257: _normed, _q/_k/_v after the
 *                 projection, the split norm and the rope, _attn, _proj, x
 *                 after each add, _gate/_up/_ff) rounded to bf16 where the
 *                 reference stores it, instead of u15-ref's fp32 throughout. */
#define ORC_LAYER_W8A8 1
#define ORC_LAYER_SAGE 2
#define ORC_LAYER_BF16 4
void orc_mot_layer_ex(const float* x, long tokens, int nseg, const int* seg_off,
                      const int* seg_expert, const orc_expert* experts,
                      const orc_dims* d, const int* pos_t, const int* pos_h,
                      const int* pos_w, long n_prefix, const float* k_prefix,
                      const float* v_prefix, int mode, const int* t_index,
                      int flags, float* out, float* k_new, float* v_new);

void orc_quant_rows_i8(const float* x, long rows, long cols, int8_t* q,
                       float* scale);
void orc_gemm_i8(const int8_t* a, const int8_t* w, long M, long K, long N,
                 int32_t* acc);
void orc_dequant_i8(const int32_t* acc, const float* s_tok, const float* s_ch,
                    long M, long N, float* y);

void orc_sage_attention(const float* q, const float* k, const float* v,
                        long hq, long hkv, long tq, long tk, long d,
                        long kv_stride, long bq, long bk, float* out);

void orc_time_schedule(int num_steps, double shift, float* out);

/* the denoise step (src/u15-generator.cc:582-705) */
enum { ORC_CFG_NONE = 0, ORC_CFG_IMG = 1, ORC_CFG_UNC = 2, ORC_CFG_BOTH = 3 };
enum { ORC_NORM_NONE = 0, ORC_NORM_GLOBAL = 1, ORC_NORM_CHANNEL = 2, ORC_NORM_ZERO_STAR = 3 };
void orc_velocity(const float* x_pred, const float* img, long n, double denom, float* v);
double orc_optimized_scale(const float* pos, const float* neg, long n);
void orc_cfg(const float* v_cond, const float* v_unc, const float* v_img, long H, long W,
             int form, int norm, double cfg, double icfg, int step, float* out);
void orc_euler(float* img, const float* v, long n, double dt);

/* the image path (src/u15-ref.cc vision_embed / conv_decoder; src/u15-image.cc) */
void orc_patchify_cf(const float* img, int c, int H, int W, int p, float* out);
void orc_gelu_erf(float* x, long n);
void orc_vision_embed(const float* px, const float* patch_w, const float* patch_b,
                      const float* dense_w, const float* dense_b, int gh, int gw, int p,
                      int C, int LLM, int m, double theta, float* out);
void orc_conv_decoder_hwc(const float* x, const float* conv1_w, const float* conv1_b,
                          const float* conv2_w, const float* conv2_b, int in_ch, int th, int tw,
                          int hidden_ch, float* out);
void orc_timestep_row(double t, double ratio, int dim, int H, const float* w0, const float* b0,
                      const float* w2, const float* b2, const float* nw0, const float* nb0,
                      const float* nw2, const float* nb2, float* out);

#ifdef __cplusplus
}
#endif
#endif
