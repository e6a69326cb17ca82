/*
 * TEST INFRASTRUCTURE ONLY -- the CPU checker for the CUDA path. See
 * u15_oracle.h for the conventions. Paths in the citations are relative to
 * the reference project's root.
 *
 * Parity is pinned by tests/test_oracle_golden.py: every routine that has a
 * counterpart in the reference's u15::ref is compared against fixtures the
 * reference itself produced (tests/golden/gen_golden.py, run against the
 * reference compiled by oracle/Makefile). The W8A8 and Sage routines have
 * no reference CPU counterpart and are restated from their published
 * definitions; see their comments.
 */
#include "u15_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

/* ------------------------------------------------------------------ */
/* primitives                                                          */
/* ------------------------------------------------------------------ */

/* src/u15-ref.cc:15-31 -- row RMSNorm with gain, mean of squares in
 * double. */
void orc_rms_norm(const float* x, const float* w, float eps, long rows,
                  long dim, float* out)
{
#pragma omp parallel for schedule(static)
  for (long r = 0; r < rows; ++r) {
    const float* xr = x + r * dim;
    float* o = out + r * dim;
    double acc = 0.0;
    for (long c = 0; c < dim; ++c) acc += (double)xr[c] * (double)xr[c];
    const double inv = 1.0 / sqrt(acc / (double)dim + (double)eps);
    for (long c = 0; c < dim; ++c)
      o[c] = (float)((double)xr[c] * inv * (double)w[c]);
  }
}

/* src/u15-ref.cc:33-49 -- y = x W^T (+ b), W [out][in], double dot. */
void orc_linear(const float* x, const float* w, const float* b, long rows,
                long in_dim, long out_dim, float* out)
{
#pragma omp parallel for collapse(2) schedule(static)
  for (long r = 0; r < rows; ++r) {
    for (long oc = 0; oc < out_dim; ++oc) {
      const float* xr = x + r * in_dim;
      const float* wr = w + oc * in_dim;
      double acc = 0.0;
#pragma omp simd reduction(+ : acc)
      for (long ic = 0; ic < in_dim; ++ic)
        acc += (double)xr[ic] * (double)wr[ic];
      if (b) acc += (double)b[oc];
      out[r * out_dim + oc] = (float)acc;
    }
  }
}

/* src/u15-ref.cc:51-58 */
void orc_silu(float* x, long n)
{
  for (long i = 0; i < n; ++i) {
    const double v = (double)x[i];
    x[i] = (float)(v / (1.0 + exp(-v)));
  }
}

/* silu(g) * u, the MLP body of src/u15-ref.cc:292-299 */
void orc_swiglu(const float* g, const float* u, float* y, long n)
{
#pragma omp parallel for schedule(static)
  for (long i = 0; i < n; ++i) {
    const double v = (double)g[i];
    y[i] = (float)((v / (1.0 + exp(-v))) * (double)u[i]);
  }
}

/* ------------------------------------------------------------------ */
/* split-3 RoPE                                                        */
/* ------------------------------------------------------------------ */

/* src/u15-metal-ops.cc:547-605 -- [tokens][head_dim] cos/sin tables, each
 * of the three ranges (t: [0,d_t), h: [d_t,d_t+d_h), w: [d_t+d_h, hd))
 * filled with its own ladder, doubled cat(freqs, freqs)-style, angles
 * formed in double and narrowed once.
 *
 * inv_freq_f32 = 1 narrows the inverse frequencies to float first, the way
 * src/u15-ref.cc:64-74 (rope_inv_freq) does; 0 keeps them in double as the
 * GPU path's table builder does. */
void orc_rope_tables(const int* pos_t, const int* pos_h, const int* pos_w,
                     long tokens, int head_dim, int d_t, int d_h,
                     double theta_t, double theta_hw, int inv_freq_f32,
                     float* cos_tab, float* sin_tab)
{
  const int offs[3] = {0, d_t, d_t + d_h};
  const int width[3] = {d_t, d_h, d_h};
  const double theta[3] = {theta_t, theta_hw, theta_hw};
  const int* pos[3] = {pos_t, pos_h, pos_w};
  for (int r = 0; r < 3; ++r) {
    const int half = width[r] / 2;
    for (long t = 0; t < tokens; ++t) {
      const double p = (double)pos[r][t];
      for (int i = 0; i < half; ++i) {
        double inv = 1.0 / pow(theta[r], (double)(2 * i) / (double)width[r]);
        if (inv_freq_f32) inv = (double)(float)inv;
        const double a = p * inv;
        const float cv = (float)cos(a), sv = (float)sin(a);
        const long base = t * head_dim + offs[r];
        cos_tab[base + i] = cv;
        sin_tab[base + i] = sv;
        cos_tab[base + i + half] = cv;
        sin_tab[base + i + half] = sv;
      }
    }
  }
}

/* src/u15-kernels.metal:50-87 (and src/u15-ref.cc:136-160) -- per
 * (token, head) row of head_dim: one RMS reduction over [0, hd/2) with w_t
 * and one over [hd/2, hd) with w_hw. Token-major [tokens][heads*hd], in
 * place. */
void orc_split_qk_norm(float* x, const float* w_t, const float* w_hw,
                       long heads, long tokens, long head_dim, float eps)
{
  const long half = head_dim / 2;
#pragma omp parallel for schedule(static)
  for (long row = 0; row < tokens * heads; ++row) {
    float* r = x + row * head_dim;
    double at = 0.0, ah = 0.0;
    for (long i = 0; i < half; ++i) {
      at += (double)r[i] * (double)r[i];
      ah += (double)r[i + half] * (double)r[i + half];
    }
    const double it = 1.0 / sqrt(at / (double)half + (double)eps);
    const double ih = 1.0 / sqrt(ah / (double)half + (double)eps);
    for (long i = 0; i < half; ++i) {
      r[i] = (float)((double)r[i] * it * (double)w_t[i]);
      r[i + half] = (float)((double)r[i + half] * ih * (double)w_hw[i]);
    }
  }
}

/* src/u15-kernels.metal:118-157 -- rotate_half within each of the three
 * ranges, reading the first half of each range's table entries. */
void orc_split_rope(float* x, const float* cos_tab, const float* sin_tab,
                    long heads, long tokens, long head_dim, int d_t, int d_h)
{
  const int offs[3] = {0, d_t, d_t + d_h};
  const int width[3] = {d_t, d_h, d_h};
#pragma omp parallel for schedule(static)
  for (long row = 0; row < tokens * heads; ++row) {
    const long t = row / heads;
    float* r = x + row * head_dim;
    for (int g = 0; g < 3; ++g) {
      const int half = width[g] / 2;
      for (int i = 0; i < half; ++i) {
        const long ti = t * head_dim + offs[g] + i;
        const double c = (double)cos_tab[ti], s = (double)sin_tab[ti];
        const double a = (double)r[offs[g] + i];
        const double b = (double)r[offs[g] + i + half];
        r[offs[g] + i] = (float)(a * c - b * s);
        r[offs[g] + i + half] = (float)(b * c + a * s);
      }
    }
  }
}

/* ------------------------------------------------------------------ */
/* attention                                                           */
/* ------------------------------------------------------------------ */

/* src/u15-ref.cc:184-230 (GQA attention in double) with the mask rules of
 * src/u15-ref.cc:169-182 and src/u15-kernels.metal:186-252, evaluated from
 * the rule instead of a materialised mask:
 *   ORC_BIDIR         every key j < tk
 *   ORC_CAUSAL        j <= q_offset + i
 *   ORC_BLOCK_CAUSAL  t[j] == t[q_offset + i]  or  j <= q_offset + i
 * q [hq][tq][d]; k/v [hkv][kv_stride][d]; out [tq][hq*d]. */
void orc_attention(const float* q, const float* k, const float* v, long hq,
                   long hkv, long tq, long tk, long d, long kv_stride,
                   int mode, long q_offset, const int* t_index, float* out)
{
  const double scale = 1.0 / sqrt((double)d);
  const long group = hq / hkv;
#pragma omp parallel
  {
    double* row = (double*)malloc(sizeof(double) * (size_t)tk);
    double* acc = (double*)malloc(sizeof(double) * (size_t)d);
#pragma omp for collapse(2) schedule(static)
    for (long h = 0; h < hq; ++h) {
      for (long i = 0; i < tq; ++i) {
        const long hk = h / group;
        const long qpos = q_offset + i;
        const float* qi = q + (h * tq + i) * d;
        double mx = -INFINITY;
        for (long j = 0; j < tk; ++j) {
          int ok = 1;
          if (mode == ORC_CAUSAL) ok = (j <= qpos);
          else if (mode == ORC_BLOCK_CAUSAL)
            ok = (t_index[j] == t_index[qpos]) || (j <= qpos);
          if (!ok) { row[j] = -INFINITY; continue; }
          const float* kj = k + (hk * kv_stride + j) * d;
          double s = 0.0;
          for (long c = 0; c < d; ++c) s += (double)qi[c] * (double)kj[c];
          row[j] = s * scale;
          if (row[j] > mx) mx = row[j];
        }
        double sum = 0.0;
        for (long j = 0; j < tk; ++j) {
          row[j] = (row[j] == -INFINITY) ? 0.0 : exp(row[j] - mx);
          sum += row[j];
        }
        const double inv = sum > 0.0 ? 1.0 / sum : 0.0;
        for (long c = 0; c < d; ++c) acc[c] = 0.0;
        for (long j = 0; j < tk; ++j) {
          if (row[j] == 0.0) continue;
          const double p = row[j] * inv;
          const float* vj = v + (hk * kv_stride + j) * d;
          for (long c = 0; c < d; ++c) acc[c] += p * (double)vj[c];
        }
        float* o = out + i * (hq * d) + h * d;
        for (long c = 0; c < d; ++c) o[c] = (float)acc[c];
      }
    }
    free(row);
    free(acc);
  }
}

/* ------------------------------------------------------------------ */
/* the joint MoT layer                                                 */
/* ------------------------------------------------------------------ */

/* One MoT decoder layer over `tokens` rows split into contiguous segments,
 * each routed to expert seg_expert[s] (0 = und, 1 = _mot_gen). The body is
 * the single-expert src/u15-ref.cc:236-308 (decoder_layer) applied per
 * segment for every per-token step (norms, projections, split norm, MLP),
 * with ONE shared attention over [prefix || this block] -- the order of
 * src/u15-backbone.cc:173-257, where K/V go to the cache before attention
 * and queries attend the cache. The prefix K/V, when n_prefix > 0, are
 * already normed and roped (what a cache holds): [hkv][n_prefix][hd].
 *
 * The rope tables use the GPU path's double inverse frequencies
 * (src/u15-metal-ops.cc:547-605).
 *
 * Outputs: out [tokens][hidden]; k_new/v_new (optional) [hkv][tokens][hd],
 * the block this layer appended to the cache. */
/* Round to the nearest bf16 (ties to even), returned as float. */
static float bf16_rne(float v)
{
  uint32_t u;
  memcpy(&u, &v, sizeof u);
  u = (u + 0x7FFFu + ((u >> 16) & 1u)) & 0xFFFF0000u;
  memcpy(&v, &u, sizeof v);
  return v;
}

/* With `on`, round a buffer to bf16 in place (the reference's activation
 * buffers are bf16 SharedBuffers). */
static void store_bf16(float* a, long n, int on)
{
  if (!on) return;
  for (long i = 0; i < n; ++i) a[i] = bf16_rne(a[i]);
}

/* One projection of the layer: y[n][N] = x[n][K] w[N][K]^T, in fp32 with
 * double accumulation (orc_linear), or under the W8A8 rule. The int8 tier
 * quantizes the activation buffer the GEMM reads, which the reference keeps
 * in bf16 (MetalOps::linear_mma_ hands its bf16 `x` to I8GemmContext::gemm,
 * src/u15-metal-ops.cc:283-306), so the activations are rounded to bf16
 * before the per-token codes are formed. The codes move with that rounding
 * (a W8A8 layer computed from the f32 activations differs from this one by
 * ~3e-2 of the layer's update at full width), so the rounding point is part
 * of the rule. */
static void layer_linear(const float* x, const float* w, long n, long K, long N,
                         float* y, int w8a8)
{
  if (!w8a8) {
    orc_linear(x, w, NULL, n, K, N, y);
    return;
  }
  float* xb = malloc(sizeof(float) * n * K);
  int8_t* xq = malloc((size_t)(n * K));
  int8_t* wq = malloc((size_t)(N * K));
  float* st = malloc(sizeof(float) * n);
  float* sc = malloc(sizeof(float) * N);
  int32_t* acc = malloc(sizeof(int32_t) * n * N);
  for (long i = 0; i < n * K; ++i) xb[i] = bf16_rne(x[i]);
  orc_quant_rows_i8(xb, n, K, xq, st);
  orc_quant_rows_i8(w, N, K, wq, sc);
  orc_gemm_i8(xq, wq, n, K, N, acc);
  orc_dequant_i8(acc, st, sc, n, N, y);
  free(xb); free(xq); free(wq); free(st); free(sc); free(acc);
}

void orc_mot_layer(const float* x, long T, int nseg, const int* seg_off,
                   const int* seg_expert, const orc_expert* E,
                   const orc_dims* d, const int* pos_t, const int* pos_h,
                   const int* pos_w, long n_prefix, const float* k_prefix,
                   const float* v_prefix, int mode, const int* t_index,
                   float* out, float* k_new, float* v_new)
{
  orc_mot_layer_ex(x, T, nseg, seg_off, seg_expert, E, d, pos_t, pos_h, pos_w,
                   n_prefix, k_prefix, v_prefix, mode, t_index, 0, out, k_new,
                   v_new);
}

void orc_mot_layer_ex(const float* x, long T, int nseg, const int* seg_off,
                      const int* seg_expert, const orc_expert* E,
                      const orc_dims* d, const int* pos_t, const int* pos_h,
                      const int* pos_w, long n_prefix, const float* k_prefix,
                      const float* v_prefix, int mode, const int* t_index,
                      int flags, float* out, float* k_new, float* v_new)
{
  const int i8 = (flags & ORC_LAYER_W8A8) != 0;
  const int bf = (flags & ORC_LAYER_BF16) != 0;
  const long H = d->hidden, NH = d->heads, KV = d->kv_heads,
             HD = d->head_dim, I = d->inter;
  const float eps = (float)d->eps;
  const int d_t = (int)(HD / 2), d_h = (int)(HD / 4);
  const long TK = n_prefix + T;

  float* normed = malloc(sizeof(float) * T * H);
  float* q = malloc(sizeof(float) * T * NH * HD);
  float* kk = malloc(sizeof(float) * T * KV * HD);
  float* vv = malloc(sizeof(float) * T * KV * HD);
  float* qh = malloc(sizeof(float) * T * NH * HD);
  float* kc = malloc(sizeof(float) * TK * KV * HD);
  float* vc = malloc(sizeof(float) * TK * KV * HD);
  float* att = malloc(sizeof(float) * T * NH * HD);
  float* proj = malloc(sizeof(float) * T * H);
  float* g = malloc(sizeof(float) * T * I);
  float* u = malloc(sizeof(float) * T * I);
  float* ctab = malloc(sizeof(float) * T * HD);
  float* stab = malloc(sizeof(float) * T * HD);

  orc_rope_tables(pos_t, pos_h, pos_w, T, (int)HD, d_t, d_h, d->theta_t,
                  d->theta_hw, 0, ctab, stab);

  /* attention half */
  for (int s = 0; s < nseg; ++s) {
    const long r0 = seg_off[s], n = seg_off[s + 1] - seg_off[s];
    if (n <= 0) continue;
    const orc_expert* w = &E[seg_expert[s]];
    orc_rms_norm(x + r0 * H, w->input_layernorm, eps, n, H,
                 normed + r0 * H);
    store_bf16(normed + r0 * H, n * H, bf);
    layer_linear(normed + r0 * H, w->q_proj, n, H, NH * HD, q + r0 * NH * HD,
                 i8);
    layer_linear(normed + r0 * H, w->k_proj, n, H, KV * HD, kk + r0 * KV * HD,
                 i8);
    layer_linear(normed + r0 * H, w->v_proj, n, H, KV * HD, vv + r0 * KV * HD,
                 i8);
    store_bf16(q + r0 * NH * HD, n * NH * HD, bf);
    store_bf16(kk + r0 * KV * HD, n * KV * HD, bf);
    store_bf16(vv + r0 * KV * HD, n * KV * HD, bf);
    orc_split_qk_norm(q + r0 * NH * HD, w->q_norm, w->q_norm_hw, NH, n, HD,
                      eps);
    orc_split_qk_norm(kk + r0 * KV * HD, w->k_norm, w->k_norm_hw, KV, n, HD,
                      eps);
  }
  store_bf16(q, T * NH * HD, bf);
  store_bf16(kk, T * KV * HD, bf);
  orc_split_rope(q, ctab, stab, NH, T, HD, d_t, d_h);
  orc_split_rope(kk, ctab, stab, KV, T, HD, d_t, d_h);
  store_bf16(q, T * NH * HD, bf);
  store_bf16(kk, T * KV * HD, bf);

  /* head-major q; the cache holds [prefix || block] per kv head */
  for (long t = 0; t < T; ++t)
    for (long h = 0; h < NH; ++h)
      memcpy(qh + (h * T + t) * HD, q + (t * NH + h) * HD,
             sizeof(float) * HD);
  for (long h = 0; h < KV; ++h) {
    if (n_prefix > 0) {
      memcpy(kc + h * TK * HD, k_prefix + h * n_prefix * HD,
             sizeof(float) * n_prefix * HD);
      memcpy(vc + h * TK * HD, v_prefix + h * n_prefix * HD,
             sizeof(float) * n_prefix * HD);
    }
    for (long t = 0; t < T; ++t) {
      memcpy(kc + (h * TK + n_prefix + t) * HD, kk + (t * KV + h) * HD,
             sizeof(float) * HD);
      memcpy(vc + (h * TK + n_prefix + t) * HD, vv + (t * KV + h) * HD,
             sizeof(float) * HD);
    }
  }
  if (k_new && v_new) {
    for (long h = 0; h < KV; ++h) {
      memcpy(k_new + h * T * HD, kc + (h * TK + n_prefix) * HD,
             sizeof(float) * T * HD);
      memcpy(v_new + h * T * HD, vc + (h * TK + n_prefix) * HD,
             sizeof(float) * T * HD);
    }
  }
  if ((flags & ORC_LAYER_SAGE) && mode == ORC_BIDIR)
    orc_sage_attention(qh, kc, vc, NH, KV, T, TK, HD, TK, 64, 32, att);
  else
    orc_attention(qh, kc, vc, NH, KV, T, TK, HD, TK, mode, n_prefix, t_index,
                  att);
  store_bf16(att, T * NH * HD, bf);

  /* o_proj + residual, then the MLP half, per segment */
  for (int s = 0; s < nseg; ++s) {
    const long r0 = seg_off[s], n = seg_off[s + 1] - seg_off[s];
    if (n <= 0) continue;
    const orc_expert* w = &E[seg_expert[s]];
    layer_linear(att + r0 * NH * HD, w->o_proj, n, NH * HD, H, proj + r0 * H,
                 i8);
    store_bf16(proj + r0 * H, n * H, bf);
    for (long i = 0; i < n * H; ++i) proj[r0 * H + i] += x[r0 * H + i];
    store_bf16(proj + r0 * H, n * H, bf);
    orc_rms_norm(proj + r0 * H, w->post_attention_layernorm, eps, n, H,
                 normed + r0 * H);
    store_bf16(normed + r0 * H, n * H, bf);
    layer_linear(normed + r0 * H, w->gate_proj, n, H, I, g + r0 * I, i8);
    layer_linear(normed + r0 * H, w->up_proj, n, H, I, u + r0 * I, i8);
    store_bf16(g + r0 * I, n * I, bf);
    store_bf16(u + r0 * I, n * I, bf);
    orc_swiglu(g + r0 * I, u + r0 * I, g + r0 * I, n * I);
    store_bf16(g + r0 * I, n * I, bf);
    layer_linear(g + r0 * I, w->down_proj, n, I, H, out + r0 * H, i8);
    store_bf16(out + r0 * H, n * H, bf);
    for (long i = 0; i < n * H; ++i) out[r0 * H + i] += proj[r0 * H + i];
    store_bf16(out + r0 * H, n * H, bf);
  }

  free(normed); free(q); free(kk); free(vv); free(qh); free(kc); free(vc);
  free(att); free(proj); free(g); free(u); free(ctab); free(stab);
}

/* ------------------------------------------------------------------ */
/* W8A8                                                                */
/* ------------------------------------------------------------------ */

/* Symmetric per-row int8 quantization, the rule the BASELINE W8A8 config
 * states (the reference's own i8_gemm uses per-512-group scales inside a
 * host library whose source is not in the tree, src/u15-metal-ops.h:71-98,
 * so this is restated from that spec):
 *   scale = absmax(row) / 127         (fp32 division)
 *   q     = round_half_even(x / scale) (fp32 division), clamped to +-127
 *   an all-zero row has scale 0 and codes 0.
 * Every step is one IEEE fp32 operation, so the GPU kernel reproduces the
 * codes bit for bit. Used per token for activations and per output
 * channel for weights. */
void orc_quant_rows_i8(const float* x, long rows, long cols, int8_t* q,
                       float* scale)
{
#pragma omp parallel for schedule(static)
  for (long r = 0; r < rows; ++r) {
    const float* xr = x + r * cols;
    float amax = 0.0f;
    for (long c = 0; c < cols; ++c) {
      const float a = fabsf(xr[c]);
      if (a > amax) amax = a;
    }
    const float s = amax / 127.0f;
    scale[r] = s;
    for (long c = 0; c < cols; ++c) {
      int v = 0;
      if (s > 0.0f) {
        const float t = xr[c] / s;
        v = (int)rintf(t);
        if (v > 127) v = 127;
        if (v < -127) v = -127;
      }
      q[r * cols + c] = (int8_t)v;
    }
  }
}

/* acc[m][n] = sum_k a[m][k] * w[n][k], exact (int64 sums, |acc| < 2^31 for
 * K <= 2^17 at |code| <= 127). */
void orc_gemm_i8(const int8_t* a, const int8_t* w, long M, long K, long N,
                 int32_t* acc)
{
#pragma omp parallel for collapse(2) schedule(static)
  for (long m = 0; m < M; ++m) {
    for (long n = 0; n < N; ++n) {
      const int8_t* ar = a + m * K;
      const int8_t* wr = w + n * K;
      long long s = 0;
#pragma omp simd reduction(+ : s)
      for (long k = 0; k < K; ++k) s += (long long)ar[k] * (long long)wr[k];
      acc[m * N + n] = (int32_t)s;
    }
  }
}

/* y = ((float)acc * s_tok[m]) * s_ch[n], in fp32, in that order -- the
 * dequant the GPU epilogue applies before its bf16 rounding. */
void orc_dequant_i8(const int32_t* acc, const float* s_tok, const float* s_ch,
                    long M, long N, float* y)
{
#pragma omp parallel for schedule(static)
  for (long m = 0; m < M; ++m)
    for (long n = 0; n < N; ++n)
      y[m * N + n] = ((float)acc[m * N + n] * s_tok[m]) * s_ch[n];
}

/* ------------------------------------------------------------------ */
/* Sage int8-QK attention                                              */
/* ------------------------------------------------------------------ */

/* The SageAttention method (Zhang et al., "SageAttention: Accurate 8-bit
 * attention for plug-and-play inference acceleration", 2024) as the
 * reference describes its use (src/u15-metal-ops.h:294-315,
 * src/u15-metal-ops.cc:789-833): QK^T in int8 with one scale per attention
 * block, the key side smoothed as K - mean_tokens(K) per kv head and
 * channel (exact under softmax: it shifts each score row by a constant),
 * and P.V kept in floating point. The reference's own kernels are not in
 * its tree, so this is restated from the method:
 *   kmean[hk][c]  = (sum over the tk keys of K[hk][j][c]) / tk
 *   ks            = K - kmean
 *   Q blocks of bq query rows per head, K blocks of bk key rows per kv
 *   head, each quantized with orc_quant_rows_i8's rule over the whole
 *   block (one scale per block);
 *   s_ij = int_dot(q8_i, k8_j) * sq * sk / sqrt(d), then softmax and P.V. */
void orc_sage_attention(const float* q, const float* k, const float* v,
                        long hq, long hkv, long tq, long tk, long d,
                        long kv_stride, long bq, long bk, float* out)
{
  const long group = hq / hkv;
  const double scale = 1.0 / sqrt((double)d);
  float* ks = malloc(sizeof(float) * hkv * tk * d);
  int8_t* k8 = malloc((size_t)(hkv * tk * d));
  int8_t* q8 = malloc((size_t)(hq * tq * d));
  const long nqb = (tq + bq - 1) / bq, nkb = (tk + bk - 1) / bk;
  float* sq = malloc(sizeof(float) * hq * nqb);
  float* sk = malloc(sizeof(float) * hkv * nkb);

  for (long h = 0; h < hkv; ++h) {
    for (long c = 0; c < d; ++c) {
      double s = 0.0;
      for (long j = 0; j < tk; ++j) s += (double)k[(h * kv_stride + j) * d + c];
      const float mean = (float)(s / (double)tk);
      for (long j = 0; j < tk; ++j)
        ks[(h * tk + j) * d + c] = k[(h * kv_stride + j) * d + c] - mean;
    }
  }
  /* block quantization: a block is rows x d values sharing one scale */
  for (long h = 0; h < hq; ++h) {
    for (long b = 0; b < nqb; ++b) {
      const long r0 = b * bq, n = (r0 + bq <= tq) ? bq : tq - r0;
      float s;
      float amax = 0.0f;
      const float* src = q + (h * tq + r0) * d;
      for (long i = 0; i < n * d; ++i)
        if (fabsf(src[i]) > amax) amax = fabsf(src[i]);
      s = amax / 127.0f;
      sq[h * nqb + b] = s;
      for (long i = 0; i < n * d; ++i) {
        int vq = 0;
        if (s > 0.0f) {
          vq = (int)rintf(src[i] / s);
          if (vq > 127) vq = 127;
          if (vq < -127) vq = -127;
        }
        q8[(h * tq + r0) * d + i] = (int8_t)vq;
      }
    }
  }
  for (long h = 0; h < hkv; ++h) {
    for (long b = 0; b < nkb; ++b) {
      const long r0 = b * bk, n = (r0 + bk <= tk) ? bk : tk - r0;
      float amax = 0.0f;
      const float* src = ks + (h * tk + r0) * d;
      for (long i = 0; i < n * d; ++i)
        if (fabsf(src[i]) > amax) amax = fabsf(src[i]);
      const float s = amax / 127.0f;
      sk[h * nkb + b] = s;
      for (long i = 0; i < n * d; ++i) {
        int vq = 0;
        if (s > 0.0f) {
          vq = (int)rintf(src[i] / s);
          if (vq > 127) vq = 127;
          if (vq < -127) vq = -127;
        }
        k8[(h * tk + r0) * d + i] = (int8_t)vq;
      }
    }
  }

#pragma omp parallel
  {
    double* row = malloc(sizeof(double) * (size_t)tk);
    double* acc = malloc(sizeof(double) * (size_t)d);
#pragma omp for collapse(2) schedule(static)
    for (long h = 0; h < hq; ++h) {
      for (long i = 0; i < tq; ++i) {
        const long hk = h / group;
        const int8_t* qi = q8 + (h * tq + i) * d;
        const double sqv = (double)sq[h * nqb + i / bq];
        double mx = -INFINITY;
        for (long j = 0; j < tk; ++j) {
          const int8_t* kj = k8 + (hk * tk + j) * d;
          long long dot = 0;
          for (long c = 0; c < d; ++c) dot += (long long)qi[c] * kj[c];
          row[j] = (double)dot * sqv * (double)sk[hk * nkb + j / bk] * scale;
          if (row[j] > mx) mx = row[j];
        }
        double sum = 0.0;
        for (long j = 0; j < tk; ++j) {
          row[j] = exp(row[j] - mx);
          sum += row[j];
        }
        for (long c = 0; c < d; ++c) acc[c] = 0.0;
        for (long j = 0; j < tk; ++j) {
          const double p = row[j] / sum;
          const float* vj = v + (hk * kv_stride + j) * d;
          for (long c = 0; c < d; ++c) acc[c] += p * (double)vj[c];
        }
        float* o = out + i * (hq * d) + h * d;
        for (long c = 0; c < d; ++c) o[c] = (float)acc[c];
      }
    }
    free(row);
    free(acc);
  }
  free(ks); free(k8); free(q8); free(sq); free(sk);
}

/* ------------------------------------------------------------------ */
/* sampling                                                            */
/* ------------------------------------------------------------------ */

/* src/u15-ref.cc:722-733 -- sigma = 1 - i/n, shifted, t = 1 - sigma. */
void orc_time_schedule(int num_steps, double shift, float* out)
{
  for (int i = 0; i <= num_steps; ++i) {
    double sigma = 1.0 - (double)i / (double)num_steps;
    sigma = shift * sigma / (1.0 + (shift - 1.0) * sigma);
    out[i] = (float)(1.0 - sigma);
  }
}

/* ------------------------------------------------------------------ */
/* the denoise step                                                    */
/* ------------------------------------------------------------------ */

/* src/u15-generator.cc:582-584 -- v = (x_pred - img) / denom in double. */
void orc_velocity(const float* x_pred, const float* img, long n, double denom, float* v)
{
  for (long i = 0; i < n; ++i)
    v[i] = (float)(((double)x_pred[i] - (double)img[i]) / denom);
}

/* src/u15-ref.cc:755-765 -- alpha = <pos, neg> / (||neg||^2 + 1e-8). */
double orc_optimized_scale(const float* pos, const float* neg, long n)
{
  double dot = 0.0, nrm = 0.0;
  for (long i = 0; i < n; ++i) {
    dot += (double)pos[i] * (double)neg[i];
    nrm += (double)neg[i] * (double)neg[i];
  }
  return dot / (nrm + 1e-8);
}

/* src/u15-generator.cc:596-693 -- the CFG combination and its renorms over an
 * [H][W][3] image (32x32-pixel tokens for the per-token renorm).
 *   ORC_CFG_IMG   v_img + cfg (v_cond - v_img)                 (img_cfg == 1)
 *   ORC_CFG_UNC   v_unc + cfg (v_cond - v_unc), or with ORC_NORM_ZERO_STAR
 *                 a = alpha v_unc; a + cfg (v_cond - a), exactly 0 at step 0
 *   ORC_CFG_BOTH  v_unc + cfg (v_cond - v_img) + icfg (v_img - v_unc)
 *   ORC_CFG_NONE  v_cond
 * then ORC_NORM_GLOBAL scales by min(1, |v_cond| / (|out| + 1e-8)) over the
 * image and ORC_NORM_CHANNEL does the same per token. */
void orc_cfg(const float* vc, const float* vu, const float* vi, long H, long W, int form,
             int norm, double cfg, double icfg, int step, float* out)
{
  const long n = H * W * 3;
  if (form == ORC_CFG_IMG) {
    for (long i = 0; i < n; ++i)
      out[i] = (float)((double)vi[i] + cfg * ((double)vc[i] - (double)vi[i]));
  } else if (form == ORC_CFG_UNC) {
    if (norm == ORC_NORM_ZERO_STAR) {
      const double alpha = orc_optimized_scale(vc, vu, n);
      if (step <= 0) {
        for (long i = 0; i < n; ++i) out[i] = 0.0f;
      } else {
        for (long i = 0; i < n; ++i) {
          const double a = alpha * (double)vu[i];
          out[i] = (float)(a + cfg * ((double)vc[i] - a));
        }
      }
    } else {
      for (long i = 0; i < n; ++i)
        out[i] = (float)((double)vu[i] + cfg * ((double)vc[i] - (double)vu[i]));
    }
  } else if (form == ORC_CFG_BOTH) {
    for (long i = 0; i < n; ++i)
      out[i] = (float)((double)vu[i] + cfg * ((double)vc[i] - (double)vi[i]) +
                       icfg * ((double)vi[i] - (double)vu[i]));
  } else {
    for (long i = 0; i < n; ++i) out[i] = vc[i];
  }
  if (norm == ORC_NORM_GLOBAL) {
    double nc = 0.0, nv = 0.0;
    for (long i = 0; i < n; ++i) {
      nc += (double)vc[i] * vc[i];
      nv += (double)out[i] * out[i];
    }
    double sc = sqrt(nc) / (sqrt(nv) + 1e-8);
    if (sc > 1.0) sc = 1.0;
    for (long i = 0; i < n; ++i) out[i] = (float)(out[i] * sc);
  } else if (norm == ORC_NORM_CHANNEL) {
    const long ps = 32, th = H / ps, tw = W / ps;
    for (long ty = 0; ty < th; ++ty) {
      for (long tx = 0; tx < tw; ++tx) {
        double nc = 0.0, nv = 0.0;
        for (long y = 0; y < ps; ++y)
          for (long x = 0; x < ps; ++x)
            for (long c = 0; c < 3; ++c) {
              const long i = ((ty * ps + y) * W + (tx * ps + x)) * 3 + c;
              nc += (double)vc[i] * vc[i];
              nv += (double)out[i] * out[i];
            }
        double sc = sqrt(nc) / (sqrt(nv) + 1e-8);
        if (sc > 1.0) sc = 1.0;
        for (long y = 0; y < ps; ++y)
          for (long x = 0; x < ps; ++x)
            for (long c = 0; c < 3; ++c) {
              const long i = ((ty * ps + y) * W + (tx * ps + x)) * 3 + c;
              out[i] = (float)(out[i] * sc);
            }
      }
    }
  }
}

/* src/u15-generator.cc:701-705 -- img += dt v, in double. */
void orc_euler(float* img, const float* v, long n, double dt)
{
  for (long i = 0; i < n; ++i) img[i] = (float)((double)img[i] + dt * (double)v[i]);
}

/* ------------------------------------------------------------------ */
/* the image path (src/u15-ref.cc: patchify_channel_first_hwc,         */
/* gelu_erf, rope_interleaved_inplace, vision_embed, pixel_shuffle,    */
/* conv3x3, conv_decoder, timestep_sinusoid; the timestep MLP of       */
/* src/u15-image.cc ImagePath::timestep_row)                           */
/* ------------------------------------------------------------------ */

/* img [H][W][c] -> [gh*gw][c*p*p], each patch packed channel-FIRST
 * (ci, pi, qi): the patch embedder's input (src/u15-ref.cc
 * patchify_channel_first_hwc). */
void orc_patchify_cf(const float* img, int c, int H, int W, int p, float* out)
{
  const int gh = H / p, gw = W / p;
  const long stride = (long)c * p * p;
  for (int hi = 0; hi < gh; ++hi)
    for (int wi = 0; wi < gw; ++wi) {
      float* o = out + ((long)hi * gw + wi) * stride;
      for (int ci = 0; ci < c; ++ci)
        for (int pi = 0; pi < p; ++pi)
          for (int qi = 0; qi < p; ++qi)
            o[((long)ci * p + pi) * p + qi] =
                img[((long)(hi * p + pi) * W + (wi * p + qi)) * c + ci];
    }
}

/* the exact erf GELU, in double */
void orc_gelu_erf(float* x, long n)
{
  for (long i = 0; i < n; ++i) {
    const double v = x[i];
    x[i] = (float)(0.5 * v * (1.0 + erf(v / sqrt(2.0))));
  }
}

/* rotate (2i, 2i+1) pairs of x[0:dim) by position * inv[i] (double) */
static void rope_pairs(float* x, const float* inv, int dim, double pos)
{
  for (int i = 0; i < dim / 2; ++i) {
    const double a = pos * (double)inv[i], c = cos(a), s = sin(a);
    const double u = x[2 * i], v = x[2 * i + 1];
    x[2 * i] = (float)(u * c - v * s);
    x[2 * i + 1] = (float)(u * s + v * c);
  }
}

/* The patch embedder (src/u15-ref.cc vision_embed): per-patch linear
 * (C x 3p^2) + bias, GELU, interleaved 2-D RoPE (first half of each
 * embedding by the patch column, second half by its row; inverse
 * frequencies of C/2 dims, as float), m x m tiles gathered channel-slowest,
 * dense linear (LLM x C m^2) + bias. px [gh*gw][3p^2] -> out [(gh/m)(gw/m)][LLM]. */
void orc_vision_embed(const float* px, const float* patch_w, const float* patch_b,
                      const float* dense_w, const float* dense_b, int gh, int gw, int p,
                      int C, int LLM, int m, double theta, float* out)
{
  const long n = (long)gh * gw, pin = 3L * p * p;
  float* emb = (float*)malloc(sizeof(float) * n * C);
  orc_linear(px, patch_w, patch_b, n, pin, C, emb);
  orc_gelu_erf(emb, n * C);
  const int half = C / 2;
  float* inv = (float*)malloc(sizeof(float) * (half / 2));
  for (int i = 0; i < half / 2; ++i)
    inv[i] = (float)(1.0 / pow(theta, (double)(2 * i) / (double)half));
  for (int r = 0; r < gh; ++r)
    for (int c = 0; c < gw; ++c) {
      float* e = emb + ((long)r * gw + c) * C;
      rope_pairs(e, inv, half, (double)c);
      rope_pairs(e + half, inv, half, (double)r);
    }
  const int oh = gh / m, ow = gw / m;
  const long tile = (long)C * m * m;
  float* g = (float*)malloc(sizeof(float) * oh * ow * tile);
  for (int r = 0; r < oh; ++r)
    for (int c = 0; c < ow; ++c)
      for (int ch = 0; ch < C; ++ch)
        for (int i = 0; i < m; ++i)
          for (int j = 0; j < m; ++j)
            g[((long)r * ow + c) * tile + ((long)ch * m + i) * m + j] =
                emb[((long)(r * m + i) * gw + (c * m + j)) * C + ch];
  orc_linear(g, dense_w, dense_b, (long)oh * ow, tile, LLM, out);
  free(g);
  free(inv);
  free(emb);
}

/* PixelShuffle(r) on a channel-last map: input channel c*r*r + i*r + j of
 * pixel (y, x) -> output channel c of pixel (y*r + i, x*r + j). */
static void ps_hwc(const float* in, int H, int W, int Cin, int r, float* out)
{
  const int Co = Cin / (r * r);
  for (int y = 0; y < H; ++y)
    for (int x = 0; x < W; ++x)
      for (int ci = 0; ci < Cin; ++ci) {
        const int c = ci / (r * r), i = (ci % (r * r)) / r, j = ci % r;
        out[((long)(y * r + i) * (W * r) + (x * r + j)) * Co + c] =
            in[((long)y * W + x) * Cin + ci];
      }
}

/* 3x3 convolution, padding 1, channel-last; weight [cout][cin][3][3]
 * (the checkpoint's order), double accumulation. */
static void conv3x3_hwc(const float* x, const float* w, const float* b, int cin, int cout,
                        int H, int W, float* out)
{
#pragma omp parallel for collapse(2) schedule(static)
  for (int y = 0; y < H; ++y)
    for (int xx = 0; xx < W; ++xx)
      for (int oc = 0; oc < cout; ++oc) {
        double acc = b ? (double)b[oc] : 0.0;
        for (int ky = 0; ky < 3; ++ky) {
          const int sy = y + ky - 1;
          if (sy < 0 || sy >= H) continue;
          for (int kx = 0; kx < 3; ++kx) {
            const int sx = xx + kx - 1;
            if (sx < 0 || sx >= W) continue;
            const float* src = x + ((long)sy * W + sx) * cin;
            const float* wk = w + (long)oc * cin * 9 + ky * 3 + kx;
            for (int ic = 0; ic < cin; ++ic) acc += (double)wk[(long)ic * 9] * (double)src[ic];
          }
        }
        out[((long)y * W + xx) * cout + oc] = (float)acc;
      }
}

/* The pixel head (src/u15-ref.cc conv_decoder) in the channel-last layout
 * the device runs: x [th][tw][in_ch] -> PS(2) -> conv1 3x3 (in_ch/4 ->
 * hidden_ch) + bias -> GELU -> PS(2) -> conv2 3x3 (hidden_ch/4 -> 192) +
 * bias -> PS(8) -> out [32 th][32 tw][3]. */
void orc_conv_decoder_hwc(const float* x, const float* conv1_w, const float* conv1_b,
                          const float* conv2_w, const float* conv2_b, int in_ch, int th, int tw,
                          int hidden_ch, float* out)
{
  const int c1 = in_ch / 4, c2 = hidden_ch / 4;
  float* a = (float*)malloc(sizeof(float) * (long)c1 * 4 * th * tw);
  float* b = (float*)malloc(sizeof(float) * (long)hidden_ch * 4 * th * tw);
  float* c = (float*)malloc(sizeof(float) * (long)c2 * 16 * th * tw);
  float* e = (float*)malloc(sizeof(float) * 192L * 16 * th * tw);
  ps_hwc(x, th, tw, in_ch, 2, a);
  conv3x3_hwc(a, conv1_w, conv1_b, c1, hidden_ch, 2 * th, 2 * tw, b);
  orc_gelu_erf(b, (long)hidden_ch * 4 * th * tw);
  ps_hwc(b, 2 * th, 2 * tw, hidden_ch, 2, c);
  conv3x3_hwc(c, conv2_w, conv2_b, c2, 192, 4 * th, 4 * tw, e);
  ps_hwc(e, 4 * th, 4 * tw, 192, 8, out);
  free(e);
  free(c);
  free(b);
  free(a);
}

/* sinusoid of `dim` (cos first, then sin; max period 1e4) -> Linear(dim
 * -> H) -> SiLU -> Linear(H -> H), f32 values with double accumulation
 * (src/u15-image.cc ImagePath::timestep_row); the noise-scale embedder,
 * when its weights are given, is evaluated the same way at `ratio` and
 * added. */
static void scalar_mlp(double v, int dim, int H, const float* w0, const float* b0,
                       const float* w2, const float* b2, float* out)
{
  float* s = (float*)malloc(sizeof(float) * dim);
  float* h = (float*)malloc(sizeof(float) * H);
  const int half = dim / 2;
  for (int i = 0; i < half; ++i) {
    const double f = exp(-log(10000.0) * (double)i / (double)half);
    s[i] = (float)cos(v * f);
    s[i + half] = (float)sin(v * f);
  }
  orc_linear(s, w0, b0, 1, dim, H, h);
  orc_silu(h, H);
  orc_linear(h, w2, b2, 1, H, H, out);
  free(h);
  free(s);
}

void orc_timestep_row(double t, double ratio, int dim, int H, const float* w0, const float* b0,
                      const float* w2, const float* b2, const float* nw0, const float* nb0,
                      const float* nw2, const float* nb2, float* out)
{
  scalar_mlp(t, dim, H, w0, b0, w2, b2, out);
  if (nw0 != NULL) {
    float* ns = (float*)malloc(sizeof(float) * H);
    scalar_mlp(ratio, dim, H, nw0, nb0, nw2, nb2, ns);
    for (int i = 0; i < H; ++i) out[i] += ns[i];
    free(ns);
  }
}
