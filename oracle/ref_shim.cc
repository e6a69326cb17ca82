// Test infrastructure: a C ABI over the reference's own CPU implementation
// (u15::ref in src/u15-ref.h of the reference), so Python fixtures
// generators and tests can call it through ctypes. This file is ours; the
// functions it forwards to are compiled unchanged from the reference tree.
//
// Every entry point forwards one-to-one; argument meaning follows
// src/u15-ref.h.
#include "u15-ref.h"

#include <cstring>
#include <vector>

using namespace u15::ref;

extern "C" {

void refx_rms_norm(const float* x, const float* w, float eps, long rows,
                   long dim, float* out)
{
  rms_norm(x, w, eps, (std::size_t)rows, (std::size_t)dim, out);
}

void refx_linear(const float* x, const float* w, const float* b, long rows,
                 long in_dim, long out_dim, float* out)
{
  linear(x, w, b, (std::size_t)rows, (std::size_t)in_dim,
         (std::size_t)out_dim, out);
}

void refx_silu(float* x, long n) { silu(x, (std::size_t)n); }

void refx_rope_inv_freq(int dim, double theta, float* out)
{
  const std::vector<float> f = rope_inv_freq(dim, theta);
  std::memcpy(out, f.data(), f.size() * sizeof(float));
}

void refx_split_rope_project(const float* x, const float* w_proj,
                             const float* w_norm, const float* w_norm_hw,
                             const int* pos_t, const int* pos_h,
                             const int* pos_w, long tokens, long hidden,
                             int heads, int head_dim, double theta_t,
                             double theta_hw, double eps, float* out)
{
  SplitRopeParams p;
  p.heads = heads;
  p.head_dim = head_dim;
  p.theta_t = theta_t;
  p.theta_hw = theta_hw;
  p.rms_eps = eps;
  const std::vector<int> t(pos_t, pos_t + tokens), h(pos_h, pos_h + tokens),
      w(pos_w, pos_w + tokens);
  split_rope_project(x, w_proj, w_norm, w_norm_hw, t, h, w,
                     (std::size_t)tokens, (std::size_t)hidden, p, out);
}

void refx_attention(const float* q, const float* k, const float* v,
                    const float* mask, long hq, long hkv, long tq, long tk,
                    long d, float* out)
{
  attention(q, k, v, mask, (std::size_t)hq, (std::size_t)hkv,
            (std::size_t)tq, (std::size_t)tk, (std::size_t)d, out);
}

void refx_block_causal_mask(const int* t_index, long n, float* out)
{
  const std::vector<int> t(t_index, t_index + n);
  const std::vector<float> m = block_causal_mask(t);
  std::memcpy(out, m.data(), m.size() * sizeof(float));
}

// The 13 tensors of one expert-layer, in LayerWeights order.
void refx_decoder_layer(const float* x, const float* const* wts,
                        long hidden, long heads, long kv_heads, long head_dim,
                        long inter, double eps, double theta_t,
                        double theta_hw, const int* pos_t, const int* pos_h,
                        const int* pos_w, const float* mask, long tokens,
                        float* out)
{
  LayerWeights w;
  w.input_layernorm = wts[0];
  w.post_attention_layernorm = wts[1];
  w.q_proj = wts[2];
  w.k_proj = wts[3];
  w.v_proj = wts[4];
  w.o_proj = wts[5];
  w.q_norm = wts[6];
  w.k_norm = wts[7];
  w.q_norm_hw = wts[8];
  w.k_norm_hw = wts[9];
  w.gate_proj = wts[10];
  w.up_proj = wts[11];
  w.down_proj = wts[12];
  LayerDims d;
  d.hidden = (std::size_t)hidden;
  d.heads = (std::size_t)heads;
  d.kv_heads = (std::size_t)kv_heads;
  d.head_dim = (std::size_t)head_dim;
  d.intermediate = (std::size_t)inter;
  d.rms_eps = eps;
  d.theta_t = theta_t;
  d.theta_hw = theta_hw;
  const std::vector<int> t(pos_t, pos_t + tokens), h(pos_h, pos_h + tokens),
      ww(pos_w, pos_w + tokens);
  decoder_layer(x, w, d, t, h, ww, mask, (std::size_t)tokens, out);
}

void refx_time_schedule(int num_steps, double shift, float* out)
{
  const std::vector<float> t = time_schedule(num_steps, shift);
  std::memcpy(out, t.data(), t.size() * sizeof(float));
}

double refx_optimized_scale(const float* pos, const float* neg, long n)
{
  return optimized_scale(pos, neg, (std::size_t)n);
}


// ---- the image path (src/u15-ref.cc: vision_embed, conv_decoder,
// patchify_channel_first_hwc, timestep_sinusoid, gelu_erf) ----

void refx_vision_embed(const float* px, const float* patch_w, const float* patch_b,
                       const float* dense_w, const float* dense_b, int grid_h, int grid_w,
                       int patch_px, int hidden, int llm_hidden, int merge, double theta,
                       float* out)
{
  VisionWeights w;
  w.patch_w = patch_w;
  w.patch_b = patch_b;
  w.dense_w = dense_w;
  w.dense_b = dense_b;
  vision_embed(px, w, grid_h, grid_w, patch_px, hidden, llm_hidden, merge, theta, out);
}

void refx_conv_decoder(const float* x_chw, const float* conv1_w, const float* conv1_b,
                       const float* conv2_w, const float* conv2_b, int in_ch, int th, int tw,
                       int hidden_ch, float* out_chw)
{
  HeadWeights w;
  w.conv1_w = conv1_w;
  w.conv1_b = conv1_b;
  w.conv2_w = conv2_w;
  w.conv2_b = conv2_b;
  conv_decoder(x_chw, w, in_ch, th, tw, hidden_ch, out_chw);
}

void refx_patchify_channel_first_hwc(const float* img_hwc, int c, int h, int w, int p,
                                     float* out)
{
  patchify_channel_first_hwc(img_hwc, c, h, w, p, out);
}

void refx_timestep_sinusoid(double t, int dim, double max_period, float* out)
{
  const std::vector<float> e = timestep_sinusoid(t, dim, max_period);
  std::memcpy(out, e.data(), e.size() * sizeof(float));
}

void refx_gelu_erf(float* x, long n) { gelu_erf(x, (std::size_t)n); }

}  // extern "C"
