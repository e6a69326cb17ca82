/*
 * u15c.h -- C ABI of libu15c.so, the B200 (sm_100a) implementation of the
 * SenseNova-U1.5 Mixture-of-Transformers backbone layer.
 *
 * The entry points replace the operator surface the reference's backbone
 * calls (class MetalOps, src/u15-metal-ops.h:59-403 of the reference), the
 * backbone itself (class U15Backbone, src/u15-backbone.h:67-170) and the
 * weight bind step (U15Weights::load, src/u15-weights.h:152-197). Each
 * declaration names the reference interface it replaces.
 *
 * Conventions (as the reference's):
 *   - weights [out][in]; activations token-major [tokens][dim]; bf16 unless
 *     a name says i8/f32; every pointer argument is a DEVICE pointer unless
 *     documented as host;
 *   - attention q is head-major [heads][tokens][128]; the K/V cache is either
 *     the reference's contiguous [kv_heads][capacity][128] (page_table ==
 *     NULL, `cap` = capacity in tokens) or a paged pool
 *     [num_pages][kv_heads][64][128] addressed through a device int32 page
 *     table of logical page -> physical page (64 tokens per page);
 *   - head_dim is 128 (the model's); the split RoPE ranges are t [0,64),
 *     h [64,96), w [96,128);
 *   - every call returns U15C_OK (0) or an error code; u15c_last_error()
 *     gives this thread's message for the last failure. Calls that launch
 *     work are asynchronous on `stream` and allocate nothing.
 *   - a device-side wait that runs out (a kernel-internal watchdog, about
 *     2 s) writes a code into the device status word instead of hanging;
 *     u15c_sync() and u15c_device_status() report it.
 */
#ifndef U15C_H
#define U15C_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef void* u15c_stream; /* a cudaStream_t (NULL: the legacy default stream) */

#define U15C_OK 0
#define U15C_EINVAL 1   /* bad argument, refused before any launch */
#define U15C_ECUDA 2    /* a CUDA runtime/driver call failed */
#define U15C_ENOMEM 3   /* device allocation failed */
#define U15C_EDEVICE 4  /* a kernel's bounded wait ran out (device status word) */
#define U15C_ESTOPPED 5 /* the cooperative stop fired (U15Backbone::kStopped) */

#define U15C_EPI_STORE 0    /* y = acc (+ bias) */
#define U15C_EPI_RESIDUAL 1 /* y = resid + acc (o_proj / down_proj + add) */
#define U15C_EPI_SWIGLU 2   /* gate|up rows interleaved in 128-row blocks: y = silu(g)*u */
#define U15C_EPI_STORE_F32 3 /* y f32 [M][N] = acc (+ bias): a row-parallel partial product */

#define U15C_ATTN_BIDIRECTIONAL 0 /* Attn::Bidirectional, src/u15-backbone.h:48-57 */
#define U15C_ATTN_CAUSAL 1        /* Attn::Causal */
#define U15C_ATTN_BLOCK_CAUSAL 2  /* Attn::BlockCausal */

#define U15C_EXPERT_UND 0 /* Expert::Und, src/u15-backbone.h:46 */
#define U15C_EXPERT_GEN 1 /* Expert::Gen (the _mot_gen weight set) */

/* ------------------------------------------------------------------ */
/* library                                                             */
/* ------------------------------------------------------------------ */

/* Message of this thread's last failed call ("" if none). */
const char* u15c_last_error(void);
const char* u15c_version(void);

/* Prepare `device` (makes it current, reads its SM count, allocates the
 * device status word). Replaces MetalOps::init (src/u15-metal-ops.cc:39-245),
 * which validates every kernel: here every kernel is compiled in, so init
 * checks the device is sm_100 and records its properties. Other calls
 * initialise the current device on first use. */
int u15c_init(int device, unsigned flags);

/* Read and clear the device status word of `device` (0 = no watchdog fired). */
int u15c_device_status(int device, unsigned* code);

/* cudaStreamSynchronize + the status word: U15C_EDEVICE if a watchdog fired. */
int u15c_sync(u15c_stream stream);

/* The bound of every device-side wait of `device`'s kernels, in ns (0: the
 * default, 2 s). Waits that run out record a code in the status word and
 * unwind instead of hanging. Set it between passes, with no kernel of this
 * library in flight on the device. No reference counterpart: the reference's
 * kernels do not wait on one another. */
int u15c_set_wait_limit(int device, unsigned long long ns);

/* One device thread waits (bounded by the wait limit) until *counter >=
 * target with acquire semantics at system scope, so the stream's later work
 * sees what the counter's writers stored before incrementing it; the gate
 * the fused tensor-parallel reduction puts after each row-parallel product.
 * On a wait that runs out the status word holds 0x106 and the stream moves
 * on. counter: device or peer-mapped memory, 8-byte aligned. */
int u15c_wait_counter(u15c_stream stream, const unsigned long long* counter,
                      unsigned long long target);

/* ------------------------------------------------------------------ */
/* GEMMs                                                               */
/* ------------------------------------------------------------------ */

/* MetalOps::linear (src/u15-metal-ops.h:102-108, .cc:448-468):
 * y[M][N] = x[M][K] w[N][K]^T (+ bias[N]). K must be a multiple of 8. */
int u15c_linear_bf16(u15c_stream stream, const void* x, const void* w, const void* bias,
                     void* y, int M, int K, int N);

/* The MoT token-routed projection (the reference selects the expert per
 * pass at src/u15-backbone.cc:189; here one launch routes per segment).
 * w_stack: [n_experts][N][K]; rows [seg_off[i], seg_off[i+1]) use expert
 * seg_expert[i] (host arrays, nseg <= 8, segments cover [0, M)).
 * epilogue: U15C_EPI_STORE (y [M][N], optional bias [n_experts][N]),
 * U15C_EPI_RESIDUAL (y = resid + acc; y may equal resid), U15C_EPI_SWIGLU
 * (N = 2*inter rows interleaved [gate 128 | up 128]..., y [M][N/2]; the
 * layout MetalOps::swiglu_fused expects, src/u15-metal-ops.h:121-135, with
 * 128-row blocks instead of single rows). */
int u15c_mot_linear_bf16(u15c_stream stream, const void* x, const void* w_stack,
                         int n_experts, const int* seg_off, const int* seg_expert, int nseg,
                         int epilogue, const void* bias, const void* resid, void* y, int M,
                         int K, int N);

/* Symmetric per-row int8 quantisation (per token for activations, per
 * output channel for weights): scale = absmax/127, q = rn_even(x/scale)
 * clamped to +-127. The activation half of i8_gemm
 * (src/u15-metal-ops.h:71-98; BASELINE's W8A8 rule). */
int u15c_quant_rows_i8(u15c_stream stream, const void* x, int8_t* q, float* scale, int rows,
                       int cols);

/* i8_gemm W8A8 (src/u15-metal-ops.cc:291-306, I8GemmContext::gemm):
 * acc = xq[M][K] . wq[N][K]^T in int32 (exact), y = bf16(acc*s_tok[m]*s_ch[n]
 * (+ bias)). acc_dump, when non-NULL, receives the raw int32 [M][N]. */
int u15c_linear_i8(u15c_stream stream, const int8_t* xq, const float* s_tok, const int8_t* wq,
                   const float* s_ch, const void* bias, void* y, int32_t* acc_dump, int M, int K,
                   int N);

/* The routed W8A8 projection: wq_stack [n_experts][N][K], s_ch_stack
 * [n_experts][N]; segments and epilogues as u15c_mot_linear_bf16. */
int u15c_mot_linear_i8(u15c_stream stream, const int8_t* xq, const float* s_tok,
                       const int8_t* wq_stack, const float* s_ch_stack, int n_experts,
                       const int* seg_off, const int* seg_expert, int nseg, int epilogue,
                       const void* resid, void* y, int32_t* acc_dump, int M, int K, int N);

/* ------------------------------------------------------------------ */
/* norms, RoPE, layout                                                 */
/* ------------------------------------------------------------------ */

/* MetalOps::rms_norm (src/u15-metal-ops.h:146-154). dim % 8 == 0. */
int u15c_rms_norm(u15c_stream stream, const void* x, const void* w, void* y, int rows, int dim,
                  float eps);
/* The same with one gain row per expert, w_stack [n_experts][dim]. */
int u15c_mot_rms_norm(u15c_stream stream, const void* x, const void* w_stack, int n_experts,
                      const int* seg_off, const int* seg_expert, int nseg, void* y, int rows,
                      int dim, float eps);

/* RMSNorm fused with the W8A8 activation quantisation: the normed row, rounded
 * to bf16 as u15c_mot_rms_norm stores it, quantised per token by the rule of
 * u15c_quant_rows_i8 (codes bit-identical to the two calls in sequence).
 * dim <= 4096, dim % 8 == 0. Feeds u15c_mot_linear_i8 directly. */
int u15c_mot_rms_norm_quant_i8(u15c_stream stream, const void* x, const void* w_stack,
                               int n_experts, const int* seg_off, const int* seg_expert, int nseg,
                               int8_t* q, float* scale, int rows, int dim, float eps);

/* MetalOps::split_qk_norm (src/u15-metal-ops.h:156-161,
 * src/u15-kernels.metal:50-87): in place on token-major [tokens][heads*128]. */
int u15c_split_qk_norm(u15c_stream stream, void* x, const void* w_t, const void* w_hw,
                       int heads, int tokens, int head_dim, float eps);

/* MetalOps::split_rope (src/u15-metal-ops.h:163-169,
 * src/u15-kernels.metal:118-157): in place; cos/sin f32 [tokens][128]. */
int u15c_split_rope(u15c_stream stream, void* x, const float* cos_tab, const float* sin_tab,
                    int heads, int tokens, int head_dim, int d_t, int d_h);

/* MetalOps::build_rope_tables (src/u15-metal-ops.h:171-185, .cc:547-605),
 * on the device with fp64 angles. pos_* are device int32 [tokens]. */
int u15c_build_rope_tables(u15c_stream stream, const int32_t* pos_t, const int32_t* pos_h,
                           const int32_t* pos_w, int tokens, int head_dim, int d_t, int d_h,
                           double theta_t, double theta_hw, float* cos_tab, float* sin_tab);

/* The QKV post-processing of one layer, fused: split q/k norm (per-expert
 * gains, norms_stack [n_experts][4][64] = q_norm, q_norm_hw, k_norm,
 * k_norm_hw), split RoPE, q -> head-major q_out [heads][T][128], k/v
 * appended to the cache at token kv_off. Replaces split_qk_norm x2,
 * split_rope x2, transpose_thd and transpose_into_cache x2
 * (src/u15-backbone.cc:199-214). qkv is token-major [T][(heads+2*kv_heads)*128]. */
int u15c_qkv_post(u15c_stream stream, const void* qkv, const void* norms_stack, int n_experts,
                  const int* seg_off, const int* seg_expert, int nseg, const float* cos_tab,
                  const float* sin_tab, void* q_out, void* k_cache, void* v_cache,
                  const int32_t* page_table, int cap, int heads, int kv_heads, int T, int kv_off,
                  float eps);

/* MetalOps::transpose_thd / transpose_htd (src/u15-metal-ops.h:332-342). */
int u15c_transpose_thd(u15c_stream stream, const void* in, void* out, int T, int H, int D);
int u15c_transpose_htd(u15c_stream stream, const void* in, void* out, int T, int H, int D);

/* MetalOps::transpose_into_cache (src/u15-metal-ops.h:344-348): [T][H*128]
 * -> contiguous cache [H][cap][128] at token `offset` (the KV append). */
int u15c_transpose_into_cache(u15c_stream stream, const void* in, void* cache, int T, int H,
                              int D, int cap, int offset);
/* The same into a paged pool [pages][H][64][128] through `page_table`. */
int u15c_kv_append(u15c_stream stream, const void* in, void* pages, const int32_t* page_table,
                   int T, int H, int offset);

/* ------------------------------------------------------------------ */
/* elementwise (src/u15-metal-ops.h:207-212, 359-370)                   */
/* ------------------------------------------------------------------ */
int u15c_swiglu(u15c_stream stream, const void* gate, const void* up, void* y, int rows,
                int inter);
int u15c_add(u15c_stream stream, void* dst, const void* src, long n);
int u15c_add_row(u15c_stream stream, void* dst, const void* row, int rows, int dim);
int u15c_silu(u15c_stream stream, void* x, long n);

/* ------------------------------------------------------------------ */
/* attention                                                           */
/* ------------------------------------------------------------------ */

/* Bytes of device workspace the Sage int8-QK path needs at this geometry
 * (the role of MetalOps::sage_lend's arena, src/u15-metal-ops.h:316-318). */
size_t u15c_sage_workspace_bytes(int hq, int hkv, int tq, int tk);

/* Grouped-query flash attention, head_dim 128.
 * q [hq][tq][128]; K/V as described at the top (contiguous when page_table
 * is NULL, then `cap` is the capacity); out token-major [tq][hq*128].
 * mode: U15C_ATTN_*; q_offset places the queries in the key range (causal
 * rules); t_index: device int32 [tk] (block-causal). sage_ws non-NULL
 * selects the Sage int8-QK path (bidirectional only; size from
 * u15c_sage_workspace_bytes). Replaces MetalOps::sdpa, ::sdpa_steel and
 * ::sdpa_block_causal (src/u15-metal-ops.h:214-331). */
int u15c_attention(u15c_stream stream, const void* q, const void* k, const void* v,
                   const int32_t* page_table, int cap, void* out, int hq, int hkv, int tq,
                   int tk, int head_dim, int mode, int q_offset, const int32_t* t_index,
                   void* sage_ws);

/* The same over the model's paged cache layout: K pages
 * [n_pages][hkv][64][128], V pages TRANSPOSED [n_pages][hkv][128][64] (dims as
 * rows of 64 tokens, the operand layout of the tensor-core P.V), page table
 * device int32 (NULL = identity). Every rule runs the tcgen05/TMEM flash
 * kernel: bidirectional (Sage int8-QK when sage_ws is non-NULL), causal and
 * block-causal (fully masked key blocks skipped per 128-row query tile; a
 * block-causal t_index that is not 16-byte aligned, or more than 32768 keys,
 * runs on the mma.sync kernel instead). Replaces MetalOps::sdpa_steel for
 * the denoise pass (src/u15-metal-ops.cc:835-882) and ::sdpa /
 * ::sdpa_block_causal for the prefill (:648-677, 884-908). */
int u15c_attention_paged(u15c_stream stream, const void* q, const void* k_pages,
                         const void* vt_pages, const int32_t* page_table, int n_pages, void* out,
                         int hq, int hkv, int tq, int tk, int head_dim, int mode, int q_offset,
                         const int32_t* t_index, void* sage_ws);

/* The reference's three attention entry points with their own argument
 * order, over the contiguous cache (kv stride = cap tokens):
 * MetalOps::sdpa (src/u15-metal-ops.h:214-232): full or causal. */
int u15c_sdpa(u15c_stream stream, const void* q, const void* k, const void* v, void* out,
              int hq, int hkv, int tq, int tk, int d, int cap, int causal, int q_offset);
/* MetalOps::sdpa_steel (src/u15-metal-ops.h:282-289): bidirectional; Sage
 * when sage_ws is non-NULL. */
int u15c_sdpa_steel(u15c_stream stream, const void* q, const void* k, const void* v, void* out,
                    int hq, int hkv, int tq, int tk, int d, int cap, void* sage_ws);
/* MetalOps::sdpa_block_causal (src/u15-metal-ops.h:320-331). */
int u15c_sdpa_block_causal(u15c_stream stream, const void* q, const void* k, const void* v,
                           void* out, const int32_t* t_index, int hq, int hkv, int tq, int tk,
                           int d, int cap, int q_offset);

/* Sage int8-QK bidirectional attention that allocates nothing: the same
 * computation as u15c_attention with a Sage workspace, but the workspace is a
 * fixed 24 MiB device array inside this library (16 MiB of int8 queries plus
 * keys and scales covers 32 query heads x 4096 tokens over 8 kv heads x 4416
 * keys). It is for callers that cannot call cudaMalloc: a host that plans its
 * device memory up front and may not grow it, a process whose free memory is
 * held by another allocator, a latency-bound caller that cannot take the
 * implicit synchronisation of cudaMalloc/cudaFree. This entry point has no
 * counterpart in the reference.
 * Geometries whose workspace (u15c_sage_workspace_bytes) exceeds 24 MiB are
 * refused with U15C_EINVAL. The first call on a device sets up the array's
 * address for that device (make it before any stream capture). Every call
 * shares the array: calls that overlap on the GPU race and must be
 * serialised by the caller. Every GPU that loads the library holds the
 * 24 MiB until the process exits. Arguments as u15c_attention. */
int u15c_attention_sage_static(u15c_stream stream, const void* q, const void* k, const void* v,
                               const int32_t* page_table, int cap, void* out, int hq, int hkv,
                               int tq, int tk, int head_dim);

/* ------------------------------------------------------------------ */
/* the denoise step (Generator::generate, src/u15-generator.cc:468-706)  */
/* ------------------------------------------------------------------ */

#define U15C_CFG_NONE 0 /* v = v_cond */
#define U15C_CFG_IMG 1  /* v_img + cfg (v_cond - v_img)               (img_cfg == 1) */
#define U15C_CFG_UNC 2  /* v_unc + cfg (v_cond - v_unc)               (t2i, cfg == img_cfg) */
#define U15C_CFG_BOTH 3 /* v_unc + cfg (v_cond - v_img) + icfg (v_img - v_unc) */
#define U15C_NORM_NONE 0      /* CfgNorm::None */
#define U15C_NORM_GLOBAL 1    /* CfgNorm::Global: min(1, |v_cond| / |v|) over the image */
#define U15C_NORM_CHANNEL 2   /* CfgNorm::Channel: the same per 32x32 token */
#define U15C_NORM_ZERO_STAR 3 /* CfgNorm::CfgZeroStar (U15C_CFG_UNC only) */

/* v = (x_pred - img) / denom, fp64 arithmetic (src/u15-generator.cc:582-584);
 * denom = max(1 - t, t_eps). f32 device arrays of n elements. */
int u15c_velocity(u15c_stream stream, const float* x_pred, const float* img, float* v, long n,
                  double denom);
/* The CFG combination and renorm (src/u15-generator.cc:596-693) over [H][W][3]
 * f32 velocities; unused inputs may be NULL. Reductions are fp64 and
 * deterministic; workspace: u15c_cfg_workspace_bytes() bytes of device memory. */
size_t u15c_cfg_workspace_bytes(void);
int u15c_cfg_combine(u15c_stream stream, const float* v_cond, const float* v_unc,
                     const float* v_img, float* out, int H, int W, int form, int norm, double cfg,
                     double icfg, int step, void* workspace);
/* img += dt * v in fp64 (src/u15-generator.cc:701-705). */
int u15c_euler(u15c_stream stream, float* img, const float* v, long n, double dt);

/* The start image (Generator::generate, src/u15-generator.cc:394-417), on the
 * host: out[i] = (float)(noise_scale * d(rng)) for i in [0, n) in order,
 * rng = std::mt19937_64(seed), d = std::normal_distribution<float>(0, 1) --
 * the reference's engine and distribution (the distribution's algorithm is
 * the C++ library's: the same seed gives the reference's image wherever the
 * standard library is the same; the init_noise file is the exact path
 * across libraries). out: HOST float[n] ([H][W][3] channel-last). */
int u15c_init_noise(uint64_t seed, double noise_scale, float* out, long n);

/* GenConfig::init_noise_scale (src/u15-config.cc:106-122): the noise scale
 * for an image of `image_tokens` tokens. mode (GenConfig::noise_scale_mode):
 * U15C_NOISE_CONSTANT = min(noise_scale, max_value); U15C_NOISE_RESOLUTION
 * ("resolution" / "dynamic") = min(sqrt(L / base) * noise_scale, max_value);
 * U15C_NOISE_DYNAMIC_SQRT = min(sqrt(sqrt(L / base) * noise_scale), max_value);
 * base = base_seq_len (64 when <= 0). The reference's defaults: RESOLUTION,
 * noise_scale 1, max_value 16, base 64. Host arithmetic. */
#define U15C_NOISE_CONSTANT 0
#define U15C_NOISE_RESOLUTION 1
#define U15C_NOISE_DYNAMIC_SQRT 2
int u15c_init_noise_scale(int image_tokens, int mode, double noise_scale, double max_value,
                          int base_seq_len, double* out);
/* [H][W][3] f32 <-> [(H/32)*(W/32)][32*32*3] bf16 token rows, channel-last
 * packing (the reference's patchify_channel_last, src/u15-ref.cc). */
int u15c_patchify(u15c_stream stream, const float* img, void* rows, int H, int W);
int u15c_unpatchify(u15c_stream stream, const void* rows, float* img, int H, int W);

/* ------------------------------------------------------------------ */
/* the prefill's inputs from token ids (src/u15-generator.cc:308-392)   */
/* ------------------------------------------------------------------ */

/* out[i][:] = table[ids[i]][:] (bf16 [vocab][hidden] -> [n][hidden]),
 * the embed_tokens lookup; ids are device int32. An id outside [0, vocab)
 * gives a zero row and U15C_EDEVICE at the next u15c_sync. */
int u15c_embed_tokens(u15c_stream stream, const void* table, int vocab, int hidden,
                      const int32_t* ids, int n, void* out);
/* Prompt::thw_indexes (src/u15-prompt.cc:349-386), host arrays: t grows by
 * one per token that is not <IMG_CONTEXT> and by one more right after an
 * <img>, so an image's context tokens share one t; h / w count the context
 * tokens of each image row-major on its merged grid (grid_w / 2 per row),
 * restarting per image. grid_hw: [n_imgs][2] patch grids (h, w). The
 * generated image's tokens then sit at t = max(t) + 1. */
int u15c_thw_indexes(const int32_t* ids, int n, int img_id, int img_ctx_id, const int* grid_hw,
                     int n_imgs, int32_t* t, int32_t* h, int32_t* w);
/* copy image k's patch embeddings [image_tokens[k]][hidden] (device) over
 * the k-th run of <IMG_CONTEXT> rows of x [n][hidden] (ids on the host) */
int u15c_splice_image_rows(u15c_stream stream, void* x, int hidden, const int32_t* ids_host,
                           int n, int img_ctx_id, const void* const* image_embeds,
                           const int* image_tokens, int n_imgs);

/* ------------------------------------------------------------------ */
/* the image path (ImagePath, src/u15-image.h:24-100; CPU forms          */
/* src/u15-ref.cc vision_embed / conv_decoder): patch embedder in,      */
/* pixel head out, timestep + noise-scale embedding. Channel-last.      */
/* ------------------------------------------------------------------ */

typedef struct u15c_image u15c_image;
typedef struct u15c_image_config {
  int vision_hidden;         /* 1024: patch embedding width */
  int llm_hidden;            /* 4096: backbone hidden size */
  int patch;                 /* 16 */
  int merge;                 /* 2: tiles merged by the dense embedding */
  int head_hidden;           /* 1024: the pixel head's conv1 width */
  int freq_dim;              /* 256: the timestep sinusoid's width */
  int noise_scale_embedding; /* 1: add the noise-scale embedder's row */
  double vision_theta;       /* 1e4: the patch embedder's 2-D RoPE */
} u15c_image_config;

/* tensor ids for u15c_image_bind, the checkpoint's shapes; patch/dense
 * take expert 0 (vision_model, understanding) or 1 (vision_model_mot_gen) */
#define U15C_I_PATCH_W 0   /* [vision_hidden][3][p][p] */
#define U15C_I_PATCH_B 1
#define U15C_I_DENSE_W 2   /* [llm_hidden][vision_hidden][m][m] */
#define U15C_I_DENSE_B 3
#define U15C_I_CONV1_W 4   /* [head_hidden][llm_hidden/4][3][3] */
#define U15C_I_CONV1_B 5
#define U15C_I_CONV2_W 6   /* [192][head_hidden/4][3][3] */
#define U15C_I_CONV2_B 7
#define U15C_I_TSTEP_W0 8  /* [llm_hidden][freq_dim] */
#define U15C_I_TSTEP_B0 9
#define U15C_I_TSTEP_W2 10 /* [llm_hidden][llm_hidden] */
#define U15C_I_TSTEP_B2 11
#define U15C_I_NSCALE_W0 12
#define U15C_I_NSCALE_B0 13
#define U15C_I_NSCALE_W2 14
#define U15C_I_NSCALE_B2 15

/* ImagePath::create */
int u15c_image_create(const u15c_image_config* cfg, u15c_image** out);
void u15c_image_destroy(u15c_image* im);
/* bind one tensor (f32/f16/bf16, host or device) into the device layout;
 * the conv kernels are repacked to [cout][ky][kx][cin] for the im2col GEMM
 * (ImagePath::build_conv_weights_, src/u15-image.cc:56-131) */
int u15c_image_bind(u15c_image* im, u15c_stream stream, int tensor, int expert, const void* src,
                    int dtype, int src_on_host);
int u15c_image_bind_random(u15c_image* im, u15c_stream stream, uint64_t seed, float std);
/* ImagePath::patchify_for_embed: img [H][W][3] f32 -> px [(H/p)(W/p)][3p^2]
 * bf16, each patch channel-FIRST */
int u15c_image_patchify(u15c_stream stream, const float* img, void* px, int H, int W, int patch);
/* ImagePath::embed (src/u15-image.cc:145-197): px [gh*gw][3p^2] ->
 * out [(gh/m)(gw/m)][llm_hidden] bf16 */
int u15c_image_embed(u15c_image* im, u15c_stream stream, const void* px, int grid_h, int grid_w,
                     int expert, void* out);
/* ImagePath::timestep_row (src/u15-image.cc:199-251), on the device:
 * out [llm_hidden] f32 */
int u15c_image_timestep_row(u15c_image* im, u15c_stream stream, double t, double noise_ratio,
                            float* out);
/* the row rounded to bf16 and added to every row of x [rows][llm_hidden]
 * (the generator's add_row, src/u15-generator.cc:489-499) */
int u15c_image_add_timestep(u15c_image* im, u15c_stream stream, void* x, int rows, double t,
                            double noise_ratio);
/* ImagePath::decode (src/u15-image.cc:253-303): hidden [th*tw][llm_hidden]
 * bf16 -> out_px [32 th][32 tw][3] f32 (bf16-exact values), model space */
int u15c_image_decode(u15c_image* im, u15c_stream stream, const void* hidden, int th, int tw,
                      float* out_px);
/* ImagePath::to_u8_planar: [H][W][3] model space -> [3][H][W] u8 */
int u15c_image_to_u8_planar(u15c_stream stream, const float* px, uint8_t* out, int H, int W);

/* ------------------------------------------------------------------ */
/* model: weights, KV cache, backbone                                   */
/* ------------------------------------------------------------------ */

typedef struct u15c_model u15c_model; /* U15Weights + U15Backbone */
typedef struct u15c_kv u15c_kv;       /* KvCache, src/u15-backbone.h:60-66 (paged) */

typedef struct u15c_config {
  int n_layers;   /* 42 */
  int hidden;     /* 4096 */
  int heads;      /* 32 */
  int kv_heads;   /* 8 */
  int head_dim;   /* 128 */
  int inter;      /* 12288 */
  int n_experts;  /* 2: und, _mot_gen */
  double eps;     /* 1e-6 */
  double theta_t; /* 5e6 */
  double theta_hw;/* 1e4 */
} u15c_config;

#define U15C_MODEL_INT8 1u /* also bind the W8A8 twin of every projection */

/* tensor ids for u15c_model_bind, the 13 per-expert tensors of
 * src/u15-weights.cc:539-578 */
#define U15C_T_INPUT_LN 0
#define U15C_T_POST_LN 1
#define U15C_T_Q 2
#define U15C_T_K 3
#define U15C_T_V 4
#define U15C_T_O 5
#define U15C_T_Q_NORM 6
#define U15C_T_K_NORM 7
#define U15C_T_Q_NORM_HW 8
#define U15C_T_K_NORM_HW 9
#define U15C_T_GATE 10
#define U15C_T_UP 11
#define U15C_T_DOWN 12
#define U15C_T_FINAL_NORM 13 /* trunk: `norm` (und) / `norm_mot_gen`; layer ignored */

#define U15C_DT_F32 0
#define U15C_DT_F16 1
#define U15C_DT_BF16 2

/* U15Weights::load + U15Backbone::create: allocate the bound layout for
 * cfg (all layers, all experts). */
int u15c_model_create(const u15c_config* cfg, unsigned flags, u15c_model** out);
void u15c_model_destroy(u15c_model* m);

/* Tensor parallelism for one large render (no reference counterpart: the
 * reference runs one device). Rank tp_rank of tp_size (1, 2, 4, 8) holds
 * heads/tp q heads and kv_heads/tp kv heads (column-parallel q/k/v, KV cache
 * sharded by kv head), inter/tp of the MLP (column-parallel gate/up), and
 * the matching columns of o_proj and down_proj (row-parallel). cfg is the
 * FULL model; u15c_model_bind takes full tensors and keeps this rank's
 * share. Before a pass, install the all-reduce the row-parallel products
 * need with u15c_model_set_allreduce. */
int u15c_model_create_tp(const u15c_config* cfg, unsigned flags, int tp_rank, int tp_size,
                         u15c_model** out);
int u15c_model_tp(const u15c_model* m, int* tp_rank, int* tp_size);
/* fn(ctx, count, stream): sum buf[0 : count) over the tensor-parallel ranks
 * in place (f32), ordered after the work already on `stream` and before the
 * work enqueued on it next (e.g. ncclAllReduce on that stream); 0 = ok.
 * buf: device, at least tokens x hidden floats of the largest pass. */
typedef int (*u15c_allreduce_fn)(void* ctx, long count, u15c_stream stream);
int u15c_model_set_allreduce(u15c_model* m, u15c_allreduce_fn fn, void* ctx, float* buf,
                             long buf_elems);
/* The fused form: o_proj / down_proj and their all-reduce in ONE kernel over
 * NVLink peer memory (each rank's partial tile, rounded to bf16, goes to the
 * tile's owner; the owner adds the ranks' partials in f32 and the residual
 * and stores the bf16 result into every rank's activations). Each rank exports a region sized
 * for passes of up to max_tokens tokens and gets a U15C_TP_BLOB_BYTES blob
 * (a CUDA IPC handle and the GPU's UUID); the caller gathers the blobs of
 * all ranks in rank order (e.g. an all-gather) and imports them. Then every
 * pass uses the fused kernel; the ranks must run the same passes in the same
 * order, each on its own GPU (refused otherwise). */
#define U15C_TP_BLOB_BYTES 128
int u15c_model_tp_export(u15c_model* m, int max_tokens, void* blob);
int u15c_model_tp_import(u15c_model* m, const void* blobs);
/* Unmap the peers' regions (waits for this device's work first). Every rank
 * calls it and the ranks meet (a barrier) before any of them destroys its
 * model: a region may not be freed while a peer still maps it. */
int u15c_model_tp_disconnect(u15c_model* m);

/* U15Weights bind_bf16_/bind_matrix_ (src/u15-weights.cc:102-151,
 * 516-603): convert one tensor (f32/f16/bf16, host or device) to bf16 with
 * round-to-nearest-even and place it in the bound layout (q|k|v fused,
 * gate|up interleaved, experts stacked). */
int u15c_model_bind(u15c_model* m, u15c_stream stream, int layer, int expert, int tensor,
                    const void* src, int dtype, int src_on_host);
/* The checkpoint's affine-quantized matrices (bind_matrix_,
 * src/u15-weights.cc:248-325): codes u32 [N][K*bits/32] (code k of a row at
 * bits (k % (32/bits)) * bits of word k / (32/bits)), scales and biases
 * [N][K/group] (F16 / BF16 / F32, rounded to bf16 as the reference binds
 * them); out bf16 [N][K] = scale * code + bias. bits 4 or 8, group 32 or 64.
 * Dequantized once at bind time; pass `out` to u15c_model_bind (BF16). */
int u15c_dequant_affine(u15c_stream stream, const uint32_t* codes, const void* scales,
                        const void* biases, int scale_dtype, int N, int K, int bits, int group,
                        void* out);
/* Seeded synthetic weights (no checkpoint): projections N(0, std), norm
 * gains N(norm_mean, norm_std). */
int u15c_model_bind_random(u15c_model* m, u15c_stream stream, uint64_t seed, float std,
                           float norm_mean, float norm_std);
/* Build the W8A8 twins (per-output-channel int8) from the bound bf16. */
int u15c_model_finalize(u15c_model* m, u15c_stream stream);

size_t u15c_model_weight_bytes(const u15c_model* m);
/* U15Backbone::scratch_bytes (src/u15-backbone.cc:150-165) of this layout. */
size_t u15c_model_scratch_bytes(const u15c_model* m, int n);
/* U15Backbone::kv_bytes (src/u15-backbone.cc:54-61), rounded to pages. */
size_t u15c_model_kv_bytes(const u15c_model* m, int capacity);

/* U15Backbone::make_cache (src/u15-backbone.cc:63-90): a paged bf16 cache of
 * `capacity` tokens for every layer: per layer K pages [pages][kv_heads][64][128]
 * and V pages stored transposed [pages][kv_heads][128][64], zero-initialised. */
int u15c_kv_create(u15c_model* m, int capacity, u15c_kv** out);
void u15c_kv_destroy(u15c_kv* kv);
int u15c_kv_capacity(const u15c_kv* kv);
/* Replace the logical->physical page map (host int32[n], a permutation of
 * the cache's pages); the paged layout is then exercised non-contiguously. */
int u15c_kv_set_page_table(u15c_kv* kv, const int32_t* pages_host, int n);
/* The device pools of one layer (K pages, transposed V pages), the page
 * table and the number of pages, for u15c_attention_paged. Any out
 * pointer may be NULL. */
int u15c_kv_pages(u15c_kv* kv, int layer, void** k_pages, void** vt_pages,
                  const int32_t** page_table, int* n_pages);
/* Read one layer's K or V for tokens [0, n) into a contiguous
 * [kv_heads][n][128] buffer (tests, diagnostics). */
int u15c_kv_read(u15c_kv* kv, u15c_stream stream, int layer, int which_v, void* out, int n);
/* Write a prefix of one layer's K or V from a contiguous [kv_heads][n][128]
 * buffer at tokens [0, n) (a frozen prefix prepared elsewhere). */
int u15c_kv_write(u15c_kv* kv, u15c_stream stream, int layer, int which_v, const void* in,
                  int n);

#define U15C_FWD_INT8 1u /* W8A8 projections (i8_gemm) */
#define U15C_FWD_SAGE 2u /* Sage int8-QK on the bidirectional pass */

/* The Sage tier's `dense_layers` (vpipe::genai::sage::Config, set through
 * MetalOps::set_sage, src/u15-metal-ops.cc:789-814, and honoured by
 * sdpa_steel, :852-855): under U15C_FWD_SAGE, layers [0, n) keep the bf16
 * attention and layers >= n take the int8-QK one. Default 0 (the
 * reference's default, every layer Sage). */
int u15c_model_set_sage_dense_layers(u15c_model* m, int n);

/* One MoT layer for one branch: U15Backbone::layer_step_
 * (src/u15-backbone.cc:173-257), x [n][hidden] updated in place, tokens
 * routed per segment (host seg arrays), K/V written at kv_off, attention
 * over kv_len keys by rule `attn`. pos_* are device int32 [n]; t_index is
 * device int32 [kv_len] (block-causal). */
int u15c_layer_forward(u15c_model* m, u15c_stream stream, int layer, void* x, int n,
                       const int* seg_off, const int* seg_expert, int nseg, u15c_kv* kv,
                       int kv_off, int kv_len, const int32_t* pos_t, const int32_t* pos_h,
                       const int32_t* pos_w, int attn, const int32_t* t_index, unsigned flags);

/* U15Backbone::forward (src/u15-backbone.cc:259-277): every layer, with a
 * cooperative stop polled before each layer (stop(ctx) != 0 returns
 * U15C_ESTOPPED, src/u15-backbone.cc:386-397). stop may be NULL. */
int u15c_forward(u15c_model* m, u15c_stream stream, void* x, int n, const int* seg_off,
                 const int* seg_expert, int nseg, u15c_kv* kv, int kv_off, int kv_len,
                 const int32_t* pos_t, const int32_t* pos_h, const int32_t* pos_w, int attn,
                 const int32_t* t_index, unsigned flags, int (*stop)(void*), void* stop_ctx);

/* One branch of a multi-branch pass (U15Backbone::PassSlot,
 * src/u15-backbone.h:112-124). */
typedef struct u15c_slot {
  u15c_kv* kv;
  int kv_off;              /* where this branch's K/V are written */
  int kv_len;              /* keys attended */
  const int32_t* pos_t;    /* device int32 [n] */
  const int32_t* pos_h;
  const int32_t* pos_w;
  const int32_t* t_index;  /* block-causal only (device int32 [kv_len]) */
} u15c_slot;

/* U15Backbone::forward_many (src/u15-backbone.cc:279-432): every layer for
 * every branch, layer-outermost. The branches' activations are one
 * contiguous buffer x [nslots * n][hidden] (slot i at rows [i*n, (i+1)*n)),
 * all routed to `expert`; the row-wise work of each layer (norms and the four
 * projection GEMMs) runs once over all nslots * n rows, the attention and the
 * K/V append per branch against its own cache. stop as u15c_forward. */
int u15c_forward_many(u15c_model* m, u15c_stream stream, void* x, int n, const u15c_slot* slots,
                      int nslots, int expert, int attn, unsigned flags, int (*stop)(void*),
                      void* stop_ctx);

/* U15Backbone::final_norm (src/u15-backbone.cc:140-148). */
int u15c_final_norm(u15c_model* m, u15c_stream stream, void* x, int n, int expert);

/* End to end through host memory: copy x_host [n][hidden] bf16 to the
 * device, run u15c_layer_forward, copy the result back to out_host (both
 * should be pinned for full speed). Synchronous. */
int u15c_layer_forward_host(u15c_model* m, u15c_stream stream, int layer, const void* x_host,
                            void* out_host, int n, const int* seg_off, const int* seg_expert,
                            int nseg, u15c_kv* kv, int kv_off, int kv_len, const int32_t* pos_t,
                            const int32_t* pos_h, const int32_t* pos_w, int attn,
                            const int32_t* t_index, unsigned flags);

/* The same layer through host memory, enqueued without waiting (a serving
 * loop's form of u15c_layer_forward_host; the reference's layer calls are
 * synchronous, so this entry has no counterpart there). The upload runs on
 * the model's upload stream, the layer on `stream` once it has landed, the
 * download on the model's download stream once the layer is done. Two device
 * staging buffers are used in turn, so call k + 1's upload and call k - 1's
 * download run during call k's layer: back-to-back calls keep the copies off
 * the critical path. x_host must stay unchanged and out_host unread until the
 * call's results are drained: u15c_layer_host_drain makes `stream` wait for
 * every download enqueued so far, after which synchronising `stream` (or
 * u15c_sync) completes them. Both host buffers should be pinned. Not for
 * tensor-parallel models (U15C_EINVAL). */
int u15c_layer_forward_host_async(u15c_model* m, u15c_stream stream, int layer,
                                  const void* x_host, void* out_host, int n, const int* seg_off,
                                  const int* seg_expert, int nseg, u15c_kv* kv, int kv_off,
                                  int kv_len, const int32_t* pos_t, const int32_t* pos_h,
                                  const int32_t* pos_w, int attn, const int32_t* t_index,
                                  unsigned flags);

/* Make `stream` wait for every download u15c_layer_forward_host_async has
 * enqueued on this model so far (no host wait). */
int u15c_layer_host_drain(u15c_model* m, u15c_stream stream);

#ifdef __cplusplus
}
#endif
#endif /* U15C_H */
