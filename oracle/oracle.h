/* CPU oracle for the VoxCPM2 patch loop (TEST INFRASTRUCTURE ONLY).
 *
 * A plain fp32 restatement of the reference's ncnn CPU path, used by the
 * tests, by __graft_entry__.smoke() and by bench.py's cpu_baseline / reference
 * arm as the checker. The product library (libvoxcpm2_cuda.so) never links,
 * loads or calls anything declared here.
 *
 * Weights are the same fp16 blobs the CUDA library receives (IEEE half bits),
 * widened to fp32 on use, exactly as ncnn does when a graph whose .bin was
 * exported with fp16=1 runs with fp16 storage disabled (synthesizer.cpp:999-1004).
 */
#pragma once
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct orc_desc {
    int32_t hidden;        /* LM hidden H */
    int32_t ffn;           /* LM SwiGLU intermediate F */
    int32_t q_heads;
    int32_t kv_heads;
    int32_t head_dim;
    int32_t base_layers;
    int32_t res_layers;
    int32_t dit_hidden;    /* Hd */
    int32_t dit_ffn;
    int32_t dit_layers;
    int32_t dit_q_heads;
    int32_t dit_kv_heads;
    int32_t feat_dim;      /* D = 64 */
    int32_t patch_size;    /* P = 4 */
    int32_t vocab;
    int32_t fsq_dim;
    float fsq_scale;
    float rms_eps;
    float rope_theta;
    int32_t rope_original_max;
    float base_residual_scale; /* muP depth scale, 1 = off */
    float res_residual_scale;
    float dit_residual_scale;
    float embed_scale;
    int32_t audio_start_token;
    int32_t max_generation_patches;
} orc_desc;

typedef struct orc_model orc_model;

void orc_set_threads(int threads);
int orc_get_threads(void);

/* ---- per-op restatements ------------------------------------------------ */

/* VoxCPM2SDPA::forward CPU path (src/ncnn_layers/sdpa/voxcpm2_sdpa.cpp:115-260).
 * Layout is ncnn's w=dim, h=seq, c=heads, planes packed contiguously:
 *   q [heads][src][d], k/v [groups][cur][d|dv], mask [mask_c][src][past+cur] or NULL,
 *   past_k/v [groups][past][d] (past may be 0), out [heads][src][dv],
 *   out_k/out_v [groups][past+cur][d] or NULL.  scale 0 -> 1/sqrt(d). */
int orc_sdpa(const float* q, int heads, int src, int d,
             const float* k, const float* v, int groups, int cur, int dv,
             const float* mask, int mask_c,
             const float* past_k, const float* past_v, int past,
             float scale, float* out, float* out_k, float* out_v);

/* VoxCPM2TimestepEmbedding::forward (timestep_embedding.cpp:128-160). */
void orc_timestep_embedding(const float* in, int batch, int half_dim, float scale,
                            float max_period, int schedule_mode, float* out);

/* make_decoder_mask (kvcache.cpp:216-230): out [cur][past+cur]. */
void orc_decoder_mask(int cur, int past, float* out);

/* Synthesizer::Impl::make_rope_cache (synthesizer.cpp:940-974) with
 * prepare_rope_inverse_frequency (:928-938). short/long factor arrays hold
 * head_dim/2 entries; NULL long -> short is always used. cos/sin [len][head_dim]. */
void orc_rope_cache(int head_dim, float theta, int original_max, const float* short_factor,
                    const float* long_factor, int position_start, int length, float* cos_out,
                    float* sin_out);

/* CfmWorkspace t_span (synthesizer.cpp:49-60): out [timesteps+1]. */
void orc_sway_t_span(int timesteps, float* out);
/* zero_init_steps (synthesizer.cpp:123). */
int orc_zero_init_steps(int timesteps);
/* optimized_scale (synthesizer.cpp:76-84). */
float orc_optimized_scale(const float* positive, const float* negative, int n);
/* max_patches_for_target (synthesizer.cpp:216-220). */
int orc_max_patches(int target_text_tokens, int hard_cap);
/* std::mt19937 rng(seed) + a fresh std::normal_distribution<float>(0,1) per
 * patch, 'per_patch' draws each (synthesizer.cpp:108-112, 452). */
void orc_noise_table(uint32_t seed, int patches, int per_patch, float* out);

/* ---- model ------------------------------------------------------------- */

orc_model* orc_model_create(const orc_desc* desc);
void orc_model_destroy(orc_model* model);
/* number of fp16 elements of a component blob; component ids follow
 * src/components.h:16-29 (text_embed=0 ... dit_estimator=8). */
size_t orc_component_count(const orc_desc* desc, int component);
/* The blob is referenced, not copied: it must outlive the model. */
int orc_set_weights(orc_model* model, int component, const uint16_t* fp16, size_t count);

/* LongRoPE factors of the base decoder (n >= head_dim / 2 each, the first head_dim / 2
 * used; long may be NULL): setting.rope.short_factor / long_factor. Returns -1 on a
 * short table or a factor <= 0. */
int orc_set_rope_factors(orc_model* model, const float* short_factor, const float* long_factor, int n);

/* KV caches of one utterance (HostDecoderKvCache, kvcache.cpp:39-93). */
void orc_reset_caches(orc_model* model);
int orc_token_count(const orc_model* model, int which);
/* read back layer 'layer' of a cache: k/v [kv_heads][tokens][head_dim] */
int orc_read_cache(const orc_model* model, int which, int layer, float* k, float* v);

/* run_decoder_with_kv (kvcache.cpp:232-279) over the DecoderKv graph
 * (tools/export_components.py:496-550). which 0 = base (RoPE), 1 = residual.
 * embed [n][H]; mask [n][past+n] or NULL (-> make_decoder_mask(n, past));
 * cos/sin [n][head_dim] or NULL (-> rope table for [past, past+n); base only).
 * out [n][H] (after the final norm). */
int orc_decoder_forward(orc_model* model, int which, const float* embed, int n, const float* mask,
                        const float* cos, const float* sin, float* out);

/* Small component graphs (export_components.py:553-599). rows = tokens. */
int orc_text_embed(const orc_model* model, const int32_t* ids, int n, float* out);
int orc_fsq(const orc_model* model, const float* in, int rows, float* out);
int orc_fusion_proj(const orc_model* model, const float* lm, const float* feat, int rows, float* out);
int orc_dit_proj(const orc_model* model, const float* lm, const float* res, float* out /*[2*Hd]*/);
int orc_stop_head(const orc_model* model, const float* hidden, float* logits /*[2]*/);
/* latent d-major [D][P] (synthesizer.cpp:172-185 transposes it to frame-major) */
int orc_feat_encoder(const orc_model* model, const float* latent_dp, float* out /*[H]*/);

/* DitEstimator.forward (export_components.py:661-689); inputs exactly as
 * cfm_sample binds them (synthesizer.cpp:137-145):
 *  x_in [2][D][P], mu_in [2][2*Hd], t_in [2] (= {step-1, T}, schedule mode),
 *  cond_in [2][D][P], dt_in [2] (raw delta times) -> out [2][D*P]. */
int orc_dit_estimator(const orc_model* model, const float* x_in, const float* mu_in,
                      const float* t_in, const float* cond_in, const float* dt_in, float* out);

/* cfm_sample (synthesizer.cpp:86-170) with the patch's 256 noise draws given. */
int orc_cfm_sample(const orc_model* model, const float* mu, const float* cond, const float* noise,
                   int timesteps, float cfg, float* out_latent);

/* generate_with_caches for a text-only prefix (synthesizer.cpp:353-659, without
 * the audio VAE decode). Outputs (all optional, may be NULL):
 *   latents [max_patches][D*P], lm_hidden / res_hidden [max_patches][H] (the
 *   hidden states entering each patch), stop_logits [max_patches][2].
 * *out_patches = number of patches generated. */
int orc_generate(orc_model* model, const int32_t* text_ids, int n_text, int min_patches,
                 int timesteps, float cfg, int max_patches_override, uint32_t seed,
                 float* latents, float* lm_hidden, float* res_hidden, float* stop_logits,
                 int* out_patches);

/* Test hook: record the pre-rounding FSQ values (tanh(z) * fsq_scale, [rows][fsq_dim])
 * of the next 'rows' FSQ rows into buf (NULL stops); returns the rows recorded into
 * the previous buffer. During orc_generate row p is the FSQ of patch p, whose output
 * is the LM hidden state entering patch p + 1. */
int orc_trace_fsq(orc_model* model, float* buf, int rows);

/* Test hook: the next 'rows' FSQ rows take their codes from codes [rows][fsq_dim]
 * (integers: the rounded tanh(z) * fsq_scale) instead of their own rounding, so the
 * oracle can follow another implementation through a value that sits on a rounding
 * boundary; NULL stops. Returns the rows the previous buffer served. */
int orc_force_fsq(orc_model* model, const float* codes, int rows);

/* The same from a prefix given row by row (synthesizer.cpp:43-47, 359-535): token
 * ids of every row, is_audio flags, the audio rows' latent patches in row order
 * ([n_audio][D*P], d-major); n_target_text sizes max_patches (the target text's
 * token count). A prefix of text ids + audio_start with no audio rows gives
 * orc_generate's result. */
int orc_generate_rows(orc_model* model, const int32_t* token_ids, const int32_t* is_audio,
                      const float* audio_latents, int n_rows, int n_target_text, int min_patches, int timesteps,
                      float cfg, int max_patches_override, uint32_t seed, float* latents, float* lm_hidden,
                      float* res_hidden, float* stop_logits, int* out_patches);

#ifdef __cplusplus
}
#endif
