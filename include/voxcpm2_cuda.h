/* C ABI of libvoxcpm2_cuda: the B200 (sm_100a) VoxCPM2 patch loop.
 *
 * This is the thin shim the reference's C++ host runtime calls instead of its
 * ncnn graphs for the autoregressive patch loop. Each entry point names the
 * reference routine it replaces. Conventions (mirroring include/voxcpm2/c_api.h):
 *   - every function returning int32_t returns a vxc_status and never throws;
 *     on failure vxc_last_error() holds this thread's message (valid until the
 *     thread's next failing call);
 *   - unless stated otherwise pointers are HOST memory, fp32, C order;
 *   - calls on one vxc_stream are serialised by the library; distinct streams
 *     (e.g. one host thread each) run concurrently and share their device's
 *     read-only weights;
 *   - nothing falls back to the CPU: without a usable CUDA device calls fail.
 */
#pragma once

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__) || defined(__clang__)
#define VXC_API __attribute__((visibility("default")))
#else
#define VXC_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define VXC_ABI_VERSION 1u

typedef struct vxc_device vxc_device;
typedef struct vxc_stream vxc_stream;
typedef struct vxc_group vxc_group;

/* Same values and meaning as voxcpm2_status (include/voxcpm2/c_api.h:37-44). */
typedef enum vxc_status {
    VXC_STATUS_OK = 0,
    VXC_STATUS_INVALID_ARGUMENT = 1,
    VXC_STATUS_INVALID_STATE = 2,
    VXC_STATUS_CANCELLED = 3,
    VXC_STATUS_OUT_OF_MEMORY = 4,
    VXC_STATUS_RUNTIME_ERROR = 5,
} vxc_status;

/* Component ids of src/components.h:16-29 (the audio VAE ids 9/10 are not served here). */
enum {
    VXC_TEXT_EMBED = 0,
    VXC_BASE_DECODER = 1,
    VXC_RESIDUAL_DECODER = 2,
    VXC_FSQ = 3,
    VXC_FUSION_PROJ = 4,
    VXC_DIT_PROJ = 5,
    VXC_STOP_HEAD = 6,
    VXC_FEAT_ENCODER = 7,
    VXC_DIT_ESTIMATOR = 8,
};

/* Which decoder a KV-cache call addresses. */
enum { VXC_BASE = 0, VXC_RESIDUAL = 1 };

/* Model dimensions: the fields of model.json's "setting" block
 * (src/model_manifest.cpp:145-172) plus the per-component sizes the ncnn
 * graphs carry implicitly. */
typedef struct vxc_model_desc {
    int32_t hidden;        /* LM hidden size H */
    int32_t ffn;           /* LM SwiGLU intermediate size */
    int32_t q_heads;
    int32_t kv_heads;
    int32_t head_dim;      /* 64 */
    int32_t base_layers;   /* base_attn_cnt */
    int32_t res_layers;    /* residual_attn_cnt */
    int32_t dit_hidden;    /* Hd; mu is 2 tokens of Hd */
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
    int32_t rope_original_max;   /* original_max_position_embeddings */
    float base_residual_scale;   /* muP scale_depth / sqrt(layers), 1 = off */
    float res_residual_scale;
    float dit_residual_scale;
    float embed_scale;           /* text_embed scale_emb, 1 = off */
    int32_t audio_start_token;
    int32_t max_generation_patches; /* hard cap, 2000 in the reference */
} vxc_model_desc;

/* Snapshot of a stream's device control block. */
typedef struct vxc_stream_state {
    int32_t kv_len[2];      /* tokens in the base / residual KV caches */
    int32_t patches;        /* patches generated since the last prefill */
    int32_t stopped;        /* the last patch step hit the stop rule */
    float stop_logits[2];   /* the last stop_head logits */
    int32_t prefix_len;
    int32_t error;          /* last device-side check code (0 = none) */
    int32_t graph_kernels;  /* kernel launches in one captured patch step (0 before the first) */
} vxc_stream_state;

/* Hot kernels vxc_profile_kernel can time. */
enum {
    VXC_PROF_DIT_GATEUP = 0,   /* DiT gate/up projection over the 2 x 11 tokens (post-attention RMSNorm fused) */
    VXC_PROF_DIT_DOWN = 1,     /* DiT down projection + residual */
    VXC_PROF_DIT_QKV = 2,      /* DiT q/k/v projection (input RMSNorm fused) */
    VXC_PROF_BASE_GATEUP = 3,  /* base decoder gate/up GEMV (RMSNorm fused) */
    VXC_PROF_BASE_DOWN = 4,    /* base decoder down GEMV */
    VXC_PROF_BASE_QKV = 5,     /* base decoder q/k/v GEMV + RoPE + KV append */
    VXC_PROF_BASE_ATTN = 6,    /* base decoder flash-decode attention */
    VXC_PROF_DIT_O = 7,        /* DiT attention + o projection + residual */
    /* 8 is not used */
    VXC_PROF_BASE_STEP = 9,    /* one whole base decoder KV-cache step (24 layers + final norm) */
    VXC_PROF_RES_STEP = 10,    /* one whole residual decoder KV-cache step */
    VXC_PROF_DIT_EVAL = 11,    /* one whole DiT estimator evaluation (embed, 12 layers, out projection) */
};

/* Progress callback of vxc_generate: return non-zero to continue, zero to cancel
 * (the same contract as voxcpm2_progress_callback, include/voxcpm2/c_api.h:98-106). */
typedef int32_t (*vxc_progress_fn)(void* user_data, int32_t completed, int32_t total);

VXC_API uint32_t vxc_abi_version(void);
VXC_API const char* vxc_last_error(void);

/* Number of fp16 values vxc_load_weights expects for a component. */
VXC_API size_t vxc_component_weight_count(const vxc_model_desc* desc, int32_t component);

/* Loads the model on one CUDA device (replaces Synthesizer::Impl::load_manifest /
 * load_net, src/synthesizer.cpp:812-870, for the patch-loop components). */
VXC_API int32_t vxc_device_create(int32_t device, const vxc_model_desc* desc, vxc_device** out);
VXC_API void vxc_device_destroy(vxc_device* dev);

/* Copies one component's fp16 weights (IEEE half bits, the tensor order documented
 * in voxcpm2_b200/config.py) to the device (replaces ncnn::Net::load_model). */
VXC_API int32_t vxc_load_weights(vxc_device* dev, int32_t component, const void* fp16, size_t count);

/* The base decoder's LongRoPE factors, n >= head_dim / 2 values each (the first
 * head_dim / 2 are used; shorter tables are rejected, synthesizer.cpp:949-951): model.json's
 * setting.rope.short_factor and long_factor (src/model_manifest.cpp:92-109, kept by
 * load_manifest, synthesizer.cpp:825-830). Until this is called every factor is 1.
 * As make_rope_cache (synthesizer.cpp:940-974), a call covering positions
 * [start, start + n) rotates with long_factor when start + n > rope_original_max and
 * long_factor is set, else with short_factor; long_factor may be NULL. The patch
 * loop stays below rope_original_max (synthesizer.cpp:542-544), so there only the
 * short factors apply. Streams pick the factors up at their next prefill, decoder
 * step or patch step; the call may come from any thread. Every factor must be positive. */
VXC_API int32_t vxc_set_rope_factors(vxc_device* dev, const float* short_factor, const float* long_factor,
                                     int32_t n);

/* One synthesis stream: its CUDA stream, KV caches of kv_capacity tokens for both
 * decoders (replaces HostDecoderKvCache, src/kvcache.h:18-40), scratch and graphs. */
VXC_API int32_t vxc_stream_create(vxc_device* dev, int32_t kv_capacity, vxc_stream** out);
VXC_API void vxc_stream_destroy(vxc_stream* s);
/* How a stream's estimator linears spread over the GPU (no counterpart in the
 * reference, which runs the estimator on the CPU). VXC_PLAN_THROUGHPUT, the default:
 * ~32 CTAs and a 2-stage shared-memory ring per tcgen05 linear, the highest rate when
 * many streams share the GPU. VXC_PLAN_LATENCY: ~296 CTAs and a 3-stage ring (the
 * down projection as 16-CTA clusters), the lowest per-patch latency for a stream
 * that runs alone. The plans split the linears'
 * K range differently, so latents differ in the last bits between them. Takes effect
 * at the next patch (its graph is captured again); INVALID_STATE while a submitted
 * patch has not been collected. */
#define VXC_PLAN_THROUGHPUT 0
#define VXC_PLAN_LATENCY 1
VXC_API int32_t vxc_stream_set_plan(vxc_stream* s, int32_t plan);
/* Empties both KV caches (a new HostDecoderKvCache pair, synthesizer.cpp:348-350). */
VXC_API int32_t vxc_stream_reset(vxc_stream* s);
/* Cancels the active vxc_generate at its next patch boundary (thread-safe;
 * voxcpm2_operation_cancel, include/voxcpm2/c_api.h:110-114). */
VXC_API void vxc_stream_cancel(vxc_stream* s);

/* HostDecoderKvCache::token_count (src/kvcache.cpp:55-60). */
VXC_API int32_t vxc_token_count(vxc_stream* s, int32_t which, int32_t* out);
/* HostDecoderKvCache::cache_or_empty (src/kvcache.cpp:62-72) as fp32 copies:
 * k, v [kv_heads][token_count][head_dim]. */
VXC_API int32_t vxc_read_cache(vxc_stream* s, int32_t which, int32_t layer, float* k, float* v);

/* run_decoder_with_kv (src/kvcache.h:87-94, src/kvcache.cpp:232-279): runs the
 * base (RoPE) or residual decoder over n new rows embed [n][H], with the causal
 * mask make_decoder_mask(n, token_count) and, for the base decoder, the RoPE
 * rows of positions [token_count, token_count + n) -- exactly what every call
 * site in synthesizer.cpp passes -- appends to the KV cache and writes the
 * final-norm output out [n][H]. */
VXC_API int32_t vxc_decoder_step(vxc_stream* s, int32_t which, const float* embed, int32_t n, float* out);

/* text_embed graph (export_components.py:475-482): out [n][H]. */
VXC_API int32_t vxc_text_embed(vxc_stream* s, const int32_t* ids, int32_t n, float* out);

/* One-row small graphs (run_net_vec in synthesizer.cpp:546-640):
 *   VXC_FSQ          in0 [H]                 -> out [H]
 *   VXC_FUSION_PROJ  in0 lm [H], in1 feat [H] -> out [H]
 *   VXC_DIT_PROJ     in0 lm [H], in1 res [H]  -> out [2*Hd]
 *   VXC_STOP_HEAD    in0 [H]                 -> out [2]
 *   VXC_FEAT_ENCODER in0 latent [D][P] d-major -> out [H] */
VXC_API int32_t vxc_run_component(vxc_stream* s, int32_t component, const float* in0, const float* in1,
                                  float* out);

/* One dit_estimator call as cfm_sample binds it (synthesizer.cpp:137-145):
 * x_in [2][D][P], mu_in [2][2*Hd], t_in [2] = {step index, timesteps} (schedule
 * mode), cond_in [2][D][P], dt_in [2] raw -> out [2][D*P]. */
VXC_API int32_t vxc_dit_estimator(vxc_stream* s, const float* x_in, const float* mu_in, const float* t_in,
                                  const float* cond_in, const float* dt_in, float* out);

/* cfm_sample (synthesizer.cpp:86-170) for one patch: mu [2*Hd], cond [D*P],
 * noise [D*P] (the patch's N(0,1) draws) -> out_latent [D*P]. */
VXC_API int32_t vxc_cfm_sample(vxc_stream* s, const float* mu, const float* cond, const float* noise,
                               int32_t timesteps, float cfg_value, float* out_latent);

/* Prefix phase of generate_with_caches for a text-only prompt
 * (synthesizer.cpp:387-535): prefix = text_ids + audio_start; text_embed, base
 * prefill, fusion_proj, residual prefill; resets the caches and the patch count. */
VXC_API int32_t vxc_prefill(vxc_stream* s, const int32_t* text_ids, int32_t n_text);

/* The prefix phase for a prefix given row by row, as the reference's PrefixRow
 * list (synthesizer.cpp:43-47, 359-535), so prompt and reference audio can lead
 * the utterance: token_ids of every row (audio rows' ids are embedded and then
 * replaced; the reference uses 0), is_audio flags (NULL: all text), and the audio
 * rows' latent patches in row order, [n_audio][D*P] d-major (as encoded by the
 * audio VAE). An audio row is embedded by feat_encoder, its LM hidden after the base
 * prefill is its FSQ output, and its feat_encoder embedding is its residual
 * feature input; when the last row is audio, the first patch is conditioned on its
 * latent. Resets the caches and the patch count. */
VXC_API int32_t vxc_prefill_rows(vxc_stream* s, const int32_t* token_ids, const int32_t* is_audio,
                                 const float* audio_latents, int32_t n_rows);

/* One iteration of the patch loop (synthesizer.cpp:537-659), replayed as one
 * CUDA graph: dit_proj, cfm_sample (timesteps-1 estimator calls after the
 * zero-init skip), stop_head, and -- unless the stop rule fires --
 * feat_encoder, base decode, fsq, fusion_proj and residual decode. 'step' must
 * equal the number of patches generated since vxc_prefill. noise [D*P] are the
 * patch's draws (NULL: use the table uploaded with vxc_upload_noise).
 * out_latent [D*P] (may be NULL); *out_stop = 1 when the loop must break. */
VXC_API int32_t vxc_patch_step(vxc_stream* s, const float* noise, int32_t min_patches, int32_t step,
                               float cfg_value, int32_t timesteps, float* out_latent, int32_t* out_stop);

/* generate_with_caches without the audio VAE (synthesizer.cpp:353-659): prefill,
 * then patch steps with noise from std::mt19937(seed) (:452, :108-112) until the
 * stop rule or max_patches (max_patches_for_target, :216-220; max_patches_override
 * > 0 lowers it). out_latents [max][D*P]; optional traces per patch of the hidden
 * states entering it: lm_trace / res_trace [max][H], stop_trace [max][2]. */
VXC_API int32_t vxc_generate(vxc_stream* s, const int32_t* text_ids, int32_t n_text, int32_t min_patches,
                             int32_t timesteps, float cfg_value, int32_t max_patches_override, uint32_t seed,
                             float* out_latents, int32_t* out_patches, float* lm_trace, float* res_trace,
                             float* stop_trace, vxc_progress_fn progress, void* progress_user_data);

/* VoxCPM2SDPA::forward (src/ncnn_layers/sdpa/voxcpm2_sdpa.cpp:115-260) on DEVICE
 * pointers, ncnn layout (w = dim, h = seq, c = heads): q [heads][src][d],
 * k/v [groups][cur][d|dv], mask [mask_c][src][past+cur] or NULL, past_k/v
 * [groups][past][d] (past may be 0), out [heads][src][dv], out_k/out_v
 * [groups][past+cur][d] or NULL. scale 0 -> 1/sqrt(d). cuda_stream is a
 * cudaStream_t (NULL = legacy default stream); the call is asynchronous. */
VXC_API int32_t vxc_sdpa(const float* q, int32_t heads, int32_t src, int32_t d, const float* k, const float* v,
                         int32_t groups, int32_t cur, int32_t dv, const float* mask, int32_t mask_c,
                         const float* past_k, const float* past_v, int32_t past, float scale, float* out,
                         float* out_k, float* out_v, void* cuda_stream);
/* No counterpart in the reference. vxc_sdpa for one query row (src = 1,
 * head dim 64, at most 64 query heads, <= 16 per KV group, mask [past+cur] or
 * NULL), for callers that cannot let a library allocate device memory -- a
 * plugin host that forbids allocation inside its enqueue call, or a real-time
 * thread that cannot absorb cudaMalloc's device synchronisation. It allocates
 * nothing: its split-K scratch is a fixed 528.3 KiB device array that every GPU
 * loading the library keeps until exit. The first call on a device resolves
 * that array's address (and raises kernel shared-memory limits), so make it
 * before any stream capture. Larger shapes return VXC_STATUS_INVALID_ARGUMENT.
 * All calls share the one array: calls that overlap on the GPU (different
 * streams, or host threads racing on one device) corrupt each other's results;
 * serialise them, e.g. on one stream. Device pointers, asynchronous on
 * cuda_stream (a cudaStream_t; NULL = legacy default stream). */
VXC_API int32_t vxc_sdpa_decode_noalloc(const float* q, int32_t heads, int32_t d, const float* k, const float* v,
                                        int32_t groups, int32_t cur, const float* mask, const float* past_k,
                                        const float* past_v, int32_t past, float scale, float* out, float* out_k,
                                        float* out_v, void* cuda_stream);
/* The same on HOST pointers (what the ncnn CPU layer receives); synchronous. */
VXC_API int32_t vxc_sdpa_host(const float* q, int32_t heads, int32_t src, int32_t d, const float* k,
                              const float* v, int32_t groups, int32_t cur, int32_t dv, const float* mask,
                              int32_t mask_c, const float* past_k, const float* past_v, int32_t past,
                              float scale, float* out, float* out_k, float* out_v);

/* VoxCPM2TimestepEmbedding::forward (src/ncnn_layers/timestep_embedding/
 * voxcpm2_timestep_embedding.cpp:128-160; params half_dim, scale, max_period,
 * schedule_mode from load_param) on HOST pointers, computed on the current
 * CUDA device; synchronous. in [n_in]; out [n_in][2 * half_dim] =
 * [sin(t f_i) | cos(t f_i)], f_i = exp(-ln(max_period) i / (half_dim - 1)),
 * t = in[b] * scale (schedule_mode 0) or t(in[0] = step, in[1] = timesteps) *
 * scale for every row (schedule_mode != 0, n_in >= 2). */
VXC_API int32_t vxc_timestep_embedding(const float* in, int32_t n_in, int32_t half_dim, float scale,
                                       float max_period, int32_t schedule_mode, float* out);

/* ---- device-resident driving (benchmarks, multi-stream servers) ---------- */
/* Uploads noise [patches][D*P] into the stream's device noise table. */
VXC_API int32_t vxc_upload_noise(vxc_stream* s, const float* noise, int32_t patches);
/* Enqueues one patch-step graph reading the device noise table; no host sync,
 * no host copies. The caller checks the stop flag later with vxc_read_state. */
VXC_API int32_t vxc_patch_step_async(vxc_stream* s, int32_t min_patches, float cfg_value, int32_t timesteps);
/* Pipelined patch loop: vxc_patch_submit queues one patch step (as vxc_patch_step:
 * host noise [D*P] through a pinned slot, the patch graph, and copies of its latent
 * and control block back to pinned slots) and returns without waiting; at most 4
 * patches may be in flight. vxc_patch_collect waits for the oldest queued patch
 * only and returns its latent and stop flag. A host keeps the next patch queued
 * while it handles the previous one; when a collected patch has stop set, it
 * discards the patch it queued after it (vxc_prefill or vxc_stream_reset drops
 * queued patches). Collecting with nothing queued is VXC_STATUS_INVALID_STATE. */
VXC_API int32_t vxc_patch_submit(vxc_stream* s, const float* noise, int32_t min_patches, float cfg_value,
                                 int32_t timesteps);
VXC_API int32_t vxc_patch_collect(vxc_stream* s, float* out_latent, int32_t* out_stop);
/* The patch loop body (src/synthesizer.cpp:537-659, one vxc_patch_step per
 * patch) for n independent streams of one device, driven from the calling
 * thread with no per-stream host thread: each stream keeps two patches queued
 * through vxc_patch_submit / vxc_patch_collect, visited round robin. noise
 * [n][patches][D*P] and out_latents [n][patches][D*P] are host arrays; a
 * stream ends at its stop decision or after 'patches' patches, and
 * out_patches[i] is the number of latents written for stream i. Every stream
 * must be prefilled, with nothing in flight; the call holds every stream's call
 * lock until it returns. */
VXC_API int32_t vxc_patch_run(vxc_stream* const* streams, int32_t n, const float* noise, int32_t patches,
                              int32_t min_patches, float cfg_value, int32_t timesteps, float* out_latents,
                              int32_t* out_patches);

VXC_API int32_t vxc_stream_synchronize(vxc_stream* s);
VXC_API int32_t vxc_read_state(vxc_stream* s, vxc_stream_state* out);
/* Current hidden states entering the next patch: lm [H], res [H] (either may be NULL). */
VXC_API int32_t vxc_read_hidden(vxc_stream* s, float* lm, float* res);
/* Latents of patches [first, first + count) generated since the last prefill. */
VXC_API int32_t vxc_read_latents(vxc_stream* s, int32_t first, int32_t count, float* out);
/* Times one hot kernel on the stream's own buffers in the form the patch graph
 * runs it: 'iters' launches cycling through the layers' weights (for the
 * benchmark model more than the L2 holds), captured in one CUDA graph with
 * programmatic dependent launch between them, timed with CUDA events on the
 * stream after one warm-up replay. Writes the mean milliseconds per launch and
 * the algorithmic bytes one launch must move (weights + activations in + out).
 * Call it between patch steps: it leaves the stream's positions and valid KV
 * rows as they were, but overwrites scratch activations and the next free KV
 * row of every base layer. */
VXC_API int32_t vxc_profile_kernel(vxc_stream* s, int32_t kernel, int32_t iters, float* ms_per_launch,
                                   double* bytes_per_launch);
/* The same kernel on n streams of one device at once: each stream replays its own
 * graph of 'iters' launches, all started after one event on streams[0] and joined
 * before a second; writes the elapsed milliseconds of the whole set (n * iters
 * launches) and the algorithmic bytes of one launch. */
VXC_API int32_t vxc_profile_kernel_concurrent(vxc_stream** streams, int32_t n, int32_t kernel, int32_t iters,
                                              float* ms_total, double* bytes_per_launch);
/* The stream's cudaStream_t, for callers timing it with CUDA events. */
/* Groups: up to 8 streams whose patch steps run together as one CUDA graph. Each
 * member keeps its own prompt, KV caches, noise, stop state and latents (use the
 * stream calls above on vxc_group_stream's handle: vxc_prefill, vxc_upload_noise,
 * vxc_read_state, vxc_read_latents ...); the 9 estimator evaluations of all
 * members run as one batched pass over 22 rows per member, so the DiT weights are
 * read once per group patch. No reference counterpart: the reference synthesises
 * one utterance at a time. Group steps are stream-ordered with the members' own
 * calls: a step waits for work queued on every member stream, and later calls on a
 * member stream wait for the step. */
VXC_API int32_t vxc_group_create(vxc_device* dev, int32_t n_streams, int32_t kv_capacity, vxc_group** out);
VXC_API void vxc_group_destroy(vxc_group* g);
VXC_API int32_t vxc_group_stream(vxc_group* g, int32_t member, vxc_stream** out);
/* One patch of every member (as vxc_patch_step_async), noise from each member's uploaded table. */
VXC_API int32_t vxc_group_patch_step_async(vxc_group* g, int32_t min_patches, float cfg_value, int32_t timesteps);
/* Waits for the group's work; reports a device-side failure of any member. */
VXC_API int32_t vxc_group_synchronize(vxc_group* g);
/* Kernel launches in one captured group patch step (0 before the first). */
VXC_API int32_t vxc_group_graph_kernels(vxc_group* g, int32_t* out);

VXC_API int32_t vxc_stream_cuda_handle(vxc_stream* s, void** out);

#ifdef __cplusplus
}
#endif
