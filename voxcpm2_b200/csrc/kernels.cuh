// Kernel launch interface of libvoxcpm2_cuda (host side, sm_100a).
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <vector>

#include "common.cuh"

namespace vxc {

// ---------------------------------------------------------------- GEMV ---
// Batch-1 matrix-vector products over fp16 weights [rows][K] with an fp32
// input vector, fp32 accumulation. The input can be RMS-normalised on the fly
// (gain g, eps), formed by concatenating two vectors, or read from a d-major
// latent patch transposed to frame-major.
enum GemvMode : int {
    GEMV_PLAIN = 0,   // y[r] = act(dot + bias[r])
    GEMV_RESID = 1,   // resid[r] += rscale * dot                    (o_proj, down_proj)
    GEMV_GATEUP = 2,  // y[r] = silu(dot(gate r)) * dot(up r)        (rows r and r + pairs)
    GEMV_QKV = 3,     // q/k/v rows in RoPE pairs; q -> y, k/v -> fp32 KV cache at ctl->kv_len
};
enum GemvAct : int { ACT_NONE = 0, ACT_SILU = 1, ACT_FSQ = 2 };
enum GemvInput : int { IN_PLAIN = 0, IN_CONCAT = 1, IN_LATENT_T = 2 };

struct GemvArgs {
    int mode = GEMV_PLAIN;
    const __half* w = nullptr;
    const __half* bias = nullptr;
    const float* x = nullptr;
    const float* x2 = nullptr;      // IN_CONCAT: second part, starting at k1
    int k1 = 0;
    int in_mode = IN_PLAIN;
    int lat_d = 0, lat_p = 0;       // IN_LATENT_T: latent [lat_d][lat_p]
    const __half* norm_g = nullptr;  // RMSNorm gain of the input, or null
    float eps = 1e-5f;
    int K = 0;
    int rows = 0;                   // output rows (row pairs for GATEUP / QKV)
    int act = ACT_NONE;
    float act_scale = 1.0f;         // ACT_FSQ quantisation scale
    float rscale = 1.0f;            // GEMV_RESID residual scale
    float* y = nullptr;
    float* y2 = nullptr;            // optional second copy of y
    float* resid = nullptr;
    // GEMV_QKV
    int q_heads = 0, kv_heads = 0, head_dim = 0;
    const float* rope_cos = nullptr;  // [capacity][head_dim] or null (no RoPE)
    const float* rope_sin = nullptr;
    // LongRoPE: the row of position pos comes from these tables when pos + 1 > rope_long_from
    const float* rope_cos_long = nullptr;
    const float* rope_sin_long = nullptr;
    int rope_long_from = 1 << 30;
    float* k_cache = nullptr;       // this layer: [kv_heads][cap][head_dim]
    float* v_cache = nullptr;
    int cap = 0;
    int which = 0;                  // which decoder's kv_len indexes the cache
    // control
    StreamCtl* ctl = nullptr;
    int skip_if_stopped = 0;
};

void launch_gemv(const GemvArgs& a, cudaStream_t s, bool pdl);
// The same product with at most one block per SM whose weight rows are copied
// into shared memory by the bulk-copy engine before the dependency wait (the
// decoder-step form); IN_PLAIN input, K <= 4096.
void launch_gemv_bulk(const GemvArgs& a, cudaStream_t s, bool pdl);
constexpr int kGroupMembers = 8;  // most streams in a group (the member-indexed argument arrays)
// Up to kGemvBatch members (streams of a group) through the same weights: one read
// of each weight row, one dot product per member. Member m replaces a's x, y,
// resid, k_cache, v_cache and ctl; each member skips (and appends no KV row) when
// a.skip_if_stopped and its own ctl->stopped are set.
constexpr int kGemvBatch = kGroupMembers;
struct GemvBatch {
    int n = 0;
    const float* x[kGemvBatch] = {};
    float* y[kGemvBatch] = {};
    float* resid[kGemvBatch] = {};
    float* k_cache[kGemvBatch] = {};
    float* v_cache[kGemvBatch] = {};
    StreamCtl* ctl[kGemvBatch] = {};
};
void launch_gemv_bulk_batch(const GemvArgs& a, const GemvBatch& b, cudaStream_t s, bool pdl);
// The register-streaming form of the same member batch (weights loaded once per warp).
void launch_gemv_batch(const GemvArgs& a, const GemvBatch& b, cudaStream_t s, bool pdl);

// ------------------------------------------------------ flash decode -----
// One query token of each of q_heads heads attends over keys [0, T) of a GQA
// cache split into two segments (seg0 of len0 rows, then seg1), split-K over
// 'splits' CTAs per KV head with a last-CTA combine. Rows are fp32 (the decoder
// caches and the layer contract; an fp16 instantiation exists for fp16 callers); 'T' is read from ctl->kv_len[which] + 1
// when ctl is non-null (then len0 must hold the cache capacity, which sizes the
// shared-memory score buffer), else T = len0 + len1.
struct AttnArgs {
    const float* q = nullptr;          // [q_heads][d]
    const void* k0 = nullptr; const void* v0 = nullptr;  // [kv_heads][stride0][d]
    const void* k1 = nullptr; const void* v1 = nullptr;  // [kv_heads][stride1][d]
    int len0 = 0, len1 = 0;
    long stride0 = 0, stride1 = 0;     // rows per KV head plane
    const float* mask = nullptr;       // additive [T] (one query row) or null
    int q_heads = 0, kv_heads = 0, head_dim = 0;
    float scale = 0.125f;
    int splits = 16;
    float* partial = nullptr;          // [kv_heads][splits][group][head_dim + 2]
    int* counters = nullptr;           // [kv_heads], zero between launches
    float* out = nullptr;              // [q_heads][head_dim]
    StreamCtl* ctl = nullptr;
    int which = 0;
    int skip_if_stopped = 0;
};
void launch_attn_decode(const AttnArgs& a, bool fp16_kv, cudaStream_t s, bool pdl);
// The same (fp32 KV) with the split-K combine inside one 8-CTA cluster per KV head
// (distributed shared memory; no scratch, no atomics). Ignores splits/partial/counters.
void launch_attn_decode_cluster(const AttnArgs& a, cudaStream_t s, bool pdl);
// The same for up to kGroupMembers members (grid z = member): member m replaces a's
// q, k0, v0, out and ctl (its own KV length and stop flag).
struct AttnBatch {
    int n = 0;
    const float* q[kGroupMembers] = {};
    const void* k0[kGroupMembers] = {};
    const void* v0[kGroupMembers] = {};
    float* out[kGroupMembers] = {};
    StreamCtl* ctl[kGroupMembers] = {};
};
void launch_attn_decode_cluster_batch(const AttnArgs& a, const AttnBatch& b, cudaStream_t s, bool pdl);
// The layer-contract op (sdpa_op.cu): one query row over at most 512 fp32 keys given as
// [k0 rows | k1 rows] per KV head, no control block; every load issued up front, one
// 8-CTA cluster per KV head combining through shared memory.
bool sdpa_op_supported(const AttnArgs& a);
void launch_sdpa_op(const AttnArgs& a, cudaStream_t s, bool pdl);
void init_sdpa_op_attributes();

// final RMSNorm of a decoder step: out = norm(h) * g; optionally bump kv_len.
void launch_final_norm(const float* h, const __half* g, float eps, int H, float* out, float* out2,
                       StreamCtl* ctl, int which, int bump, int skip_if_stopped, cudaStream_t s,
                       bool pdl);

// ----------------------------------------------------- token batches -----
// Y[m][r] for M tokens (prefill rows, the DiT's 2 x 11 tokens).
struct RowsArgs {
    const __half* w = nullptr;
    const __half* bias = nullptr;
    const float* x = nullptr;  // [M][ldx]
    int ldx = 0;
    int K = 0;
    int rows = 0;              // output rows (pairs for GATEUP)
    int M = 0;
    int mode = GEMV_PLAIN;     // PLAIN (act) / RESID / GATEUP
    int act = ACT_NONE;
    float rscale = 1.0f;
    float* y = nullptr;        // [M][ldy] (RESID: accumulated in place)
    int ldy = 0;
    StreamCtl* ctl = nullptr;
    int skip_if_stopped = 0;
};
void launch_rows_linear(const RowsArgs& a, cudaStream_t s, bool pdl);

// out[m] = x[m] / rms(x[m]) * g for M rows of width K
void launch_rmsnorm_rows(const float* x, int ldx, const __half* g, float eps, int K, int M,
                         float* out, int ldo, StreamCtl* ctl, int skip_if_stopped,
                         cudaStream_t s, bool pdl);

// RoPE on the q and k parts of qkv rows [M][(hq+2hkv)d], in place, at position
// past + (m % pos_mod) of row m (tables indexed by position). With a cache, k/v
// of row m are also appended at cache row past + m (prefill).
void launch_qkv_rows_post(float* qkv, int M, int q_heads, int kv_heads, int d, int past,
                          int pos_mod, const float* rope_cos, const float* rope_sin,
                          float* k_cache, float* v_cache, int cap, StreamCtl* ctl,
                          cudaStream_t s, bool pdl);

// Causal attention of M prefill rows (positions past..past+M-1) over the KV cache.
void launch_attn_rows_cache(const float* qkv, int M, int q_heads, int kv_heads, int d, int past,
                            const float* k_cache, const float* v_cache, int cap, float scale,
                            float* out, cudaStream_t s, bool pdl);


// DiT, tensor-core operand producers. Both write the next tcgen05 linear's B
// operand: split fp16 rows [48][ld] (row m = fp16(v), row 24 + m = fp16(v - fp16(v))).
// RMSNorm of the M residual rows:
// RMSNorm of M rows (g == nullptr: no normalisation) into a split-fp16 operand:
// fp16(v) in row m, fp16(v - fp16(v)) in row lo + m (lo = 24 for the DiT linears,
// kRowBlock for the prefill's row-block linears)
void launch_rmsnorm_rows_split(const float* x, int ldx, const __half* g, float eps, int K, int M, __half* xb,
                               StreamCtl* ctl, cudaStream_t s, bool pdl, int lo = 24);
// RoPE (positions 0..seq-1) + full attention within each sequence, one CTA per
// (head, sequence), from the fp32 q/k/v rows [nseq*seq][(hq+2hkv)d]:
void launch_dit_attention_split(const float* qkv, int nseq, int seq, int q_heads, int kv_heads, int d,
                                const float* rope_cos, const float* rope_sin, float scale, __half* xb,
                                StreamCtl* ctl, cudaStream_t s, bool pdl, int lo = 24);

// h[m] = table[ids[m]] * scale
void launch_embed_gather(const __half* table, const int32_t* ids, int M, int H, float scale,
                         float* out, cudaStream_t s);

// ------------------------------------------------------------- DiT ------
struct DitEmbedArgs {
    const __half* in_w; const __half* in_b; const __half* cond_w; const __half* cond_b;
    const float* x;       // [D*P] d-major sample of CFG row 0
    const float* cond;    // [D*P] d-major condition of CFG row 0
    const float* mu;      // [2*Hd] mu tokens of CFG row 0
    const float* t_tok0;  // [Hd] time_mlp(emb(t)) of CFG row 0
    const float* t_tok1;  // ... of CFG row 1
    const float* dt_tok0; // [Hd] delta_time_mlp(emb(dt)) of CFG row 0
    const float* dt_tok1;
    int Hd, D, P;
    float* hidden;        // [2][3 + 2P][Hd]
    StreamCtl* ctl;
    const float* mu_uncond;  // [2*Hd] of CFG row 1, or null (zeros)
    const float* x_uncond;   // [D*P] of CFG row 1, or null (same as x)
    const float* cond_uncond;// [D*P] of CFG row 1, or null (same as cond)
    const float* tsum;       // [Hd] precomputed t_tok + dt_tok of both CFG rows, or null
    float* ssq_out;          // or null: per 32-feature block, row sums of squares [block][24]
    // group members (grid y = member, 0 = none): member m replaces x, cond, mu and ctl,
    // and writes hidden + m * member_stride
    int members;
    const float* mx[kGroupMembers];
    const float* mcond[kGroupMembers];
    const float* mmu[kGroupMembers];
    StreamCtl* mctl[kGroupMembers];
    size_t member_stride;
};
void launch_dit_embed(const DitEmbedArgs& a, cudaStream_t s, bool pdl);

// sinusoidal timestep embedding rows (VoxCPM2TimestepEmbedding): t_rows[r] (or
// t_val for one row when t_rows is null) times the host-computed frequencies
// freq[half_dim]; out [rows][2 * half_dim].
void launch_timestep_embedding(const float* t_rows, float t_val, int rows, const float* freq, int half_dim,
                               float* out, StreamCtl* ctl, cudaStream_t s, bool pdl);
// the layer's host-side arithmetic (timestep_embedding.cpp:137-152), in float as the layer does it
float timestep_scheduled_t(float step_index, float timesteps);
std::vector<float> timestep_frequencies(int half_dim, float max_period);

struct DitOutArgs {
    const float* hidden;    // [2][seq][Hd] pre-final-norm residual stream
    int seq, Hd, D, P;
    const __half* norm_g; float eps;
    const __half* out_w; const __half* out_b;
    float* est_out;         // optional [2][D*P] raw estimator output
    float* x;               // [D*P] sample updated in place (null: no update)
    float dt, cfg;
    StreamCtl* ctl;
    float* est_buf;         // [2][D*P] estimator output (est_out or a scratch buffer)
    int* counter;           // arrival counter, zero between launches
    // group members (grid y = member, 0 = none): member m reads hidden + m * member_stride
    // and replaces x, ctl, est_buf and counter
    int members = 0;
    float* mx[kGroupMembers] = {};
    StreamCtl* mctl[kGroupMembers] = {};
    float* mest[kGroupMembers] = {};
    int* mcounter[kGroupMembers] = {};
    size_t member_stride = 0;
};
void launch_dit_out(const DitOutArgs& a, cudaStream_t s, bool pdl);

// stop decision: logits = head_w [2][H] . mid; ctl->stopped = step > min_patches && l1 > l0
// out[i] = a[i] + b[i]
void launch_vec_add(const float* a, const float* b, float* out, int n, cudaStream_t s);

void launch_stop_decide(const __half* head_w, const float* mid, int H, StreamCtl* ctl,
                        float* logits_out, cudaStream_t s, bool pdl);

// per-patch prologue: x = noise[ctl->patch]; cond = latents[ctl->patch - 1], or
// init_cond for the first patch (synthesizer.cpp:561-563, 445-447); clears the stop flag.
void launch_patch_begin(const float* noise_table, const float* latents, const float* init_cond,
                        int per_patch, float* x, float* cond, StreamCtl* ctl, cudaStream_t s,
                        bool pdl);
// per-patch epilogue: latents[ctl->patch] = x; patch and step counters advance.
void launch_patch_end(const float* x, float* latents, int per_patch, StreamCtl* ctl,
                      cudaStream_t s, bool pdl);

// VoxCPM2SDPA layer contract (fp32, any src rows, optional mask and cache concat).
void launch_sdpa_rows_f32(const float* q, int heads, int src, int d, const float* k,
                          const float* v, int groups, int cur, int dv, const float* mask,
                          int mask_c, const float* past_k, const float* past_v, int past,
                          float scale, float* out, cudaStream_t s);
void launch_concat_kv(const float* past, const float* cur, int groups, int past_len, int cur_len,
                      int d, float* out, cudaStream_t s);

// ------------------------------------------------------- tcgen05 linear ---
// Y = X W^T for <= 24 token rows on the 5th-generation tensor cores. A = W (fp16
// [rows][K], tensor map box 64 rows x 64 cols, 128B swizzle); B = the token rows as
// split fp16 [48][K] (rows m: fp16(x), rows 24 + m: fp16(x - fp16(x)); pad rows 0).
struct TcLinearArgs {
    int K = 0;           // multiple of 64
    int M = 0;           // token rows (<= 24)
    int rows = 0;        // output features (GATEUP: gate/up pairs)
    int splits = 1;      // K split = cluster size (<= 16; gate/up <= 8)
    int gateup = 0;      // tile = 64 gate rows + the matching 64 up rows; out = SiLU(g) * u
    int resid = 0;       // y += rscale * out (else y = out)
    float rscale = 1.0f;
    float* y = nullptr;  // fp32 [M][ldy] (plain / residual)
    int ldy = 0;
    __half* yb = nullptr;  // GATEUP: split-fp16 [48][ldyb], the next linear's B operand
    int ldyb = 0;
    StreamCtl* ctl = nullptr;  // receives error 3 if a bounded wait gave up
    // The B operand (the token rows) comes by TMA from a split-fp16 [48][K] buffer (map_b).
    // row_scale: the producer's per-slice sums of squares of the rows, ssq_parts parts
    // of ssq_in [part][24], and the RMSNorm eps
    float eps = 0.f;
    const float* ssq_in = nullptr;
    int ssq_parts = 0;
    int max_stages = 8;  // shared-memory ring depth (1..8)
    // residual epilogue: partial sums of squares of the updated rows, one part per
    // (tile, owner CTA) = tile * splits + rank, written to ssq_out [part][24]
    float* ssq_out = nullptr;
    // residual epilogue with ssq_out: also write the next linear's TMA-fed B operand,
    // split fp16 of (updated row * next_g) into next_b [48][ldnb]: its RMSNorm with
    // the gain applied and the 1 / rms left to the consumer (row_scale)
    const __half* next_g = nullptr;
    __half* next_b = nullptr;
    int ldnb = 0;
    // consumer of such an operand: token row m of the result is multiplied by
    // rsqrt(sum of the ssq_parts parts of ssq_in / K + eps), the RMSNorm's 1 / rms
    // (W (x g) / rms = W (x g / rms))
    int row_scale = 0;
    // K split with a TMA-fed operand: receive the cluster's partials (and keep the
    // squares) in the idle stage area after one more cluster barrier, instead of a
    // dedicated buffer behind it (smaller CTAs, more of them per SM)
    int recv_shared = 0;
};
constexpr int kSsqStride = 24;  // floats per part in a sums-of-squares buffer
CUtensorMap make_tensor_map_f16(const void* base, int rows, int cols, int box_rows);
size_t tc_linear_smem_bytes(int K, int splits, int max_stages = 8, bool ssq_out = false, bool recv_shared = false,
                            int row_scale_parts = 0);
void launch_tc_linear(const CUtensorMap& map_a, const CUtensorMap& map_b, const TcLinearArgs& a, cudaStream_t s,
                      bool pdl);
void init_tc_attributes();

// Row-block tcgen05 linear (prefill): Y[m][r] for m < M <= kRowBlock rows, one
// CTA per 128-feature tile (gate/up: 64 gate + 64 up rows), no K split
// (tc_rows.cu). The token operand is split fp16 [2 * kRowBlock][K] (map_b, box
// rows 2 * kRowBlock): fp16(x) in rows 0.., the residuals in rows kRowBlock...
constexpr int kRowBlock = 128;
struct TcRowsArgs {
    int K = 0, M = 0, rows = 0;
    int gateup = 0;            // out = SiLU(gate) * up, as split fp16 into yb [2 * kRowBlock][ldyb]
    int resid = 0;             // y += rscale * out (else y = out)
    float rscale = 1.f;
    float* y = nullptr;        // fp32 [M][ldy]
    int ldy = 0;
    __half* yb = nullptr;
    int ldyb = 0;
    int stages = 4;            // shared-memory ring depth (1..4)
    StreamCtl* ctl = nullptr;  // receives error 3 if a bounded wait gave up
    // K split over 'splits' CTAs per output tile: each writes its fp32 partial tile into
    // part [splits][M][rows] (gate/up: [splits][M][2 rows], the gate then the up features)
    // and a second kernel sums the partials in order and applies the epilogue
    int splits = 1;
    float* part = nullptr;
};
void launch_tc_rows(const CUtensorMap& map_a, const CUtensorMap& map_b, const TcRowsArgs& a, cudaStream_t s);
// K split of a prefill linear: about 128 CTAs per launch, at most 8 per output tile.
int tc_rows_splits(int rows, int gateup, int K);
void init_tc_rows_attributes();

// Wide-token tcgen05 linear (the DiT of a group of streams): Y[m][r] for
// m < M <= lo rows, K split across a cluster of 'splits' CTAs (tc_wide.cu). The
// token operand is split fp16 [2 lo][K] (map_b, box rows lo): fp16(x) in rows
// 0..lo-1, the residuals in rows lo..2 lo-1; lo is a multiple of 16, at most
// kWideTokens (8 members x 22 rows).
constexpr int kWideTokens = 176;
struct TcWideArgs {
    int K = 0, M = 0, rows = 0;
    int lo = 0;                // the token operand's row block (a multiple of 16, M <= lo <= kWideTokens)
    int splits = 1;
    int gateup = 0;            // out = SiLU(gate) * up, as split fp16 into yb [2 lo][ldyb]
    int resid = 0;             // y += rscale * out (else y = out)
    float rscale = 1.f;
    float* y = nullptr;        // fp32 [M][ldy]
    int ldy = 0;
    __half* yb = nullptr;
    int ldyb = 0;
    int stages = 2;            // shared-memory ring depth (1..4; lowered where the block does not fit)
    StreamCtl* ctl = nullptr;  // receives error 3 if a bounded wait gave up
    // K split: receive the cluster's partials in the (by then idle) stage area after one
    // more cluster barrier, instead of a dedicated buffer (more CTAs per SM; always
    // so where the dedicated buffer would not fit beside the ring)
    int recv_shared = 0;
};
void launch_tc_wide(const CUtensorMap& map_a, const CUtensorMap& map_b, const TcWideArgs& a, cudaStream_t s,
                    bool pdl);
void init_tc_wide_attributes();

// Raise the dynamic shared-memory limit of the kernels that need more than 48 KB
// (call once per device, outside stream capture).
void init_kernel_attributes();

}  // namespace vxc
