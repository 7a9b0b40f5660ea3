// Host runtime and C ABI of libvoxcpm2_cuda.
//
// Mirrors the reference's host side for the patch loop: Synthesizer::Impl's
// generate_with_caches (src/synthesizer.cpp:353-659), cfm_sample (:86-170),
// the RoPE tables (:928-974) and run_decoder_with_kv (src/kvcache.cpp:232-279),
// with every ncnn graph replaced by sm_100a kernels and each patch iteration
// captured once as a CUDA graph (positions come from a device control block,
// so the same graph is replayed for every patch).
#include <algorithm>
#include <array>
#include <atomic>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <functional>
#include <initializer_list>
#include <map>
#include <memory>
#include <mutex>
#include <new>
#include <numbers>
#include <random>
#include <stdexcept>
#include <string>
#include <vector>

#include "../../include/voxcpm2_cuda.h"
#include "kernels.cuh"

using namespace vxc;

namespace vxc {

// VoxCPM2TimestepEmbedding's host arithmetic, in float with the C library as the
// layer computes it (timestep_embedding.cpp:141-152): schedule mode's t from
// (step_index, timesteps), and the frequencies exp(-ln(max_period) i / (half - 1)).
float timestep_scheduled_t(float step_index, float timesteps) {
    constexpr float kPi = 3.14159265358979323846f;
    const float u = 1.0f - step_index / std::max(timesteps, 1.0f);
    return u + (std::cos(kPi * 0.5f * u) - 1.0f + u);
}

std::vector<float> timestep_frequencies(int half_dim, float max_period) {
    const float log_period = std::log(max_period);
    std::vector<float> f(static_cast<size_t>(half_dim));
    for (int i = 0; i < half_dim; ++i)
        f[i] = std::exp(-log_period * static_cast<float>(i) / static_cast<float>(half_dim - 1));
    return f;
}

}  // namespace vxc

namespace {

thread_local std::string g_last_error;

struct InvalidState : std::runtime_error {
    using std::runtime_error::runtime_error;
};
struct Cancelled : std::runtime_error {
    Cancelled() : std::runtime_error("operation cancelled") {}
};
struct DeviceOom : std::runtime_error {
    using std::runtime_error::runtime_error;
};

void ck(cudaError_t e, const char* what) {
    if (e == cudaSuccess) return;
    cudaGetLastError();
    if (e == cudaErrorMemoryAllocation) throw DeviceOom(std::string(what) + ": " + cudaGetErrorString(e));
    throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
}

// Exceptions -> status codes, as guard() in src/c_api.cpp:168-193.
template <typename F>
int32_t guard(F&& f) noexcept {
    try {
        f();
        return VXC_STATUS_OK;
    } catch (const Cancelled& e) {
        g_last_error = e.what();
        return VXC_STATUS_CANCELLED;
    } catch (const InvalidState& e) {
        g_last_error = e.what();
        return VXC_STATUS_INVALID_STATE;
    } catch (const std::invalid_argument& e) {
        g_last_error = e.what();
        return VXC_STATUS_INVALID_ARGUMENT;
    } catch (const DeviceOom& e) {
        g_last_error = e.what();
        return VXC_STATUS_OUT_OF_MEMORY;
    } catch (const std::bad_alloc&) {
        g_last_error = "native allocation failed";
        return VXC_STATUS_OUT_OF_MEMORY;
    } catch (const std::exception& e) {
        g_last_error = e.what();
        return VXC_STATUS_RUNTIME_ERROR;
    } catch (...) {
        g_last_error = "unknown native exception";
        return VXC_STATUS_RUNTIME_ERROR;
    }
}

void require(bool ok, const char* msg) {
    if (!ok) throw std::invalid_argument(msg);
}

// ------------------------------------------------------------ weights ----
struct LayerW {
    const __half *in_norm, *wqkv, *wo, *post_norm, *wgateup, *wdown;
};
struct DecoderShape {
    int h, f, hq, hkv, d, layers;
};

size_t decoder_count(const DecoderShape& s) {
    const size_t H = s.h, F = s.f, Q = static_cast<size_t>(s.hq) * s.d, KV = static_cast<size_t>(s.hkv) * s.d;
    return static_cast<size_t>(s.layers) * (H + Q * H + 2 * KV * H + H * Q + H + 2 * F * H + H * F) + H;
}

// The decoder blob stores per layer: input_norm, q, k, v, o, post_norm, gate,
// up, down (voxcpm2_b200/config.py). q/k/v are consecutive row blocks, i.e. one
// fused [(hq + 2 hkv) d][H] matrix; gate/up likewise form one [2F][H] matrix.
std::vector<LayerW> carve_decoder(const __half* base, const DecoderShape& s, const __half** final_norm) {
    const size_t H = s.h, F = s.f, Q = static_cast<size_t>(s.hq) * s.d, KV = static_cast<size_t>(s.hkv) * s.d;
    std::vector<LayerW> out;
    size_t off = 0;
    for (int l = 0; l < s.layers; ++l) {
        LayerW L{};
        L.in_norm = base + off;
        off += H;
        L.wqkv = base + off;
        off += (Q + 2 * KV) * H;
        L.wo = base + off;
        off += H * Q;
        L.post_norm = base + off;
        off += H;
        L.wgateup = base + off;
        off += 2 * F * H;
        L.wdown = base + off;
        off += H * F;
        out.push_back(L);
    }
    *final_norm = base + off;
    return out;
}

// TMA maps (64 x 64 boxes, 128-byte swizzle) of one decoder's per-layer matrices
std::vector<std::array<CUtensorMap, 4>> decoder_maps(const vxc_model_desc& d, const std::vector<LayerW>& layers) {
    const int H = d.hidden, F = d.ffn, Q = d.q_heads * d.head_dim;
    const int W = (d.q_heads + 2 * d.kv_heads) * d.head_dim;
    std::vector<std::array<CUtensorMap, 4>> maps;
    for (const LayerW& L : layers)
        maps.push_back({make_tensor_map_f16(L.wqkv, W, H, 64), make_tensor_map_f16(L.wo, H, Q, 64),
                        make_tensor_map_f16(L.wgateup, 2 * F, H, 64), make_tensor_map_f16(L.wdown, H, F, 64)});
    return maps;
}

DecoderShape base_shape(const vxc_model_desc& d) {
    return {d.hidden, d.ffn, d.q_heads, d.kv_heads, d.head_dim, d.base_layers};
}
DecoderShape res_shape(const vxc_model_desc& d) {
    return {d.hidden, d.ffn, d.q_heads, d.kv_heads, d.head_dim, d.res_layers};
}
DecoderShape dit_shape(const vxc_model_desc& d) {
    return {d.dit_hidden, d.dit_ffn, d.dit_q_heads, d.dit_kv_heads, d.dit_hidden / d.dit_q_heads, d.dit_layers};
}

size_t component_count(const vxc_model_desc& d, int c) {
    const size_t H = d.hidden, Hd = d.dit_hidden, D = d.feat_dim, P = d.patch_size, Q = d.fsq_dim;
    switch (c) {
        case VXC_TEXT_EMBED: return static_cast<size_t>(d.vocab) * H;
        case VXC_BASE_DECODER: return decoder_count(base_shape(d));
        case VXC_RESIDUAL_DECODER: return decoder_count(res_shape(d));
        case VXC_FSQ: return Q * H + Q + H * Q + H;
        case VXC_FUSION_PROJ: return H * 2 * H + H;
        case VXC_DIT_PROJ: return 2 * (Hd * H + Hd);
        case VXC_STOP_HEAD: return H * H + H + 2 * H;
        case VXC_FEAT_ENCODER: return H * (P * D) + H + H * H + H;
        case VXC_DIT_ESTIMATOR:
            return 2 * (Hd * D + Hd) + 4 * (Hd * Hd + Hd) + decoder_count(dit_shape(d)) + D * Hd + D;
        default: return 0;
    }
}

void validate_desc(const vxc_model_desc& d) {
    require(d.hidden > 0 && d.hidden % 8 == 0, "hidden must be a positive multiple of 8");
    require(d.ffn > 0 && d.ffn % 8 == 0, "ffn must be a positive multiple of 8");
    require(d.head_dim == 64, "head_dim must be 64");
    require(d.q_heads > 0 && d.kv_heads > 0 && d.q_heads % d.kv_heads == 0 && d.q_heads / d.kv_heads <= 16,
            "q_heads must be a multiple of kv_heads (group <= 16)");
    require(d.base_layers > 0 && d.res_layers > 0 && d.dit_layers > 0, "layer counts must be positive");
    require(d.dit_hidden > 0 && d.dit_hidden % 8 == 0 && d.dit_q_heads > 0 &&
                d.dit_hidden % d.dit_q_heads == 0 && d.dit_hidden / d.dit_q_heads == 64,
            "dit head_dim must be 64");
    require(d.dit_kv_heads > 0 && d.dit_q_heads % d.dit_kv_heads == 0, "dit heads must group");
    require(d.dit_ffn > 0 && d.dit_ffn % 8 == 0, "dit_ffn must be a positive multiple of 8");
    require(d.feat_dim > 0 && d.patch_size > 0 && 2 * d.patch_size <= 8 &&
                (d.feat_dim * d.patch_size) % 8 == 0,
            "unsupported patch shape");
    require(d.fsq_dim > 0 && d.fsq_dim % 8 == 0 && d.fsq_scale > 0.f, "bad fsq shape");
    require(d.vocab > 0, "vocab must be positive");
    require(d.rms_eps > 0.f && d.rope_theta > 0.f && d.rope_original_max > 0, "bad norm/rope settings");
    require(d.hidden <= 4096 && d.ffn <= 4096 && d.dit_hidden <= 4096 && d.dit_ffn <= 4096,
            "dimensions above 4096 are not supported");
    // tensor-core DiT linears: 128-feature tiles (64 gate/up pairs), 64-wide K chunks, <= 24 token rows
    require(d.dit_hidden % 128 == 0 && d.dit_ffn % 64 == 0 &&
                ((d.dit_q_heads + 2 * d.dit_kv_heads) * 64) % 128 == 0 && 2 * (3 + 2 * d.patch_size) <= 24,
            "DiT shape must tile by 128 features and 64-element K chunks");
    require(d.audio_start_token >= 0 && d.audio_start_token < d.vocab, "audio_start_token out of range");
}

// RoPE tables of Synthesizer::Impl::make_rope_cache (synthesizer.cpp:928-974):
// one row per position, freq_j = (pos / factor_j) * theta^(-2j / head_dim), with
// 'factor' the chosen LongRoPE table (head_dim / 2 values) or all ones when null.
void rope_table(int head_dim, float theta, int positions, std::vector<float>& cos_t, std::vector<float>& sin_t,
                const float* factor = nullptr) {
    const int half = head_dim / 2;
    std::vector<float> inv(half);
    for (int j = 0; j < half; ++j) {
        const float exponent = (2.0f * static_cast<float>(j)) / static_cast<float>(head_dim);
        inv[j] = 1.0f / std::pow(theta, exponent);
    }
    cos_t.assign(static_cast<size_t>(positions) * head_dim, 0.f);
    sin_t.assign(cos_t.size(), 0.f);
    for (int p = 0; p < positions; ++p) {
        for (int j = 0; j < half; ++j) {
            const float freq = (static_cast<float>(p) / (factor ? factor[j] : 1.0f)) * inv[j];
            const float c = std::cos(freq), s = std::sin(freq);
            cos_t[static_cast<size_t>(p) * head_dim + j] = c;
            cos_t[static_cast<size_t>(p) * head_dim + j + half] = c;
            sin_t[static_cast<size_t>(p) * head_dim + j] = s;
            sin_t[static_cast<size_t>(p) * head_dim + j + half] = s;
        }
    }
}

// Euler dt of each estimator step in cfm_sample's float arithmetic
// (synthesizer.cpp:49-60, 121-167): dts[step] for step = 1..T.
std::vector<float> euler_dts(int T) {
    std::vector<float> t_span(static_cast<size_t>(T) + 1);
    for (int i = 0; i <= T; ++i) {
        const float t = 1.0f - static_cast<float>(i) / static_cast<float>(T);
        t_span[i] = t + (std::cos(std::numbers::pi_v<float> * 0.5f * t) - 1.0f + t);
    }
    std::vector<float> dts(static_cast<size_t>(T) + 1, 0.f);
    float t = t_span[0];
    float dt = t_span[0] - (T >= 1 ? t_span[1] : 0.f);
    for (int step = 1; step <= T; ++step) {
        dts[step] = dt;
        t -= dt;
        if (step < T) dt = t - t_span[static_cast<size_t>(step) + 1];
    }
    return dts;
}

int zero_init_steps(int T) { return std::max(1, static_cast<int>((T + 1) * 0.04f)); }

int max_patches_for_target(int target_text_tokens, int hard_cap) {
    const int text_tokens = std::max(1, target_text_tokens);
    const int cap = static_cast<int>(static_cast<float>(text_tokens) * 6.0f + 10.0f);
    return std::max(1, std::min(hard_cap, cap));
}

template <typename T>
T* dev_alloc(size_t n) {
    void* p = nullptr;
    ck(cudaMalloc(&p, std::max<size_t>(n, 1) * sizeof(T)), "cudaMalloc");
    return static_cast<T*>(p);
}

struct DeviceGuard {
    int prev = -1;
    explicit DeviceGuard(int dev, bool nothrow = false) {
        if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
        const cudaError_t e = cudaSetDevice(dev);
        if (!nothrow) ck(e, "cudaSetDevice");
        else if (e != cudaSuccess) cudaGetLastError();
    }
    ~DeviceGuard() {
        if (prev >= 0) cudaSetDevice(prev);
    }
};

constexpr int dit_tokens_per_seq(int P) { return 3 + 2 * P; }

}  // namespace

// =================================================================== device ==
struct vxc_device {
    int device = 0;
    vxc_model_desc desc{};
    __half* blob[9] = {};
    bool loaded[9] = {};
    // the base decoder's LongRoPE factors (vxc_set_rope_factors); empty = all ones / none
    std::vector<float> rope_short, rope_long;
    uint64_t rope_epoch = 0;
    std::mutex rope_mu;  // guards the three above (set from any thread, read by stream calls)
    std::vector<LayerW> base, res, dit;
    const __half *base_norm = nullptr, *res_norm = nullptr, *dit_norm = nullptr;
    float *dit_rope_cos = nullptr, *dit_rope_sin = nullptr;  // positions 0..seq-1
    float* temb_freq = nullptr;  // the DiT timestep embedding's frequencies [dit_hidden / 2]
    std::atomic<int> live_groups{0};  // stream groups on this device (sets their wide linears' CTA target)
    // per DiT layer: TMA maps of W_qkv, W_o, W_gate|up, W_down (A operands)
    std::vector<std::array<CUtensorMap, 4>> dit_maps;
    // per decoder layer: TMA maps of W_qkv, W_o, W_gate|up, W_down for the prefill's row-block linears
    std::vector<std::array<CUtensorMap, 4>> base_maps, res_maps;
    uint64_t epoch = 0;  // bumped by every weight upload (invalidates derived tables)
};

namespace {

struct DitPtrs {
    const __half *in_w, *in_b, *cond_w, *cond_b, *t1_w, *t1_b, *t2_w, *t2_b, *dt1_w, *dt1_b, *dt2_w, *dt2_b;
    const __half *out_w, *out_b;
};

DitPtrs dit_ptrs(const vxc_device* dev) {
    const vxc_model_desc& d = dev->desc;
    const size_t Hd = d.dit_hidden, D = d.feat_dim;
    const __half* p = dev->blob[VXC_DIT_ESTIMATOR];
    DitPtrs w{};
    w.in_w = p; p += Hd * D;
    w.in_b = p; p += Hd;
    w.cond_w = p; p += Hd * D;
    w.cond_b = p; p += Hd;
    w.t1_w = p; p += Hd * Hd;
    w.t1_b = p; p += Hd;
    w.t2_w = p; p += Hd * Hd;
    w.t2_b = p; p += Hd;
    w.dt1_w = p; p += Hd * Hd;
    w.dt1_b = p; p += Hd;
    w.dt2_w = p; p += Hd * Hd;
    w.dt2_b = p; p += Hd;
    p += decoder_count(dit_shape(d));
    w.out_w = p; p += D * Hd;
    w.out_b = p;
    return w;
}

}  // namespace

// =================================================================== stream ==
struct vxc_stream {
    vxc_device* dev = nullptr;
    cudaStream_t cs = nullptr;
    int cap = 0;
    int splits = 16;
    std::mutex call_mutex;  // serialises calls on one stream (src/c_api.cpp:234-283)
    std::atomic<bool> cancel{false};

    StreamCtl* ctl = nullptr;       // device
    StreamCtl* ctl_host = nullptr;  // pinned mirror
    float *kc[2] = {}, *vc[2] = {};  // fp32 KV caches [layers][kv_heads][cap][head_dim]
    float *rope_cos = nullptr, *rope_sin = nullptr;          // short-factor rows [cap][head_dim]
    float *rope_cos_l = nullptr, *rope_sin_l = nullptr;      // long-factor rows (= short when none is set)
    uint64_t rope_epoch = ~0ull;                             // device factors the tables were built from
    // batch-1 step buffers
    float *h[2] = {}, *out[2] = {}, *q = nullptr, *attn = nullptr, *act = nullptr;
    float *lm_h = nullptr, *res_h = nullptr, *feat = nullptr, *mid = nullptr, *mid2 = nullptr;
    float* partial = nullptr;
    int* counters = nullptr;
    // CFM / DiT buffers
    float *mu = nullptr, *x = nullptr, *cond = nullptr, *cond0 = nullptr, *noise = nullptr, *latents = nullptr;
    float *temb = nullptr, *tmid = nullptr, *ttok = nullptr, *dtemb = nullptr, *dtmid = nullptr, *dttok = nullptr;
    float *dtemb1 = nullptr, *dtmid1 = nullptr, *dttok1 = nullptr;
    float *dh = nullptr, *dxn = nullptr, *dqkv = nullptr, *dattn = nullptr, *dact = nullptr, *est = nullptr;
    // split-fp16 B operands of the DiT's tensor-core linears ([48][K], rows 24+m = residuals)
    __half *xb_n = nullptr, *xb_a = nullptr, *xb_act = nullptr;
    CUtensorMap map_xb_n{}, map_xb_a{}, map_xb_act{};
    float* gen_in = nullptr;  // staging for generic calls
    float* pin = nullptr;     // pinned host staging
    // pipelined driving (vxc_patch_submit / vxc_patch_collect): per in-flight patch a
    // pinned noise slot, latent slot and control-block snapshot, and its completion event
    static constexpr int kInflight = 4;
    float* pin_noise = nullptr;      // [kInflight][D*P]
    float* pin_lat = nullptr;        // [kInflight][D*P]
    StreamCtl* pin_ctl = nullptr;    // [kInflight]
    cudaEvent_t patch_ev[kInflight] = {};
    int64_t submitted = 0, collected = 0;
    // prefill buffers (grown on demand)
    int pre_rows = 0;
    float *ph = nullptr, *pxn = nullptr, *pqkv = nullptr, *pattn = nullptr, *pact = nullptr, *pcat = nullptr;
    // row-block split-fp16 operands of the prefill's tcgen05 linears ([2 * kRowBlock][K]) and their maps
    __half *xr_n = nullptr, *xr_a = nullptr, *xr_act = nullptr;
    CUtensorMap map_xr_n{}, map_xr_a{}, map_xr_act{};
    float* xr_part = nullptr;  // K-split partial tiles of the prefill linears
    int32_t* pids = nullptr;

    // host mirror
    int kv_len[2] = {0, 0};
    int patches = 0;
    int prefix_len = 0;
    bool prefilled = false;
    int graph_T = -1;
    float graph_cfg = 0.f;
    // per timestep count T: rows t_tok(step) + dt_tok(0) of the sampler's
    // estimator steps, [T + 1][Hd]; contents follow the device's weight epoch
    struct TimeTable {
        float* dev = nullptr;
        uint64_t epoch = ~0ull;
    };
    std::map<int, TimeTable> ttab;
    float* dest = nullptr;  // [2][D*P] estimator output scratch of dit_out
    float* dssq = nullptr;  // [parts][24] row sums of squares of s->dh, by slice
    // ring depth of the per-layer tensor-core launches (VXC_TC_STAGES): a shallow ring keeps a
    // CTA's shared memory small, so linears of several concurrent streams share an SM
    int tc_stages = 2;
    // CTAs a per-layer tensor-core launch aims at (VXC_TC_TARGET): 32 by default, so most
    // linears run without a K split (no cluster exchange) and concurrent streams share the SMs;
    // 148 (one per SM) trades ~45% of the multi-stream throughput for ~8% lower single-stream latency
    int tc_target = 32;
    // programmatic dependent launch between the patch graph's kernels (VXC_NO_PDL=1 turns it off)
    bool pdl = true;
    // split tcgen05 linears receive their partials in the idle stage area (VXC_RECV_SHARED=1)
    bool recv_shared = false;
    // split DiT form: RMSNorm folded into the neighbouring linears (the residual epilogue writes the
    // next operand, the consumer scales rows by 1/rms); VXC_NORM_KERNELS=1 launches separate RMSNorm kernels
    bool norm_kernels = false;
    // decoder-step GEMVs: register-streaming (the default: the highest 16-stream throughput), or
    // VXC_BULK_GEMV=1 for the bulk-copy form (weight rows into shared memory before the
    // dependency wait; stream groups always use it, batched over their members)
    bool bulk_gemv = false;
    int* dcount = nullptr;  // dit_out arrival counter
    cudaGraphExec_t graph = nullptr;
    int graph_kernels = 0;
    int min_patches_dev = -1;

    ~vxc_stream();
};

namespace {

void free_all(vxc_stream* s) {
    if (s->graph) cudaGraphExecDestroy(s->graph);
    s->graph = nullptr;
    void* ptrs[] = {s->ctl, s->kc[0], s->kc[1], s->vc[0], s->vc[1], s->rope_cos, s->rope_sin, s->rope_cos_l,
                    s->rope_sin_l, s->h[0], s->h[1],
                    s->out[0], s->out[1], s->q, s->attn, s->act, s->lm_h, s->res_h, s->feat, s->mid, s->mid2,
                    s->partial, s->counters, s->mu, s->x, s->cond, s->cond0, s->noise, s->latents, s->temb,
                    s->tmid, s->ttok, s->dtemb, s->dtmid, s->dttok, s->dtemb1, s->dtmid1, s->dttok1, s->dh,
                    s->dxn, s->dqkv, s->dattn, s->dact, s->est, s->gen_in, s->ph, s->pxn, s->pqkv, s->pattn,
                    s->pact, s->pcat, s->pids, s->xb_n, s->xb_a, s->xb_act};
    for (void* p : ptrs)
        if (p) cudaFree(p);
    for (auto& kv : s->ttab)
        if (kv.second.dev) cudaFree(kv.second.dev);
    if (s->dest) cudaFree(s->dest);
    if (s->dssq) cudaFree(s->dssq);
    for (__half* p : {s->xr_n, s->xr_a, s->xr_act})
        if (p) cudaFree(p);
    if (s->xr_part) cudaFree(s->xr_part);
    if (s->dcount) cudaFree(s->dcount);
    if (s->ctl_host) cudaFreeHost(s->ctl_host);
    if (s->pin) cudaFreeHost(s->pin);
    for (void* p : {static_cast<void*>(s->pin_noise), static_cast<void*>(s->pin_lat), static_cast<void*>(s->pin_ctl)})
        if (p) cudaFreeHost(p);
    for (cudaEvent_t& e : s->patch_ev)
        if (e) cudaEventDestroy(e);
    if (s->cs) cudaStreamDestroy(s->cs);
}

void check_loaded(const vxc_device* dev, std::initializer_list<int> comps) {
    for (int c : comps)
        if (!dev->loaded[c]) throw InvalidState("weights of a required component are not loaded");
}

GemvArgs plain_gemv(const __half* w, const __half* b, const float* x, int K, int rows, float* y, int act,
                    StreamCtl* ctl, int skip) {
    GemvArgs a;
    a.mode = GEMV_PLAIN;
    a.w = w;
    a.bias = b;
    a.x = x;
    a.K = K;
    a.rows = rows;
    a.y = y;
    a.act = act;
    a.ctl = ctl;
    a.skip_if_stopped = skip;
    return a;
}

// ----------------------------------------------------------- enqueue ------
// The base decoder's RoPE tables from the device's LongRoPE factors: rebuilt when
// the factors changed since the stream last built them (same device pointers, so
// captured graphs stay valid). The stream's queue is drained first.
void sync_rope(vxc_stream* s) {
    vxc_device* dev = s->dev;
    std::vector<float> short_f, long_f;
    uint64_t epoch = 0;
    {
        std::lock_guard<std::mutex> lk(dev->rope_mu);
        if (s->rope_epoch == dev->rope_epoch) return;
        short_f = dev->rope_short;
        long_f = dev->rope_long;
        epoch = dev->rope_epoch;
    }
    const vxc_model_desc& d = dev->desc;
    const int hd = d.head_dim;
    std::vector<float> c, sn;
    ck(cudaStreamSynchronize(s->cs), "rope tables");
    rope_table(hd, d.rope_theta, s->cap, c, sn, short_f.empty() ? nullptr : short_f.data());
    ck(cudaMemcpy(s->rope_cos, c.data(), sizeof(float) * c.size(), cudaMemcpyHostToDevice), "rope");
    ck(cudaMemcpy(s->rope_sin, sn.data(), sizeof(float) * sn.size(), cudaMemcpyHostToDevice), "rope");
    if (!long_f.empty()) rope_table(hd, d.rope_theta, s->cap, c, sn, long_f.data());
    ck(cudaMemcpy(s->rope_cos_l, c.data(), sizeof(float) * c.size(), cudaMemcpyHostToDevice), "rope");
    ck(cudaMemcpy(s->rope_sin_l, sn.data(), sizeof(float) * sn.size(), cudaMemcpyHostToDevice), "rope");
    s->rope_epoch = epoch;
}

// RoPE of a one-row base-decoder q/k/v GEMV: the position (device side) picks the
// short- or long-factor row as make_rope_cache(pos, 1) does.
void set_decode_rope(GemvArgs& a, const vxc_stream* s) {
    a.rope_cos = s->rope_cos;
    a.rope_sin = s->rope_sin;
    a.rope_cos_long = s->rope_cos_l;
    a.rope_sin_long = s->rope_sin_l;
    a.rope_long_from = s->dev->desc.rope_original_max;
}

// Batch-1 decoder step over s->h[which] (the residual stream, already holding
// the input embedding); writes the final-norm output to out (+ out2) and bumps
// kv_len[which] on the device (unless advance is 0). ctl_override replaces the
// stream's control block (the step profile runs on a private one).
void enqueue_decoder_step(vxc_stream* s, int which, float* out, float* out2, int skip,
                          StreamCtl* ctl_override = nullptr, int advance = 1) {
    StreamCtl* ctl = ctl_override ? ctl_override : s->ctl;

    auto gemv = s->bulk_gemv ? launch_gemv_bulk : launch_gemv;
    const vxc_device* dev = s->dev;
    const vxc_model_desc& d = dev->desc;
    const std::vector<LayerW>& layers = which == 0 ? dev->base : dev->res;
    const __half* fnorm = which == 0 ? dev->base_norm : dev->res_norm;
    const float rscale = which == 0 ? d.base_residual_scale : d.res_residual_scale;
    const int H = d.hidden, F = d.ffn, hq = d.q_heads, hkv = d.kv_heads, hd = d.head_dim;
    const size_t plane = static_cast<size_t>(hkv) * s->cap * hd;
    for (size_t l = 0; l < layers.size(); ++l) {
        const LayerW& L = layers[l];
        GemvArgs qa;
        qa.mode = GEMV_QKV;
        qa.w = L.wqkv;
        qa.x = s->h[which];
        qa.norm_g = L.in_norm;
        qa.eps = d.rms_eps;
        qa.K = H;
        qa.rows = (hq + 2 * hkv) * hd / 2;
        qa.y = s->q;
        qa.q_heads = hq;
        qa.kv_heads = hkv;
        qa.head_dim = hd;
        if (which == 0) set_decode_rope(qa, s);
        qa.k_cache = s->kc[which] + l * plane;
        qa.v_cache = s->vc[which] + l * plane;
        qa.cap = s->cap;
        qa.which = which;
        qa.ctl = ctl;
        qa.skip_if_stopped = skip;
        gemv(qa, s->cs, s->pdl);

        AttnArgs aa;
        aa.q = s->q;
        aa.k0 = s->kc[which] + l * plane;
        aa.v0 = s->vc[which] + l * plane;
        aa.len0 = s->cap;
        aa.stride0 = s->cap;
        aa.q_heads = hq;
        aa.kv_heads = hkv;
        aa.head_dim = hd;
        aa.scale = 1.0f / std::sqrt(static_cast<float>(hd));
        aa.splits = s->splits;
        aa.partial = s->partial;
        aa.counters = s->counters;
        aa.out = s->attn;
        aa.ctl = ctl;
        aa.which = which;
        aa.skip_if_stopped = skip;
        launch_attn_decode_cluster(aa, s->cs, s->pdl);

        GemvArgs oa;
        oa.mode = GEMV_RESID;
        oa.w = L.wo;
        oa.x = s->attn;
        oa.K = hq * hd;
        oa.rows = H;
        oa.resid = s->h[which];
        oa.rscale = rscale;
        oa.ctl = ctl;
        oa.skip_if_stopped = skip;
        gemv(oa, s->cs, s->pdl);

        GemvArgs ga;
        ga.mode = GEMV_GATEUP;
        ga.w = L.wgateup;
        ga.x = s->h[which];
        ga.norm_g = L.post_norm;
        ga.eps = d.rms_eps;
        ga.K = H;
        ga.rows = F;
        ga.y = s->act;
        ga.ctl = ctl;
        ga.skip_if_stopped = skip;
        gemv(ga, s->cs, s->pdl);

        GemvArgs da;
        da.mode = GEMV_RESID;
        da.w = L.wdown;
        da.x = s->act;
        da.K = F;
        da.rows = H;
        da.resid = s->h[which];
        da.rscale = rscale;
        da.ctl = ctl;
        da.skip_if_stopped = skip;
        gemv(da, s->cs, s->pdl);
    }
    launch_final_norm(s->h[which], fnorm, d.rms_eps, H, out, out2, ctl, which, advance, skip, s->cs, s->pdl);
}

// K split (cluster size) of a tensor-core linear: about 'target' CTAs per launch
// (one per SM for a single stream; fewer when many streams share the GPU, which
// saves each CTA's fixed setup and split-K exchange).
int choose_splits(int tiles, int k, int target = 148, int most = 8) {
    const int chunks = k / 64;
    const int want = std::max(1, (target + tiles / 2) / tiles);
    return std::max(1, std::min({most, chunks, want}));
}

// The tensor-core kernels split K over 1, 2, 4, 8 or 16 CTAs.
int pow2_floor(int v) { return v >= 16 ? 16 : v >= 8 ? 8 : v >= 4 ? 4 : v >= 2 ? 2 : 1; }

// K split and ring depth of one tensor-core launch: about tc_target CTAs per launch.
// 'most' caps the split: 16 for the down projection only (K = 4096). There a 16-CTA
// cluster gives the latency plan 128 CTAs of 4 weight chunks each instead of 64 CTAs
// of 8, so a 3-stage ring refills once after the dependency wait instead of five
// times (one estimator evaluation 364 -> 339 us on B200). The o projection (K = 1024)
// measured slower at 16 (one chunk per CTA: the exchange outweighs the bytes); q/k/v
// and gate/up keep 8.
TcLinearArgs tc_plan(const vxc_stream* s, int tiles, int K, int most) {
    TcLinearArgs a;
    a.splits = pow2_floor(choose_splits(tiles, K, s->tc_target, most));
    a.max_stages = s->tc_stages;
    a.recv_shared = s->recv_shared ? 1 : 0;
    return a;
}

// DiT decoder over the 2 x seq rows in s->dh (DitEstimator.decoder,
// export_components.py:625-659): per layer the four linears on tcgen05 and the
// attention on CUDA cores. RMSNorm is folded into the linears: the residual
// epilogues of o and down also write the next linear's split-fp16 operand of
// dh * gain and per-slice sums of squares, and the consumer scales each token
// row by 1 / rms (W (x g / rms) = (1 / rms) W (x g)); layer 0 (after the
// embedding) and VXC_NORM_KERNELS=1 launch separate RMSNorm kernels instead.
void enqueue_dit_layers(vxc_stream* s, StreamCtl* ctl) {
    const vxc_device* dev = s->dev;
    const vxc_model_desc& d = dev->desc;
    const int Hd = d.dit_hidden, F = d.dit_ffn, hq = d.dit_q_heads, hkv = d.dit_kv_heads, hd = Hd / hq;
    const int seq = dit_tokens_per_seq(d.patch_size), M = 2 * seq;
    const int W = (hq + 2 * hkv) * hd;
    const float scale = 1.0f / std::sqrt(static_cast<float>(hd));
    // sums-of-squares parts of s->dh: dit_embed leaves one per 32 features
    int parts = (Hd + 31) / 32;
    for (size_t l = 0; l < dev->dit.size(); ++l) {
        const LayerW& L = dev->dit[l];
        const std::array<CUtensorMap, 4>& maps = dev->dit_maps[l];
        TcLinearArgs qa = tc_plan(s, W / 128, Hd, 8);
        qa.K = Hd;
        qa.M = M;
        qa.rows = W;
        qa.y = s->dqkv;
        qa.ldy = W;
        qa.ctl = ctl;
        if (l == 0 || s->norm_kernels) {
            launch_rmsnorm_rows_split(s->dh, Hd, L.in_norm, d.rms_eps, Hd, M, s->xb_n, ctl, s->cs, s->pdl);
        } else {  // the previous down projection left split(dh * in_norm) and its sums of squares
            qa.row_scale = 1;
            qa.ssq_in = s->dssq;
            qa.ssq_parts = parts;
            qa.eps = d.rms_eps;
        }
        launch_tc_linear(maps[0], s->map_xb_n, qa, s->cs, s->pdl);
        TcLinearArgs oa = tc_plan(s, Hd / 128, hq * hd, 8);
        oa.K = hq * hd;
        oa.M = M;
        oa.rows = Hd;
        oa.resid = 1;
        oa.rscale = d.dit_residual_scale;
        oa.y = s->dh;
        oa.ldy = Hd;
        oa.ctl = ctl;
        launch_dit_attention_split(s->dqkv, 2, seq, hq, hkv, hd, dev->dit_rope_cos, dev->dit_rope_sin, scale,
                                   s->xb_a, ctl, s->cs, s->pdl);
        if (!s->norm_kernels) {
            // the residual epilogue also writes split(dh * post_norm) for gate/up, and the sums of squares
            oa.ssq_out = s->dssq;
            oa.next_g = L.post_norm;
            oa.next_b = s->xb_n;
            oa.ldnb = Hd;
        }
        launch_tc_linear(maps[1], s->map_xb_a, oa, s->cs, s->pdl);
        const int o_parts = (Hd / 128) * oa.splits;
        TcLinearArgs ga = tc_plan(s, F / 64, Hd, 8);
        ga.K = Hd;
        ga.M = M;
        ga.rows = F;
        ga.gateup = 1;
        ga.yb = s->xb_act;
        ga.ldyb = F;
        ga.ctl = ctl;
        if (s->norm_kernels) {
            launch_rmsnorm_rows_split(s->dh, Hd, L.post_norm, d.rms_eps, Hd, M, s->xb_n, ctl, s->cs, s->pdl);
        } else {
            ga.row_scale = 1;
            ga.ssq_in = s->dssq;
            ga.ssq_parts = o_parts;
            ga.eps = d.rms_eps;
        }
        launch_tc_linear(maps[2], s->map_xb_n, ga, s->cs, s->pdl);
        TcLinearArgs da = tc_plan(s, Hd / 128, F, 16);
        da.K = F;
        da.M = M;
        da.rows = Hd;
        da.resid = 1;
        da.rscale = d.dit_residual_scale;
        da.y = s->dh;
        da.ldy = Hd;
        da.ctl = ctl;
        if (!s->norm_kernels && l + 1 < dev->dit.size()) {  // the next q/k/v operand, split(dh * in_norm)
            da.ssq_out = s->dssq;
            da.next_g = dev->dit[l + 1].in_norm;
            da.next_b = s->xb_n;
            da.ldnb = Hd;
        }
        launch_tc_linear(maps[3], s->map_xb_act, da, s->cs, s->pdl);
        parts = (Hd / 128) * da.splits;
    }
}

// time_mlp(emb(t)) for estimator step 'step_index' (schedule mode) into
// s->ttok, and delta_time_mlp(emb(dt)) rows into s->dttok / s->dttok1.
void enqueue_time_tokens(vxc_stream* s, float step_index, float T, const float* dt_raw, StreamCtl* ctl) {
    const vxc_model_desc& d = s->dev->desc;
    const DitPtrs w = dit_ptrs(s->dev);
    const int Hd = d.dit_hidden;
    const int sk = ctl ? 1 : 0;
    const float* freq = s->dev->temb_freq;
    // the estimator's time layers: scale 1000, schedule mode 1 for t and 0 for dt
    const float t_sched = timestep_scheduled_t(step_index, T) * 1000.0f;
    launch_timestep_embedding(nullptr, t_sched, 1, freq, Hd / 2, s->temb, ctl, s->cs, s->pdl);
    launch_gemv(plain_gemv(w.t1_w, w.t1_b, s->temb, Hd, Hd, s->tmid, ACT_SILU, ctl, sk), s->cs, s->pdl);
    launch_gemv(plain_gemv(w.t2_w, w.t2_b, s->tmid, Hd, Hd, s->ttok, ACT_NONE, ctl, sk), s->cs, s->pdl);
    launch_timestep_embedding(nullptr, dt_raw[0] * 1000.0f, 1, freq, Hd / 2, s->dtemb, ctl, s->cs, s->pdl);
    launch_gemv(plain_gemv(w.dt1_w, w.dt1_b, s->dtemb, Hd, Hd, s->dtmid, ACT_SILU, ctl, sk), s->cs, s->pdl);
    launch_gemv(plain_gemv(w.dt2_w, w.dt2_b, s->dtmid, Hd, Hd, s->dttok, ACT_NONE, ctl, sk), s->cs, s->pdl);
    if (dt_raw[1] != dt_raw[0]) {
        launch_timestep_embedding(nullptr, dt_raw[1] * 1000.0f, 1, freq, Hd / 2, s->dtemb1, ctl, s->cs, s->pdl);
        launch_gemv(plain_gemv(w.dt1_w, w.dt1_b, s->dtemb1, Hd, Hd, s->dtmid1, ACT_SILU, ctl, sk), s->cs, s->pdl);
        launch_gemv(plain_gemv(w.dt2_w, w.dt2_b, s->dtmid1, Hd, Hd, s->dttok1, ACT_NONE, ctl, sk), s->cs, s->pdl);
    }
}

// One estimator evaluation + (if x_update) the CFG-zero* Euler update.
void enqueue_dit_eval(vxc_stream* s, const float* x, const float* x_unc, const float* mu, const float* mu_unc,
                      const float* cond, const float* cond_unc, bool dt_rows_differ, float* est_out,
                      float* x_update, float dt, float cfg, StreamCtl* ctl, const float* tsum) {
    const vxc_model_desc& d = s->dev->desc;
    const DitPtrs w = dit_ptrs(s->dev);
    DitEmbedArgs e{};
    e.in_w = w.in_w;
    e.in_b = w.in_b;
    e.cond_w = w.cond_w;
    e.cond_b = w.cond_b;
    e.x = x;
    e.cond = cond;
    e.mu = mu;
    e.t_tok0 = s->ttok;
    e.t_tok1 = s->ttok;
    e.dt_tok0 = s->dttok;
    e.dt_tok1 = dt_rows_differ ? s->dttok1 : s->dttok;
    e.Hd = d.dit_hidden;
    e.D = d.feat_dim;
    e.P = d.patch_size;
    e.hidden = s->dh;
    e.ctl = ctl;
    e.mu_uncond = mu_unc;
    e.x_uncond = x_unc;
    e.cond_uncond = cond_unc;
    e.tsum = tsum;
    e.ssq_out = s->dssq;
    launch_dit_embed(e, s->cs, s->pdl);
    enqueue_dit_layers(s, ctl);
    DitOutArgs o{};
    o.hidden = s->dh;
    o.seq = dit_tokens_per_seq(d.patch_size);
    o.Hd = d.dit_hidden;
    o.D = d.feat_dim;
    o.P = d.patch_size;
    o.norm_g = s->dev->dit_norm;
    o.eps = d.rms_eps;
    o.out_w = w.out_w;
    o.out_b = w.out_b;
    o.est_out = est_out;
    o.x = x_update;
    o.dt = dt;
    o.cfg = cfg;
    o.ctl = ctl;
    o.est_buf = est_out ? est_out : s->dest;
    o.counter = s->dcount;
    launch_dit_out(o, s->cs, s->pdl);
}

// cfm_sample over s->x (holding the noise), mu = s->mu (row 1 of mu_in stays
// zero: the unconditional CFG branch, synthesizer.cpp:52, 114).
// The sampler's time tokens depend only on the weights and (step, T): the
// time_mlp(emb(t_step)) + delta_time_mlp(emb(0)) rows are computed once per T
// (by the same kernels, eagerly, outside any capture) and re-used by every
// patch. Refreshed when the weights change.
const float* time_table(vxc_stream* s, int T) {
    vxc_stream::TimeTable& t = s->ttab[T];
    const int Hd = s->dev->desc.dit_hidden;
    if (!t.dev) t.dev = dev_alloc<float>(static_cast<size_t>(T + 1) * Hd);
    if (t.epoch != s->dev->epoch) {
        const float dt0[2] = {0.f, 0.f};
        for (int step = 1; step <= T; ++step) {
            enqueue_time_tokens(s, static_cast<float>(step - 1), static_cast<float>(T), dt0, nullptr);
            launch_vec_add(s->ttok, s->dttok, t.dev + static_cast<size_t>(step) * Hd, Hd, s->cs);
        }
        ck(cudaStreamSynchronize(s->cs), "time table");
        t.epoch = s->dev->epoch;
    }
    return t.dev;
}

// cfm_sample's Euler loop; time_table(s, T) must be current.
void enqueue_cfm(vxc_stream* s, const float* cond_dev, int T, float cfg) {
    const std::vector<float> dts = euler_dts(T);
    const int z = zero_init_steps(T);
    const int Hd = s->dev->desc.dit_hidden;
    const float* tab = s->ttab.at(T).dev;
    for (int step = 1; step <= T; ++step) {
        if (step <= z) continue;  // zero-init steps leave x untouched (synthesizer.cpp:123-126)
        enqueue_dit_eval(s, s->x, nullptr, s->mu, nullptr, cond_dev, nullptr, false, nullptr, s->x, dts[step], cfg,
                         s->ctl, tab + static_cast<size_t>(step) * Hd);
    }
}

// The patch iteration before the sampler: noise and condition of this patch,
// then dit_proj: mu = cat(lm_to_dit_proj(lm), res_to_dit_proj(res)).
void enqueue_patch_pre(vxc_stream* s) {
    const vxc_device* dev = s->dev;
    const vxc_model_desc& d = dev->desc;
    const int H = d.hidden, Hd = d.dit_hidden, L = d.feat_dim * d.patch_size;
    launch_patch_begin(s->noise, s->latents, s->cond0, L, s->x, s->cond, s->ctl, s->cs, s->pdl);
    const __half* dp = dev->blob[VXC_DIT_PROJ];
    const size_t dps = static_cast<size_t>(Hd) * H;
    launch_gemv(plain_gemv(dp, dp + dps, s->lm_h, H, Hd, s->mu, ACT_NONE, s->ctl, 0), s->cs, s->pdl);
    launch_gemv(plain_gemv(dp + dps + Hd, dp + 2 * dps + Hd, s->res_h, H, Hd, s->mu + Hd, ACT_NONE, s->ctl, 0),
                s->cs, s->pdl);
}

// The whole patch iteration (synthesizer.cpp:546-658) on s->cs.
void enqueue_patch_post(vxc_stream* s);
void enqueue_patch(vxc_stream* s, int T, float cfg) {
    enqueue_patch_pre(s);
    enqueue_cfm(s, s->cond, T, cfg);
    enqueue_patch_post(s);
}

// Post-sampler part A: stop decision, feat_encoder (-> the base decoder input).
void enqueue_post_stop_feat(vxc_stream* s) {
    const vxc_device* dev = s->dev;
    const vxc_model_desc& d = dev->desc;
    const int H = d.hidden, L = d.feat_dim * d.patch_size;
    // stop head on the hidden state entering this patch
    const __half* sh = dev->blob[VXC_STOP_HEAD];
    launch_gemv(plain_gemv(sh, sh + static_cast<size_t>(H) * H, s->lm_h, H, H, s->mid, ACT_SILU, s->ctl, 0), s->cs,
                true);
    launch_stop_decide(sh + static_cast<size_t>(H) * H + H, s->mid, H, s->ctl, nullptr, s->cs, s->pdl);
    // feat_encoder(latent) -> feat and the base decoder input
    const __half* fe = dev->blob[VXC_FEAT_ENCODER];
    const size_t fin = static_cast<size_t>(H) * L;
    GemvArgs fa = plain_gemv(fe, fe + fin, s->x, L, H, s->mid2, ACT_SILU, s->ctl, 1);
    fa.in_mode = IN_LATENT_T;
    fa.lat_d = d.feat_dim;
    fa.lat_p = d.patch_size;
    launch_gemv(fa, s->cs, s->pdl);
    GemvArgs fb = plain_gemv(fe + fin + H, fe + fin + H + static_cast<size_t>(H) * H, s->mid2, H, H, s->feat,
                             ACT_NONE, s->ctl, 1);
    fb.y2 = s->h[0];
    launch_gemv(fb, s->cs, s->pdl);
}

// Part B, after the base decoder step: FSQ and fusion (-> the residual decoder input).
void enqueue_post_fsq_fusion(vxc_stream* s) {
    const vxc_device* dev = s->dev;
    const vxc_model_desc& d = dev->desc;
    const int H = d.hidden;
    // fsq
    const __half* fq = dev->blob[VXC_FSQ];
    const size_t Q = d.fsq_dim;
    GemvArgs qa = plain_gemv(fq, fq + Q * H, s->out[0], H, static_cast<int>(Q), s->mid, ACT_FSQ, s->ctl, 1);
    qa.act_scale = d.fsq_scale;
    launch_gemv(qa, s->cs, s->pdl);
    launch_gemv(plain_gemv(fq + Q * H + Q, fq + Q * H + Q + H * Q, s->mid, static_cast<int>(Q), H, s->lm_h, ACT_NONE,
                           s->ctl, 1),
                s->cs, s->pdl);
    // fusion_proj(cat(lm, feat)) -> residual decoder input
    const __half* fu = dev->blob[VXC_FUSION_PROJ];
    GemvArgs ua = plain_gemv(fu, fu + static_cast<size_t>(H) * 2 * H, s->lm_h, 2 * H, H, s->h[1], ACT_NONE, s->ctl, 1);
    ua.in_mode = IN_CONCAT;
    ua.x2 = s->feat;
    ua.k1 = H;
    launch_gemv(ua, s->cs, s->pdl);
}

// Part C, after the residual decoder step: the latent's store (on stream cs, or
// the member's own stream).
void enqueue_post_end(vxc_stream* s, cudaStream_t cs = nullptr) {
    const int L = s->dev->desc.feat_dim * s->dev->desc.patch_size;
    launch_patch_end(s->x, s->latents, L, s->ctl, cs ? cs : s->cs, s->pdl);
}

// The patch iteration after the sampler: the stop decision, feat_encoder, both
// decoder steps, FSQ and fusion, and the latent's store.
void enqueue_patch_post(vxc_stream* s) {
    enqueue_post_stop_feat(s);
    enqueue_decoder_step(s, 0, s->out[0], nullptr, 1);
    enqueue_post_fsq_fusion(s);
    enqueue_decoder_step(s, 1, s->res_h, nullptr, 1);
    enqueue_post_end(s);
}

void sync_ctl(vxc_stream* s) {
    ck(cudaMemcpyAsync(s->ctl_host, s->ctl, sizeof(StreamCtl), cudaMemcpyDeviceToHost, s->cs), "ctl readback");
    ck(cudaStreamSynchronize(s->cs), "cudaStreamSynchronize");
    const int err = s->ctl_host->error;
    if (err != 0) {
        s->ctl_host->error = 0;
        cudaMemcpyAsync(&s->ctl->error, &s->ctl_host->error, sizeof(int), cudaMemcpyHostToDevice, s->cs);
        cudaStreamSynchronize(s->cs);
        if (err == 1) throw std::runtime_error("KV cache capacity exceeded on the device");
        if (err == 2) throw std::runtime_error("dit_estimator produced non-finite values");
        if (err == 3) throw std::runtime_error("a tensor-core pipeline wait timed out");
        throw std::runtime_error("device-side check failed");
    }
    s->kv_len[0] = s->ctl_host->kv_len[0];
    s->kv_len[1] = s->ctl_host->kv_len[1];
    s->patches = s->ctl_host->patch;
}

void write_ctl(vxc_stream* s) {
    ck(cudaMemcpyAsync(s->ctl, s->ctl_host, sizeof(StreamCtl), cudaMemcpyHostToDevice, s->cs), "ctl upload");
    ck(cudaStreamSynchronize(s->cs), "cudaStreamSynchronize");
}

void ensure_prefill_rows(vxc_stream* s, int n) {
    if (n <= s->pre_rows) return;
    const vxc_model_desc& d = s->dev->desc;
    for (float* p : {s->ph, s->pxn, s->pqkv, s->pattn, s->pact, s->pcat})
        if (p) cudaFree(p);
    if (s->pids) cudaFree(s->pids);
    s->ph = s->pxn = s->pqkv = s->pattn = s->pact = s->pcat = nullptr;
    s->pids = nullptr;
    s->pre_rows = 0;
    const size_t H = d.hidden, F = d.ffn, W = static_cast<size_t>(d.q_heads + 2 * d.kv_heads) * d.head_dim;
    s->ph = dev_alloc<float>(n * H);
    s->pxn = dev_alloc<float>(n * H);
    s->pqkv = dev_alloc<float>(n * W);
    s->pattn = dev_alloc<float>(n * static_cast<size_t>(d.q_heads) * d.head_dim);
    s->pact = dev_alloc<float>(n * F);
    s->pcat = dev_alloc<float>(n * 2 * H);
    s->pids = dev_alloc<int32_t>(n);
    s->pre_rows = n;
    if (!s->xr_n) {  // row-block operands: one block of kRowBlock rows, reused block after block
        const size_t Q = static_cast<size_t>(d.q_heads) * d.head_dim;
        s->xr_n = dev_alloc<__half>(2 * kRowBlock * H);
        s->xr_a = dev_alloc<__half>(2 * kRowBlock * Q);
        s->xr_act = dev_alloc<__half>(2 * kRowBlock * F);
        ck(cudaMemset(s->xr_n, 0, 2 * kRowBlock * H * sizeof(__half)), "cudaMemset");
        ck(cudaMemset(s->xr_a, 0, 2 * kRowBlock * Q * sizeof(__half)), "cudaMemset");
        ck(cudaMemset(s->xr_act, 0, 2 * kRowBlock * F * sizeof(__half)), "cudaMemset");
        s->map_xr_n = make_tensor_map_f16(s->xr_n, 2 * kRowBlock, static_cast<int>(H), 2 * kRowBlock);
        s->map_xr_a = make_tensor_map_f16(s->xr_a, 2 * kRowBlock, static_cast<int>(Q), 2 * kRowBlock);
        s->map_xr_act = make_tensor_map_f16(s->xr_act, 2 * kRowBlock, static_cast<int>(F), 2 * kRowBlock);
        // the largest split partial buffer of the four linears: splits x kRowBlock x outputs
        const int Hi = static_cast<int>(H), Fi = static_cast<int>(F), Wi = static_cast<int>(W), Qi = static_cast<int>(Q);
        const size_t part = std::max({static_cast<size_t>(tc_rows_splits(Wi, 0, Hi)) * Wi,
                                      static_cast<size_t>(tc_rows_splits(Hi, 0, Qi)) * Hi,
                                      static_cast<size_t>(tc_rows_splits(Fi, 1, Hi)) * 2 * Fi,
                                      static_cast<size_t>(tc_rows_splits(Hi, 0, Fi)) * Hi}) * kRowBlock;
        s->xr_part = dev_alloc<float>(part);
    }
}

// Multi-row decoder call (prefill): rows already in s->ph; out [n][H] device.
// The four linears of each layer run on tcgen05 over blocks of up to kRowBlock
// rows (tc_rows_kernel, weights read once per block); RMSNorm, RoPE + cache
// append and the causal attention run over all rows.
void run_decoder_rows(vxc_stream* s, int which, int n, float* out_dev) {
    const vxc_device* dev = s->dev;
    const vxc_model_desc& d = dev->desc;
    const std::vector<LayerW>& layers = which == 0 ? dev->base : dev->res;
    const std::vector<std::array<CUtensorMap, 4>>& maps = which == 0 ? dev->base_maps : dev->res_maps;
    const __half* fnorm = which == 0 ? dev->base_norm : dev->res_norm;
    const float rscale = which == 0 ? d.base_residual_scale : d.res_residual_scale;
    const int H = d.hidden, F = d.ffn, hq = d.q_heads, hkv = d.kv_heads, hd = d.head_dim, Q = hq * hd;
    const int W = (hq + 2 * hkv) * hd;
    const int past = s->kv_len[which];
    const size_t plane = static_cast<size_t>(hkv) * s->cap * hd;
    // make_rope_cache(past, n): every row takes the long-factor table when past + n > original_max
    const bool long_rows = past + n > d.rope_original_max;
    const float* rope_c = long_rows ? s->rope_cos_l : s->rope_cos;
    const float* rope_s = long_rows ? s->rope_sin_l : s->rope_sin;
    for (size_t l = 0; l < layers.size(); ++l) {
        const LayerW& L = layers[l];
        for (int r0 = 0; r0 < n; r0 += kRowBlock) {
            const int mb = std::min(kRowBlock, n - r0);
            launch_rmsnorm_rows_split(s->ph + static_cast<size_t>(r0) * H, H, L.in_norm, d.rms_eps, H, mb, s->xr_n,
                                      nullptr, s->cs, false, kRowBlock);
            TcRowsArgs qa;
            qa.K = H;
            qa.M = mb;
            qa.rows = W;
            qa.y = s->pqkv + static_cast<size_t>(r0) * W;
            qa.ldy = W;
            qa.ctl = s->ctl;
            qa.splits = tc_rows_splits(qa.rows, 0, qa.K);
            qa.part = s->xr_part;
            launch_tc_rows(maps[l][0], s->map_xr_n, qa, s->cs);
        }
        launch_qkv_rows_post(s->pqkv, n, hq, hkv, hd, past, 1 << 30, which == 0 ? rope_c : nullptr,
                             which == 0 ? rope_s : nullptr, s->kc[which] + l * plane, s->vc[which] + l * plane,
                             s->cap, s->ctl, s->cs, false);
        launch_attn_rows_cache(s->pqkv, n, hq, hkv, hd, past, s->kc[which] + l * plane, s->vc[which] + l * plane,
                               s->cap, 1.0f / std::sqrt(static_cast<float>(hd)), s->pattn, s->cs, false);
        for (int r0 = 0; r0 < n; r0 += kRowBlock) {
            const int mb = std::min(kRowBlock, n - r0);
            float* hb = s->ph + static_cast<size_t>(r0) * H;
            launch_rmsnorm_rows_split(s->pattn + static_cast<size_t>(r0) * Q, Q, nullptr, 0.f, Q, mb, s->xr_a, nullptr,
                                      s->cs, false, kRowBlock);
            TcRowsArgs oa;
            oa.K = Q;
            oa.M = mb;
            oa.rows = H;
            oa.resid = 1;
            oa.rscale = rscale;
            oa.y = hb;
            oa.ldy = H;
            oa.ctl = s->ctl;
            oa.splits = tc_rows_splits(oa.rows, 0, oa.K);
            oa.part = s->xr_part;
            launch_tc_rows(maps[l][1], s->map_xr_a, oa, s->cs);
            launch_rmsnorm_rows_split(hb, H, L.post_norm, d.rms_eps, H, mb, s->xr_n, nullptr, s->cs, false, kRowBlock);
            TcRowsArgs ga;
            ga.K = H;
            ga.M = mb;
            ga.rows = F;
            ga.gateup = 1;
            ga.yb = s->xr_act;
            ga.ldyb = F;
            ga.ctl = s->ctl;
            ga.splits = tc_rows_splits(ga.rows, 1, ga.K);
            ga.part = s->xr_part;
            launch_tc_rows(maps[l][2], s->map_xr_n, ga, s->cs);
            TcRowsArgs da;
            da.K = F;
            da.M = mb;
            da.rows = H;
            da.resid = 1;
            da.rscale = rscale;
            da.y = hb;
            da.ldy = H;
            da.ctl = s->ctl;
            da.splits = tc_rows_splits(da.rows, 0, da.K);
            da.part = s->xr_part;
            launch_tc_rows(maps[l][3], s->map_xr_act, da, s->cs);
        }
    }
    launch_rmsnorm_rows(s->ph, H, fnorm, d.rms_eps, H, n, out_dev, H, nullptr, 0, s->cs, false);
    s->ctl_host->kv_len[which] = past + n;
    ck(cudaMemcpyAsync(&s->ctl->kv_len[which], &s->ctl_host->kv_len[which], sizeof(int), cudaMemcpyHostToDevice,
                       s->cs),
       "kv_len update");
    ck(cudaStreamSynchronize(s->cs), "cudaStreamSynchronize");
    s->kv_len[which] = past + n;
}

void decoder_call(vxc_stream* s, int which, const float* embed, int n, float* out) {
    const vxc_model_desc& d = s->dev->desc;
    const int H = d.hidden;
    check_loaded(s->dev, {which == 0 ? VXC_BASE_DECODER : VXC_RESIDUAL_DECODER});
    if (s->kv_len[which] + n > s->cap) throw std::invalid_argument("decoder KV cache capacity exceeded");
    if (n == 1) {
        ck(cudaMemcpyAsync(s->h[which], embed, sizeof(float) * H, cudaMemcpyHostToDevice, s->cs), "upload");
        enqueue_decoder_step(s, which, s->out[which], nullptr, 0);
        ck(cudaMemcpyAsync(out, s->out[which], sizeof(float) * H, cudaMemcpyDeviceToHost, s->cs), "download");
        sync_ctl(s);
    } else {
        ensure_prefill_rows(s, n);
        ck(cudaMemcpyAsync(s->ph, embed, sizeof(float) * H * n, cudaMemcpyHostToDevice, s->cs), "upload");
        run_decoder_rows(s, which, n, s->pxn);
        ck(cudaMemcpy(out, s->pxn, sizeof(float) * H * n, cudaMemcpyDeviceToHost), "download");
    }
}

void capture_patch_graph(vxc_stream* s, int T, float cfg) {
    time_table(s, T);  // the graph reads the table; keep it current before every replay
    if (s->graph && s->graph_T == T && s->graph_cfg == cfg) return;
    if (s->graph) {
        cudaGraphExecDestroy(s->graph);
        s->graph = nullptr;
    }
    cudaGraph_t g = nullptr;
    ck(cudaStreamBeginCapture(s->cs, cudaStreamCaptureModeThreadLocal), "cudaStreamBeginCapture");
    try {
        enqueue_patch(s, T, cfg);
    } catch (...) {
        cudaStreamEndCapture(s->cs, &g);
        if (g) cudaGraphDestroy(g);
        throw;
    }
    ck(cudaStreamEndCapture(s->cs, &g), "cudaStreamEndCapture");
    size_t n_nodes = 0;
    ck(cudaGraphGetNodes(g, nullptr, &n_nodes), "cudaGraphGetNodes");
    std::vector<cudaGraphNode_t> nodes(n_nodes);
    if (n_nodes) ck(cudaGraphGetNodes(g, nodes.data(), &n_nodes), "cudaGraphGetNodes");
    int kernels = 0;
    for (cudaGraphNode_t nd : nodes) {
        cudaGraphNodeType t;
        ck(cudaGraphNodeGetType(nd, &t), "cudaGraphNodeGetType");
        if (t == cudaGraphNodeTypeKernel) ++kernels;
    }
    s->graph_kernels = kernels;
    const cudaError_t e = cudaGraphInstantiate(&s->graph, g, 0);
    cudaGraphDestroy(g);
    ck(e, "cudaGraphInstantiate");
    s->graph_T = T;
    s->graph_cfg = cfg;
}

void set_min_patches(vxc_stream* s, int min_patches) {
    if (s->min_patches_dev == min_patches) return;
    s->ctl_host->min_patches = min_patches;
    ck(cudaMemcpyAsync(&s->ctl->min_patches, &s->ctl_host->min_patches, sizeof(int), cudaMemcpyHostToDevice, s->cs),
       "min_patches");
    ck(cudaStreamSynchronize(s->cs), "sync");
    s->min_patches_dev = min_patches;
}

void check_patch_preconditions(vxc_stream* s, int T) {
    check_loaded(s->dev, {1, 2, 3, 4, 5, 6, 7, 8});
    if (!s->prefilled) throw InvalidState("vxc_prefill must run before patch steps");
    if (T <= 0) throw std::invalid_argument("inference timesteps must be positive");
    const vxc_model_desc& d = s->dev->desc;
    // synthesizer.cpp:542-544
    if (s->prefix_len + s->patches >= d.rope_original_max)
        throw std::runtime_error("VoxCPM2 KV cache reached the exported RoPE range");
    if (s->kv_len[0] + 1 > s->cap || s->kv_len[1] + 1 > s->cap || s->patches >= s->cap)
        throw std::invalid_argument("KV cache capacity exceeded: create the stream with a larger kv_capacity");
    sync_rope(s);  // factors set since the prefill apply from this patch on (every group member alike)
}

void patch_step(vxc_stream* s, const float* noise, int min_patches, float cfg, int T, float* out_latent,
                int* out_stop) {
    check_patch_preconditions(s, T);
    const int L = s->dev->desc.feat_dim * s->dev->desc.patch_size;
    if (noise) {
        std::memcpy(s->pin, noise, sizeof(float) * L);
        ck(cudaMemcpyAsync(s->noise + static_cast<size_t>(s->patches) * L, s->pin, sizeof(float) * L,
                           cudaMemcpyHostToDevice, s->cs),
           "noise upload");
    }
    set_min_patches(s, min_patches);
    capture_patch_graph(s, T, cfg);
    ck(cudaGraphLaunch(s->graph, s->cs), "cudaGraphLaunch");
    const int idx = s->patches;
    ck(cudaMemcpyAsync(s->pin + L, s->latents + static_cast<size_t>(idx) * L, sizeof(float) * L,
                       cudaMemcpyDeviceToHost, s->cs),
       "latent download");
    sync_ctl(s);
    if (out_latent) std::memcpy(out_latent, s->pin + L, sizeof(float) * L);
    if (out_stop) *out_stop = s->ctl_host->stopped;
}

// Pipelined driving: one patch step is queued (noise through a pinned slot, the patch
// graph, and copies of its latent and control block into pinned slots, then an event)
// without waiting; patch_collect waits for the oldest queued patch only. A host can
// keep the next patch queued while it handles the previous one, so the stream's GPU
// work never drains between patches; after a stop it discards the patch it queued
// speculatively.
void patch_submit(vxc_stream* s, const float* noise, int min_patches, float cfg, int T) {
    if (s->submitted - s->collected >= vxc_stream::kInflight)
        throw InvalidState("four patches are in flight: collect one before submitting another");
    check_patch_preconditions(s, T);
    require(noise != nullptr, "noise must not be null");
    const int L = s->dev->desc.feat_dim * s->dev->desc.patch_size;
    const int slot = static_cast<int>(s->submitted % vxc_stream::kInflight);
    float* pn = s->pin_noise + static_cast<size_t>(slot) * L;
    // the slot's previous copies finished before its patch was collected
    std::memcpy(pn, noise, sizeof(float) * L);
    ck(cudaMemcpyAsync(s->noise + static_cast<size_t>(s->patches) * L, pn, sizeof(float) * L, cudaMemcpyHostToDevice,
                       s->cs),
       "noise upload");
    set_min_patches(s, min_patches);
    capture_patch_graph(s, T, cfg);
    ck(cudaGraphLaunch(s->graph, s->cs), "cudaGraphLaunch");
    ck(cudaMemcpyAsync(s->pin_lat + static_cast<size_t>(slot) * L, s->latents + static_cast<size_t>(s->patches) * L,
                       sizeof(float) * L, cudaMemcpyDeviceToHost, s->cs),
       "latent download");
    ck(cudaMemcpyAsync(s->pin_ctl + slot, s->ctl, sizeof(StreamCtl), cudaMemcpyDeviceToHost, s->cs), "ctl download");
    ck(cudaEventRecord(s->patch_ev[slot], s->cs), "cudaEventRecord");
    s->submitted += 1;
    s->patches += 1;  // host mirrors advance optimistically; collect re-syncs them
    s->kv_len[0] += 1;
    s->kv_len[1] += 1;
}

void patch_collect(vxc_stream* s, float* out_latent, int* out_stop) {
    if (s->collected >= s->submitted) throw InvalidState("no patch in flight");
    const int L = s->dev->desc.feat_dim * s->dev->desc.patch_size;
    const int slot = static_cast<int>(s->collected % vxc_stream::kInflight);
    ck(cudaEventSynchronize(s->patch_ev[slot]), "cudaEventSynchronize");
    s->collected += 1;
    const StreamCtl& c = s->pin_ctl[slot];
    if (c.error != 0) {  // reports the device-side failure and clears it, like sync_ctl
        sync_ctl(s);
        throw std::runtime_error("device-side check failed");
    }
    if (out_latent) std::memcpy(out_latent, s->pin_lat + static_cast<size_t>(slot) * L, sizeof(float) * L);
    if (out_stop) *out_stop = c.stopped;
    if (s->collected == s->submitted) {  // nothing queued behind it: the snapshot is the stream's state
        s->kv_len[0] = c.kv_len[0];
        s->kv_len[1] = c.kv_len[1];
        s->patches = c.patch;
    }
}

// The prefix phase of generate_with_caches (synthesizer.cpp:403-535) for a prefix
// given row by row (PrefixRow, :43-47, built at :359-400): every row's token id is
// embedded by text_embed; an audio row's embedding is feat_encoder(its latent patch)
// instead, which is also the row's residual feature input (:415-443); the base
// decoder runs over all rows, and the LM hidden of audio rows is their FSQ output
// (:476-495); the residual decoder reads fusion_proj(lm, feat) (:497-522). The first
// patch is conditioned on the last row's latent when that row is audio, else on
// zeros (:444-447). audio_latents: the audio rows' patches in row order, d-major.
void prefill_rows(vxc_stream* s, const int32_t* ids_in, const int32_t* is_audio, const float* audio_latents, int L) {
    const vxc_device* dev = s->dev;
    const vxc_model_desc& d = dev->desc;
    require(ids_in != nullptr && L > 0, "the prefix must not be empty");
    sync_rope(s);
    std::vector<int> audio_rows;
    for (int i = 0; i < L; ++i)
        if (is_audio && is_audio[i]) audio_rows.push_back(i);
    check_loaded(dev, audio_rows.empty() ? std::initializer_list<int>{0, 1, 2, 4}
                                         : std::initializer_list<int>{0, 1, 2, 3, 4, 7});
    require(audio_rows.empty() || audio_latents != nullptr, "audio rows need their latent patches");
    require(L <= s->cap, "prompt longer than the KV capacity");
    require(L <= d.rope_original_max, "prompt longer than the RoPE range");
    for (int i = 0; i < L; ++i) require(ids_in[i] >= 0 && ids_in[i] < d.vocab, "token id out of range");
    const int H = d.hidden, latent = d.feat_dim * d.patch_size;
    const size_t A = audio_rows.size();
    ensure_prefill_rows(s, L);
    // new utterance: empty caches, zero counters (synthesizer.cpp:348-350)
    std::memset(s->ctl_host, 0, sizeof(StreamCtl));
    s->ctl_host->min_patches = s->min_patches_dev;
    write_ctl(s);
    s->kv_len[0] = s->kv_len[1] = 0;
    s->patches = 0;
    s->prefilled = false;
    s->submitted = s->collected = 0;  // write_ctl synchronised the stream: queued patches are dropped
    float* lat = nullptr;  // the audio rows' latents on the device (stream-ordered allocation)
    if (A) {
        ck(cudaMallocAsync(reinterpret_cast<void**>(&lat), sizeof(float) * latent * A, s->cs), "audio latents");
        ck(cudaMemcpyAsync(lat, audio_latents, sizeof(float) * latent * A, cudaMemcpyHostToDevice, s->cs), "latents");
    }
    try {
        ck(cudaMemcpyAsync(s->pids, ids_in, sizeof(int32_t) * L, cudaMemcpyHostToDevice, s->cs), "ids");
        launch_embed_gather(dev->blob[VXC_TEXT_EMBED], s->pids, L, H, d.embed_scale, s->ph, s->cs);
        // residual feature input: zeros, and feat_encoder(latent) on audio rows
        ck(cudaMemset2DAsync(s->pcat + H, sizeof(float) * 2 * H, 0, sizeof(float) * H, L, s->cs), "feat zeros");
        const __half* fe = dev->blob[VXC_FEAT_ENCODER];
        const size_t fin = static_cast<size_t>(H) * latent;
        for (size_t a = 0; a < A; ++a) {
            const size_t r = static_cast<size_t>(audio_rows[a]);
            GemvArgs fa = plain_gemv(fe, fe + fin, lat + a * latent, latent, H, s->mid2, ACT_SILU, nullptr, 0);
            fa.in_mode = IN_LATENT_T;
            fa.lat_d = d.feat_dim;
            fa.lat_p = d.patch_size;
            launch_gemv(fa, s->cs, false);
            GemvArgs fb = plain_gemv(fe + fin + H, fe + fin + H + static_cast<size_t>(H) * H, s->mid2, H, H,
                                     s->ph + r * H, ACT_NONE, nullptr, 0);
            fb.y2 = s->pcat + r * 2 * H + H;
            launch_gemv(fb, s->cs, false);
        }
        run_decoder_rows(s, 0, L, s->pxn);  // base_hidden -> pxn
        // the LM hidden of audio rows is their FSQ output
        const __half* fq = dev->blob[VXC_FSQ];
        const size_t Q = d.fsq_dim;
        for (size_t a = 0; a < A; ++a) {
            float* row = s->pxn + static_cast<size_t>(audio_rows[a]) * H;
            GemvArgs qa = plain_gemv(fq, fq + Q * H, row, H, static_cast<int>(Q), s->mid, ACT_FSQ, nullptr, 0);
            qa.act_scale = d.fsq_scale;
            launch_gemv(qa, s->cs, false);
            launch_gemv(plain_gemv(fq + Q * H + Q, fq + Q * H + Q + H * Q, s->mid, static_cast<int>(Q), H, row,
                                   ACT_NONE, nullptr, 0),
                        s->cs, false);
        }
        ck(cudaMemcpy2DAsync(s->pcat, sizeof(float) * 2 * H, s->pxn, sizeof(float) * H, sizeof(float) * H, L,
                             cudaMemcpyDeviceToDevice, s->cs),
           "concat");
        ck(cudaMemcpyAsync(s->lm_h, s->pxn + static_cast<size_t>(L - 1) * H, sizeof(float) * H,
                           cudaMemcpyDeviceToDevice, s->cs),
           "lm row");
        const __half* fu = dev->blob[VXC_FUSION_PROJ];
        RowsArgs fa;
        fa.w = fu;
        fa.bias = fu + static_cast<size_t>(H) * 2 * H;
        fa.x = s->pcat;
        fa.ldx = 2 * H;
        fa.K = 2 * H;
        fa.rows = H;
        fa.M = L;
        fa.y = s->ph;
        fa.ldy = H;
        launch_rows_linear(fa, s->cs, false);
        run_decoder_rows(s, 1, L, s->pxn);
        ck(cudaMemcpyAsync(s->res_h, s->pxn + static_cast<size_t>(L - 1) * H, sizeof(float) * H,
                           cudaMemcpyDeviceToDevice, s->cs),
           "res row");
        if (A && audio_rows.back() == L - 1)  // conditioned on the prompt's last patch
            ck(cudaMemcpyAsync(s->cond0, lat + (A - 1) * latent, sizeof(float) * latent, cudaMemcpyDeviceToDevice,
                               s->cs),
               "cond");
        else
            ck(cudaMemsetAsync(s->cond0, 0, sizeof(float) * latent, s->cs), "cond");
    } catch (...) {
        if (lat) cudaFreeAsync(lat, s->cs);
        throw;
    }
    if (lat) ck(cudaFreeAsync(lat, s->cs), "audio latents");
    sync_ctl(s);
    s->prefix_len = L;
    s->prefilled = true;
}

// A text-only prompt: prefix = text ids + audio_start (synthesizer.cpp:387-390).
void prefill(vxc_stream* s, const int32_t* text_ids, int n_text) {
    require(text_ids != nullptr && n_text > 0, "text must not be empty");
    std::vector<int32_t> ids(text_ids, text_ids + n_text);
    ids.push_back(s->dev->desc.audio_start_token);
    prefill_rows(s, ids.data(), nullptr, nullptr, static_cast<int>(ids.size()));
}

}  // namespace

vxc_stream::~vxc_stream() { free_all(this); }

// Error message slot shared with the other translation units of the library.
void vxc_internal_set_error(const char* msg) { g_last_error = msg; }

// ==================================================================== C ABI ==
// ------------------------------------------------------------- groups ----
// A group of up to 8 streams whose patch steps run as one CUDA graph: each
// member's decoder steps and small graphs on its own stream (forked branches),
// and the 9 estimator evaluations of all members batched into one pass over
// 22 rows per member, so every DiT weight byte is read once per group patch.
constexpr int kGroupMax = kWideTokens / 22;

struct vxc_group {
    vxc_device* dev = nullptr;
    std::vector<vxc_stream*> members;
    std::mutex call_mutex;
    float* gdh = nullptr;   // [22 n][Hd] residual stream of all members' DiT rows
    float* gqkv = nullptr;  // [22 n][(Hq + 2 Hkv) d]
    int lo = 0;  // the split operands' row block: 22 rows per member rounded up to 16
    __half *xw_n = nullptr, *xw_a = nullptr, *xw_act = nullptr;  // [2 lo][K] split operands
    CUtensorMap map_xw_n{}, map_xw_a{}, map_xw_act{};
    int tc_target = 32;              // CTAs aimed at per wide linear: group_tc_target(), or a fixed
                                     // VXC_GROUP_TC_TARGET
    bool target_fixed = false;       // VXC_GROUP_TC_TARGET was given
    int graph_target = -1;           // the target the captured graph was built with
    int tc_stages = 2;               // TMA ring depth of the wide linears (VXC_GROUP_TC_STAGES)
    bool recv_shared = true;         // split wide linears receive in their stage area (VXC_GROUP_RECV_SHARED=0: not)
    bool bulk_gemv = false;          // decoder GEMVs: register-streaming batch form (0, the faster), or
                                     // bulk-copy (VXC_GROUP_BULK_GEMV=1)
    StreamCtl* gctl = nullptr;       // error reports of the batched linears
    StreamCtl* gctl_host = nullptr;
    std::vector<cudaEvent_t> events;  // fork / join points of the group graph
    cudaGraphExec_t graph = nullptr;
    int graph_T = -1;
    float graph_cfg = 0.f;
    int graph_kernels = 0;
    ~vxc_group();
};

namespace {

// One decoder step (base: which 0, residual: 1) of every member at once
// (base_decoder_kv / residual_decoder_kv, tools/export_components.py:496-550):
// each linear reads its weights once for all members (member-batched GEMV), the
// attention runs one cluster per (member, KV head) over the member's own cache,
// and every member keeps its own KV length and stop flag.
void enqueue_group_decoder_step(vxc_group* g, int which) {
    vxc_stream* s0 = g->members[0];
    const vxc_device* dev = g->dev;
    const vxc_model_desc& d = dev->desc;
    const std::vector<LayerW>& layers = which == 0 ? dev->base : dev->res;
    const __half* fnorm = which == 0 ? dev->base_norm : dev->res_norm;
    const float rscale = which == 0 ? d.base_residual_scale : d.res_residual_scale;
    const int H = d.hidden, F = d.ffn, hq = d.q_heads, hkv = d.kv_heads, hd = d.head_dim;
    const int n = static_cast<int>(g->members.size());
    cudaStream_t cs = s0->cs;
    const bool pdl = s0->pdl;
    auto gemv = g->bulk_gemv ? launch_gemv_bulk_batch : launch_gemv_batch;
    for (size_t l = 0; l < layers.size(); ++l) {
        const LayerW& L = layers[l];
        GemvBatch qb, ob, gb, db;
        AttnBatch ab;
        qb.n = ob.n = gb.n = db.n = ab.n = n;
        for (int m = 0; m < n; ++m) {
            vxc_stream* s = g->members[static_cast<size_t>(m)];
            const size_t plane = static_cast<size_t>(hkv) * s->cap * hd;
            qb.x[m] = s->h[which];
            qb.y[m] = s->q;
            qb.k_cache[m] = s->kc[which] + l * plane;
            qb.v_cache[m] = s->vc[which] + l * plane;
            qb.ctl[m] = s->ctl;
            ab.q[m] = s->q;
            ab.k0[m] = s->kc[which] + l * plane;
            ab.v0[m] = s->vc[which] + l * plane;
            ab.out[m] = s->attn;
            ab.ctl[m] = s->ctl;
            ob.x[m] = s->attn;
            ob.resid[m] = s->h[which];
            ob.ctl[m] = s->ctl;
            gb.x[m] = s->h[which];
            gb.y[m] = s->act;
            gb.ctl[m] = s->ctl;
            db.x[m] = s->act;
            db.resid[m] = s->h[which];
            db.ctl[m] = s->ctl;
        }
        GemvArgs qa;
        qa.mode = GEMV_QKV;
        qa.w = L.wqkv;
        qa.norm_g = L.in_norm;
        qa.eps = d.rms_eps;
        qa.K = H;
        qa.rows = (hq + 2 * hkv) * hd / 2;
        qa.q_heads = hq;
        qa.kv_heads = hkv;
        qa.head_dim = hd;
        if (which == 0) set_decode_rope(qa, s0);  // the members share a capacity and the device's factors
        qa.cap = s0->cap;
        qa.which = which;
        qa.skip_if_stopped = 1;
        gemv(qa, qb, cs, pdl);

        AttnArgs aa;
        aa.k0 = ab.k0[0];
        aa.v0 = ab.v0[0];
        aa.len0 = s0->cap;
        aa.stride0 = s0->cap;
        aa.q_heads = hq;
        aa.kv_heads = hkv;
        aa.head_dim = hd;
        aa.scale = 1.0f / std::sqrt(static_cast<float>(hd));
        aa.ctl = s0->ctl;
        aa.which = which;
        aa.skip_if_stopped = 1;
        launch_attn_decode_cluster_batch(aa, ab, cs, pdl);

        GemvArgs oa;
        oa.mode = GEMV_RESID;
        oa.w = L.wo;
        oa.K = hq * hd;
        oa.rows = H;
        oa.rscale = rscale;
        oa.skip_if_stopped = 1;
        gemv(oa, ob, cs, pdl);

        GemvArgs ga;
        ga.mode = GEMV_GATEUP;
        ga.w = L.wgateup;
        ga.norm_g = L.post_norm;
        ga.eps = d.rms_eps;
        ga.K = H;
        ga.rows = F;
        ga.skip_if_stopped = 1;
        gemv(ga, gb, cs, pdl);

        GemvArgs da;
        da.mode = GEMV_RESID;
        da.w = L.wdown;
        da.K = F;
        da.rows = H;
        da.rscale = rscale;
        da.skip_if_stopped = 1;
        gemv(da, db, cs, pdl);
    }
    for (vxc_stream* s : g->members)
        launch_final_norm(s->h[which], fnorm, d.rms_eps, H, which == 0 ? s->out[0] : s->res_h, nullptr, s->ctl, which,
                          1, 1, cs, pdl);
}

// The estimator layers over all members' rows (the split form: RMSNorm and
// attention kernels around four wide tensor-core linears).
void enqueue_group_layers(vxc_group* g) {
    vxc_stream* s0 = g->members[0];
    const vxc_device* dev = g->dev;
    const vxc_model_desc& d = dev->desc;
    const int n = static_cast<int>(g->members.size());
    const int Hd = d.dit_hidden, F = d.dit_ffn, hq = d.dit_q_heads, hkv = d.dit_kv_heads, hd = Hd / hq;
    const int seq = dit_tokens_per_seq(d.patch_size), M = 2 * seq * n;
    const int W = (hq + 2 * hkv) * hd;
    const float scale = 1.0f / std::sqrt(static_cast<float>(hd));
    cudaStream_t cs = s0->cs;
    const bool pdl = s0->pdl;
    auto plan = [&](int tiles, int K) {
        TcWideArgs a;
        a.splits = pow2_floor(choose_splits(tiles, K, g->tc_target));
        a.stages = g->tc_stages;
        a.M = M;
        a.lo = g->lo;
        a.K = K;
        a.ctl = g->gctl;
        a.recv_shared = g->recv_shared ? 1 : 0;
        return a;
    };
    for (size_t l = 0; l < dev->dit.size(); ++l) {
        const LayerW& L = dev->dit[l];
        const std::array<CUtensorMap, 4>& maps = dev->dit_maps[l];
        launch_rmsnorm_rows_split(g->gdh, Hd, L.in_norm, d.rms_eps, Hd, M, g->xw_n, nullptr, cs, pdl, g->lo);
        TcWideArgs qa = plan(W / 128, Hd);
        qa.rows = W;
        qa.y = g->gqkv;
        qa.ldy = W;
        launch_tc_wide(maps[0], g->map_xw_n, qa, cs, pdl);
        launch_dit_attention_split(g->gqkv, 2 * n, seq, hq, hkv, hd, dev->dit_rope_cos, dev->dit_rope_sin, scale,
                                   g->xw_a, nullptr, cs, pdl, g->lo);
        TcWideArgs oa = plan(Hd / 128, hq * hd);
        oa.rows = Hd;
        oa.resid = 1;
        oa.rscale = d.dit_residual_scale;
        oa.y = g->gdh;
        oa.ldy = Hd;
        launch_tc_wide(maps[1], g->map_xw_a, oa, cs, pdl);
        launch_rmsnorm_rows_split(g->gdh, Hd, L.post_norm, d.rms_eps, Hd, M, g->xw_n, nullptr, cs, pdl, g->lo);
        TcWideArgs ga = plan(F / 64, Hd);
        ga.rows = F;
        ga.gateup = 1;
        ga.yb = g->xw_act;
        ga.ldyb = F;
        launch_tc_wide(maps[2], g->map_xw_n, ga, cs, pdl);
        TcWideArgs da = plan(Hd / 128, F);
        da.rows = Hd;
        da.resid = 1;
        da.rscale = d.dit_residual_scale;
        da.y = g->gdh;
        da.ldy = Hd;
        launch_tc_wide(maps[3], g->map_xw_act, da, cs, pdl);
    }
}

// cfm_sample of every member at once (synthesizer.cpp:86-170): per step, each
// member's input rows, the batched layers, then each member's output projection
// with its own CFG-zero* scale and Euler update. Members whose stop flag is set
// skip their embed and update.
void enqueue_group_cfm(vxc_group* g, int T, float cfg) {
    vxc_stream* s0 = g->members[0];
    const vxc_device* dev = g->dev;
    const vxc_model_desc& d = dev->desc;
    const int Hd = d.dit_hidden, seq = dit_tokens_per_seq(d.patch_size);
    const std::vector<float> dts = euler_dts(T);
    const int z = zero_init_steps(T);
    const float* tab = s0->ttab.at(T).dev;
    const DitPtrs w = dit_ptrs(dev);
    for (int step = 1; step <= T; ++step) {
        if (step <= z) continue;  // zero-init steps leave x untouched (synthesizer.cpp:123-126)
        const int n = static_cast<int>(g->members.size());
        const size_t stride = 2 * seq * static_cast<size_t>(Hd);
        DitEmbedArgs e{};
        e.in_w = w.in_w;
        e.in_b = w.in_b;
        e.cond_w = w.cond_w;
        e.cond_b = w.cond_b;
        e.Hd = Hd;
        e.D = d.feat_dim;
        e.P = d.patch_size;
        e.hidden = g->gdh;
        e.tsum = tab + static_cast<size_t>(step) * Hd;
        e.members = n;
        e.member_stride = stride;
        for (int m = 0; m < n; ++m) {
            vxc_stream* s = g->members[static_cast<size_t>(m)];
            e.mx[m] = s->x;
            e.mcond[m] = s->cond;
            e.mmu[m] = s->mu;
            e.mctl[m] = s->ctl;
        }
        e.x = e.mx[0];
        e.cond = e.mcond[0];
        e.mu = e.mmu[0];
        launch_dit_embed(e, s0->cs, s0->pdl);
        enqueue_group_layers(g);
        DitOutArgs o{};
        o.hidden = g->gdh;
        o.seq = seq;
        o.Hd = Hd;
        o.D = d.feat_dim;
        o.P = d.patch_size;
        o.norm_g = dev->dit_norm;
        o.eps = d.rms_eps;
        o.out_w = w.out_w;
        o.out_b = w.out_b;
        o.dt = dts[step];
        o.cfg = cfg;
        o.members = n;
        o.member_stride = stride;
        for (int m = 0; m < n; ++m) {
            vxc_stream* s = g->members[static_cast<size_t>(m)];
            o.mx[m] = s->x;
            o.mctl[m] = s->ctl;
            o.mest[m] = s->dest;
            o.mcounter[m] = s->dcount;
        }
        o.x = o.mx[0];
        o.est_buf = o.mest[0];
        o.counter = o.mcounter[0];
        launch_dit_out(o, s0->cs, s0->pdl);
    }
}

// The members' streams join the capture on members[0]'s stream (fork) and it
// waits for all of them (join); 'k' indexes the event pair used.
void group_fork(vxc_group* g, int k) {
    const int n = static_cast<int>(g->members.size());
    cudaEvent_t ev = g->events[static_cast<size_t>(k) * (n + 1)];
    ck(cudaEventRecord(ev, g->members[0]->cs), "fork");
    for (int m = 1; m < n; ++m) ck(cudaStreamWaitEvent(g->members[m]->cs, ev, 0), "fork");
}
void group_join(vxc_group* g, int k) {
    const int n = static_cast<int>(g->members.size());
    for (int m = 1; m < n; ++m) {
        cudaEvent_t ev = g->events[static_cast<size_t>(k) * (n + 1) + m];
        ck(cudaEventRecord(ev, g->members[m]->cs), "join");
        ck(cudaStreamWaitEvent(g->members[0]->cs, ev, 0), "join");
    }
}

// CTAs per wide linear for a group: 256 over the device's groups, clamped to 16..32.
// For the benchmark model that splits the o and down projections 4 ways up to 9 groups
// and 2 ways from 10, so many groups do not crowd each other's CTAs off the SMs and a
// few keep their latency. Measured per device (patches/s): 12 x 4 streams 2096-2112 at
// 32 and 2136-2177 at 16 (1881 at 8); 12 x 8 1969 at 32 and 2133-2147 at 16; 8 x 4 1931
// at 32 and 1883-1892 at 16-24; 4 x 4 1334 at 32 and 1200 at 16.
int group_tc_target(const vxc_group* g) {
    if (g->target_fixed) return g->tc_target;
    const int n = std::max(1, g->dev->live_groups.load());
    return std::max(16, std::min(32, 256 / n));
}

void capture_group_graph(vxc_group* g, int T, float cfg) {
    time_table(g->members[0], T);  // the graph reads it; keep it current before every replay
    const int target = group_tc_target(g);
    if (g->graph && g->graph_T == T && g->graph_cfg == cfg && g->graph_target == target) return;
    g->tc_target = target;
    if (g->graph) {
        // a patch of the old graph may still run (the target changes when another group
        // is created or destroyed between this group's asynchronous patches)
        ck(cudaStreamSynchronize(g->members[0]->cs), "cudaStreamSynchronize");
        cudaGraphExecDestroy(g->graph);
        g->graph = nullptr;
    }
    cudaStream_t c0 = g->members[0]->cs;
    cudaGraph_t gr = nullptr;
    ck(cudaStreamBeginCapture(c0, cudaStreamCaptureModeThreadLocal), "cudaStreamBeginCapture");
    try {
        // per-member small graphs on forked branches, the heavy passes batched on members[0]'s stream
        group_fork(g, 0);
        for (vxc_stream* s : g->members) enqueue_patch_pre(s);
        group_join(g, 0);
        enqueue_group_cfm(g, T, cfg);
        group_fork(g, 1);
        for (vxc_stream* s : g->members) enqueue_post_stop_feat(s);
        group_join(g, 1);
        enqueue_group_decoder_step(g, 0);
        group_fork(g, 2);
        for (vxc_stream* s : g->members) enqueue_post_fsq_fusion(s);
        group_join(g, 2);
        enqueue_group_decoder_step(g, 1);
        for (vxc_stream* s : g->members) enqueue_post_end(s, g->members[0]->cs);
    } catch (...) {
        cudaStreamEndCapture(c0, &gr);
        if (gr) cudaGraphDestroy(gr);
        throw;
    }
    ck(cudaStreamEndCapture(c0, &gr), "cudaStreamEndCapture");
    size_t n_nodes = 0;
    ck(cudaGraphGetNodes(gr, nullptr, &n_nodes), "cudaGraphGetNodes");
    std::vector<cudaGraphNode_t> nodes(n_nodes);
    if (n_nodes) ck(cudaGraphGetNodes(gr, nodes.data(), &n_nodes), "cudaGraphGetNodes");
    int kernels = 0;
    for (cudaGraphNode_t nd : nodes) {
        cudaGraphNodeType t;
        ck(cudaGraphNodeGetType(nd, &t), "cudaGraphNodeGetType");
        if (t == cudaGraphNodeTypeKernel) ++kernels;
    }
    g->graph_kernels = kernels;
    const cudaError_t e = cudaGraphInstantiate(&g->graph, gr, 0);
    cudaGraphDestroy(gr);
    ck(e, "cudaGraphInstantiate");
    g->graph_T = T;
    g->graph_cfg = cfg;
    g->graph_target = target;
}

void free_group(vxc_group* g) {
    if (g->graph) cudaGraphExecDestroy(g->graph);
    g->graph = nullptr;
    for (cudaEvent_t e : g->events)
        if (e) cudaEventDestroy(e);
    g->events.clear();
    for (void* p : {static_cast<void*>(g->gdh), static_cast<void*>(g->gqkv), static_cast<void*>(g->xw_n),
                    static_cast<void*>(g->xw_a), static_cast<void*>(g->xw_act), static_cast<void*>(g->gctl)})
        if (p) cudaFree(p);
    if (g->gctl_host) cudaFreeHost(g->gctl_host);
    g->gdh = g->gqkv = nullptr;
    g->xw_n = g->xw_a = g->xw_act = nullptr;
    g->gctl = nullptr;
    g->gctl_host = nullptr;
}

}  // namespace

vxc_group::~vxc_group() = default;

extern "C" {

VXC_API uint32_t vxc_abi_version(void) { return VXC_ABI_VERSION; }

VXC_API const char* vxc_last_error(void) { return g_last_error.c_str(); }

VXC_API size_t vxc_component_weight_count(const vxc_model_desc* desc, int32_t component) {
    return desc ? component_count(*desc, component) : 0;
}

VXC_API int32_t vxc_device_create(int32_t device, const vxc_model_desc* desc, vxc_device** out) {
    return guard([&] {
        require(desc != nullptr && out != nullptr, "desc and out must not be null");
        *out = nullptr;
        validate_desc(*desc);
        int n = 0;
        ck(cudaGetDeviceCount(&n), "cudaGetDeviceCount");
        require(device >= 0 && device < n, "CUDA device index out of range");
        cudaDeviceProp prop{};
        ck(cudaGetDeviceProperties(&prop, device), "cudaGetDeviceProperties");
        if (prop.major != 10) throw std::runtime_error("libvoxcpm2_cuda is built for sm_100a (B200) devices only");
        DeviceGuard g(device);
        init_kernel_attributes();
        auto dev = std::make_unique<vxc_device>();
        dev->device = device;
        dev->desc = *desc;
        const int seq = dit_tokens_per_seq(desc->patch_size);
        std::vector<float> c, s;
        rope_table(64, desc->rope_theta, seq, c, s);
        dev->dit_rope_cos = dev_alloc<float>(c.size());
        dev->dit_rope_sin = dev_alloc<float>(s.size());
        ck(cudaMemcpy(dev->dit_rope_cos, c.data(), sizeof(float) * c.size(), cudaMemcpyHostToDevice), "rope");
        ck(cudaMemcpy(dev->dit_rope_sin, s.data(), sizeof(float) * s.size(), cudaMemcpyHostToDevice), "rope");
        const std::vector<float> f = timestep_frequencies(desc->dit_hidden / 2, 10000.0f);
        dev->temb_freq = dev_alloc<float>(f.size());
        ck(cudaMemcpy(dev->temb_freq, f.data(), sizeof(float) * f.size(), cudaMemcpyHostToDevice), "frequencies");
        *out = dev.release();
    });
}

VXC_API void vxc_device_destroy(vxc_device* dev) {
    if (!dev) return;
    {
        DeviceGuard g(dev->device, true);  // teardown never throws (also at process exit)
        for (__half* p : dev->blob)
            if (p) cudaFree(p);
        if (dev->dit_rope_cos) cudaFree(dev->dit_rope_cos);
        if (dev->dit_rope_sin) cudaFree(dev->dit_rope_sin);
        if (dev->temb_freq) cudaFree(dev->temb_freq);
    }
    delete dev;
}

VXC_API int32_t vxc_load_weights(vxc_device* dev, int32_t component, const void* fp16, size_t count) {
    return guard([&] {
        require(dev != nullptr && fp16 != nullptr, "device and weights must not be null");
        require(component >= 0 && component <= 8, "unknown component id");
        require(count == component_count(dev->desc, component), "weight count does not match the model description");
        DeviceGuard g(dev->device);
        if (!dev->blob[component]) dev->blob[component] = dev_alloc<__half>(count);
        ck(cudaMemcpy(dev->blob[component], fp16, count * sizeof(__half), cudaMemcpyHostToDevice), "weights upload");
        dev->loaded[component] = true;
        ++dev->epoch;
        const __half* fn = nullptr;
        if (component == VXC_BASE_DECODER) {
            dev->base = carve_decoder(dev->blob[component], base_shape(dev->desc), &fn);
            dev->base_norm = fn;
            dev->base_maps = decoder_maps(dev->desc, dev->base);
        } else if (component == VXC_RESIDUAL_DECODER) {
            dev->res = carve_decoder(dev->blob[component], res_shape(dev->desc), &fn);
            dev->res_norm = fn;
            dev->res_maps = decoder_maps(dev->desc, dev->res);
        } else if (component == VXC_DIT_ESTIMATOR) {
            const size_t Hd = dev->desc.dit_hidden, D = dev->desc.feat_dim;
            const __half* base = dev->blob[component] + 2 * (Hd * D + Hd) + 4 * (Hd * Hd + Hd);
            dev->dit = carve_decoder(base, dit_shape(dev->desc), &fn);
            dev->dit_norm = fn;
            const int dh = dev->desc.dit_hidden, df = dev->desc.dit_ffn;
            const int W = (dev->desc.dit_q_heads + 2 * dev->desc.dit_kv_heads) * 64;
            dev->dit_maps.clear();
            for (const LayerW& L : dev->dit)
                dev->dit_maps.push_back({make_tensor_map_f16(L.wqkv, W, dh, 64), make_tensor_map_f16(L.wo, dh, dh, 64),
                                         make_tensor_map_f16(L.wgateup, 2 * df, dh, 64),
                                         make_tensor_map_f16(L.wdown, dh, df, 64)});
        }
    });
}

VXC_API int32_t vxc_set_rope_factors(vxc_device* dev, const float* short_factor, const float* long_factor,
                                     int32_t n) {
    return guard([&] {
        require(dev != nullptr && short_factor != nullptr, "device and short_factor must not be null");
        // make_rope_cache reads the first head_dim / 2 entries and rejects shorter tables
        // (synthesizer.cpp:949-951)
        const int half = dev->desc.head_dim / 2;
        require(n >= half, "VoxCPM2 rope tables are missing or too short");
        for (int j = 0; j < half; ++j)
            require(short_factor[j] > 0.f && (!long_factor || long_factor[j] > 0.f), "rope factors must be positive");
        std::lock_guard<std::mutex> lk(dev->rope_mu);
        dev->rope_short.assign(short_factor, short_factor + half);
        if (long_factor) dev->rope_long.assign(long_factor, long_factor + half);
        else dev->rope_long.clear();
        ++dev->rope_epoch;
    });
}

VXC_API int32_t vxc_stream_create(vxc_device* dev, int32_t kv_capacity, vxc_stream** out) {
    return guard([&] {
        require(dev != nullptr && out != nullptr, "device and out must not be null");
        *out = nullptr;
        require(kv_capacity > 1 && kv_capacity <= 32768, "kv_capacity must be in [2, 32768]");
        DeviceGuard g(dev->device);
        const vxc_model_desc& d = dev->desc;
        auto s = std::make_unique<vxc_stream>();
        s->dev = dev;
        s->cap = kv_capacity;
        s->splits = std::min(32, std::max(4, (kv_capacity + 31) / 32));
        ck(cudaStreamCreateWithFlags(&s->cs, cudaStreamNonBlocking), "cudaStreamCreate");
        s->ctl = dev_alloc<StreamCtl>(1);
        ck(cudaMallocHost(&s->ctl_host, sizeof(StreamCtl)), "cudaMallocHost");
        std::memset(s->ctl_host, 0, sizeof(StreamCtl));
        ck(cudaMemset(s->ctl, 0, sizeof(StreamCtl)), "ctl");
        const size_t H = d.hidden, F = d.ffn, hd = d.head_dim, hq = d.q_heads, hkv = d.kv_heads;
        const int layers[2] = {d.base_layers, d.res_layers};
        for (int w = 0; w < 2; ++w) {
            const size_t n = static_cast<size_t>(layers[w]) * hkv * kv_capacity * hd;
            s->kc[w] = dev_alloc<float>(n);
            s->vc[w] = dev_alloc<float>(n);
            ck(cudaMemset(s->kc[w], 0, n * sizeof(float)), "cache");
            ck(cudaMemset(s->vc[w], 0, n * sizeof(float)), "cache");
            s->h[w] = dev_alloc<float>(H);
            s->out[w] = dev_alloc<float>(H);
        }
        const size_t rope_n = static_cast<size_t>(kv_capacity) * hd;
        s->rope_cos = dev_alloc<float>(rope_n);
        s->rope_sin = dev_alloc<float>(rope_n);
        s->rope_cos_l = dev_alloc<float>(rope_n);
        s->rope_sin_l = dev_alloc<float>(rope_n);
        sync_rope(s.get());
        s->q = dev_alloc<float>(hq * hd);
        s->attn = dev_alloc<float>(hq * hd);
        s->act = dev_alloc<float>(F);
        s->lm_h = dev_alloc<float>(H);
        s->res_h = dev_alloc<float>(H);
        s->feat = dev_alloc<float>(H);
        s->mid = dev_alloc<float>(std::max<size_t>(H, d.fsq_dim));
        s->mid2 = dev_alloc<float>(H);
        const size_t G = hq / hkv;
        s->partial = dev_alloc<float>(hkv * s->splits * G * (hd + 2));
        s->counters = dev_alloc<int>(hkv);
        ck(cudaMemset(s->counters, 0, sizeof(int) * hkv), "counters");
        const size_t Hd = d.dit_hidden, L = static_cast<size_t>(d.feat_dim) * d.patch_size;
        const size_t M = 2 * static_cast<size_t>(dit_tokens_per_seq(d.patch_size));
        const size_t Wd = static_cast<size_t>(d.dit_q_heads + 2 * d.dit_kv_heads) * (Hd / d.dit_q_heads);
        s->mu = dev_alloc<float>(2 * Hd);
        s->x = dev_alloc<float>(L);
        s->cond = dev_alloc<float>(L);
        s->cond0 = dev_alloc<float>(L);
        ck(cudaMemset(s->cond0, 0, sizeof(float) * L), "cond");
        s->noise = dev_alloc<float>(static_cast<size_t>(kv_capacity) * L);
        ck(cudaMemset(s->noise, 0, sizeof(float) * kv_capacity * L), "noise");
        s->latents = dev_alloc<float>(static_cast<size_t>(kv_capacity) * L);
        for (float** p : {&s->temb, &s->tmid, &s->ttok, &s->dtemb, &s->dtmid, &s->dttok, &s->dtemb1, &s->dtmid1,
                          &s->dttok1})
            *p = dev_alloc<float>(Hd);
        s->dh = dev_alloc<float>(M * Hd);
        s->dxn = dev_alloc<float>(M * Hd);
        s->dqkv = dev_alloc<float>(M * Wd);
        s->dattn = dev_alloc<float>(M * Hd);
        s->dact = dev_alloc<float>(M * d.dit_ffn);
        s->est = dev_alloc<float>(2 * L);
        s->dest = dev_alloc<float>(2 * L);
        s->dcount = dev_alloc<int>(1);
        ck(cudaMemset(s->dcount, 0, sizeof(int)), "cudaMemset");
        if (const char* np = std::getenv("VXC_NO_PDL")) s->pdl = std::string(np) != "1";
        if (const char* nk = std::getenv("VXC_NORM_KERNELS")) s->norm_kernels = std::string(nk) == "1";
        if (const char* rs = std::getenv("VXC_RECV_SHARED")) s->recv_shared = std::string(rs) == "1";
        if (const char* bg = std::getenv("VXC_BULK_GEMV")) s->bulk_gemv = std::string(bg) == "1";
        if (const char* tt = std::getenv("VXC_TC_TARGET")) {
            s->tc_target = std::atoi(tt);
            if (s->tc_target < 1 || s->tc_target > 4096) throw std::invalid_argument("VXC_TC_TARGET must be in [1, 4096]");
        }
        if (const char* st = std::getenv("VXC_TC_STAGES")) {
            s->tc_stages = std::atoi(st);
            if (s->tc_stages < 1 || s->tc_stages > 8) throw std::invalid_argument("VXC_TC_STAGES must be in [1, 8]");
        }
        // row sums of squares of dh, by slice: the embedding's Hd / 32 parts or a residual
        // epilogue's (Hd / 128 tiles) x (K split <= 16) parts
        const size_t ssq_n = static_cast<size_t>(Hd / 8 + Hd / 32 + 1) * kSsqStride;
        s->dssq = dev_alloc<float>(ssq_n);
        ck(cudaMemset(s->dssq, 0, ssq_n * sizeof(float)), "cudaMemset");
        for (__half** xb : {&s->xb_n, &s->xb_a, &s->xb_act}) {
            const size_t k = xb == &s->xb_act ? d.dit_ffn : Hd;
            *xb = dev_alloc<__half>(48 * k);
            ck(cudaMemset(*xb, 0, 48 * k * sizeof(__half)), "operand");  // pad rows stay zero
        }
        s->map_xb_n = make_tensor_map_f16(s->xb_n, 48, static_cast<int>(Hd), 48);
        s->map_xb_a = make_tensor_map_f16(s->xb_a, 48, static_cast<int>(Hd), 48);
        s->map_xb_act = make_tensor_map_f16(s->xb_act, 48, d.dit_ffn, 48);
        s->gen_in = dev_alloc<float>(std::max(8 * Hd + 8 * L, 4 * H));
        ck(cudaMallocHost(&s->pin, sizeof(float) * (4 * std::max<size_t>(L, 2 * Hd) + 4 * H)), "cudaMallocHost");
        ck(cudaMallocHost(&s->pin_noise, sizeof(float) * L * vxc_stream::kInflight), "cudaMallocHost");
        ck(cudaMallocHost(&s->pin_lat, sizeof(float) * L * vxc_stream::kInflight), "cudaMallocHost");
        ck(cudaMallocHost(&s->pin_ctl, sizeof(StreamCtl) * vxc_stream::kInflight), "cudaMallocHost");
        for (cudaEvent_t& e : s->patch_ev) ck(cudaEventCreateWithFlags(&e, cudaEventDisableTiming), "cudaEventCreate");
        *out = s.release();
    });
}

VXC_API void vxc_stream_destroy(vxc_stream* s) {
    if (!s) return;
    s->cancel.store(true);
    {
        std::lock_guard<std::mutex> lk(s->call_mutex);  // wait for an active call to leave
        DeviceGuard g(s->dev->device, true);
        cudaStreamSynchronize(s->cs);
    }
    DeviceGuard g(s->dev->device, true);  // teardown never throws (also at process exit)
    delete s;
}

VXC_API void vxc_stream_cancel(vxc_stream* s) {
    if (s) s->cancel.store(true, std::memory_order_release);
}

VXC_API int32_t vxc_stream_set_plan(vxc_stream* s, int32_t plan) {
    return guard([&] {
        require(s != nullptr, "stream must not be null");
        require(plan == VXC_PLAN_THROUGHPUT || plan == VXC_PLAN_LATENCY, "plan must be VXC_PLAN_THROUGHPUT or VXC_PLAN_LATENCY");
        std::lock_guard<std::mutex> lk(s->call_mutex);
        if (s->submitted != s->collected) throw InvalidState("collect the submitted patches before changing the plan");
        DeviceGuard g(s->dev->device);
        ck(cudaStreamSynchronize(s->cs), "cudaStreamSynchronize");
        s->tc_target = plan == VXC_PLAN_LATENCY ? 296 : 32;
        s->tc_stages = plan == VXC_PLAN_LATENCY ? 3 : 2;
        if (s->graph) cudaGraphExecDestroy(s->graph);
        s->graph = nullptr;  // the next patch captures its graph with the new plan
    });
}

VXC_API int32_t vxc_stream_reset(vxc_stream* s) {
    return guard([&] {
        require(s != nullptr, "stream must not be null");
        std::lock_guard<std::mutex> lk(s->call_mutex);
        DeviceGuard g(s->dev->device);
        std::memset(s->ctl_host, 0, sizeof(StreamCtl));
        s->ctl_host->min_patches = s->min_patches_dev;
        write_ctl(s);
        s->kv_len[0] = s->kv_len[1] = 0;
        s->patches = 0;
        s->prefilled = false;
        s->submitted = s->collected = 0;
    });
}

VXC_API int32_t vxc_token_count(vxc_stream* s, int32_t which, int32_t* out) {
    return guard([&] {
        require(s != nullptr && out != nullptr && (which == 0 || which == 1), "bad arguments");
        std::lock_guard<std::mutex> lk(s->call_mutex);
        DeviceGuard g(s->dev->device);
        sync_ctl(s);
        *out = s->kv_len[which];
    });
}

VXC_API int32_t vxc_read_cache(vxc_stream* s, int32_t which, int32_t layer, float* k, float* v) {
    return guard([&] {
        require(s != nullptr && k != nullptr && v != nullptr && (which == 0 || which == 1), "bad arguments");
        std::lock_guard<std::mutex> lk(s->call_mutex);
        const vxc_model_desc& d = s->dev->desc;
        const int layers = which == 0 ? d.base_layers : d.res_layers;
        require(layer >= 0 && layer < layers, "decoder kv layer index out of range");
        DeviceGuard g(s->dev->device);
        sync_ctl(s);
        const int T = s->kv_len[which], hd = d.head_dim, hkv = d.kv_heads;
        std::vector<float> hk(static_cast<size_t>(hkv) * s->cap * hd), hv(hk.size());
        const size_t plane = hk.size();
        ck(cudaMemcpy(hk.data(), s->kc[which] + layer * plane, plane * sizeof(float), cudaMemcpyDeviceToHost), "k");
        ck(cudaMemcpy(hv.data(), s->vc[which] + layer * plane, plane * sizeof(float), cudaMemcpyDeviceToHost), "v");
        for (int h = 0; h < hkv; ++h)
            for (int t = 0; t < T; ++t)
                for (int e = 0; e < hd; ++e) {
                    const size_t src = (static_cast<size_t>(h) * s->cap + t) * hd + e;
                    const size_t dst = (static_cast<size_t>(h) * T + t) * hd + e;
                    k[dst] = hk[src];
                    v[dst] = hv[src];
                }
    });
}

VXC_API int32_t vxc_decoder_step(vxc_stream* s, int32_t which, const float* embed, int32_t n, float* out) {
    return guard([&] {
        require(s != nullptr && embed != nullptr && out != nullptr, "null argument");
        require(which == 0 || which == 1, "which must be VXC_BASE or VXC_RESIDUAL");
        require(n > 0, "invalid decoder attention mask shape");
        std::lock_guard<std::mutex> lk(s->call_mutex);
        DeviceGuard g(s->dev->device);
        sync_rope(s);
        decoder_call(s, which, embed, n, out);
    });
}

VXC_API int32_t vxc_text_embed(vxc_stream* s, const int32_t* ids, int32_t n, float* out) {
    return guard([&] {
        require(s != nullptr && ids != nullptr && out != nullptr && n > 0, "bad arguments");
        std::lock_guard<std::mutex> lk(s->call_mutex);
        const vxc_model_desc& d = s->dev->desc;
        check_loaded(s->dev, {VXC_TEXT_EMBED});
        for (int i = 0; i < n; ++i) require(ids[i] >= 0 && ids[i] < d.vocab, "token id out of range");
        DeviceGuard g(s->dev->device);
        ensure_prefill_rows(s, n);
        ck(cudaMemcpyAsync(s->pids, ids, sizeof(int32_t) * n, cudaMemcpyHostToDevice, s->cs), "ids");
        launch_embed_gather(s->dev->blob[VXC_TEXT_EMBED], s->pids, n, d.hidden, d.embed_scale, s->pxn, s->cs);
        ck(cudaMemcpyAsync(out, s->pxn, sizeof(float) * n * d.hidden, cudaMemcpyDeviceToHost, s->cs), "download");
        ck(cudaStreamSynchronize(s->cs), "sync");
    });
}

VXC_API int32_t vxc_run_component(vxc_stream* s, int32_t component, const float* in0, const float* in1, float* out) {
    return guard([&] {
        require(s != nullptr && in0 != nullptr && out != nullptr, "null argument");
        require(component >= VXC_FSQ && component <= VXC_FEAT_ENCODER,
                "vxc_run_component serves fsq, fusion_proj, dit_proj, stop_head, feat_encoder");
        std::lock_guard<std::mutex> lk(s->call_mutex);
        vxc_device* dev = s->dev;
        const vxc_model_desc& d = dev->desc;
        const int H = d.hidden, Hd = d.dit_hidden, L = d.feat_dim * d.patch_size, Q = d.fsq_dim;
        DeviceGuard g(dev->device);
        check_loaded(dev, {component});
        float* a = s->gen_in;      // [H]
        float* b = s->gen_in + H;  // [H]
        int out_n = H;
        switch (component) {
            case VXC_FSQ: {
                ck(cudaMemcpyAsync(a, in0, sizeof(float) * H, cudaMemcpyHostToDevice, s->cs), "upload");
                const __half* fq = dev->blob[VXC_FSQ];
                const size_t qh = static_cast<size_t>(Q) * H;
                GemvArgs qa = plain_gemv(fq, fq + qh, a, H, Q, s->mid, ACT_FSQ, nullptr, 0);
                qa.act_scale = d.fsq_scale;
                launch_gemv(qa, s->cs, false);
                launch_gemv(plain_gemv(fq + qh + Q, fq + qh + Q + qh, s->mid, Q, H, s->feat, ACT_NONE, nullptr, 0),
                            s->cs, false);
                break;
            }
            case VXC_FUSION_PROJ: {
                require(in1 != nullptr, "fusion_proj needs two inputs");
                ck(cudaMemcpyAsync(a, in0, sizeof(float) * H, cudaMemcpyHostToDevice, s->cs), "upload");
                ck(cudaMemcpyAsync(b, in1, sizeof(float) * H, cudaMemcpyHostToDevice, s->cs), "upload");
                const __half* fu = dev->blob[VXC_FUSION_PROJ];
                GemvArgs ua = plain_gemv(fu, fu + static_cast<size_t>(H) * 2 * H, a, 2 * H, H, s->feat, ACT_NONE,
                                         nullptr, 0);
                ua.in_mode = IN_CONCAT;
                ua.x2 = b;
                ua.k1 = H;
                launch_gemv(ua, s->cs, false);
                break;
            }
            case VXC_DIT_PROJ: {
                require(in1 != nullptr, "dit_proj needs two inputs");
                ck(cudaMemcpyAsync(a, in0, sizeof(float) * H, cudaMemcpyHostToDevice, s->cs), "upload");
                ck(cudaMemcpyAsync(b, in1, sizeof(float) * H, cudaMemcpyHostToDevice, s->cs), "upload");
                const __half* dp = dev->blob[VXC_DIT_PROJ];
                const size_t dps = static_cast<size_t>(Hd) * H;
                launch_gemv(plain_gemv(dp, dp + dps, a, H, Hd, s->mu, ACT_NONE, nullptr, 0), s->cs, false);
                launch_gemv(plain_gemv(dp + dps + Hd, dp + 2 * dps + Hd, b, H, Hd, s->mu + Hd, ACT_NONE, nullptr, 0),
                            s->cs, false);
                ck(cudaMemcpyAsync(out, s->mu, sizeof(float) * 2 * Hd, cudaMemcpyDeviceToHost, s->cs), "download");
                ck(cudaStreamSynchronize(s->cs), "sync");
                return;
            }
            case VXC_STOP_HEAD: {
                ck(cudaMemcpyAsync(a, in0, sizeof(float) * H, cudaMemcpyHostToDevice, s->cs), "upload");
                const __half* sh = dev->blob[VXC_STOP_HEAD];
                launch_gemv(plain_gemv(sh, sh + static_cast<size_t>(H) * H, a, H, H, s->mid, ACT_SILU, nullptr, 0),
                            s->cs, false);
                launch_stop_decide(sh + static_cast<size_t>(H) * H + H, s->mid, H, nullptr, s->feat, s->cs, false);
                out_n = 2;
                break;
            }
            default: {  // VXC_FEAT_ENCODER
                ck(cudaMemcpyAsync(a, in0, sizeof(float) * L, cudaMemcpyHostToDevice, s->cs), "upload");
                const __half* fe = dev->blob[VXC_FEAT_ENCODER];
                const size_t fin = static_cast<size_t>(H) * L;
                GemvArgs fa = plain_gemv(fe, fe + fin, a, L, H, s->mid, ACT_SILU, nullptr, 0);
                fa.in_mode = IN_LATENT_T;
                fa.lat_d = d.feat_dim;
                fa.lat_p = d.patch_size;
                launch_gemv(fa, s->cs, false);
                launch_gemv(plain_gemv(fe + fin + H, fe + fin + H + static_cast<size_t>(H) * H, s->mid, H, H, s->feat,
                                       ACT_NONE, nullptr, 0),
                            s->cs, false);
                break;
            }
        }
        ck(cudaMemcpyAsync(out, s->feat, sizeof(float) * out_n, cudaMemcpyDeviceToHost, s->cs), "download");
        ck(cudaStreamSynchronize(s->cs), "sync");
    });
}

VXC_API int32_t vxc_dit_estimator(vxc_stream* s, const float* x_in, const float* mu_in, const float* t_in,
                                  const float* cond_in, const float* dt_in, float* out) {
    return guard([&] {
        require(s && x_in && mu_in && t_in && cond_in && dt_in && out, "null argument");
        std::lock_guard<std::mutex> lk(s->call_mutex);
        check_loaded(s->dev, {VXC_DIT_ESTIMATOR});
        const vxc_model_desc& d = s->dev->desc;
        const int Hd = d.dit_hidden, L = d.feat_dim * d.patch_size;
        DeviceGuard g(s->dev->device);
        float* xin = s->gen_in;    // [2][L]
        float* cin = xin + 2 * L;  // [2][L]
        float* min_ = cin + 2 * L; // [2][2Hd]
        ck(cudaMemcpyAsync(xin, x_in, sizeof(float) * 2 * L, cudaMemcpyHostToDevice, s->cs), "x");
        ck(cudaMemcpyAsync(cin, cond_in, sizeof(float) * 2 * L, cudaMemcpyHostToDevice, s->cs), "cond");
        ck(cudaMemcpyAsync(min_, mu_in, sizeof(float) * 4 * Hd, cudaMemcpyHostToDevice, s->cs), "mu");
        enqueue_time_tokens(s, t_in[0], t_in[1], dt_in, nullptr);
        enqueue_dit_eval(s, xin, xin + L, min_, min_ + 2 * Hd, cin, cin + L, dt_in[1] != dt_in[0], s->est, nullptr,
                         0.f, 0.f, nullptr, nullptr);
        ck(cudaMemcpyAsync(out, s->est, sizeof(float) * 2 * L, cudaMemcpyDeviceToHost, s->cs), "download");
        ck(cudaStreamSynchronize(s->cs), "sync");
    });
}

VXC_API int32_t vxc_cfm_sample(vxc_stream* s, const float* mu, const float* cond, const float* noise,
                               int32_t timesteps, float cfg_value, float* out_latent) {
    return guard([&] {
        require(s && mu && cond && noise && out_latent, "null argument");
        require(timesteps > 0, "inference timesteps must be positive");
        std::lock_guard<std::mutex> lk(s->call_mutex);
        check_loaded(s->dev, {VXC_DIT_ESTIMATOR});
        const vxc_model_desc& d = s->dev->desc;
        const int Hd = d.dit_hidden, L = d.feat_dim * d.patch_size;
        DeviceGuard g(s->dev->device);
        float* c = s->gen_in;
        ck(cudaMemcpyAsync(s->mu, mu, sizeof(float) * 2 * Hd, cudaMemcpyHostToDevice, s->cs), "mu");
        ck(cudaMemcpyAsync(c, cond, sizeof(float) * L, cudaMemcpyHostToDevice, s->cs), "cond");
        ck(cudaMemcpyAsync(s->x, noise, sizeof(float) * L, cudaMemcpyHostToDevice, s->cs), "noise");
        // standalone call: a stale stop flag must not skip the kernels
        s->ctl_host->stopped = 0;
        ck(cudaMemcpyAsync(&s->ctl->stopped, &s->ctl_host->stopped, sizeof(int), cudaMemcpyHostToDevice, s->cs), "ctl");
        time_table(s, timesteps);
        enqueue_cfm(s, c, timesteps, cfg_value);
        ck(cudaMemcpyAsync(out_latent, s->x, sizeof(float) * L, cudaMemcpyDeviceToHost, s->cs), "download");
        sync_ctl(s);
    });
}

VXC_API int32_t vxc_prefill(vxc_stream* s, const int32_t* text_ids, int32_t n_text) {
    return guard([&] {
        require(s != nullptr, "stream must not be null");
        std::lock_guard<std::mutex> lk(s->call_mutex);
        DeviceGuard g(s->dev->device);
        prefill(s, text_ids, n_text);
    });
}

VXC_API int32_t vxc_prefill_rows(vxc_stream* s, const int32_t* token_ids, const int32_t* is_audio,
                                 const float* audio_latents, int32_t n_rows) {
    return guard([&] {
        require(s != nullptr, "stream must not be null");
        std::lock_guard<std::mutex> lk(s->call_mutex);
        DeviceGuard g(s->dev->device);
        prefill_rows(s, token_ids, is_audio, audio_latents, n_rows);
    });
}

VXC_API int32_t vxc_patch_step(vxc_stream* s, const float* noise, int32_t min_patches, int32_t step, float cfg_value,
                               int32_t timesteps, float* out_latent, int32_t* out_stop) {
    return guard([&] {
        require(s != nullptr, "stream must not be null");
        std::lock_guard<std::mutex> lk(s->call_mutex);
        DeviceGuard g(s->dev->device);
        if (step != s->patches) throw InvalidState("step must equal the number of patches generated so far");
        int stop = 0;
        patch_step(s, noise, min_patches, cfg_value, timesteps, out_latent, &stop);
        if (out_stop) *out_stop = stop;
    });
}

VXC_API int32_t vxc_generate(vxc_stream* s, const int32_t* text_ids, int32_t n_text, int32_t min_patches,
                             int32_t timesteps, float cfg_value, int32_t max_patches_override, uint32_t seed,
                             float* out_latents, int32_t* out_patches, float* lm_trace, float* res_trace,
                             float* stop_trace, vxc_progress_fn progress, void* progress_user_data) {
    return guard([&] {
        require(s != nullptr && out_latents != nullptr && out_patches != nullptr, "null argument");
        require(timesteps > 0, "inference timesteps must be positive");
        std::lock_guard<std::mutex> lk(s->call_mutex);
        DeviceGuard g(s->dev->device);
        s->cancel.store(false);
        *out_patches = 0;
        const vxc_model_desc& d = s->dev->desc;
        const int H = d.hidden, L = d.feat_dim * d.patch_size;
        int max_patches = max_patches_for_target(n_text, d.max_generation_patches);
        if (max_patches_override > 0) max_patches = std::min(max_patches, max_patches_override);
        require(n_text + 1 + max_patches <= s->cap,
                "KV cache capacity exceeded: prefix + max_patches exceeds the stream's kv_capacity");
        prefill(s, text_ids, n_text);
        std::mt19937 rng(seed);
        std::vector<float> noise(static_cast<size_t>(L));
        for (int step = 0; step < max_patches; ++step) {
            if (s->cancel.load(std::memory_order_acquire)) throw Cancelled();
            if (progress && progress(progress_user_data, step, max_patches) == 0) throw Cancelled();
            if (lm_trace)
                ck(cudaMemcpyAsync(lm_trace + static_cast<size_t>(step) * H, s->lm_h, sizeof(float) * H,
                                   cudaMemcpyDeviceToHost, s->cs),
                   "trace");
            if (res_trace)
                ck(cudaMemcpyAsync(res_trace + static_cast<size_t>(step) * H, s->res_h, sizeof(float) * H,
                                   cudaMemcpyDeviceToHost, s->cs),
                   "trace");
            // cfm_sample draws the patch's values from a fresh normal_distribution (synthesizer.cpp:108-112)
            std::normal_distribution<float> normal(0.0f, 1.0f);
            for (float& v : noise) v = normal(rng);
            int stop = 0;
            patch_step(s, noise.data(), min_patches, cfg_value, timesteps, out_latents + static_cast<size_t>(step) * L,
                       &stop);
            if (stop_trace) {
                stop_trace[2 * step] = s->ctl_host->stop_logits[0];
                stop_trace[2 * step + 1] = s->ctl_host->stop_logits[1];
            }
            *out_patches = step + 1;
            if (stop) break;
        }
        if (progress) progress(progress_user_data, *out_patches, max_patches);
    });
}

// One-query SDPA calls of up to this many keys take the cluster-combined decode kernel.
constexpr int kClusterDecodeKeys = 512;

VXC_API int32_t vxc_sdpa(const float* q, int32_t heads, int32_t src, int32_t d, const float* k, const float* v,
                         int32_t groups, int32_t cur, int32_t dv, const float* mask, int32_t mask_c,
                         const float* past_k, const float* past_v, int32_t past, float scale, float* out,
                         float* out_k, float* out_v, void* cuda_stream) {
    return guard([&] {
        require(q && k && v && out, "null argument");
        require(heads > 0 && groups > 0 && heads % groups == 0 && src > 0 && cur > 0 && d > 0 && dv > 0 && past >= 0,
                "bad SDPA shape");
        require(past == 0 || (past_k && past_v), "past cache pointers missing");
        cudaStream_t cs = static_cast<cudaStream_t>(cuda_stream);
        const float rs = scale == 0.f ? 1.f / std::sqrt(static_cast<float>(d)) : scale;
        const int G = heads / groups;
        {
            // the op may be used without a vxc_device: raise the kernels' shared-memory
            // limits once per device on first use
            static std::mutex attr_mu;
            static std::vector<int> ready;
            int dev_id = 0;
            ck(cudaGetDevice(&dev_id), "cudaGetDevice");
            std::lock_guard<std::mutex> lk(attr_mu);
            if (std::find(ready.begin(), ready.end(), dev_id) == ready.end()) {
                init_kernel_attributes();
                ready.push_back(dev_id);
            }
        }
        if (src == 1 && d == 64 && dv == 64 && G <= 16 && mask_c <= 1 && past + cur <= kClusterDecodeKeys) {
            // up to 512 keys: one 8-CTA cluster per KV head (at most 2 key tiles per CTA),
            // the splits combined through distributed shared memory; no scratch
            AttnArgs aa;
            aa.q = q;
            aa.k0 = past > 0 ? past_k : k;
            aa.v0 = past > 0 ? past_v : v;
            aa.len0 = past > 0 ? past : cur;
            aa.stride0 = past > 0 ? past : cur;
            aa.k1 = past > 0 ? k : nullptr;
            aa.v1 = past > 0 ? v : nullptr;
            aa.len1 = past > 0 ? cur : 0;
            aa.stride1 = cur;
            aa.mask = mask;
            aa.q_heads = heads;
            aa.kv_heads = groups;
            aa.head_dim = d;
            aa.scale = rs;
            aa.out = out;
            // programmatic dependent launch: the kernel waits (griddepcontrol.wait) before it
            // reads anything, so its launch overlaps the tail of the stream's previous kernel.
            // Rows on 16-byte boundaries (always, from vxc_sdpa_host) take the load-all-first
            // op kernel; others the cluster decode kernel, which loads q by element.
            const bool aligned = ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(aa.k0) |
                                   reinterpret_cast<uintptr_t>(aa.v0) | reinterpret_cast<uintptr_t>(aa.k1) |
                                   reinterpret_cast<uintptr_t>(aa.v1)) & 15) == 0;
            if (aligned && sdpa_op_supported(aa))
                launch_sdpa_op(aa, cs, true);
            else
                launch_attn_decode_cluster(aa, cs, true);
        } else if (src == 1 && d == 64 && dv == 64 && G <= 16 && mask_c <= 1 && groups <= 64) {
            // longer: split-K flash decode over [past | cur] (fp32 rows). Its split partials
            // live in a scratch buffer kept per (device, CUDA stream): calls on one
            // stream run in order, calls on different streams never share it.
            int dev_id = 0;
            ck(cudaGetDevice(&dev_id), "cudaGetDevice");
            struct Scratch {
                float* partial = nullptr;
                int* counters = nullptr;
                size_t cap = 0;
            };
            static std::mutex mu;
            static std::map<std::pair<int, cudaStream_t>, Scratch> scratch;
            const int T = past + cur;
            const int splits = std::min(32, std::max(1, (T + 31) / 32));
            const size_t need = static_cast<size_t>(groups) * splits * G * (d + 2);
            std::lock_guard<std::mutex> lk(mu);
            Scratch& sc = scratch[{dev_id, cs}];
            if (sc.cap < need || sc.counters == nullptr) {
                ck(cudaStreamSynchronize(cs), "sync");
                if (sc.partial) cudaFree(sc.partial);
                if (sc.counters) cudaFree(sc.counters);
                sc = Scratch{};
                sc.partial = dev_alloc<float>(need);
                sc.counters = dev_alloc<int>(64);
                ck(cudaMemset(sc.counters, 0, sizeof(int) * 64), "counters");
                sc.cap = need;
            }
            AttnArgs aa;
            aa.q = q;
            aa.k0 = past > 0 ? past_k : k;
            aa.v0 = past > 0 ? past_v : v;
            aa.len0 = past > 0 ? past : cur;
            aa.stride0 = past > 0 ? past : cur;
            aa.k1 = past > 0 ? k : nullptr;
            aa.v1 = past > 0 ? v : nullptr;
            aa.len1 = past > 0 ? cur : 0;
            aa.stride1 = cur;
            aa.mask = mask;
            aa.q_heads = heads;
            aa.kv_heads = groups;
            aa.head_dim = d;
            aa.scale = rs;
            aa.splits = splits;
            aa.partial = sc.partial;
            aa.counters = sc.counters;
            aa.out = out;
            launch_attn_decode(aa, false, cs, true);
        } else {
            launch_sdpa_rows_f32(q, heads, src, d, k, v, groups, cur, dv, mask, mask_c, past_k, past_v, past, rs, out, cs);
        }
        if (out_k) launch_concat_kv(past_k, k, groups, past, cur, d, out_k, cs);
        if (out_v) launch_concat_kv(past_v, v, groups, past, cur, dv, out_v, cs);
    });
}

VXC_API int32_t vxc_sdpa_host(const float* q, int32_t heads, int32_t src, int32_t d, const float* k, const float* v,
                              int32_t groups, int32_t cur, int32_t dv, const float* mask, int32_t mask_c,
                              const float* past_k, const float* past_v, int32_t past, float scale, float* out,
                              float* out_k, float* out_v) {
    return guard([&] {
        require(q && k && v && out, "null argument");
        require(heads > 0 && groups > 0 && src > 0 && cur > 0 && d > 0 && dv > 0 && past >= 0, "bad SDPA shape");
        const int dst = past + cur;
        const size_t nq = static_cast<size_t>(heads) * src * d, nk = static_cast<size_t>(groups) * cur * d,
                     nv = static_cast<size_t>(groups) * cur * dv, npk = static_cast<size_t>(groups) * past * d,
                     npv = static_cast<size_t>(groups) * past * dv,
                     nm = mask ? static_cast<size_t>(std::max(1, mask_c)) * src * dst : 0,
                     no = static_cast<size_t>(heads) * src * dv, nok = static_cast<size_t>(groups) * dst * d,
                     nov = static_cast<size_t>(groups) * dst * dv;
        std::vector<float*> bufs;
        auto release = [&] {
            for (float* p : bufs) cudaFree(p);
            bufs.clear();
        };
        auto up = [&](const float* h, size_t n) -> float* {
            if (!h || n == 0) return nullptr;
            float* p = dev_alloc<float>(n);
            bufs.push_back(p);
            ck(cudaMemcpy(p, h, n * sizeof(float), cudaMemcpyHostToDevice), "upload");
            return p;
        };
        auto alloc = [&](size_t n) -> float* {
            float* p = dev_alloc<float>(n);
            bufs.push_back(p);
            return p;
        };
        try {
            float* dq = up(q, nq);
            float* dk = up(k, nk);
            float* dvv = up(v, nv);
            float* dpk = up(past_k, npk);
            float* dpv = up(past_v, npv);
            float* dm = up(mask, nm);
            float* dout = alloc(no);
            float* dok = out_k ? alloc(nok) : nullptr;
            float* dov = out_v ? alloc(nov) : nullptr;
            const int32_t rc = vxc_sdpa(dq, heads, src, d, dk, dvv, groups, cur, dv, dm, mask_c, dpk, dpv, past, scale,
                                        dout, dok, dov, nullptr);
            if (rc != VXC_STATUS_OK) {
                const std::string msg = g_last_error;
                release();
                if (rc == VXC_STATUS_INVALID_ARGUMENT) throw std::invalid_argument(msg);
                throw std::runtime_error(msg);
            }
            ck(cudaMemcpy(out, dout, no * sizeof(float), cudaMemcpyDeviceToHost), "download");
            if (out_k) ck(cudaMemcpy(out_k, dok, nok * sizeof(float), cudaMemcpyDeviceToHost), "download");
            if (out_v) ck(cudaMemcpy(out_v, dov, nov * sizeof(float), cudaMemcpyDeviceToHost), "download");
        } catch (...) {
            release();
            throw;
        }
        release();
    });
}

VXC_API int32_t vxc_timestep_embedding(const float* in, int32_t n_in, int32_t half_dim, float scale,
                                       float max_period, int32_t schedule_mode, float* out) {
    return guard([&] {
        require(in != nullptr && out != nullptr, "null argument");
        require(n_in > 0 && half_dim > 1 && max_period > 0.f, "bad timestep embedding shape");
        require(schedule_mode == 0 || n_in >= 2, "schedule mode reads (step_index, timesteps) from two inputs");
        // one t per input row; schedule mode gives every row t(step_index, timesteps)
        std::vector<float> t(static_cast<size_t>(n_in));
        const float sched = schedule_mode != 0 ? timestep_scheduled_t(in[0], in[1]) : 0.f;
        for (int b = 0; b < n_in; ++b) t[b] = (schedule_mode != 0 ? sched : in[b]) * scale;
        const std::vector<float> f = timestep_frequencies(half_dim, max_period);
        const size_t n_out = static_cast<size_t>(n_in) * 2 * half_dim;
        float* dt = dev_alloc<float>(t.size() + f.size() + n_out);
        try {
            float* dfreq = dt + t.size();
            float* dout = dfreq + f.size();
            ck(cudaMemcpy(dt, t.data(), sizeof(float) * t.size(), cudaMemcpyHostToDevice), "upload");
            ck(cudaMemcpy(dfreq, f.data(), sizeof(float) * f.size(), cudaMemcpyHostToDevice), "upload");
            launch_timestep_embedding(dt, 0.f, n_in, dfreq, half_dim, dout, nullptr, nullptr, false);
            ck(cudaMemcpy(out, dout, sizeof(float) * n_out, cudaMemcpyDeviceToHost), "download");
        } catch (...) {
            cudaFree(dt);
            throw;
        }
        cudaFree(dt);
    });
}

VXC_API int32_t vxc_upload_noise(vxc_stream* s, const float* noise, int32_t patches) {
    return guard([&] {
        require(s && noise && patches > 0, "bad arguments");
        std::lock_guard<std::mutex> lk(s->call_mutex);
        require(patches <= s->cap, "more noise rows than the stream holds (kv_capacity)");
        const int L = s->dev->desc.feat_dim * s->dev->desc.patch_size;
        DeviceGuard g(s->dev->device);
        ck(cudaMemcpy(s->noise, noise, sizeof(float) * L * patches, cudaMemcpyHostToDevice), "noise");
    });
}

VXC_API int32_t vxc_patch_step_async(vxc_stream* s, int32_t min_patches, float cfg_value, int32_t timesteps) {
    return guard([&] {
        require(s != nullptr, "stream must not be null");
        std::lock_guard<std::mutex> lk(s->call_mutex);
        DeviceGuard g(s->dev->device);
        check_patch_preconditions(s, timesteps);
        set_min_patches(s, min_patches);
        capture_patch_graph(s, timesteps, cfg_value);
        ck(cudaGraphLaunch(s->graph, s->cs), "cudaGraphLaunch");
        // host mirror advances optimistically; vxc_read_state re-syncs it
        s->patches += 1;
        s->kv_len[0] += 1;
        s->kv_len[1] += 1;
    });
}

VXC_API int32_t vxc_patch_submit(vxc_stream* s, const float* noise, int32_t min_patches, float cfg_value,
                                 int32_t timesteps) {
    return guard([&] {
        require(s != nullptr, "stream must not be null");
        std::lock_guard<std::mutex> lk(s->call_mutex);
        DeviceGuard g(s->dev->device);
        patch_submit(s, noise, min_patches, cfg_value, timesteps);
    });
}

VXC_API int32_t vxc_patch_collect(vxc_stream* s, float* out_latent, int32_t* out_stop) {
    return guard([&] {
        require(s != nullptr, "stream must not be null");
        std::lock_guard<std::mutex> lk(s->call_mutex);
        DeviceGuard g(s->dev->device);
        int stop = 0;
        patch_collect(s, out_latent, &stop);
        if (out_stop) *out_stop = stop;
    });
}

VXC_API int32_t vxc_patch_run(vxc_stream* const* streams, int32_t n, const float* noise, int32_t patches,
                              int32_t min_patches, float cfg_value, int32_t timesteps, float* out_latents,
                              int32_t* out_patches) {
    return guard([&] {
        require(streams != nullptr && noise != nullptr && out_latents != nullptr && out_patches != nullptr,
                "null argument");
        require(n > 0 && patches > 0, "need at least one stream and one patch");
        std::vector<vxc_stream*> order(streams, streams + n);
        for (vxc_stream* s : order) require(s != nullptr, "stream must not be null");
        std::sort(order.begin(), order.end());
        require(std::adjacent_find(order.begin(), order.end()) == order.end(), "a stream is listed twice");
        for (vxc_stream* s : order) require(s->dev->device == streams[0]->dev->device, "streams on different devices");
        // every stream's call lock, taken in address order (no lock-order inversion with other such calls)
        std::vector<std::unique_lock<std::mutex>> locks;
        for (vxc_stream* s : order) locks.emplace_back(s->call_mutex);
        DeviceGuard g(streams[0]->dev->device);
        const int L = streams[0]->dev->desc.feat_dim * streams[0]->dev->desc.patch_size;
        for (int i = 0; i < n; ++i) {
            require(streams[i]->submitted == streams[i]->collected, "a stream has patches in flight");
            out_patches[i] = 0;
        }
        // Each stream keeps kDepth patches queued: while the host copies one patch's
        // latent out and the next one's noise in, the stream's GPU queue never drains.
        constexpr int kDepth = 2;
        std::vector<int> sub(n, 0), col(n, 0), done(n, 0);
        auto submit = [&](int i) {
            patch_submit(streams[i], noise + (static_cast<size_t>(i) * patches + sub[i]) * L, min_patches, cfg_value,
                         timesteps);
            sub[i] += 1;
        };
        auto drain = [&](int i) {  // patches queued after a stop (their kernels skip) or after an error
            while (streams[i]->collected < streams[i]->submitted) {
                try {
                    patch_collect(streams[i], nullptr, nullptr);
                } catch (...) {
                }
            }
        };
        try {
            for (int k = 0; k < std::min(kDepth, static_cast<int>(patches)); ++k)
                for (int i = 0; i < n; ++i) submit(i);
            int live = n;
            while (live > 0) {
                for (int i = 0; i < n; ++i) {
                    if (done[i]) continue;
                    int stop = 0;
                    patch_collect(streams[i], out_latents + (static_cast<size_t>(i) * patches + col[i]) * L, &stop);
                    col[i] += 1;
                    out_patches[i] = col[i];
                    if (stop || col[i] == patches) {
                        drain(i);
                        done[i] = 1;
                        --live;
                    } else if (sub[i] < patches) {
                        submit(i);
                    }
                }
            }
        } catch (...) {
            for (int i = 0; i < n; ++i) drain(i);
            throw;
        }
    });
}

VXC_API int32_t vxc_stream_synchronize(vxc_stream* s) {
    return guard([&] {
        require(s != nullptr, "stream must not be null");
        DeviceGuard g(s->dev->device);
        ck(cudaStreamSynchronize(s->cs), "cudaStreamSynchronize");
    });
}

VXC_API int32_t vxc_read_state(vxc_stream* s, vxc_stream_state* out) {
    return guard([&] {
        require(s != nullptr && out != nullptr, "null argument");
        std::lock_guard<std::mutex> lk(s->call_mutex);
        DeviceGuard g(s->dev->device);
        ck(cudaMemcpyAsync(s->ctl_host, s->ctl, sizeof(StreamCtl), cudaMemcpyDeviceToHost, s->cs), "ctl");
        ck(cudaStreamSynchronize(s->cs), "sync");
        out->kv_len[0] = s->ctl_host->kv_len[0];
        out->kv_len[1] = s->ctl_host->kv_len[1];
        out->patches = s->ctl_host->patch;
        out->stopped = s->ctl_host->stopped;
        out->stop_logits[0] = s->ctl_host->stop_logits[0];
        out->stop_logits[1] = s->ctl_host->stop_logits[1];
        out->prefix_len = s->prefix_len;
        out->error = s->ctl_host->error;
        out->graph_kernels = s->graph_kernels;
        s->kv_len[0] = out->kv_len[0];
        s->kv_len[1] = out->kv_len[1];
        s->patches = out->patches;
    });
}

VXC_API int32_t vxc_read_hidden(vxc_stream* s, float* lm, float* res) {
    return guard([&] {
        require(s != nullptr, "stream must not be null");
        std::lock_guard<std::mutex> lk(s->call_mutex);
        const int H = s->dev->desc.hidden;
        DeviceGuard g(s->dev->device);
        if (lm) ck(cudaMemcpyAsync(lm, s->lm_h, sizeof(float) * H, cudaMemcpyDeviceToHost, s->cs), "lm");
        if (res) ck(cudaMemcpyAsync(res, s->res_h, sizeof(float) * H, cudaMemcpyDeviceToHost, s->cs), "res");
        ck(cudaStreamSynchronize(s->cs), "sync");
    });
}

VXC_API int32_t vxc_read_latents(vxc_stream* s, int32_t first, int32_t count, float* out) {
    return guard([&] {
        require(s != nullptr && out != nullptr && first >= 0 && count >= 0 && first + count <= s->cap, "bad range");
        std::lock_guard<std::mutex> lk(s->call_mutex);
        const int L = s->dev->desc.feat_dim * s->dev->desc.patch_size;
        DeviceGuard g(s->dev->device);
        ck(cudaMemcpyAsync(out, s->latents + static_cast<size_t>(first) * L, sizeof(float) * L * count,
                           cudaMemcpyDeviceToHost, s->cs),
           "latents");
        ck(cudaStreamSynchronize(s->cs), "sync");
    });
}

namespace {

// One launch function per layer of 'kernel', in the form the patch graph runs it
// (the argument turns programmatic dependent launch on); 'bytes' receives the
// algorithmic bytes of one launch. Called with the stream's mutex held.
std::vector<std::function<void(bool)>> profile_launches(vxc_stream* s, int kernel, double& bytes) {
    const vxc_device* dev = s->dev;
    const vxc_model_desc& d = dev->desc;
    const int Hd = d.dit_hidden, Fd = d.dit_ffn, H = d.hidden, F = d.ffn;
    const int seq = dit_tokens_per_seq(d.patch_size), M = 2 * seq;
    const int hq = d.q_heads, hkv = d.kv_heads, hd = d.head_dim;
    const int dq = d.dit_q_heads, dkv = d.dit_kv_heads;
    const size_t plane = static_cast<size_t>(hkv) * s->cap * hd;
    const int Wd = (dq + 2 * dkv) * (Hd / dq);
    bytes = 0.0;
    // one launch per layer, in the form the patch graph runs it
    std::vector<std::function<void(bool)>> launch;
    // the profiled decode kernels read kv_len from a private control block set to
    // the next free cache row (the q/k/v launch writes there), so valid rows stay intact
    const int pos = std::min(s->kv_len[0], s->cap - 1);
    const int T = pos + 1;
    StreamCtl* pctl = reinterpret_cast<StreamCtl*>(s->est);  // >= sizeof(StreamCtl) floats
    if (kernel == VXC_PROF_DIT_EVAL) {
        // one whole estimator evaluation (embed, the 12 layers in the stream's DiT form, out
        // projection), on the stream's current x / cond / mu and the cached time row of step 1
        // of 10; no Euler update (the estimate goes to scratch), a private control block
        const float* tab = time_table(s, 10);
        StreamCtl probe{};
        ck(cudaMemcpyAsync(pctl, &probe, sizeof(StreamCtl), cudaMemcpyHostToDevice, s->cs), "probe ctl");
        ck(cudaStreamSynchronize(s->cs), "sync");
        const double D = d.feat_dim;
        const double per_layer = static_cast<double>(Wd) * Hd + static_cast<double>(Hd) * dq * 64 + 3.0 * Fd * Hd + 2.0 * Hd;
        bytes = 2.0 * (per_layer * dev->dit.size() + 2.0 * (Hd * D + Hd) + D * Hd + D + Hd);
        launch.push_back([=](bool) {
            enqueue_dit_eval(s, s->x, nullptr, s->mu, nullptr, s->cond, nullptr, false, s->dest, nullptr, 0.f, 2.f, pctl,
                             tab + Hd);
        });
        return launch;
    }
    if (kernel == VXC_PROF_BASE_STEP || kernel == VXC_PROF_RES_STEP) {
        // a whole decoder step over the stream's current KV length, on a private
        // control block that it does not advance (each replay re-appends the same row)
        const int which = kernel == VXC_PROF_BASE_STEP ? 0 : 1;
        const std::vector<LayerW>& layers = which == 0 ? dev->base : dev->res;
        StreamCtl probe{};
        probe.kv_len[0] = std::min(s->kv_len[0], s->cap - 1);
        probe.kv_len[1] = std::min(s->kv_len[1], s->cap - 1);
        ck(cudaMemcpyAsync(pctl, &probe, sizeof(StreamCtl), cudaMemcpyHostToDevice, s->cs), "probe ctl");
        ck(cudaStreamSynchronize(s->cs), "sync");
        const double per_layer = static_cast<double>(hq + 2 * hkv) * hd * H + static_cast<double>(H) * hq * hd +
                                 3.0 * F * H + 2.0 * H;  // q/k/v, o, gate/up + down, two norms
        const double kv_rows = probe.kv_len[which] + 1.0;
        bytes = 2.0 * per_layer * layers.size() + 2.0 * H                        // fp16 weights + final norm
                + 4.0 * 2 * hkv * hd * kv_rows * layers.size();                    // fp32 K and V rows read
        // output into scratch: the residual step's real output feeds the next patch
        launch.push_back([=](bool) { enqueue_decoder_step(s, which, s->mid2, nullptr, 0, pctl, 0); });
        return launch;
    }
    if (kernel == VXC_PROF_BASE_QKV || kernel == VXC_PROF_BASE_ATTN) {
        StreamCtl probe{};
        probe.kv_len[0] = pos;
        ck(cudaMemcpyAsync(pctl, &probe, sizeof(StreamCtl), cudaMemcpyHostToDevice, s->cs), "probe ctl");
        ck(cudaStreamSynchronize(s->cs), "sync");
    }
    const bool dit = kernel <= VXC_PROF_DIT_QKV || kernel == VXC_PROF_DIT_O;
    const size_t nl = dit ? dev->dit.size() : dev->base.size();
    for (size_t l = 0; l < nl; ++l) {
        switch (kernel) {
            case VXC_PROF_DIT_GATEUP: {
                TcLinearArgs a = tc_plan(s, Fd / 64, Hd, 8);
                a.K = Hd; a.M = M; a.rows = Fd; a.gateup = 1;
                a.yb = s->xb_act; a.ldyb = Fd; a.ctl = s->ctl;
                bytes = 2.0 * 2 * Fd * Hd + 2.0 * 48 * Hd + 2.0 * 48 * Fd;
                const CUtensorMap ma = dev->dit_maps[l][2], mb = s->map_xb_n;
                launch.push_back([=](bool pdl) { launch_tc_linear(ma, mb, a, s->cs, pdl); });
                break;
            }
            case VXC_PROF_DIT_DOWN: {
                TcLinearArgs a = tc_plan(s, Hd / 128, Fd, 16);
                a.K = Fd; a.M = M; a.rows = Hd; a.resid = 1;
                a.y = s->dxn; a.ldy = Hd; a.ctl = s->ctl;
                bytes = 2.0 * Hd * Fd + 2.0 * 48 * Fd + 8.0 * M * Hd;
                const CUtensorMap ma = dev->dit_maps[l][3], mb = s->map_xb_act;
                launch.push_back([=](bool pdl) { launch_tc_linear(ma, mb, a, s->cs, pdl); });
                break;
            }
            case VXC_PROF_DIT_QKV: {
                TcLinearArgs a = tc_plan(s, Wd / 128, Hd, 8);
                a.K = Hd; a.M = M; a.rows = Wd;
                a.y = s->dqkv; a.ldy = Wd; a.ctl = s->ctl;
                bytes = 2.0 * Wd * Hd + 2.0 * 48 * Hd + 4.0 * M * Wd;
                const CUtensorMap ma = dev->dit_maps[l][0], mb = s->map_xb_n;
                launch.push_back([=](bool pdl) { launch_tc_linear(ma, mb, a, s->cs, pdl); });
                break;
            }
            case VXC_PROF_DIT_O: {
                TcLinearArgs a = tc_plan(s, Hd / 128, dq * 64, 8);
                a.K = dq * 64; a.M = M; a.rows = Hd; a.resid = 1;
                a.y = s->dxn; a.ldy = Hd; a.ctl = s->ctl;
                bytes = 2.0 * Hd * dq * 64 + 2.0 * 48 * dq * 64 + 8.0 * M * Hd;
                const CUtensorMap ma = dev->dit_maps[l][1], mb = s->map_xb_a;
                launch.push_back([=](bool pdl) { launch_tc_linear(ma, mb, a, s->cs, pdl); });
                break;
            }
            case VXC_PROF_BASE_GATEUP: {
                const LayerW& BL = dev->base[l];
                GemvArgs a;
                a.mode = GEMV_GATEUP; a.w = BL.wgateup; a.x = s->out[0]; a.norm_g = BL.post_norm; a.eps = d.rms_eps;
                a.K = H; a.rows = F; a.y = s->act;
                bytes = 2.0 * 2 * F * H + 4.0 * H + 4.0 * F;
                launch.push_back([=](bool pdl) { launch_gemv(a, s->cs, pdl); });
                break;
            }
            case VXC_PROF_BASE_DOWN: {
                GemvArgs a;
                a.mode = GEMV_RESID; a.w = dev->base[l].wdown; a.x = s->act; a.K = F; a.rows = H; a.resid = s->out[0];
                bytes = 2.0 * H * F + 4.0 * F + 8.0 * H;
                launch.push_back([=](bool pdl) { launch_gemv(a, s->cs, pdl); });
                break;
            }
            case VXC_PROF_BASE_QKV: {
                const LayerW& BL = dev->base[l];
                GemvArgs a;
                a.mode = GEMV_QKV; a.w = BL.wqkv; a.x = s->out[0]; a.norm_g = BL.in_norm; a.eps = d.rms_eps;
                a.K = H; a.rows = (hq + 2 * hkv) * hd / 2; a.y = s->q; a.q_heads = hq; a.kv_heads = hkv;
                a.head_dim = hd; set_decode_rope(a, s);
                a.k_cache = s->kc[0] + l * plane; a.v_cache = s->vc[0] + l * plane; a.cap = s->cap; a.which = 0;
                a.ctl = pctl;
                bytes = 2.0 * (hq + 2 * hkv) * hd * H + 4.0 * H + 4.0 * hq * hd + 4.0 * 2 * hkv * hd;
                launch.push_back([=](bool pdl) { launch_gemv(a, s->cs, pdl); });
                break;
            }
            case VXC_PROF_BASE_ATTN: {
                AttnArgs a;
                a.q = s->q; a.k0 = s->kc[0] + l * plane; a.v0 = s->vc[0] + l * plane; a.len0 = s->cap;
                a.stride0 = s->cap; a.q_heads = hq; a.kv_heads = hkv; a.head_dim = hd; a.scale = 0.125f;
                a.splits = s->splits; a.partial = s->partial; a.counters = s->counters; a.out = s->attn;
                a.ctl = pctl; a.which = 0;
                bytes = 4.0 * 2 * hkv * static_cast<double>(T) * hd + 8.0 * hq * hd;
                launch.push_back([=](bool pdl) { launch_attn_decode_cluster(a, s->cs, pdl); });
                break;
            }
        }
    }
    return launch;
}

// Captures 'iters' launches of 'kernel' cycling through the layers in one graph,
// starting at layer 'first' (after one eager warm-up launch per layer), and
// instantiates it.
cudaGraphExec_t profile_graph(vxc_stream* s, int kernel, int iters, double& bytes, int first = 0) {
    std::vector<std::function<void(bool)>> launch = profile_launches(s, kernel, bytes);
    for (auto& f : launch) f(false);  // warm-up, eager
    cudaGraph_t gr = nullptr;
    ck(cudaStreamBeginCapture(s->cs, cudaStreamCaptureModeThreadLocal), "cudaStreamBeginCapture");
    try {
        for (int i = 0; i < iters; ++i) launch[static_cast<size_t>(i + first) % launch.size()](i > 0);
    } catch (...) {
        cudaStreamEndCapture(s->cs, &gr);
        if (gr) cudaGraphDestroy(gr);
        throw;
    }
    ck(cudaStreamEndCapture(s->cs, &gr), "cudaStreamEndCapture");
    cudaGraphExec_t ge = nullptr;
    const cudaError_t ie = cudaGraphInstantiate(&ge, gr, 0);
    cudaGraphDestroy(gr);
    ck(ie, "cudaGraphInstantiate");
    return ge;
}

}  // namespace

VXC_API int32_t vxc_profile_kernel(vxc_stream* s, int32_t kernel, int32_t iters, float* ms_per_launch,
                                   double* bytes_per_launch) {
    return guard([&] {
        require(s != nullptr && ms_per_launch != nullptr && bytes_per_launch != nullptr, "null argument");
        require(iters > 0 && iters <= 100000, "iters must be in [1, 100000]");
        require(kernel >= VXC_PROF_DIT_GATEUP && kernel <= VXC_PROF_DIT_EVAL, "unknown kernel id");
        std::lock_guard<std::mutex> lk(s->call_mutex);
        const vxc_device* dev = s->dev;
        const vxc_model_desc& d = dev->desc;
        check_loaded(dev, {VXC_BASE_DECODER, VXC_DIT_ESTIMATOR});
        DeviceGuard g(dev->device);
        require(kernel != 8, "kernel id 8 is not used");
        // iters launches cycling through the layers, captured in one graph with
        // programmatic dependent launch between them like the patch graph
        double bytes = 0.0;
        cudaGraphExec_t ge = profile_graph(s, kernel, iters, bytes);
        cudaEvent_t e0 = nullptr, e1 = nullptr;
        float ms = 0.f;
        cudaError_t err = cudaGraphLaunch(ge, s->cs);  // warm-up replay
        if (err == cudaSuccess) err = cudaEventCreate(&e0);
        if (err == cudaSuccess) err = cudaEventCreate(&e1);
        if (err == cudaSuccess) err = cudaEventRecord(e0, s->cs);
        if (err == cudaSuccess) err = cudaGraphLaunch(ge, s->cs);
        if (err == cudaSuccess) err = cudaEventRecord(e1, s->cs);
        if (err == cudaSuccess) err = cudaEventSynchronize(e1);
        if (err == cudaSuccess) err = cudaEventElapsedTime(&ms, e0, e1);
        if (e0) cudaEventDestroy(e0);
        if (e1) cudaEventDestroy(e1);
        cudaGraphExecDestroy(ge);
        ck(err, "profile replay");
        sync_ctl(s);  // a bounded wait that gave up inside the profiled kernels surfaces here
        *ms_per_launch = ms / static_cast<float>(iters);
        *bytes_per_launch = bytes;
    });
}

VXC_API int32_t vxc_profile_kernel_concurrent(vxc_stream** streams, int32_t n, int32_t kernel, int32_t iters,
                                              float* ms_total, double* bytes_per_launch) {
    return guard([&] {
        require(streams != nullptr && ms_total != nullptr && bytes_per_launch != nullptr, "null argument");
        require(n >= 1 && n <= 256, "stream count must be in [1, 256]");
        require(iters > 0 && iters <= 100000, "iters must be in [1, 100000]");
        require(kernel >= VXC_PROF_DIT_GATEUP && kernel <= VXC_PROF_DIT_O, "unknown kernel id");
        std::vector<vxc_stream*> ss(streams, streams + n);
        for (vxc_stream* x : ss) require(x != nullptr && x->dev == ss[0]->dev, "streams must share one device");
        std::vector<vxc_stream*> order(ss);
        std::sort(order.begin(), order.end());
        require(std::adjacent_find(order.begin(), order.end()) == order.end(), "streams must be distinct");
        std::vector<std::unique_lock<std::mutex>> locks;
        for (vxc_stream* x : order) locks.emplace_back(x->call_mutex);  // address order: no lock cycles
        check_loaded(ss[0]->dev, {VXC_BASE_DECODER, VXC_DIT_ESTIMATOR});
        DeviceGuard g(ss[0]->dev->device);
        double bytes = 0.0;
        std::vector<cudaGraphExec_t> graphs;
        std::vector<cudaEvent_t> done(ss.size(), nullptr);
        cudaEvent_t e0 = nullptr, e1 = nullptr;
        cudaError_t err = cudaSuccess;
        float ms = 0.f;
        try {
            // stream i starts at layer i * layers / n, so the streams do not read the same
            // layer's weights in lockstep (which would let them share them through the L2)
            const int layers = kernel <= VXC_PROF_DIT_QKV || kernel == VXC_PROF_DIT_O
                                   ? static_cast<int>(ss[0]->dev->dit.size())
                                   : static_cast<int>(ss[0]->dev->base.size());
            for (size_t i = 0; i < ss.size(); ++i)
                graphs.push_back(profile_graph(ss[i], kernel, iters, bytes,
                                               static_cast<int>(i * layers / ss.size())));
            for (size_t i = 0; i < ss.size() && err == cudaSuccess; ++i) err = cudaGraphLaunch(graphs[i], ss[i]->cs);
            for (vxc_stream* x : ss)
                if (err == cudaSuccess) err = cudaStreamSynchronize(x->cs);  // warm-up replays done
            for (auto& e : done)
                if (err == cudaSuccess) err = cudaEventCreateWithFlags(&e, cudaEventDisableTiming);
            if (err == cudaSuccess) err = cudaEventCreate(&e0);
            if (err == cudaSuccess) err = cudaEventCreate(&e1);
            // all graphs start after e0 on the first stream and end before e1 on it
            if (err == cudaSuccess) err = cudaEventRecord(e0, ss[0]->cs);
            for (size_t i = 1; i < ss.size() && err == cudaSuccess; ++i) err = cudaStreamWaitEvent(ss[i]->cs, e0, 0);
            for (size_t i = 0; i < ss.size() && err == cudaSuccess; ++i) err = cudaGraphLaunch(graphs[i], ss[i]->cs);
            for (size_t i = 1; i < ss.size() && err == cudaSuccess; ++i) {
                err = cudaEventRecord(done[i], ss[i]->cs);
                if (err == cudaSuccess) err = cudaStreamWaitEvent(ss[0]->cs, done[i], 0);
            }
            if (err == cudaSuccess) err = cudaEventRecord(e1, ss[0]->cs);
            if (err == cudaSuccess) err = cudaEventSynchronize(e1);
            if (err == cudaSuccess) err = cudaEventElapsedTime(&ms, e0, e1);
        } catch (...) {
            for (cudaGraphExec_t ge : graphs) cudaGraphExecDestroy(ge);
            throw;
        }
        for (auto e : done)
            if (e) cudaEventDestroy(e);
        if (e0) cudaEventDestroy(e0);
        if (e1) cudaEventDestroy(e1);
        for (cudaGraphExec_t ge : graphs) cudaGraphExecDestroy(ge);
        ck(err, "concurrent profile");
        for (vxc_stream* x : ss) sync_ctl(x);
        *ms_total = ms;
        *bytes_per_launch = bytes;
    });
}

VXC_API int32_t vxc_stream_cuda_handle(vxc_stream* s, void** out) {
    return guard([&] {
        require(s != nullptr && out != nullptr, "null argument");
        *out = static_cast<void*>(s->cs);
    });
}

VXC_API int32_t vxc_group_create(vxc_device* dev, int32_t n_streams, int32_t kv_capacity, vxc_group** out) {
    return guard([&] {
        require(dev != nullptr && out != nullptr, "device and out must not be null");
        *out = nullptr;
        require(n_streams >= 1 && n_streams <= kGroupMax, "a group holds 1 to 8 streams");
        const vxc_model_desc& d = dev->desc;
        require(dit_tokens_per_seq(d.patch_size) == 11 && d.dit_hidden / d.dit_q_heads == 64,
                "groups need the 2 x 11-token DiT with 64-wide heads");
        DeviceGuard g(dev->device);
        auto grp = std::make_unique<vxc_group>();
        grp->dev = dev;
        if (const char* tt = std::getenv("VXC_GROUP_TC_TARGET")) {
            grp->tc_target = std::atoi(tt);
            require(grp->tc_target >= 1 && grp->tc_target <= 4096, "VXC_GROUP_TC_TARGET must be in [1, 4096]");
            grp->target_fixed = true;
        }
        if (const char* bg = std::getenv("VXC_GROUP_BULK_GEMV")) grp->bulk_gemv = std::string(bg) == "1";
        if (const char* rs = std::getenv("VXC_GROUP_RECV_SHARED")) grp->recv_shared = std::string(rs) != "0";
        if (const char* st = std::getenv("VXC_GROUP_TC_STAGES")) {
            grp->tc_stages = std::atoi(st);
            require(grp->tc_stages >= 1 && grp->tc_stages <= 4, "VXC_GROUP_TC_STAGES must be in [1, 4]");
        }
        try {
            for (int m = 0; m < n_streams; ++m) {
                vxc_stream* s = nullptr;
                if (vxc_stream_create(dev, kv_capacity, &s) != VXC_STATUS_OK)
                    throw std::runtime_error(std::string("group member: ") + g_last_error);
                grp->members.push_back(s);
            }
            const size_t Hd = d.dit_hidden, F = d.dit_ffn, Q = static_cast<size_t>(d.dit_q_heads) * 64;
            const size_t W = static_cast<size_t>(d.dit_q_heads + 2 * d.dit_kv_heads) * 64;
            const size_t M = 22 * static_cast<size_t>(n_streams);
            grp->gdh = dev_alloc<float>(M * Hd);
            grp->gqkv = dev_alloc<float>(M * W);
            const int lo = (static_cast<int>(M) + 15) / 16 * 16;
            const size_t rows = 2 * static_cast<size_t>(lo);
            grp->lo = lo;
            grp->xw_n = dev_alloc<__half>(rows * Hd);
            grp->xw_a = dev_alloc<__half>(rows * Q);
            grp->xw_act = dev_alloc<__half>(rows * F);
            ck(cudaMemset(grp->xw_n, 0, rows * Hd * sizeof(__half)), "cudaMemset");
            ck(cudaMemset(grp->xw_a, 0, rows * Q * sizeof(__half)), "cudaMemset");
            ck(cudaMemset(grp->xw_act, 0, rows * F * sizeof(__half)), "cudaMemset");
            grp->map_xw_n = make_tensor_map_f16(grp->xw_n, static_cast<int>(rows), static_cast<int>(Hd), lo);
            grp->map_xw_a = make_tensor_map_f16(grp->xw_a, static_cast<int>(rows), static_cast<int>(Q), lo);
            grp->map_xw_act = make_tensor_map_f16(grp->xw_act, static_cast<int>(rows), static_cast<int>(F), lo);
            grp->gctl = dev_alloc<StreamCtl>(1);
            ck(cudaMemset(grp->gctl, 0, sizeof(StreamCtl)), "cudaMemset");
            ck(cudaMallocHost(&grp->gctl_host, sizeof(StreamCtl)), "cudaMallocHost");
            grp->events.assign(4 * static_cast<size_t>(n_streams + 1), nullptr);
            for (auto& e : grp->events) ck(cudaEventCreateWithFlags(&e, cudaEventDisableTiming), "cudaEventCreate");
        } catch (...) {
            free_group(grp.get());
            for (vxc_stream* s : grp->members) vxc_stream_destroy(s);
            throw;
        }
        dev->live_groups.fetch_add(1);
        *out = grp.release();
    });
}

VXC_API void vxc_group_destroy(vxc_group* g) {
    if (!g) return;
    {
        std::lock_guard<std::mutex> lk(g->call_mutex);
        DeviceGuard dg(g->dev->device, true);
        if (!g->members.empty()) cudaStreamSynchronize(g->members[0]->cs);
        free_group(g);
    }
    g->dev->live_groups.fetch_sub(1);
    for (vxc_stream* s : g->members) vxc_stream_destroy(s);
    delete g;
}

VXC_API int32_t vxc_group_stream(vxc_group* g, int32_t member, vxc_stream** out) {
    return guard([&] {
        require(g != nullptr && out != nullptr, "null argument");
        require(member >= 0 && member < static_cast<int>(g->members.size()), "member index out of range");
        *out = g->members[static_cast<size_t>(member)];
    });
}

VXC_API int32_t vxc_group_patch_step_async(vxc_group* g, int32_t min_patches, float cfg_value, int32_t timesteps) {
    return guard([&] {
        require(g != nullptr, "group must not be null");
        std::lock_guard<std::mutex> lk(g->call_mutex);
        std::vector<std::unique_lock<std::mutex>> locks;
        for (vxc_stream* s : g->members) locks.emplace_back(s->call_mutex);
        DeviceGuard dg(g->dev->device);
        for (vxc_stream* s : g->members) {
            check_patch_preconditions(s, timesteps);
            set_min_patches(s, min_patches);
        }
        capture_group_graph(g, timesteps, cfg_value);
        // The graph runs on members[0]'s stream: it waits for work queued on the
        // other members' streams (noise uploads ...), and their later calls wait for it.
        const size_t n = g->members.size(), base = 3 * (n + 1);
        cudaStream_t c0 = g->members[0]->cs;
        for (size_t m = 1; m < n; ++m) {
            ck(cudaEventRecord(g->events[base + m], g->members[m]->cs), "group order");
            ck(cudaStreamWaitEvent(c0, g->events[base + m], 0), "group order");
        }
        ck(cudaGraphLaunch(g->graph, c0), "cudaGraphLaunch");
        ck(cudaEventRecord(g->events[base], c0), "group order");
        for (size_t m = 1; m < n; ++m) ck(cudaStreamWaitEvent(g->members[m]->cs, g->events[base], 0), "group order");
        for (vxc_stream* s : g->members) {  // host mirrors advance optimistically; read_state re-syncs them
            s->patches += 1;
            s->kv_len[0] += 1;
            s->kv_len[1] += 1;
        }
    });
}

VXC_API int32_t vxc_group_synchronize(vxc_group* g) {
    return guard([&] {
        require(g != nullptr, "group must not be null");
        std::lock_guard<std::mutex> lk(g->call_mutex);
        DeviceGuard dg(g->dev->device);
        ck(cudaStreamSynchronize(g->members[0]->cs), "cudaStreamSynchronize");
        ck(cudaMemcpy(g->gctl_host, g->gctl, sizeof(StreamCtl), cudaMemcpyDeviceToHost), "group ctl");
        if (g->gctl_host->error != 0) {
            g->gctl_host->error = 0;
            cudaMemcpy(&g->gctl->error, &g->gctl_host->error, sizeof(int), cudaMemcpyHostToDevice);
            throw std::runtime_error("a tensor-core pipeline wait timed out in the group's estimator");
        }
        for (vxc_stream* s : g->members) {
            std::lock_guard<std::mutex> sl(s->call_mutex);
            sync_ctl(s);
        }
    });
}

VXC_API int32_t vxc_group_graph_kernels(vxc_group* g, int32_t* out) {
    return guard([&] {
        require(g != nullptr && out != nullptr, "null argument");
        *out = g->graph_kernels;
    });
}

}  // extern "C"
