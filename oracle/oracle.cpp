// CPU oracle for the VoxCPM2 patch loop -- TEST INFRASTRUCTURE ONLY.
//
// This file restates, in plain fp32 C++, what the reference's ncnn CPU path
// computes for the autoregressive patch loop. Only the tests, the smoke check
// and bench.py's CPU baseline load it; the CUDA product never does. Each
// function names the reference lines it follows. Where the math lives in the
// un-vendored upstream `voxcpm 2.0.3` package (RMSNorm, SwiGLU, rotate_half
// RoPE, FSQ, feat_encoder, stop activation, time MLP), the restatement uses
// the published definitions of those layers and the synthetic stand-ins named
// in the header of voxcpm2_b200/config.py; those parts are "parity unpinned"
// against the reference itself and pinned only by the torch cross-check.

#include "oracle.h"

#include <algorithm>
#include <cfloat>
#include <cmath>
#include <cstring>
#include <numbers>
#include <random>
#include <stdexcept>
#include <vector>

#ifdef _OPENMP
#include <omp.h>
#endif
#include <immintrin.h>

namespace {

// ---------------------------------------------------------------- fp16 ---
float half_bits_to_float(uint16_t h) {
    const uint32_t sign = static_cast<uint32_t>(h & 0x8000u) << 16;
    const uint32_t exp = (h >> 10) & 0x1fu;
    const uint32_t man = h & 0x3ffu;
    uint32_t bits;
    if (exp == 0) {
        if (man == 0) {
            bits = sign;
        } else {  // subnormal: value = man * 2^-24
            float v = static_cast<float>(man) * 5.9604644775390625e-8f;
            std::memcpy(&bits, &v, 4);
            bits |= sign;
        }
    } else if (exp == 31) {
        bits = sign | 0x7f800000u | (man << 13);
    } else {
        bits = sign | ((exp + 112u) << 23) | (man << 13);
    }
    float out;
    std::memcpy(&out, &bits, 4);
    return out;
}

struct HalfTable {
    float v[65536];
    HalfTable() {
        for (uint32_t i = 0; i < 65536; ++i) v[i] = half_bits_to_float(static_cast<uint16_t>(i));
    }
};
const HalfTable& half_table() {
    static const HalfTable table;
    return table;
}
inline float h2f(uint16_t h) { return half_table().v[h]; }

int g_threads = 1;

// ------------------------------------------------------------ layers -----
// fp32 dot product with 16 independent partial sums (a SIMD-friendly order, as
// ncnn's vectorised InnerProduct/Gemm kernels use; fp32 summation order is not
// specified by the reference).
inline float dot(const float* a, const float* b, int n) {
    float acc[16] = {0.f};
    int k = 0;
    for (; k + 16 <= n; k += 16)
        for (int j = 0; j < 16; ++j) acc[j] += a[k + j] * b[k + j];
    float s = 0.f;
    for (int j = 0; j < 16; ++j) s += acc[j];
    for (; k < n; ++k) s += a[k] * b[k];
    return s;
}

// widen n fp16 values (F16C)
inline void widen(const uint16_t* src, int n, float* dst) {
    int k = 0;
    for (; k + 8 <= n; k += 8)
        _mm256_storeu_ps(dst + k, _mm256_cvtph_ps(_mm_loadu_si128(reinterpret_cast<const __m128i*>(src + k))));
    for (; k < n; ++k) dst[k] = half_table().v[src[k]];
}

// y[m][n] = sum_k W[n][k] x[m][k] (+ b[n]); nn.Linear / ncnn InnerProduct/Gemm.
void linear(const uint16_t* w, const uint16_t* b, int n_out, int k_in, const float* x, int m,
            float* y) {
    const HalfTable& t = half_table();
#pragma omp parallel num_threads(g_threads)
    {
        std::vector<float> row(static_cast<std::size_t>(k_in));
#pragma omp for schedule(static)
        for (int n = 0; n < n_out; ++n) {
            widen(w + static_cast<std::size_t>(n) * k_in, k_in, row.data());
            const float bias = b ? t.v[b[n]] : 0.0f;
            for (int i = 0; i < m; ++i)
                y[static_cast<std::size_t>(i) * n_out + n] =
                    dot(row.data(), x + static_cast<std::size_t>(i) * k_in, k_in) + bias;
        }
    }
}

// MiniCPM RMSNorm as run by ncnn's RMSNorm layer in fp32 (31=3 forces fp32,
// export_components.py:203-221): y = x / sqrt(mean(x^2) + eps) * gamma.
void rmsnorm(const float* x, const uint16_t* gamma, int h, float eps, int m, float* y) {
    for (int i = 0; i < m; ++i) {
        const float* xr = x + static_cast<std::size_t>(i) * h;
        float* yr = y + static_cast<std::size_t>(i) * h;
        float sq = 0.0f;
        for (int k = 0; k < h; ++k) sq += xr[k] * xr[k];
        const float a = 1.0f / std::sqrt(sq / static_cast<float>(h) + eps);
        for (int k = 0; k < h; ++k) yr[k] = xr[k] * a * h2f(gamma[k]);
    }
}

inline float silu(float v) { return v / (1.0f + std::exp(-v)); }

// apply_rotary_pos_emb with rotate_half on [heads][n][d] planes, tables [n][d].
void rope_apply(float* x, int heads, int n, int d, const float* cos, const float* sin) {
    const int half = d / 2;
    std::vector<float> tmp(static_cast<std::size_t>(d));
    for (int h = 0; h < heads; ++h) {
        for (int i = 0; i < n; ++i) {
            float* r = x + (static_cast<std::size_t>(h) * n + i) * d;
            const float* c = cos + static_cast<std::size_t>(i) * d;
            const float* s = sin + static_cast<std::size_t>(i) * d;
            for (int j = 0; j < half; ++j) tmp[j] = r[j] * c[j] + (-r[j + half]) * s[j];
            for (int j = half; j < d; ++j) tmp[j] = r[j] * c[j] + r[j - half] * s[j];
            std::memcpy(r, tmp.data(), sizeof(float) * d);
        }
    }
}

// ------------------------------------------------------------- weights ---
struct DecoderLayerW {
    const uint16_t *in_norm, *wq, *wk, *wv, *wo, *post_norm, *gate, *up, *down;
};
struct DecoderW {
    std::vector<DecoderLayerW> layers;
    const uint16_t* final_norm = nullptr;
};
struct DitW {
    const uint16_t *in_w, *in_b, *cond_w, *cond_b;
    const uint16_t *t1_w, *t1_b, *t2_w, *t2_b, *dt1_w, *dt1_b, *dt2_w, *dt2_b;
    DecoderW dec;
    const uint16_t *out_w, *out_b;
};

struct Cursor {
    const uint16_t* base;
    std::size_t off = 0;
    const uint16_t* take(std::size_t n) {
        const uint16_t* p = base ? base + off : nullptr;
        off += n;
        return p;
    }
};

struct DecShape {
    int h, f, hq, hkv, d, layers;
};

DecoderW carve_decoder(Cursor& c, const DecShape& s) {
    DecoderW w;
    const std::size_t H = s.h, F = s.f, Q = static_cast<std::size_t>(s.hq) * s.d,
                      KV = static_cast<std::size_t>(s.hkv) * s.d;
    for (int l = 0; l < s.layers; ++l) {
        DecoderLayerW L{};
        L.in_norm = c.take(H);
        L.wq = c.take(Q * H);
        L.wk = c.take(KV * H);
        L.wv = c.take(KV * H);
        L.wo = c.take(H * Q);
        L.post_norm = c.take(H);
        L.gate = c.take(F * H);
        L.up = c.take(F * H);
        L.down = c.take(H * F);
        w.layers.push_back(L);
    }
    w.final_norm = c.take(H);
    return w;
}

DecShape base_shape(const orc_desc& d) {
    return {d.hidden, d.ffn, d.q_heads, d.kv_heads, d.head_dim, d.base_layers};
}
DecShape res_shape(const orc_desc& d) {
    return {d.hidden, d.ffn, d.q_heads, d.kv_heads, d.head_dim, d.res_layers};
}
DecShape dit_shape(const orc_desc& d) {
    return {d.dit_hidden, d.dit_ffn, d.dit_q_heads, d.dit_kv_heads, d.dit_hidden / d.dit_q_heads,
            d.dit_layers};
}

DitW carve_dit(Cursor& c, const orc_desc& d) {
    DitW w{};
    const std::size_t Hd = d.dit_hidden, D = d.feat_dim;
    w.in_w = c.take(Hd * D);
    w.in_b = c.take(Hd);
    w.cond_w = c.take(Hd * D);
    w.cond_b = c.take(Hd);
    w.t1_w = c.take(Hd * Hd);
    w.t1_b = c.take(Hd);
    w.t2_w = c.take(Hd * Hd);
    w.t2_b = c.take(Hd);
    w.dt1_w = c.take(Hd * Hd);
    w.dt1_b = c.take(Hd);
    w.dt2_w = c.take(Hd * Hd);
    w.dt2_b = c.take(Hd);
    w.dec = carve_decoder(c, dit_shape(d));
    w.out_w = c.take(D * Hd);
    w.out_b = c.take(D);
    return w;
}

std::size_t component_count(const orc_desc& d, int component) {
    Cursor c{nullptr};
    const std::size_t H = d.hidden, Hd = d.dit_hidden, D = d.feat_dim, P = d.patch_size,
                      Q = d.fsq_dim;
    switch (component) {
        case 0: return static_cast<std::size_t>(d.vocab) * H;
        case 1: carve_decoder(c, base_shape(d)); return c.off;
        case 2: carve_decoder(c, res_shape(d)); return c.off;
        case 3: return Q * H + Q + H * Q + H;
        case 4: return H * 2 * H + H;
        case 5: return 2 * (Hd * H + Hd);
        case 6: return H * H + H + 2 * H;
        case 7: return H * (P * D) + H + H * H + H;
        case 8: carve_dit(c, d); return c.off;
        default: return 0;
    }
}

// ------------------------------------------------------------------ SDPA ---
int sdpa_impl(const float* q, int heads, int src, int d, const float* k, const float* v,
              int groups, int cur, int dv, const float* mask, int mask_c, const float* past_k,
              const float* past_v, int past, float scale, float* out, float* out_k,
              float* out_v) {
    if (heads <= 0 || groups <= 0 || heads % groups != 0 || src <= 0 || cur <= 0 || d <= 0 ||
        dv <= 0 || past < 0)
        return -1;
    const int dst = past + cur;
    const float rs = scale == 0.f ? 1.f / std::sqrt(static_cast<float>(d)) : scale;
    const int per_group = heads / groups;

    // Concatenate past and current K/V (voxcpm2_sdpa.cpp:151-185).
    std::vector<float> key(static_cast<std::size_t>(groups) * dst * d);
    std::vector<float> value(static_cast<std::size_t>(groups) * dst * dv);
    for (int g = 0; g < groups; ++g) {
        if (past > 0) {
            std::memcpy(&key[static_cast<std::size_t>(g) * dst * d],
                        past_k + static_cast<std::size_t>(g) * past * d, sizeof(float) * past * d);
            std::memcpy(&value[static_cast<std::size_t>(g) * dst * dv],
                        past_v + static_cast<std::size_t>(g) * past * dv,
                        sizeof(float) * past * dv);
        }
        std::memcpy(&key[(static_cast<std::size_t>(g) * dst + past) * d],
                    k + static_cast<std::size_t>(g) * cur * d, sizeof(float) * cur * d);
        std::memcpy(&value[(static_cast<std::size_t>(g) * dst + past) * dv],
                    v + static_cast<std::size_t>(g) * cur * dv, sizeof(float) * cur * dv);
    }

    // Per head: scores, +mask, softmax, P.V (voxcpm2_sdpa.cpp:187-252).
#pragma omp parallel num_threads(g_threads)
    {
        std::vector<float> qk(static_cast<std::size_t>(src) * dst);
#pragma omp for schedule(static)
        for (int h = 0; h < heads; ++h) {
            const float* qh = q + static_cast<std::size_t>(h) * src * d;
            const float* kh = &key[static_cast<std::size_t>(h / per_group) * dst * d];
            const float* vh = &value[static_cast<std::size_t>(h / per_group) * dst * dv];
            float* oh = out + static_cast<std::size_t>(h) * src * dv;
            for (int i = 0; i < src; ++i) {
                const float* qp = qh + static_cast<std::size_t>(i) * d;
                float* op = &qk[static_cast<std::size_t>(i) * dst];
                for (int j = 0; j < dst; ++j) {
                    const float* kp = kh + static_cast<std::size_t>(j) * d;
                    float sum = 0.f;
                    for (int e = 0; e < d; ++e) sum += qp[e] * kp[e];
                    op[j] = sum * rs;
                }
            }
            if (mask) {
                const float* mh = mask_c > 1 ? mask + static_cast<std::size_t>(h) * src * dst : mask;
                for (int i = 0; i < src; ++i)
                    for (int j = 0; j < dst; ++j)
                        qk[static_cast<std::size_t>(i) * dst + j] +=
                            mh[static_cast<std::size_t>(i) * dst + j];
            }
            for (int i = 0; i < src; ++i) {
                float* p = &qk[static_cast<std::size_t>(i) * dst];
                float mx = -FLT_MAX;
                for (int j = 0; j < dst; ++j) mx = std::max(mx, p[j]);
                float sum = 0.f;
                for (int j = 0; j < dst; ++j) {
                    p[j] = std::exp(p[j] - mx);
                    sum += p[j];
                }
                for (int j = 0; j < dst; ++j) p[j] /= sum;
            }
            for (int i = 0; i < src; ++i) {
                const float* p = &qk[static_cast<std::size_t>(i) * dst];
                float* o = oh + static_cast<std::size_t>(i) * dv;
                for (int e = 0; e < dv; ++e) {
                    float sum = 0.f;
                    for (int j = 0; j < dst; ++j) sum += p[j] * vh[static_cast<std::size_t>(j) * dv + e];
                    o[e] = sum;
                }
            }
        }
    }
    if (out_k) std::memcpy(out_k, key.data(), sizeof(float) * key.size());
    if (out_v) std::memcpy(out_v, value.data(), sizeof(float) * value.size());
    return 0;
}

void timestep_embedding(const float* in, int batch, int half_dim, float scale, float max_period,
                        int schedule_mode, float* out) {
    constexpr float kPi = 3.14159265358979323846f;
    const int out_dim = half_dim * 2;
    const float log_period = std::log(max_period);
    float scheduled_t = 0.0f;
    if (schedule_mode != 0) {
        const float step_index = in[0];
        const float timesteps = std::max(in[1], 1.0f);
        const float u = 1.0f - step_index / timesteps;
        scheduled_t = u + (std::cos(kPi * 0.5f * u) - 1.0f + u);
    }
    for (int b = 0; b < batch; ++b) {
        const float t = (schedule_mode != 0 ? scheduled_t : in[b]) * scale;
        float* row = out + static_cast<std::size_t>(b) * out_dim;
        for (int i = 0; i < half_dim; ++i) {
            const float inv_freq =
                std::exp(-log_period * static_cast<float>(i) / static_cast<float>(half_dim - 1));
            const float phase = t * inv_freq;
            row[i] = std::sin(phase);
            row[i + half_dim] = std::cos(phase);
        }
    }
}

void decoder_mask(int cur, int past, float* out) {
    const int dst = past + cur;
    for (int r = 0; r < cur; ++r)
        for (int c = 0; c < dst; ++c)
            out[static_cast<std::size_t>(r) * dst + c] = c >= past + r + 1 ? -10000.0f : 0.0f;
}

void rope_cache(int head_dim, float theta, int original_max, const float* short_f,
                const float* long_f, int start, int length, float* cos_out, float* sin_out) {
    const int half = head_dim / 2;
    std::vector<float> inv(static_cast<std::size_t>(half));
    for (int j = 0; j < half; ++j) {
        const float exponent = (2.0f * static_cast<float>(j)) / static_cast<float>(head_dim);
        inv[static_cast<std::size_t>(j)] = 1.0f / std::pow(theta, exponent);
    }
    const float* factor = (start + length > original_max && long_f) ? long_f : short_f;
    for (int p = 0; p < length; ++p) {
        const int pos = start + p;
        float* cr = cos_out + static_cast<std::size_t>(p) * head_dim;
        float* sr = sin_out + static_cast<std::size_t>(p) * head_dim;
        for (int j = 0; j < half; ++j) {
            const float f = factor ? factor[j] : 1.0f;
            const float freq = (static_cast<float>(pos) / f) * inv[static_cast<std::size_t>(j)];
            const float c = std::cos(freq), s = std::sin(freq);
            cr[j] = c;
            cr[j + half] = c;
            sr[j] = s;
            sr[j + half] = s;
        }
    }
}

}  // namespace

// ================================================================= model ===
struct orc_model {
    orc_desc desc{};
    const uint16_t* blob[9] = {};
    DecoderW base, res;
    DitW dit{};
    // HostDecoderKvCache equivalents: per decoder, per layer, [kv_heads][T][d]
    std::vector<std::vector<float>> cache_k[2], cache_v[2];
    int tokens[2] = {0, 0};
    // LongRoPE factors of the base decoder (setting.rope.short_factor / long_factor,
    // src/model_manifest.cpp:92-109): all ones until orc_set_rope_factors; an empty
    // long table means the short one is used at every position
    std::vector<float> short_factor, long_factor;
    std::vector<float> dit_factor;  // the estimator's rotary table: all ones
    // test hook (orc_trace_fsq): every FSQ row's values tanh(z) * scale before rounding,
    // appended in call order while rows remain
    mutable float* fsq_log = nullptr;
    mutable int fsq_log_cap = 0, fsq_log_n = 0;
    // test hook (orc_force_fsq): codes (integers in units of 1 / scale) that replace the
    // rounding of the next FSQ rows, in call order while rows remain
    const float* fsq_force = nullptr;
    mutable int fsq_force_cap = 0, fsq_force_n = 0;
};

namespace {

const DecoderW& decoder_of(const orc_model* m, int which) { return which == 0 ? m->base : m->res; }

void decoder_forward(orc_model* m, int which, const float* embed, int n, const float* mask_in,
                     const float* cos_in, const float* sin_in, float* out) {
    const orc_desc& d = m->desc;
    const DecoderW& w = decoder_of(m, which);
    const int H = d.hidden, F = d.ffn, hq = d.q_heads, hkv = d.kv_heads, hd = d.head_dim;
    const int past = m->tokens[which];
    const float rscale = which == 0 ? d.base_residual_scale : d.res_residual_scale;
    const bool use_rope = which == 0;

    std::vector<float> mask;
    if (!mask_in) {
        mask.resize(static_cast<std::size_t>(n) * (past + n));
        decoder_mask(n, past, mask.data());
        mask_in = mask.data();
    }
    std::vector<float> cos, sin;
    if (use_rope && (!cos_in || !sin_in)) {
        cos.resize(static_cast<std::size_t>(n) * hd);
        sin.resize(cos.size());
        rope_cache(hd, d.rope_theta, d.rope_original_max, m->short_factor.data(),
                   m->long_factor.empty() ? nullptr : m->long_factor.data(), past, n, cos.data(), sin.data());
        cos_in = cos.data();
        sin_in = sin.data();
    }

    const std::size_t N = n;
    std::vector<float> h(embed, embed + N * H), normed(N * H), q(N * hq * hd), k(N * hkv * hd),
        v(N * hkv * hd), qh(q.size()), kh(k.size()), vh(v.size()), attn_h(q.size()),
        attn(q.size()), o(N * H), gate(N * F), up(N * F), down(N * H);
    auto& ck = m->cache_k[which];
    auto& cv = m->cache_v[which];
    for (std::size_t l = 0; l < w.layers.size(); ++l) {
        const DecoderLayerW& L = w.layers[l];
        rmsnorm(h.data(), L.in_norm, H, d.rms_eps, n, normed.data());
        linear(L.wq, nullptr, hq * hd, H, normed.data(), n, q.data());
        linear(L.wk, nullptr, hkv * hd, H, normed.data(), n, k.data());
        linear(L.wv, nullptr, hkv * hd, H, normed.data(), n, v.data());
        // view(bsz, q_len, heads, hd).transpose(1, 2) -> [heads][n][hd]
        for (int i = 0; i < n; ++i) {
            for (int hh = 0; hh < hq; ++hh)
                std::memcpy(&qh[(static_cast<std::size_t>(hh) * n + i) * hd],
                            &q[(static_cast<std::size_t>(i) * hq + hh) * hd], sizeof(float) * hd);
            for (int hh = 0; hh < hkv; ++hh) {
                std::memcpy(&kh[(static_cast<std::size_t>(hh) * n + i) * hd],
                            &k[(static_cast<std::size_t>(i) * hkv + hh) * hd], sizeof(float) * hd);
                std::memcpy(&vh[(static_cast<std::size_t>(hh) * n + i) * hd],
                            &v[(static_cast<std::size_t>(i) * hkv + hh) * hd], sizeof(float) * hd);
            }
        }
        if (use_rope) {
            rope_apply(qh.data(), hq, n, hd, cos_in, sin_in);
            rope_apply(kh.data(), hkv, n, hd, cos_in, sin_in);
        }
        std::vector<float> nk(static_cast<std::size_t>(hkv) * (past + n) * hd), nv(nk.size());
        sdpa_impl(qh.data(), hq, n, hd, kh.data(), vh.data(), hkv, n, hd, mask_in, 1,
                  past ? ck[l].data() : nullptr, past ? cv[l].data() : nullptr, past, 0.0f,
                  attn_h.data(), nk.data(), nv.data());
        ck[l] = std::move(nk);
        cv[l] = std::move(nv);
        for (int i = 0; i < n; ++i)
            for (int hh = 0; hh < hq; ++hh)
                std::memcpy(&attn[(static_cast<std::size_t>(i) * hq + hh) * hd],
                            &attn_h[(static_cast<std::size_t>(hh) * n + i) * hd],
                            sizeof(float) * hd);
        linear(L.wo, nullptr, H, hq * hd, attn.data(), n, o.data());
        for (std::size_t i = 0; i < N * H; ++i) h[i] = h[i] + (rscale == 1.0f ? o[i] : o[i] * rscale);
        rmsnorm(h.data(), L.post_norm, H, d.rms_eps, n, normed.data());
        linear(L.gate, nullptr, F, H, normed.data(), n, gate.data());
        linear(L.up, nullptr, F, H, normed.data(), n, up.data());
        for (std::size_t i = 0; i < N * F; ++i) gate[i] = silu(gate[i]) * up[i];
        linear(L.down, nullptr, H, F, gate.data(), n, down.data());
        for (std::size_t i = 0; i < N * H; ++i)
            h[i] = h[i] + (rscale == 1.0f ? down[i] : down[i] * rscale);
    }
    rmsnorm(h.data(), w.final_norm, H, d.rms_eps, n, out);
    m->tokens[which] = past + n;
}

// DiT decoder over the CFG sequences (DitEstimator.decoder,
// export_components.py:625-659): no mask, no cache, RoPE positions 0..seq-1.
// The linear layers run over all nseq * seq rows at once (rows are
// independent); attention stays within each sequence.
void dit_decoder(const orc_model* m, float* hidden, int nseq, int seq, float* out) {
    const orc_desc& d = m->desc;
    const DecShape s = dit_shape(d);
    const int H = s.h, F = s.f, hq = s.hq, hkv = s.hkv, hd = s.d;
    const int n = nseq * seq;
    std::vector<float> cos(static_cast<std::size_t>(seq) * hd), sin(cos.size());
    rope_cache(hd, d.rope_theta, d.rope_original_max, m->dit_factor.data(), nullptr, 0, seq,
               cos.data(), sin.data());
    const std::size_t N = n, S = seq;
    std::vector<float> normed(N * H), q(N * hq * hd), k(N * hkv * hd), v(N * hkv * hd),
        qh(S * hq * hd), kh(S * hkv * hd), vh(S * hkv * hd), attn_h(qh.size()), attn(q.size()),
        o(N * H), gate(N * F), up(N * F), down(N * H);
    for (const DecoderLayerW& L : m->dit.dec.layers) {
        rmsnorm(hidden, L.in_norm, H, d.rms_eps, n, normed.data());
        linear(L.wq, nullptr, hq * hd, H, normed.data(), n, q.data());
        linear(L.wk, nullptr, hkv * hd, H, normed.data(), n, k.data());
        linear(L.wv, nullptr, hkv * hd, H, normed.data(), n, v.data());
        for (int b = 0; b < nseq; ++b) {
            const std::size_t r0 = static_cast<std::size_t>(b) * seq;
            for (int i = 0; i < seq; ++i) {
                for (int hh = 0; hh < hq; ++hh)
                    std::memcpy(&qh[(static_cast<std::size_t>(hh) * seq + i) * hd],
                                &q[((r0 + i) * hq + hh) * hd], sizeof(float) * hd);
                for (int hh = 0; hh < hkv; ++hh) {
                    std::memcpy(&kh[(static_cast<std::size_t>(hh) * seq + i) * hd],
                                &k[((r0 + i) * hkv + hh) * hd], sizeof(float) * hd);
                    std::memcpy(&vh[(static_cast<std::size_t>(hh) * seq + i) * hd],
                                &v[((r0 + i) * hkv + hh) * hd], sizeof(float) * hd);
                }
            }
            rope_apply(qh.data(), hq, seq, hd, cos.data(), sin.data());
            rope_apply(kh.data(), hkv, seq, hd, cos.data(), sin.data());
            sdpa_impl(qh.data(), hq, seq, hd, kh.data(), vh.data(), hkv, seq, hd, nullptr, 0,
                      nullptr, nullptr, 0, 0.0f, attn_h.data(), nullptr, nullptr);
            for (int i = 0; i < seq; ++i)
                for (int hh = 0; hh < hq; ++hh)
                    std::memcpy(&attn[((r0 + i) * hq + hh) * hd],
                                &attn_h[(static_cast<std::size_t>(hh) * seq + i) * hd],
                                sizeof(float) * hd);
        }
        linear(L.wo, nullptr, H, hq * hd, attn.data(), n, o.data());
        const float rs = d.dit_residual_scale;
        for (std::size_t i = 0; i < N * H; ++i) hidden[i] = hidden[i] + (rs == 1.0f ? o[i] : o[i] * rs);
        rmsnorm(hidden, L.post_norm, H, d.rms_eps, n, normed.data());
        linear(L.gate, nullptr, F, H, normed.data(), n, gate.data());
        linear(L.up, nullptr, F, H, normed.data(), n, up.data());
        for (std::size_t i = 0; i < N * F; ++i) gate[i] = silu(gate[i]) * up[i];
        linear(L.down, nullptr, H, F, gate.data(), n, down.data());
        for (std::size_t i = 0; i < N * H; ++i)
            hidden[i] = hidden[i] + (rs == 1.0f ? down[i] : down[i] * rs);
    }
    rmsnorm(hidden, m->dit.dec.final_norm, H, d.rms_eps, n, out);
}

// TimestepEmbedding: linear_2(silu(linear_1(emb)))
void time_mlp(const uint16_t* w1, const uint16_t* b1, const uint16_t* w2, const uint16_t* b2,
              int hd, const float* emb, int rows, float* out) {
    std::vector<float> mid(static_cast<std::size_t>(rows) * hd);
    linear(w1, b1, hd, hd, emb, rows, mid.data());
    for (float& x : mid) x = silu(x);
    linear(w2, b2, hd, hd, mid.data(), rows, out);
}

int dit_estimator(const orc_model* m, const float* x_in, const float* mu_in, const float* t_in,
                  const float* cond_in, const float* dt_in, float* out) {
    const orc_desc& d = m->desc;
    const int Hd = d.dit_hidden, D = d.feat_dim, P = d.patch_size;
    const DitW& w = m->dit;
    // x.transpose(1, 2): [2][D][P] -> [2][P][D]; then in_proj per frame.
    std::vector<float> xt(2 * P * D), ct(2 * P * D);
    for (int b = 0; b < 2; ++b)
        for (int p = 0; p < P; ++p)
            for (int e = 0; e < D; ++e) {
                xt[(static_cast<std::size_t>(b) * P + p) * D + e] = x_in[(static_cast<std::size_t>(b) * D + e) * P + p];
                ct[(static_cast<std::size_t>(b) * P + p) * D + e] = cond_in[(static_cast<std::size_t>(b) * D + e) * P + p];
            }
    std::vector<float> xh(static_cast<std::size_t>(2) * P * Hd), ch(xh.size());
    linear(w.in_w, w.in_b, Hd, D, xt.data(), 2 * P, xh.data());
    linear(w.cond_w, w.cond_b, Hd, D, ct.data(), 2 * P, ch.data());
    // time tokens (fused VoxCPM2TimestepEmbedding: 3=1 for in2, 3=0 for in4;
    // export_components.py:84-168)
    std::vector<float> temb(2 * static_cast<std::size_t>(Hd)), dtemb(temb.size()), tt(temb.size()),
        dtt(temb.size());
    timestep_embedding(t_in, 2, Hd / 2, 1000.0f, 10000.0f, 1, temb.data());
    timestep_embedding(dt_in, 2, Hd / 2, 1000.0f, 10000.0f, 0, dtemb.data());
    time_mlp(w.t1_w, w.t1_b, w.t2_w, w.t2_b, Hd, temb.data(), 2, tt.data());
    time_mlp(w.dt1_w, w.dt1_b, w.dt2_w, w.dt2_b, Hd, dtemb.data(), 2, dtt.data());
    const int seq = 3 + 2 * P;  // [mu0, mu1, time, cond x P, x x P] = 11
    std::vector<float> hidden(static_cast<std::size_t>(2) * seq * Hd), normed(hidden.size());
    std::vector<float> rows(static_cast<std::size_t>(2) * P * Hd);
    for (int b = 0; b < 2; ++b) {
        float* hp = hidden.data() + static_cast<std::size_t>(b) * seq * Hd;
        std::memcpy(hp, mu_in + static_cast<std::size_t>(b) * 2 * Hd, sizeof(float) * 2 * Hd);
        for (int e = 0; e < Hd; ++e)
            hp[2 * Hd + e] = tt[static_cast<std::size_t>(b) * Hd + e] + dtt[static_cast<std::size_t>(b) * Hd + e];
        std::memcpy(hp + 3 * Hd, &ch[static_cast<std::size_t>(b) * P * Hd], sizeof(float) * P * Hd);
        std::memcpy(hp + (3 + P) * static_cast<std::size_t>(Hd), &xh[static_cast<std::size_t>(b) * P * Hd],
                    sizeof(float) * P * Hd);
    }
    dit_decoder(m, hidden.data(), 2, seq, normed.data());
    for (int b = 0; b < 2; ++b)
        std::memcpy(&rows[static_cast<std::size_t>(b) * P * Hd],
                    normed.data() + (static_cast<std::size_t>(b) * seq + 3 + P) * Hd, sizeof(float) * P * Hd);
    std::vector<float> o(static_cast<std::size_t>(2) * P * D);
    linear(w.out_w, w.out_b, D, Hd, rows.data(), 2 * P, o.data());
    // reshape(batch, 4, -1).transpose(1, 2) -> [2][D][P]
    for (int b = 0; b < 2; ++b)
        for (int p = 0; p < P; ++p)
            for (int e = 0; e < D; ++e)
                out[(static_cast<std::size_t>(b) * D + e) * P + p] = o[(static_cast<std::size_t>(b) * P + p) * D + e];
    return 0;
}

void sway_t_span(int T, float* out) {
    for (int i = 0; i <= T; ++i) {
        const float t = 1.0f - static_cast<float>(i) / static_cast<float>(T);
        out[i] = t + (std::cos(std::numbers::pi_v<float> * 0.5f * t) - 1.0f + t);
    }
}

int zero_init_steps(int T) { return std::max(1, static_cast<int>((T + 1) * 0.04f)); }

float optimized_scale(const float* positive, const float* negative, int n) {
    double dot = 0.0;
    double norm = 1e-8;
    for (int i = 0; i < n; ++i) {
        dot += static_cast<double>(positive[i]) * negative[i];
        norm += static_cast<double>(negative[i]) * negative[i];
    }
    return static_cast<float>(dot / norm);
}

int cfm_sample(const orc_model* m, const float* mu, const float* cond, const float* noise, int T,
               float cfg, float* out) {
    const orc_desc& d = m->desc;
    const int latent = d.feat_dim * d.patch_size;
    const int Hd2 = 2 * d.dit_hidden;
    std::vector<float> x(noise, noise + latent);
    std::vector<float> x_in(2 * static_cast<std::size_t>(latent)), mu_in(2 * static_cast<std::size_t>(Hd2), 0.0f),
        cond_in(2 * static_cast<std::size_t>(latent)), t_span(static_cast<std::size_t>(T) + 1), est(2 * static_cast<std::size_t>(latent));
    sway_t_span(T, t_span.data());
    std::memcpy(mu_in.data(), mu, sizeof(float) * Hd2);
    std::memcpy(cond_in.data(), cond, sizeof(float) * latent);
    std::memcpy(cond_in.data() + latent, cond, sizeof(float) * latent);
    float t = t_span[0];
    float dt = t_span[0] - t_span[1];
    const int zsteps = zero_init_steps(T);
    const float dt_in[2] = {0.0f, 0.0f};
    for (int step = 1; step <= T; ++step) {
        if (step > zsteps) {
            std::memcpy(x_in.data(), x.data(), sizeof(float) * latent);
            std::memcpy(x_in.data() + latent, x.data(), sizeof(float) * latent);
            const float t_in[2] = {static_cast<float>(step - 1), static_cast<float>(T)};
            dit_estimator(m, x_in.data(), mu_in.data(), t_in, cond_in.data(), dt_in, est.data());
            for (float vv : est)
                if (!std::isfinite(vv)) return -2;  // "dit_estimator produced non-finite values"
            const float* pos = est.data();
            const float* neg = est.data() + latent;
            const float sc = optimized_scale(pos, neg, latent);
            for (int i = 0; i < latent; ++i) {
                const float dphi = neg[i] * sc + cfg * (pos[i] - neg[i] * sc);
                x[static_cast<std::size_t>(i)] -= dt * dphi;
            }
        }
        t -= dt;
        if (step < T) dt = t - t_span[static_cast<std::size_t>(step) + 1];
    }
    std::memcpy(out, x.data(), sizeof(float) * latent);
    return 0;
}

}  // namespace

// ============================================================== C ABI ======
extern "C" {

void orc_set_threads(int threads) {
    g_threads = std::max(1, threads);
#ifdef _OPENMP
    omp_set_num_threads(g_threads);
#endif
}
int orc_get_threads(void) { return g_threads; }

int orc_sdpa(const float* q, int heads, int src, int d, const float* k, const float* v, int groups,
             int cur, int dv, const float* mask, int mask_c, const float* past_k,
             const float* past_v, int past, float scale, float* out, float* out_k, float* out_v) {
    return sdpa_impl(q, heads, src, d, k, v, groups, cur, dv, mask, mask_c, past_k, past_v, past,
                     scale, out, out_k, out_v);
}

void orc_timestep_embedding(const float* in, int batch, int half_dim, float scale,
                            float max_period, int schedule_mode, float* out) {
    timestep_embedding(in, batch, half_dim, scale, max_period, schedule_mode, out);
}

void orc_decoder_mask(int cur, int past, float* out) { decoder_mask(cur, past, out); }

void orc_rope_cache(int head_dim, float theta, int original_max, const float* short_factor,
                    const float* long_factor, int position_start, int length, float* cos_out,
                    float* sin_out) {
    rope_cache(head_dim, theta, original_max, short_factor, long_factor, position_start, length,
               cos_out, sin_out);
}

void orc_sway_t_span(int timesteps, float* out) { sway_t_span(timesteps, out); }
int orc_zero_init_steps(int timesteps) { return zero_init_steps(timesteps); }
float orc_optimized_scale(const float* positive, const float* negative, int n) {
    return optimized_scale(positive, negative, n);
}
int orc_max_patches(int target_text_tokens, int hard_cap) {
    const int text_tokens = std::max(1, target_text_tokens);
    const int cap = static_cast<int>(static_cast<float>(text_tokens) * 6.0f + 10.0f);
    return std::max(1, std::min(hard_cap, cap));
}

void orc_noise_table(uint32_t seed, int patches, int per_patch, float* out) {
    std::mt19937 rng(seed);
    for (int p = 0; p < patches; ++p) {
        std::normal_distribution<float> normal(0.0f, 1.0f);
        for (int i = 0; i < per_patch; ++i) out[static_cast<std::size_t>(p) * per_patch + i] = normal(rng);
    }
}

orc_model* orc_model_create(const orc_desc* desc) {
    if (!desc) return nullptr;
    auto* m = new orc_model;
    m->desc = *desc;
    m->short_factor.assign(static_cast<std::size_t>(desc->head_dim), 1.0f);
    m->dit_factor.assign(static_cast<std::size_t>(std::max(desc->head_dim, desc->dit_hidden)), 1.0f);
    const int layers[2] = {desc->base_layers, desc->res_layers};
    for (int w = 0; w < 2; ++w) {
        m->cache_k[w].resize(static_cast<std::size_t>(layers[w]));
        m->cache_v[w].resize(static_cast<std::size_t>(layers[w]));
    }
    return m;
}

// Synthesizer::Impl::load_manifest keeps setting.rope.short_factor / long_factor
// (synthesizer.cpp:825-830); make_rope_cache picks the long table for a call whose
// last position reaches original_max_position_embeddings (synthesizer.cpp:945-948).
int orc_set_rope_factors(orc_model* m, const float* short_factor, const float* long_factor, int n) {
    const int half = m ? m->desc.head_dim / 2 : 0;
    if (!m || !short_factor || n < half) return -1;  // "rope tables are missing or too short"
    for (int j = 0; j < half; ++j)
        if (!(short_factor[j] > 0.f) || (long_factor && !(long_factor[j] > 0.f))) return -1;
    m->short_factor.assign(short_factor, short_factor + half);
    if (long_factor) m->long_factor.assign(long_factor, long_factor + half);
    else m->long_factor.clear();
    return 0;
}

void orc_model_destroy(orc_model* model) { delete model; }

size_t orc_component_count(const orc_desc* desc, int component) {
    return desc ? component_count(*desc, component) : 0;
}

int orc_set_weights(orc_model* m, int component, const uint16_t* fp16, size_t count) {
    if (!m || !fp16 || component < 0 || component > 8) return -1;
    if (count != component_count(m->desc, component)) return -1;
    m->blob[component] = fp16;
    Cursor c{fp16};
    if (component == 1) m->base = carve_decoder(c, base_shape(m->desc));
    if (component == 2) m->res = carve_decoder(c, res_shape(m->desc));
    if (component == 8) m->dit = carve_dit(c, m->desc);
    return 0;
}

void orc_reset_caches(orc_model* m) {
    for (int w = 0; w < 2; ++w) {
        for (auto& x : m->cache_k[w]) x.clear();
        for (auto& x : m->cache_v[w]) x.clear();
        m->tokens[w] = 0;
    }
}

int orc_token_count(const orc_model* m, int which) { return m->tokens[which]; }

int orc_read_cache(const orc_model* m, int which, int layer, float* k, float* v) {
    if (which < 0 || which > 1 || layer < 0 ||
        layer >= static_cast<int>(m->cache_k[which].size()))
        return -1;
    std::memcpy(k, m->cache_k[which][layer].data(), sizeof(float) * m->cache_k[which][layer].size());
    std::memcpy(v, m->cache_v[which][layer].data(), sizeof(float) * m->cache_v[which][layer].size());
    return 0;
}

int orc_decoder_forward(orc_model* m, int which, const float* embed, int n, const float* mask,
                        const float* cos, const float* sin, float* out) {
    if (!m || which < 0 || which > 1 || n <= 0 || !m->blob[1 + which]) return -1;
    decoder_forward(m, which, embed, n, mask, cos, sin, out);
    return 0;
}

int orc_text_embed(const orc_model* m, const int32_t* ids, int n, float* out) {
    const int H = m->desc.hidden;
    if (!m->blob[0]) return -1;
    for (int i = 0; i < n; ++i) {
        if (ids[i] < 0 || ids[i] >= m->desc.vocab) return -1;
        const uint16_t* row = m->blob[0] + static_cast<std::size_t>(ids[i]) * H;
        for (int e = 0; e < H; ++e) out[static_cast<std::size_t>(i) * H + e] = h2f(row[e]) * m->desc.embed_scale;
    }
    return 0;
}

int orc_fsq(const orc_model* m, const float* in, int rows, float* out) {
    const orc_desc& d = m->desc;
    const uint16_t* b = m->blob[3];
    if (!b) return -1;
    const std::size_t H = d.hidden, Q = d.fsq_dim;
    const uint16_t *in_w = b, *in_b = b + Q * H, *out_w = in_b + Q, *out_b = out_w + H * Q;
    std::vector<float> z(static_cast<std::size_t>(rows) * Q);
    linear(in_w, in_b, static_cast<int>(Q), static_cast<int>(H), in, rows, z.data());
    for (float& v : z) v = std::tanh(v) * d.fsq_scale;
    for (int r = 0; r < rows && m->fsq_log && m->fsq_log_n < m->fsq_log_cap; ++r, ++m->fsq_log_n)
        std::memcpy(m->fsq_log + static_cast<std::size_t>(m->fsq_log_n) * Q, z.data() + r * Q, sizeof(float) * Q);
    for (int r = 0; r < rows; ++r) {
        const bool forced = m->fsq_force && m->fsq_force_n < m->fsq_force_cap;
        const float* code = forced ? m->fsq_force + static_cast<std::size_t>(m->fsq_force_n) * Q : nullptr;
        for (std::size_t j = 0; j < Q; ++j) {
            float& v = z[r * Q + j];
            v = (forced ? code[j] : std::nearbyint(v)) / d.fsq_scale;
        }
        if (forced) ++m->fsq_force_n;
    }
    linear(out_w, out_b, static_cast<int>(H), static_cast<int>(Q), z.data(), rows, out);
    return 0;
}

int orc_fusion_proj(const orc_model* m, const float* lm, const float* feat, int rows, float* out) {
    const uint16_t* b = m->blob[4];
    if (!b) return -1;
    const std::size_t H = m->desc.hidden;
    std::vector<float> cat(static_cast<std::size_t>(rows) * 2 * H);
    for (int r = 0; r < rows; ++r) {
        std::memcpy(&cat[static_cast<std::size_t>(r) * 2 * H], lm + r * H, sizeof(float) * H);
        std::memcpy(&cat[static_cast<std::size_t>(r) * 2 * H + H], feat + r * H, sizeof(float) * H);
    }
    linear(b, b + H * 2 * H, static_cast<int>(H), static_cast<int>(2 * H), cat.data(), rows, out);
    return 0;
}

int orc_dit_proj(const orc_model* m, const float* lm, const float* res, float* out) {
    const uint16_t* b = m->blob[5];
    if (!b) return -1;
    const std::size_t H = m->desc.hidden, Hd = m->desc.dit_hidden;
    const uint16_t *lw = b, *lb = lw + Hd * H, *rw = lb + Hd, *rb = rw + Hd * H;
    linear(lw, lb, static_cast<int>(Hd), static_cast<int>(H), lm, 1, out);
    linear(rw, rb, static_cast<int>(Hd), static_cast<int>(H), res, 1, out + Hd);
    return 0;
}

int orc_stop_head(const orc_model* m, const float* hidden, float* logits) {
    const uint16_t* b = m->blob[6];
    if (!b) return -1;
    const std::size_t H = m->desc.hidden;
    std::vector<float> mid(H);
    linear(b, b + H * H, static_cast<int>(H), static_cast<int>(H), hidden, 1, mid.data());
    for (float& v : mid) v = silu(v);
    linear(b + H * H + H, nullptr, 2, static_cast<int>(H), mid.data(), 1, logits);
    return 0;
}

int orc_feat_encoder(const orc_model* m, const float* latent_dp, float* out) {
    const uint16_t* b = m->blob[7];
    if (!b) return -1;
    const orc_desc& d = m->desc;
    const std::size_t H = d.hidden, D = d.feat_dim, P = d.patch_size;
    // make_feat_encoder_input: values[p*D + d] = latent[d*P + p]
    std::vector<float> frames(P * D), mid(H);
    for (std::size_t e = 0; e < D; ++e)
        for (std::size_t p = 0; p < P; ++p) frames[p * D + e] = latent_dp[e * P + p];
    const uint16_t *in_w = b, *in_b = in_w + H * P * D, *o_w = in_b + H, *o_b = o_w + H * H;
    linear(in_w, in_b, static_cast<int>(H), static_cast<int>(P * D), frames.data(), 1, mid.data());
    for (float& v : mid) v = silu(v);
    linear(o_w, o_b, static_cast<int>(H), static_cast<int>(H), mid.data(), 1, out);
    return 0;
}

int orc_dit_estimator(const orc_model* m, const float* x_in, const float* mu_in, const float* t_in,
                      const float* cond_in, const float* dt_in, float* out) {
    if (!m || !m->blob[8]) return -1;
    return dit_estimator(m, x_in, mu_in, t_in, cond_in, dt_in, out);
}

int orc_cfm_sample(const orc_model* m, const float* mu, const float* cond, const float* noise,
                   int timesteps, float cfg, float* out_latent) {
    if (!m || !m->blob[8] || timesteps <= 0) return -1;
    return cfm_sample(m, mu, cond, noise, timesteps, cfg, out_latent);
}

}  // extern "C"

namespace {

// generate_with_caches after the prefix is built (synthesizer.cpp:403-659): rows are
// token rows (embedded by text_embed) or audio rows (latent patch, d-major; embedded
// by feat_encoder, :415-443); the base decoder runs over all rows, audio rows of the
// LM hidden take the FSQ output (:476-495), the residual decoder reads
// fusion_proj(lm, feat) (:497-509), and the first patch is conditioned on the last
// row's latent when that row is audio (:444-447). n_target_text sizes max_patches.
int generate_prefix(orc_model* m, const std::vector<int32_t>& ids, const std::vector<int>& is_audio,
                    const std::vector<const float*>& audio, int n_target_text, int min_patches, int timesteps,
                    float cfg, int max_patches_override, uint32_t seed, float* latents, float* lm_trace,
                    float* res_trace, float* stop_trace, int* out_patches) {
    const orc_desc& d = m->desc;
    const int H = d.hidden, latent = d.feat_dim * d.patch_size;
    const int L = static_cast<int>(ids.size());
    std::vector<float> embed(static_cast<std::size_t>(L) * H), resfeat(static_cast<std::size_t>(L) * H, 0.0f);
    if (orc_text_embed(m, ids.data(), L, embed.data()) != 0) return -1;
    for (int i = 0; i < L; ++i)
        if (is_audio[static_cast<std::size_t>(i)]) {
            float* row = embed.data() + static_cast<std::size_t>(i) * H;
            orc_feat_encoder(m, audio[static_cast<std::size_t>(i)], row);
            std::memcpy(resfeat.data() + static_cast<std::size_t>(i) * H, row, sizeof(float) * H);
        }
    orc_reset_caches(m);
    std::vector<float> lm_prefix(embed.size()), res_in(embed.size()), res_hidden(embed.size()), fsq_row(H);
    decoder_forward(m, 0, embed.data(), L, nullptr, nullptr, nullptr, lm_prefix.data());
    for (int i = 0; i < L; ++i)
        if (is_audio[static_cast<std::size_t>(i)]) {
            float* row = lm_prefix.data() + static_cast<std::size_t>(i) * H;
            orc_fsq(m, row, 1, fsq_row.data());
            std::memcpy(row, fsq_row.data(), sizeof(float) * H);
        }
    orc_fusion_proj(m, lm_prefix.data(), resfeat.data(), L, res_in.data());
    decoder_forward(m, 1, res_in.data(), L, nullptr, nullptr, nullptr, res_hidden.data());
    std::vector<float> cur_lm(lm_prefix.end() - H, lm_prefix.end());
    std::vector<float> cur_res(res_hidden.end() - H, res_hidden.end());

    int max_patches = orc_max_patches(n_target_text, d.max_generation_patches);
    if (max_patches_override > 0) max_patches = std::min(max_patches, max_patches_override);
    std::mt19937 rng(seed);
    std::vector<std::vector<float>> patches;
    std::vector<float> init_cond(static_cast<std::size_t>(latent), 0.0f);
    if (is_audio.back()) std::memcpy(init_cond.data(), audio.back(), sizeof(float) * latent);
    std::vector<float> dit_hidden(2 * static_cast<std::size_t>(d.dit_hidden)), noise(static_cast<std::size_t>(latent)),
        lat(static_cast<std::size_t>(latent)), feat(static_cast<std::size_t>(H)), base_out(static_cast<std::size_t>(H)),
        fus(static_cast<std::size_t>(H));
    float logits[2];
    for (int step = 0; step < max_patches; ++step) {
        if (L + static_cast<int>(patches.size()) >= d.rope_original_max) return -3;
        orc_dit_proj(m, cur_lm.data(), cur_res.data(), dit_hidden.data());
        const std::vector<float>& cond = patches.empty() ? init_cond : patches.back();
        std::normal_distribution<float> normal(0.0f, 1.0f);
        for (float& v : noise) v = normal(rng);
        const int rc = cfm_sample(m, dit_hidden.data(), cond.data(), noise.data(), timesteps, cfg, lat.data());
        if (rc != 0) return rc;
        patches.push_back(lat);
        orc_stop_head(m, cur_lm.data(), logits);
        if (latents) std::memcpy(latents + static_cast<std::size_t>(step) * latent, lat.data(), sizeof(float) * latent);
        if (lm_trace) std::memcpy(lm_trace + static_cast<std::size_t>(step) * H, cur_lm.data(), sizeof(float) * H);
        if (res_trace) std::memcpy(res_trace + static_cast<std::size_t>(step) * H, cur_res.data(), sizeof(float) * H);
        if (stop_trace) {
            stop_trace[2 * step] = logits[0];
            stop_trace[2 * step + 1] = logits[1];
        }
        if (step > min_patches && logits[1] > logits[0]) break;
        orc_feat_encoder(m, lat.data(), feat.data());
        decoder_forward(m, 0, feat.data(), 1, nullptr, nullptr, nullptr, base_out.data());
        orc_fsq(m, base_out.data(), 1, cur_lm.data());
        orc_fusion_proj(m, cur_lm.data(), feat.data(), 1, fus.data());
        decoder_forward(m, 1, fus.data(), 1, nullptr, nullptr, nullptr, cur_res.data());
    }
    *out_patches = static_cast<int>(patches.size());
    return 0;
}

bool all_loaded(const orc_model* m) {
    for (int c = 0; c <= 8; ++c)
        if (!m->blob[c]) return false;
    return true;
}

}  // namespace

extern "C" {

// Test hook: record the pre-rounding FSQ values (tanh(z) * fsq_scale, [rows][fsq_dim])
// of the next 'rows' FSQ rows the model computes into buf (NULL stops recording).
// Returns the number of rows recorded so far by the previous call's buffer.
int orc_trace_fsq(orc_model* m, float* buf, int rows) {
    const int n = m->fsq_log_n;
    m->fsq_log = buf;
    m->fsq_log_cap = buf ? rows : 0;
    m->fsq_log_n = 0;
    return n;
}

// Test hook: the next 'rows' FSQ rows the model computes take their codes from
// codes [rows][fsq_dim] (integers, the rounded tanh(z) * fsq_scale) instead of
// rounding their own values; NULL stops. Returns the rows the previous buffer served.
int orc_force_fsq(orc_model* m, const float* codes, int rows) {
    const int n = m->fsq_force_n;
    m->fsq_force = codes;
    m->fsq_force_cap = codes ? rows : 0;
    m->fsq_force_n = 0;
    return n;
}

int orc_generate(orc_model* m, const int32_t* text_ids, int n_text, int min_patches,
                 int timesteps, float cfg, int max_patches_override, uint32_t seed,
                 float* latents, float* lm_trace, float* res_trace, float* stop_trace,
                 int* out_patches) {
    if (!all_loaded(m) || n_text <= 0 || timesteps <= 0) return -1;
    // text-only prefix = target ids + audio_start (synthesizer.cpp:387-390)
    std::vector<int32_t> ids(text_ids, text_ids + n_text);
    ids.push_back(m->desc.audio_start_token);
    const std::vector<int> is_audio(ids.size(), 0);
    const std::vector<const float*> audio(ids.size(), nullptr);
    return generate_prefix(m, ids, is_audio, audio, n_text, min_patches, timesteps, cfg, max_patches_override, seed,
                           latents, lm_trace, res_trace, stop_trace, out_patches);
}

// A prefix given row by row (the reference's PrefixRow list, synthesizer.cpp:43-47,
// 359-400): token ids of every row (audio rows' ids are embedded and then replaced),
// is_audio flags, and the audio rows' latent patches in row order ([n_audio][D*P], d-major).
int orc_generate_rows(orc_model* m, const int32_t* token_ids, const int32_t* is_audio, const float* audio_latents,
                      int n_rows, int n_target_text, int min_patches, int timesteps, float cfg,
                      int max_patches_override, uint32_t seed, float* latents, float* lm_trace, float* res_trace,
                      float* stop_trace, int* out_patches) {
    if (!all_loaded(m) || n_rows <= 0 || n_target_text <= 0 || timesteps <= 0 || !token_ids || !is_audio) return -1;
    const int latent = m->desc.feat_dim * m->desc.patch_size;
    std::vector<int32_t> ids(token_ids, token_ids + n_rows);
    std::vector<int> flags(static_cast<std::size_t>(n_rows));
    std::vector<const float*> audio(static_cast<std::size_t>(n_rows), nullptr);
    int a = 0;
    for (int i = 0; i < n_rows; ++i) {
        flags[static_cast<std::size_t>(i)] = is_audio[i] != 0;
        if (is_audio[i]) {
            if (!audio_latents) return -1;
            audio[static_cast<std::size_t>(i)] = audio_latents + static_cast<std::size_t>(a++) * latent;
        }
    }
    return generate_prefix(m, ids, flags, audio, n_target_text, min_patches, timesteps, cfg, max_patches_override,
                           seed, latents, lm_trace, res_trace, stop_trace, out_patches);
}

}  // extern "C"
