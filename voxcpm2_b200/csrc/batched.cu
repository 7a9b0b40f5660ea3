// Token-batched kernels: prompt prefill rows and the DiT estimator's 2 x 11 tokens.
//
// The DiT estimator (tools/export_components.py:602-689) runs its decoder over
// two 11-token sequences per call: [mu(2), time(1), cond(4), x(4)] for the
// conditional and the unconditional CFG row. Prefill runs the decoders over
// the whole prompt (synthesizer.cpp:455-525). Both are weight-streaming
// products with a handful of token rows; this file holds the CUDA-core version
// of those products plus the row-wise RMSNorm, RoPE/append and attention
// kernels around them, and the DiT embedding / output / CFG step.
#include <algorithm>
#include <cfloat>
#include <stdexcept>

#include "kernels.cuh"

namespace vxc {
namespace {

cudaLaunchConfig_t make_cfg(dim3 grid, dim3 block, size_t smem, cudaStream_t s, bool pdl,
                            cudaLaunchAttribute* attr) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cfg;
}

void check_launch(cudaError_t e) {
    if (e != cudaSuccess) throw std::runtime_error(cudaGetErrorString(e));
}

__device__ __forceinline__ bool stopped(const StreamCtl* ctl, int skip) { return skip && ctl && ctl->stopped; }

// ------------------------------------------------------- rows linear ------
constexpr int kRowsWarps = 4;
constexpr int kRowsTile = 8;  // token rows per CTA

template <int MODE>
__global__ void __launch_bounds__(kRowsWarps * kWarp) rows_linear_kernel(const RowsArgs a) {
    pdl_launch_dependents();
    pdl_wait();
    if (stopped(a.ctl, a.skip_if_stopped)) return;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int item = blockIdx.x * kRowsWarps + warp;
    int row[4];
    bool valid[4];
    if constexpr (MODE == GEMV_GATEUP) {
        const int p0 = item * 2;
#pragma unroll
        for (int i = 0; i < 2; ++i) {
            valid[i] = valid[i + 2] = p0 + i < a.rows;
            row[i] = p0 + i;
            row[i + 2] = a.rows + p0 + i;
        }
    } else {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            row[i] = item * 4 + i;
            valid[i] = row[i] < a.rows;
        }
    }
    if (!valid[0]) return;
    const int m0 = blockIdx.y * kRowsTile;
    const int mt = min(kRowsTile, a.M - m0);
    const int K = a.K;
    float acc[4][kRowsTile];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < kRowsTile; ++j) acc[i][j] = 0.f;

    for (int e = lane * 8; e < K; e += kWarp * 8) {
        uint4 w[4];
#pragma unroll
        for (int i = 0; i < 4; ++i)
            w[i] = valid[i] ? __ldg(reinterpret_cast<const uint4*>(a.w + static_cast<size_t>(row[i]) * K + e))
                            : make_uint4(0, 0, 0, 0);
#pragma unroll
        for (int j = 0; j < kRowsTile; ++j) {
            if (j < mt) {
                const float* xr = a.x + static_cast<size_t>(m0 + j) * a.ldx + e;
                const float4 x0 = *reinterpret_cast<const float4*>(xr);
                const float4 x1 = *reinterpret_cast<const float4*>(xr + 4);
#pragma unroll
                for (int i = 0; i < 4; ++i) acc[i][j] = dot8(w[i], x0, x1, acc[i][j]);
            }
        }
    }
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < kRowsTile; ++j) acc[i][j] = warp_sum(acc[i][j]);
    if (lane != 0) return;
    for (int j = 0; j < mt; ++j) {
        float* yr = a.y + static_cast<size_t>(m0 + j) * a.ldy;
        if constexpr (MODE == GEMV_GATEUP) {
#pragma unroll
            for (int i = 0; i < 2; ++i)
                if (valid[i]) yr[row[i]] = silu(acc[i][j]) * acc[i + 2][j];
        } else {
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                if (!valid[i]) continue;
                if constexpr (MODE == GEMV_RESID) {
                    yr[row[i]] = yr[row[i]] + (a.rscale == 1.f ? acc[i][j] : acc[i][j] * a.rscale);
                } else {
                    float v = acc[i][j] + (a.bias ? __half2float(a.bias[row[i]]) : 0.f);
                    if (a.act == ACT_SILU) v = silu(v);
                    yr[row[i]] = v;
                }
            }
        }
    }
}

__global__ void rmsnorm_rows_kernel(const float* x, int ldx, const __half* g, float eps, int K,
                                    float* out, int ldo, StreamCtl* ctl, int skip) {
    __shared__ float red[32];
    pdl_launch_dependents();
    pdl_wait();
    if (stopped(ctl, skip)) return;
    const float* xr = x + static_cast<size_t>(blockIdx.x) * ldx;
    float ss = 0.f;
    for (int k = threadIdx.x; k < K; k += blockDim.x) ss += xr[k] * xr[k];
    ss = warp_sum(ss);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    float t = 0.f;
    for (int w = 0; w < static_cast<int>(blockDim.x >> 5); ++w) t += red[w];
    const float a = g ? rsqrtf(t / static_cast<float>(K) + eps) : 1.f;
    float* orow = out + static_cast<size_t>(blockIdx.x) * ldo;
    for (int k = threadIdx.x; k < K; k += blockDim.x) orow[k] = xr[k] * a * __half2float(g[k]);
}

__global__ void qkv_rows_post_kernel(float* qkv, int q_heads, int kv_heads, int d, int past,
                                     int pos_mod, const float* rope_cos, const float* rope_sin,
                                     float* k_cache, float* v_cache, int cap, StreamCtl* ctl) {
    pdl_launch_dependents();
    pdl_wait();
    const int m = blockIdx.x;
    const int width = (q_heads + 2 * kv_heads) * d;
    float* row = qkv + static_cast<size_t>(m) * width;
    const int pos = past + (m % pos_mod);
    const int half = d / 2;
    const int pairs = (q_heads + 2 * kv_heads) * half;
    for (int it = threadIdx.x; it < pairs; it += blockDim.x) {
        const int hh = it / half, j = it - hh * half;
        float* p = row + hh * d;
        float a0 = p[j], a1 = p[j + half];
        const bool is_v = hh >= q_heads + kv_heads;
        if (!is_v && rope_cos) {
            const float* c = rope_cos + static_cast<size_t>(pos) * d;
            const float* s = rope_sin + static_cast<size_t>(pos) * d;
            const float o0 = a0 * c[j] + (-a1) * s[j];
            const float o1 = a1 * c[j + half] + a0 * s[j + half];
            a0 = o0;
            a1 = o1;
            p[j] = a0;
            p[j + half] = a1;
        }
        if (k_cache && hh >= q_heads) {
            const int crow = past + m;
            if (crow >= cap) {
                if (ctl) ctl->error = 1;
                continue;
            }
            const int kvh = is_v ? hh - q_heads - kv_heads : hh - q_heads;
            float* dst = (is_v ? v_cache : k_cache) + (static_cast<size_t>(kvh) * cap + crow) * d;
            dst[j] = a0;
            dst[j + half] = a1;
        }
    }
}


// Prefill attention over the cached keys (the rows' own K/V already appended by
// qkv_rows_post): query row m sees keys 0 .. past + m (causal, kvcache.cpp:216-230).
// One CTA per (KV head, block of rb query rows): its rb x G query vectors (at most
// 16) spread over 8 warps. Keys are walked in 32-key tiles staged by cp.async into
// two buffers; lane j holds key j's row in registers and scores it against each of
// its warp's vectors; each vector keeps an online softmax (running max and sum) and
// two output columns per lane, the probabilities broadcast by shuffles.
constexpr int kPfThreads = 256, kPfWarps = 8, kPfVectors = 16, kPfPer = kPfVectors / kPfWarps, kPfMaxGroup = 16;
constexpr int kPfKeys = 32, kPfKRow = 68;

__device__ __forceinline__ void pf_cp_async16(void* smem_dst, const void* gsrc) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(static_cast<uint32_t>(__cvta_generic_to_shared(
                     smem_dst))),
                 "l"(gsrc)
                 : "memory");
}

__global__ void __launch_bounds__(kPfThreads) attn_prefill_kernel(const float* qkv, int M, int q_heads, int kv_heads,
                                                                 int past, const float* k_cache, const float* v_cache,
                                                                 int cap, float scale, float* out, int rb) {
    constexpr int D = 64;
    __shared__ __align__(16) float ks[2][kPfKeys][kPfKRow];
    __shared__ __align__(16) float vs[2][kPfKeys][D];
    __shared__ __align__(16) float qs[kPfVectors][D];
    const int kvh = blockIdx.x, r0 = blockIdx.y * rb, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int G = q_heads / kv_heads, nv = min(rb, M - r0) * G;  // this CTA's query vectors: v -> (row v / G, head v % G)
    const int width = (q_heads + 2 * kv_heads) * D;
    for (int i = tid; i < nv * D; i += kPfThreads) {
        const int v = i / D, e = i - v * D;
        const int m = r0 + v / G, hh = kvh * G + v % G;
        qs[v][e] = qkv[static_cast<size_t>(m) * width + hh * D + e] * scale;
    }
    const int T = past + min(M, r0 + rb);  // keys of the block's last row
    const float* kb = k_cache + static_cast<size_t>(kvh) * cap * D;
    const float* vb = v_cache + static_cast<size_t>(kvh) * cap * D;
    auto stage = [&](int buf, int tb) {
        const int nt = min(kPfKeys, T - tb);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int i = tid + j * kPfThreads;  // 0 .. 1023
            const int kv = i >> 9, r = (i >> 4) & 31, c = (i & 15) * 4;
            if (r < nt) {
                const float* src = (kv == 0 ? kb : vb) + static_cast<size_t>(tb + r) * D + c;
                pf_cp_async16(kv == 0 ? &ks[buf][r][c] : &vs[buf][r][c], src);
            }
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
    };
    float m_run[kPfPer], l_run[kPfPer], acc[kPfPer][2];
#pragma unroll
    for (int i = 0; i < kPfPer; ++i) {
        m_run[i] = -1e30f;
        l_run[i] = 0.f;
        acc[i][0] = acc[i][1] = 0.f;
    }
    stage(0, 0);
    asm volatile("cp.async.wait_group 0;" ::: "memory");
    __syncthreads();  // query vectors and the first tile staged
    for (int tb = 0, buf = 0; tb < T; tb += kPfKeys, buf ^= 1) {
        if (tb + kPfKeys < T) stage(buf ^ 1, tb + kPfKeys);
        const int nt = min(kPfKeys, T - tb);
        float kr[D];
        if (lane < nt) {
#pragma unroll
            for (int c = 0; c < D; c += 4) {
                const float4 k4 = *reinterpret_cast<const float4*>(&ks[buf][lane][c]);
                kr[c] = k4.x;
                kr[c + 1] = k4.y;
                kr[c + 2] = k4.z;
                kr[c + 3] = k4.w;
            }
        }
#pragma unroll
        for (int i = 0; i < kPfPer; ++i) {
            const int v = warp + i * kPfWarps;
            if (v >= nv) break;
            const int lim = past + r0 + v / G;  // the last key this row sees
            if (tb > lim) continue;             // (warp-uniform) a fully masked tile
            float x = -1e30f;
            if (lane < nt && tb + lane <= lim) {
                float s4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
                for (int c = 0; c < D; c += 4) {
                    const float4 q4 = *reinterpret_cast<const float4*>(&qs[v][c]);
                    s4[0] = fmaf(q4.x, kr[c], s4[0]);
                    s4[1] = fmaf(q4.y, kr[c + 1], s4[1]);
                    s4[2] = fmaf(q4.z, kr[c + 2], s4[2]);
                    s4[3] = fmaf(q4.w, kr[c + 3], s4[3]);
                }
                x = (s4[0] + s4[1]) + (s4[2] + s4[3]);
            }
            const float m_new = fmaxf(m_run[i], warp_max(x));
            const float p = x > -1e29f ? __expf(x - m_new) : 0.f;
            const float alpha = __expf(m_run[i] - m_new);
            l_run[i] = l_run[i] * alpha + warp_sum(p);
            m_run[i] = m_new;
            float o0 = acc[i][0] * alpha, o1 = acc[i][1] * alpha;
            const int nk = min(nt, lim - tb + 1);
            for (int j = 0; j < nk; ++j) {
                const float pj = __shfl_sync(0xffffffffu, p, j);
                const float2 v2 = *reinterpret_cast<const float2*>(&vs[buf][j][2 * lane]);
                o0 = fmaf(pj, v2.x, o0);
                o1 = fmaf(pj, v2.y, o1);
            }
            acc[i][0] = o0;
            acc[i][1] = o1;
        }
        asm volatile("cp.async.wait_group 0;" ::: "memory");
        __syncthreads();  // this tile consumed, the next one staged
    }
#pragma unroll
    for (int i = 0; i < kPfPer; ++i) {
        const int v = warp + i * kPfWarps;
        if (v >= nv) break;
        const int m = r0 + v / G, hh = kvh * G + v % G;
        const float inv = 1.f / l_run[i];
        *reinterpret_cast<float2*>(out + static_cast<size_t>(m) * q_heads * D + hh * D + 2 * lane) =
            make_float2(acc[i][0] * inv, acc[i][1] * inv);
    }
}

// split-fp16 operand row m: fp16(v) in row m, fp16(v - fp16(v)) in row lo + m
__device__ __forceinline__ void split_store(__half* xb, int ld, int m, int col, float v, int lo = 24) {
    const __half hi = __float2half_rn(v);
    xb[static_cast<size_t>(m) * ld + col] = hi;
    xb[static_cast<size_t>(lo + m) * ld + col] = __float2half_rn(v - __half2float(hi));
}

// One CTA per token row: RMSNorm (x * rsqrt(mean(x^2) + eps) * g) written as the
// tensor-core linears' split-fp16 operand. Every thread issues its loads of the
// row and of g in one batch before any arithmetic (each global round trip costs
// about a microsecond), then one block reduction.
constexpr int kNormThreads = 256;
constexpr int kNormBatch = 4;  // float4 per thread in flight: rows up to 4096 in one batch

// g == nullptr: no normalisation (a plain split of the rows); lo: row offset of the residual half
__global__ void __launch_bounds__(kNormThreads) rmsnorm_rows_split_kernel(const float* x, int ldx, const __half* g,
                                                                         float eps, int K, __half* xb,
                                                                         StreamCtl* ctl, int lo) {
    __shared__ float red[kNormThreads / 32];
    pdl_launch_dependents();
    const int m = blockIdx.x, tid = threadIdx.x, n4 = K / 4;
    // g does not depend on the previous kernel
    uint2 gw[kNormBatch];
#pragma unroll
    for (int i = 0; i < kNormBatch; ++i) {
        const int u = tid + kNormThreads * i;
        gw[i] = u < n4 && g ? __ldg(reinterpret_cast<const uint2*>(g) + u) : make_uint2(0x3c003c00u, 0x3c003c00u);
    }
    pdl_wait();
    const bool stop = ctl && ctl->stopped;  // read beside the row; nothing is written before the check
    const float4* xr = reinterpret_cast<const float4*>(x + static_cast<size_t>(m) * ldx);
    float4 v[kNormBatch];
#pragma unroll
    for (int i = 0; i < kNormBatch; ++i) {
        const int u = tid + kNormThreads * i;
        v[i] = u < n4 ? xr[u] : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < kNormBatch; ++i) ss += v[i].x * v[i].x + v[i].y * v[i].y + v[i].z * v[i].z + v[i].w * v[i].w;
    ss = warp_sum(ss);
    if ((tid & 31) == 0) red[tid >> 5] = ss;
    if (stop) return;
    __syncthreads();
    float t = 0.f;
#pragma unroll
    for (int w = 0; w < kNormThreads / 32; ++w) t += red[w];
    const float a = g ? rsqrtf(t / static_cast<float>(K) + eps) : 1.f;
#pragma unroll
    for (int i = 0; i < kNormBatch; ++i) {
        const int u = tid + kNormThreads * i;
        if (u < n4) {
            const float2 g01 = __half22float2(*reinterpret_cast<const __half2*>(&gw[i].x));
            const float2 g23 = __half22float2(*reinterpret_cast<const __half2*>(&gw[i].y));
            split_store(xb, K, m, 4 * u, v[i].x * a * g01.x, lo);
            split_store(xb, K, m, 4 * u + 1, v[i].y * a * g01.y, lo);
            split_store(xb, K, m, 4 * u + 2, v[i].z * a * g23.x, lo);
            split_store(xb, K, m, 4 * u + 3, v[i].w * a * g23.y, lo);
        }
    }
}

// One CTA per (head, sequence): RoPE on q/k (apply_rotary_pos_emb, rotate_half),
// scores, softmax and P.V for the sequence's rows (VoxCPM2SDPA without mask or
// cache, voxcpm2_sdpa.cpp:187-252), written as the o projection's split operand.
// Every load after the dependency wait (the stop flag and the head's q/k/v rows)
// is issued in one batch; each thread rotates the (e, e + 32) column pairs it
// loaded in registers before staging them. Warp i then owns query row i from
// end to end (lane j scores key j, the softmax across the lanes, lane c forms
// output columns 2c and 2c + 1), so only one block barrier follows the staging,
// and the outputs leave as fp16 pairs.
constexpr int kDitMaxSeq = 16;
constexpr int kDitThreads = 32 * kDitMaxSeq;  // a warp per query row
constexpr int kDitRow = 68;  // staged q/k/v row: 16-byte aligned, at most two-way bank conflicts
__global__ void __launch_bounds__(kDitThreads) dit_attention_split_kernel(const float* qkv, int seq, int q_heads,
                                                                          int kv_heads, const float* rope_cos,
                                                                          const float* rope_sin, float scale,
                                                                          __half* xb, StreamCtl* ctl, int lo) {
    constexpr int D = 64, H = 32;
    __shared__ __align__(16) float qs[kDitMaxSeq][kDitRow], ks[kDitMaxSeq][kDitRow], vs[kDitMaxSeq][kDitRow];
    __shared__ float ps[kDitMaxSeq][kDitMaxSeq];
    pdl_launch_dependents();
    const int h = blockIdx.x, sq = blockIdx.y, kvh = h / (q_heads / kv_heads), tid = threadIdx.x;
    const int lane = tid & 31, warp = tid >> 5;
    const int width = (q_heads + 2 * kv_heads) * D;
    // unit tid: row r = tid / 24, kind (q, k, v) = (tid % 24) / 8, columns 4c .. 4c + 3 and
    // 32 + 4c .. 32 + 4c + 3. Its RoPE factors do not depend on the previous kernel.
    const bool unit = tid < seq * 24;
    const int r = tid / 24, w = tid - r * 24, kind = w >> 3, c4 = (w & 7) * 4;
    float4 c0 = {}, s0 = {}, c1 = {}, s1 = {};
    if (unit && kind < 2) {
        c0 = __ldg(reinterpret_cast<const float4*>(rope_cos + r * D + c4));
        s0 = __ldg(reinterpret_cast<const float4*>(rope_sin + r * D + c4));
        c1 = __ldg(reinterpret_cast<const float4*>(rope_cos + r * D + c4 + H));
        s1 = __ldg(reinterpret_cast<const float4*>(rope_sin + r * D + c4 + H));
    }
    pdl_wait();
    const bool stop = ctl && ctl->stopped;  // read beside the rows; nothing is written before the check
    if (unit) {
        const int col = kind == 0 ? h * D : kind == 1 ? (q_heads + kvh) * D : (q_heads + kv_heads + kvh) * D;
        const float* src = qkv + static_cast<size_t>(sq * seq + r) * width + col + c4;
        float4 a = *reinterpret_cast<const float4*>(src);
        float4 b = *reinterpret_cast<const float4*>(src + H);
        if (kind < 2) {  // rotate_half: x[e] cos[e] - x[e + 32] sin[e]; x[e + 32] cos[e + 32] + x[e] sin[e + 32]
            const float4 ra = make_float4(a.x * c0.x + (-b.x) * s0.x, a.y * c0.y + (-b.y) * s0.y,
                                          a.z * c0.z + (-b.z) * s0.z, a.w * c0.w + (-b.w) * s0.w);
            const float4 rb = make_float4(b.x * c1.x + a.x * s1.x, b.y * c1.y + a.y * s1.y, b.z * c1.z + a.z * s1.z,
                                          b.w * c1.w + a.w * s1.w);
            a = ra;
            b = rb;
        }
        float* dst = kind == 0 ? qs[r] : kind == 1 ? ks[r] : vs[r];
        *reinterpret_cast<float4*>(dst + c4) = a;
        *reinterpret_cast<float4*>(dst + c4 + H) = b;
    }
    if (stop) return;
    __syncthreads();
    const int i = warp;  // query row
    if (i >= seq) return;
    float x = -FLT_MAX;
    if (lane < seq) {
        float s4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int c = 0; c < D; c += 4) {
            const float4 q4 = *reinterpret_cast<const float4*>(&qs[i][c]);
            const float4 k4 = *reinterpret_cast<const float4*>(&ks[lane][c]);
            s4[0] = fmaf(q4.x, k4.x, s4[0]);
            s4[1] = fmaf(q4.y, k4.y, s4[1]);
            s4[2] = fmaf(q4.z, k4.z, s4[2]);
            s4[3] = fmaf(q4.w, k4.w, s4[3]);
        }
        x = ((s4[0] + s4[1]) + (s4[2] + s4[3])) * scale;
    }
    const float mx = warp_max(x);
    const float p = lane < seq ? expf(x - mx) : 0.f;
    const float sum = warp_sum(p);
    if (lane < seq) ps[i][lane] = p / sum;
    __syncwarp();
    // P.V: lane c -> output columns 2c, 2c + 1; hi and lo halves stored as fp16 pairs
    const int e = lane * 2;
    float a0 = 0.f, a1 = 0.f;
    for (int j = 0; j < seq; ++j) {
        const float pj = ps[i][j];
        const float2 v2 = *reinterpret_cast<const float2*>(&vs[j][e]);
        a0 = fmaf(pj, v2.x, a0);
        a1 = fmaf(pj, v2.y, a1);
    }
    const __half2 hi = __floats2half2_rn(a0, a1);
    const float2 hf = __half22float2(hi);
    const __half2 lw = __floats2half2_rn(a0 - hf.x, a1 - hf.y);
    const size_t ld = static_cast<size_t>(q_heads) * D, row = static_cast<size_t>(sq * seq + i);
    const size_t col = static_cast<size_t>(h * D + e);
    *reinterpret_cast<__half2*>(xb + row * ld + col) = hi;
    *reinterpret_cast<__half2*>(xb + (lo + row) * ld + col) = lw;
}

__global__ void embed_gather_kernel(const __half* table, const int32_t* ids, int H, float scale,
                                    float* out) {
    const int m = blockIdx.x;
    const __half* row = table + static_cast<size_t>(ids[m]) * H;
    for (int k = threadIdx.x; k < H; k += blockDim.x)
        out[static_cast<size_t>(m) * H + k] = __half2float(row[k]) * scale;
}

// ------------------------------------------------------------------ DiT ---
// DiT input rows of both CFG sequences: [mu0, mu1, t + dt, cond_proj(cond) x P,
// in_proj(x) x P]. One CTA per 32 hidden features: the features' in/cond weight
// rows are staged in shared memory (row stride 2D + 1 floats: conflict-free
// column reads), then each thread computes 4P / 8 of the feature's 4P dot
// products (2 sequences x P frames x {in, cond}).
constexpr int kEmbedFeatures = 32;
constexpr int kEmbedThreads = 256;

__global__ void __launch_bounds__(kEmbedThreads) dit_embed_kernel(const DitEmbedArgs a0) {
    extern __shared__ float sm[];
    pdl_launch_dependents();
    DitEmbedArgs a = a0;
    if (a0.members > 0) {  // member blockIdx.y of a group
        const int m = blockIdx.y;
        a.x = a0.mx[m];
        a.cond = a0.mcond[m];
        a.mu = a0.mmu[m];
        a.ctl = a0.mctl[m];
        a.hidden = a0.hidden + m * a0.member_stride;
        a.ssq_out = nullptr;
    }
    const int D = a.D, P = a.P, DP = D * P, ws = 2 * D + 1;
    const int f0 = blockIdx.x * kEmbedFeatures;
    float* w_s = sm;                              // [32][2D + 1]: in row, cond row
    float* xs = sm + kEmbedFeatures * ws;         // [2][D*P]
    float* cs = xs + 2 * DP;                      // [2][D*P]
    // weights first: they do not depend on the previous kernel. This block's rows of
    // in_w and cond_w are contiguous: 16-byte loads, all issued before any is used.
    const bool vec = (D & 7) == 0 && D <= 128 &&
                     ((reinterpret_cast<uintptr_t>(a.in_w) | reinterpret_cast<uintptr_t>(a.cond_w)) & 15) == 0;
    if (vec) {
        constexpr int kV = 2;  // 16-byte loads per thread per matrix: 32 rows x D <= 2 * 256 * 8 halves (D <= 128)
        const int n8 = kEmbedFeatures * D / 8;
        uint4 wv[2][kV];
#pragma unroll
        for (int kind = 0; kind < 2; ++kind)
#pragma unroll
            for (int j = 0; j < kV; ++j) {
                const int i = threadIdx.x + j * kEmbedThreads, fl = (i * 8) / D;
                const __half* src = (kind == 0 ? a.in_w : a.cond_w) + static_cast<size_t>(f0) * D + i * 8;
                wv[kind][j] = (i < n8 && f0 + fl < a.Hd) ? *reinterpret_cast<const uint4*>(src) : make_uint4(0, 0, 0, 0);
            }
#pragma unroll
        for (int kind = 0; kind < 2; ++kind)
#pragma unroll
            for (int j = 0; j < kV; ++j) {
                const int i = threadIdx.x + j * kEmbedThreads;
                if (i >= n8) continue;
                const int fl = (i * 8) / D, e = i * 8 - fl * D;
                const __half2* h2 = reinterpret_cast<const __half2*>(&wv[kind][j]);
                float* dst = w_s + fl * ws + kind * D + e;
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    const float2 f2 = __half22float2(h2[q]);
                    dst[2 * q] = f2.x;
                    dst[2 * q + 1] = f2.y;
                }
            }
    } else {
        for (int i = threadIdx.x; i < kEmbedFeatures * 2 * D; i += kEmbedThreads) {
            const int fl = i / (2 * D), r = i - fl * 2 * D, kind = r / D, e = r - kind * D;
            const int f = f0 + fl;
            float w = 0.f;
            if (f < a.Hd) w = __half2float((kind == 0 ? a.in_w : a.cond_w)[static_cast<size_t>(f) * D + e]);
            w_s[fl * ws + kind * D + e] = w;
        }
    }
    pdl_wait();
    // the stop flag, the x / cond rows and (threads of the first two feature rows)
    // the mu and time rows are read in one batch; nothing is written before the check
    const bool stop = a.ctl && a.ctl->stopped;
    const int fl = threadIdx.x & (kEmbedFeatures - 1), j = threadIdx.x / kEmbedFeatures;
    const int f = f0 + fl;
    const bool live = f < a.Hd;
    float v0 = 0.f, v1 = 0.f, v2 = 0.f;
    if (j < 2 && live) {  // mu tokens and the time token of sequence j
        const float* mu = j == 0 ? a.mu : a.mu_uncond;
        v0 = mu ? mu[f] : 0.f;
        v1 = mu ? mu[a.Hd + f] : 0.f;
        v2 = a.tsum ? a.tsum[f] : (j == 0 ? a.t_tok0 : a.t_tok1)[f] + (j == 0 ? a.dt_tok0 : a.dt_tok1)[f];
    }
    for (int i = threadIdx.x; i < DP; i += kEmbedThreads) {
        xs[i] = a.x[i];
        xs[DP + i] = a.x_uncond ? a.x_uncond[i] : a.x[i];
        cs[i] = a.cond[i];
        cs[DP + i] = a.cond_uncond ? a.cond_uncond[i] : a.cond[i];
    }
    if (stop) return;
    __syncthreads();
    const int seq = 3 + 2 * P;
    __shared__ float vals[24][kEmbedFeatures + 1];  // this block's outputs, for the sums of squares
    if (j < 2) {
        const int b = j;
        if (live) {
            float* h = a.hidden + static_cast<size_t>(b) * seq * a.Hd;
            h[f] = v0;
            h[a.Hd + f] = v1;
            h[2 * a.Hd + f] = v2;
        }
        if (b * seq + 2 < 24) {
            vals[b * seq][fl] = v0;
            vals[b * seq + 1][fl] = v1;
            vals[b * seq + 2][fl] = v2;
        }
    }
    const float* wr = w_s + fl * ws;
    for (int o = j; o < 4 * P; o += kEmbedThreads / kEmbedFeatures) {
        const int kind = o & 1, b = (o >> 1) & 1, p = o >> 2;
        const float* src = (kind == 0 ? xs : cs) + b * DP + p;
        const float* w = wr + kind * D;
        float acc;
        if ((D & 3) == 0) {  // four independent chains
            float c4[4] = {0.f, 0.f, 0.f, 0.f};
            for (int e = 0; e < D; e += 4) {
#pragma unroll
                for (int u = 0; u < 4; ++u) c4[u] = fmaf(w[e + u], src[(e + u) * P], c4[u]);  // frame p of [D][P]
            }
            acc = (c4[0] + c4[1]) + (c4[2] + c4[3]);
        } else {
            acc = 0.f;
            for (int e = 0; e < D; ++e) acc = fmaf(w[e], src[e * P], acc);  // frame p of a d-major [D][P] patch
        }
        const int tok = kind == 0 ? 3 + P + p : 3 + p;
        const float v = live ? acc + __half2float(kind == 0 ? a.in_b[f] : a.cond_b[f]) : 0.f;
        if (live) a.hidden[static_cast<size_t>(b * seq + tok) * a.Hd + f] = v;
        if (b * seq + tok < 24) vals[b * seq + tok][fl] = v;
    }
    if (a.ssq_out) {
        __syncthreads();
        if (threadIdx.x < 2 * seq && threadIdx.x < 24) {
            float t = 0.f;
            for (int i = 0; i < kEmbedFeatures; ++i) t += vals[threadIdx.x][i] * vals[threadIdx.x][i];
            a.ssq_out[blockIdx.x * 24 + threadIdx.x] = t;
        }
    }
}

__global__ void vec_add_kernel(const float* a, const float* b, float* out, int n) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) out[i] = a[i] + b[i];
}

// Sinusoidal timestep embedding rows [sin(t f_i) | cos(t f_i)]
// (VoxCPM2TimestepEmbedding::forward, timestep_embedding.cpp:128-160). The
// frequencies f_i = exp(-ln(max_period) i / (half - 1)) and the scaled t of every
// row (schedule mode's t(step, T) included) come from the host, computed in float
// with the C library as the layer does, so the only device rounding left is one
// fp32 product and sinf / cosf. t_rows: one t per row in device memory, or null
// for a single row of value t_val.
__global__ void timestep_embedding_kernel(const float* t_rows, float t_val, int rows, const float* freq,
                                          int half_dim, float* out, StreamCtl* ctl) {
    pdl_launch_dependents();
    pdl_wait();
    if (ctl && ctl->stopped) return;
    for (int u = blockIdx.x * blockDim.x + threadIdx.x; u < rows * half_dim; u += gridDim.x * blockDim.x) {
        const int r = u / half_dim, i = u - r * half_dim;
        const float t = t_rows ? t_rows[r] : t_val;
        const float phase = t * freq[i];
        out[static_cast<size_t>(r) * 2 * half_dim + i] = sinf(phase);
        out[static_cast<size_t>(r) * 2 * half_dim + half_dim + i] = cosf(phase);
    }
}

// final norm of the x rows, out_proj, then CFG-zero* and the Euler step
// (synthesizer.cpp:147-161). Each CTA computes kOutFeatures output features of
// both CFG rows: warp r normalises x row r in registers and dots it with the CTA's
// out_proj rows (staged in shared memory before the dependency wait), 16
// independent accumulators per lane; the last CTA to arrive reads the whole
// [2][D*P] estimate back and runs the CFG-zero* scale (double, fixed summation
// order) and the Euler update.
constexpr int kOutFeatures = 4;
constexpr int kOutThreads = 256;

__global__ void __launch_bounds__(kOutThreads) dit_out_kernel(const DitOutArgs a0) {
    extern __shared__ float sm[];
    __shared__ double dred[2][kOutThreads / 32];
    __shared__ int s_last;
    pdl_launch_dependents();
    DitOutArgs a = a0;
    if (a0.members > 0) {  // member blockIdx.y of a group
        const int m = blockIdx.y;
        a.hidden = a0.hidden + m * a0.member_stride;
        a.x = a0.mx[m];
        a.ctl = a0.mctl[m];
        a.est_buf = a0.mest[m];
        a.counter = a0.mcounter[m];
        a.est_out = nullptr;
    }
    const int R = 2 * a.P;        // rows (b, p), at most 8
    const int L = a.D * a.P;      // latent size
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = kOutThreads / 32;
    float* xn = sm;               // [R][Hd]
    float* wsm = sm + R * a.Hd;   // [kOutFeatures][Hd] out_proj rows of this CTA
    const int e0 = blockIdx.x * kOutFeatures;
    // this CTA's out_proj rows are contiguous: 16-byte loads, all issued at once
    const bool vec = (a.Hd & 7) == 0 && a.Hd <= 1024 && (reinterpret_cast<uintptr_t>(a.out_w) & 15) == 0 &&
                     (reinterpret_cast<uintptr_t>(a.norm_g) & 7) == 0;
    if (vec) {
        constexpr int kV = kOutFeatures * 1024 / 8 / kOutThreads;  // Hd <= 1024
        const int n8 = kOutFeatures * a.Hd / 8;
        uint4 wv[kV];
#pragma unroll
        for (int j = 0; j < kV; ++j) {
            const int i = threadIdx.x + j * kOutThreads, el = (i * 8) / a.Hd;
            wv[j] = (i < n8 && e0 + el < a.D)
                        ? *reinterpret_cast<const uint4*>(a.out_w + static_cast<size_t>(e0) * a.Hd + i * 8)
                        : make_uint4(0, 0, 0, 0);
        }
#pragma unroll
        for (int j = 0; j < kV; ++j) {
            const int i = threadIdx.x + j * kOutThreads;
            if (i >= n8) continue;
            const __half2* h2 = reinterpret_cast<const __half2*>(&wv[j]);
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const float2 f2 = __half22float2(h2[q]);
                wsm[i * 8 + 2 * q] = f2.x;
                wsm[i * 8 + 2 * q + 1] = f2.y;
            }
        }
    } else {
        for (int i = threadIdx.x; i < kOutFeatures * a.Hd; i += kOutThreads) {
            const int el = i / a.Hd, k = i - el * a.Hd;
            wsm[i] = e0 + el < a.D ? __half2float(a.out_w[static_cast<size_t>(e0 + el) * a.Hd + k]) : 0.f;
        }
    }
    __syncthreads();  // this CTA's out_proj rows are staged (before the dependency wait)
    pdl_wait();
    const bool stop = a.ctl && a.ctl->stopped;  // read beside the rows; nothing is written before the check
    if (vec && R <= nw) {
        // warp r: row r normalised in registers, then its dot products with this CTA's
        // kOutFeatures out_proj rows, 16 independent accumulators per lane
        if (warp < R && !stop) {
            const int r = warp, b = r / a.P, p = r - b * a.P;
            const float* h = a.hidden + (static_cast<size_t>(b) * a.seq + 3 + a.P + p) * a.Hd;
            constexpr int kR = 1024 / 4 / 32;  // float4 per lane, Hd <= 1024
            const int n4 = a.Hd / 4;
            float4 hv[kR];
            uint2 gv[kR];
#pragma unroll
            for (int j = 0; j < kR; ++j) {
                const int i = lane + j * 32;
                hv[j] = i < n4 ? reinterpret_cast<const float4*>(h)[i] : make_float4(0.f, 0.f, 0.f, 0.f);
                gv[j] = i < n4 ? reinterpret_cast<const uint2*>(a.norm_g)[i] : make_uint2(0u, 0u);
            }
            float ss = 0.f;
#pragma unroll
            for (int j = 0; j < kR; ++j) ss += hv[j].x * hv[j].x + hv[j].y * hv[j].y + hv[j].z * hv[j].z + hv[j].w * hv[j].w;
            ss = warp_sum(ss);
            const float inv = rsqrtf(ss / static_cast<float>(a.Hd) + a.eps);
            float4 acc[kOutFeatures];
#pragma unroll
            for (int el = 0; el < kOutFeatures; ++el) acc[el] = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
            for (int j = 0; j < kR; ++j) {
                const int i = lane + j * 32;
                if (i >= n4) continue;
                const float2 g01 = __half22float2(*reinterpret_cast<const __half2*>(&gv[j].x));
                const float2 g23 = __half22float2(*reinterpret_cast<const __half2*>(&gv[j].y));
                const float4 xv = make_float4(hv[j].x * inv * g01.x, hv[j].y * inv * g01.y, hv[j].z * inv * g23.x,
                                              hv[j].w * inv * g23.y);
#pragma unroll
                for (int el = 0; el < kOutFeatures; ++el) {
                    const float4 w4 = reinterpret_cast<const float4*>(wsm + el * a.Hd)[i];
                    acc[el].x = fmaf(w4.x, xv.x, acc[el].x);
                    acc[el].y = fmaf(w4.y, xv.y, acc[el].y);
                    acc[el].z = fmaf(w4.z, xv.z, acc[el].z);
                    acc[el].w = fmaf(w4.w, xv.w, acc[el].w);
                }
            }
#pragma unroll
            for (int el = 0; el < kOutFeatures; ++el) {
                const float t = warp_sum((acc[el].x + acc[el].y) + (acc[el].z + acc[el].w));
                const int e = e0 + el;
                if (lane == 0 && e < a.D) a.est_buf[b * L + e * a.P + p] = t + __half2float(a.out_b[e]);  // [2][D][P]
            }
        }
        if (stop) return;
    } else {
        // warp r normalises row r into shared memory (the row read once, as float4)
        for (int r = warp; r < R; r += nw) {
            const int b = r / a.P, p = r - b * a.P;
            const float* h = a.hidden + (static_cast<size_t>(b) * a.seq + 3 + a.P + p) * a.Hd;
            if (vec) {
                constexpr int kR = 1024 / 4 / 32;  // float4 per lane, Hd <= 1024
                const int n4 = a.Hd / 4;
                float4 hv[kR];
                uint2 gv[kR];
#pragma unroll
                for (int j = 0; j < kR; ++j) {
                    const int i = lane + j * 32;
                    hv[j] = i < n4 ? reinterpret_cast<const float4*>(h)[i] : make_float4(0.f, 0.f, 0.f, 0.f);
                    gv[j] = i < n4 ? reinterpret_cast<const uint2*>(a.norm_g)[i] : make_uint2(0u, 0u);
                }
                float ss = 0.f;
#pragma unroll
                for (int j = 0; j < kR; ++j) ss += hv[j].x * hv[j].x + hv[j].y * hv[j].y + hv[j].z * hv[j].z + hv[j].w * hv[j].w;
                ss = warp_sum(ss);
                const float inv = rsqrtf(ss / static_cast<float>(a.Hd) + a.eps);
#pragma unroll
                for (int j = 0; j < kR; ++j) {
                    const int i = lane + j * 32;
                    if (i >= n4) continue;
                    const float2 g01 = __half22float2(*reinterpret_cast<const __half2*>(&gv[j].x));
                    const float2 g23 = __half22float2(*reinterpret_cast<const __half2*>(&gv[j].y));
                    reinterpret_cast<float4*>(xn + r * a.Hd)[i] =
                        make_float4(hv[j].x * inv * g01.x, hv[j].y * inv * g01.y, hv[j].z * inv * g23.x, hv[j].w * inv * g23.y);
                }
            } else {
                float ss = 0.f;
                for (int k = lane; k < a.Hd; k += 32) ss = fmaf(h[k], h[k], ss);
                ss = warp_sum(ss);
                const float inv = rsqrtf(ss / static_cast<float>(a.Hd) + a.eps);
                for (int k = lane; k < a.Hd; k += 32) xn[r * a.Hd + k] = h[k] * inv * __half2float(a.norm_g[k]);
            }
        }
        if (stop) return;
        __syncthreads();
        // (feature, row) pairs: warp w takes pairs w, w + 8, ...
        for (int q = warp; q < kOutFeatures * R; q += nw) {
            const int el = q / R, r = q - el * R, e = e0 + el;
            if (e >= a.D) continue;
            float acc = 0.f;
            for (int k = lane; k < a.Hd; k += 32) acc = fmaf(wsm[el * a.Hd + k], xn[r * a.Hd + k], acc);
            acc = warp_sum(acc);
            if (lane == 0) {
                const int b = r / a.P, p = r - b * a.P;
                a.est_buf[b * L + e * a.P + p] = acc + __half2float(a.out_b[e]);  // [2][D][P]
            }
        }
    }
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) s_last = atomicAdd(a.counter, 1) == static_cast<int>(gridDim.x) - 1;
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    if (threadIdx.x == 0) *a.counter = 0;
    if (!a.x) return;
    // optimized_scale in double (synthesizer.cpp:76-84) + finiteness check (:150)
    double dot = 0.0, nrm = 0.0;
    int bad = 0;
    for (int i = threadIdx.x; i < L; i += kOutThreads) {
        const float p = __ldcg(a.est_buf + i), n = __ldcg(a.est_buf + L + i);
        if (!isfinite(p) || !isfinite(n)) bad = 1;
        dot += static_cast<double>(p) * n;
        nrm += static_cast<double>(n) * n;
    }
    bad = __syncthreads_or(bad);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        dot += __shfl_xor_sync(0xffffffffu, dot, o);
        nrm += __shfl_xor_sync(0xffffffffu, nrm, o);
    }
    if (lane == 0) {
        dred[0][warp] = dot;
        dred[1][warp] = nrm;
    }
    __syncthreads();
    if (bad) {
        if (threadIdx.x == 0 && a.ctl) a.ctl->error = 2;
        return;
    }
    double dt_ = 0.0, nm = 1e-8;
    for (int w = 0; w < nw; ++w) {
        dt_ += dred[0][w];
        nm += dred[1][w];
    }
    const float sc = static_cast<float>(dt_ / nm);
    for (int i = threadIdx.x; i < L; i += kOutThreads) {
        const float pos = __ldcg(a.est_buf + i), neg = __ldcg(a.est_buf + L + i);
        const float dphi = neg * sc + a.cfg * (pos - neg * sc);
        a.x[i] -= a.dt * dphi;
    }
}

__global__ void stop_decide_kernel(const __half* head_w, const float* mid, int H, StreamCtl* ctl,
                                   float* logits_out) {
    pdl_launch_dependents();
    pdl_wait();
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    __shared__ float lg[2];
    if (warp < 2) {
        float s = 0.f;
        for (int k = lane; k < H; k += kWarp) s = fmaf(__half2float(head_w[static_cast<size_t>(warp) * H + k]), mid[k], s);
        s = warp_sum(s);
        if (lane == 0) lg[warp] = s;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        if (logits_out) {
            logits_out[0] = lg[0];
            logits_out[1] = lg[1];
        }
        if (ctl) {
            ctl->stop_logits[0] = lg[0];
            ctl->stop_logits[1] = lg[1];
            // synthesizer.cpp:584: step > min_patches and argmax2(logits) == 1
            ctl->stopped = (ctl->step > ctl->min_patches && lg[1] > lg[0]) ? 1 : 0;
        }
    }
}

__global__ void patch_begin_kernel(const float* noise_table, const float* latents, const float* init_cond,
                                   int per_patch, float* x, float* cond, StreamCtl* ctl) {
    pdl_launch_dependents();
    pdl_wait();
    const int patch = ctl->patch;
    const float* src = noise_table + static_cast<size_t>(patch) * per_patch;
    const float* c = patch > 0 ? latents + static_cast<size_t>(patch - 1) * per_patch : init_cond;
    for (int i = threadIdx.x; i < per_patch; i += blockDim.x) {
        x[i] = src[i];
        cond[i] = c[i];
    }
    __syncthreads();
    if (threadIdx.x == 0) ctl->stopped = 0;
}

__global__ void patch_end_kernel(const float* x, float* latents, int per_patch, StreamCtl* ctl) {
    pdl_launch_dependents();
    pdl_wait();
    float* dst = latents + static_cast<size_t>(ctl->patch) * per_patch;
    for (int i = threadIdx.x; i < per_patch; i += blockDim.x) dst[i] = x[i];
    __syncthreads();
    if (threadIdx.x == 0) {
        ctl->patch += 1;
        ctl->step += 1;
    }
}

// VoxCPM2SDPA CPU forward on the GPU (voxcpm2_sdpa.cpp:187-252): one CTA per (head, row).
__global__ void sdpa_rows_f32_kernel(const float* q, int heads, int src, int d, const float* k,
                                     const float* v, int groups, int cur, int dv, const float* mask,
                                     int mask_c, const float* past_k, const float* past_v,
                                     int past, float scale, float* out) {
    extern __shared__ float sc[];
    __shared__ float red[32];
    const int h = blockIdx.x, i = blockIdx.y;
    const int dst = past + cur;
    const int g = h / (heads / groups);
    const float* qp = q + (static_cast<size_t>(h) * src + i) * d;
    for (int j = threadIdx.x; j < dst; j += blockDim.x) {
        const float* kp = j < past ? past_k + (static_cast<size_t>(g) * past + j) * d
                                   : k + (static_cast<size_t>(g) * cur + (j - past)) * d;
        float s = 0.f;
        for (int e = 0; e < d; ++e) s = fmaf(qp[e], kp[e], s);
        s *= scale;
        if (mask) {
            const float* mp = mask + (mask_c > 1 ? static_cast<size_t>(h) * src * dst : 0);
            s += mp[static_cast<size_t>(i) * dst + j];
        }
        sc[j] = s;
    }
    __syncthreads();
    float mx = -FLT_MAX;
    for (int j = threadIdx.x; j < dst; j += blockDim.x) mx = fmaxf(mx, sc[j]);
    mx = warp_max(mx);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = mx;
    __syncthreads();
    mx = -FLT_MAX;
    for (int w = 0; w < static_cast<int>(blockDim.x >> 5); ++w) mx = fmaxf(mx, red[w]);
    __syncthreads();
    float l = 0.f;
    for (int j = threadIdx.x; j < dst; j += blockDim.x) {
        const float p = expf(sc[j] - mx);
        sc[j] = p;
        l += p;
    }
    l = warp_sum(l);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = l;
    __syncthreads();
    l = 0.f;
    for (int w = 0; w < static_cast<int>(blockDim.x >> 5); ++w) l += red[w];
    for (int e = threadIdx.x; e < dv; e += blockDim.x) {
        float acc = 0.f;
        for (int j = 0; j < dst; ++j) {
            const float* vp = j < past ? past_v + (static_cast<size_t>(g) * past + j) * dv
                                       : v + (static_cast<size_t>(g) * cur + (j - past)) * dv;
            acc = fmaf(sc[j] / l, vp[e], acc);
        }
        out[(static_cast<size_t>(h) * src + i) * dv + e] = acc;
    }
}

__global__ void concat_kv_kernel(const float* past, const float* cur, int past_len, int cur_len,
                                 int d, float* out) {
    const int g = blockIdx.y;
    const int dst = past_len + cur_len;
    const size_t n = static_cast<size_t>(dst) * d;
    for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<size_t>(gridDim.x) * blockDim.x) {
        const size_t row = i / d, e = i - row * d;
        out[static_cast<size_t>(g) * n + i] =
            row < static_cast<size_t>(past_len) ? past[(static_cast<size_t>(g) * past_len + row) * d + e]
                                                : cur[(static_cast<size_t>(g) * cur_len + (row - past_len)) * d + e];
    }
}

}  // namespace

void init_batched_attributes() {
    constexpr int kMax = 200 * 1024;
    check_launch(cudaFuncSetAttribute(dit_out_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kMax));
    check_launch(cudaFuncSetAttribute(dit_embed_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kMax));
    check_launch(cudaFuncSetAttribute(sdpa_rows_f32_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kMax));
}

void launch_rows_linear(const RowsArgs& a, cudaStream_t s, bool pdl) {
    if (a.K <= 0 || a.K % 8 != 0 || a.M <= 0 || a.rows <= 0 || a.ldx % 4 != 0)
        throw std::invalid_argument("rows_linear: bad shape");
    const int per_warp = a.mode == GEMV_GATEUP ? 2 : 4;
    const int items = (a.rows + per_warp - 1) / per_warp;
    const dim3 grid((items + kRowsWarps - 1) / kRowsWarps, (a.M + kRowsTile - 1) / kRowsTile);
    cudaLaunchAttribute attr[1];
    cudaLaunchConfig_t cfg = make_cfg(grid, dim3(kRowsWarps * kWarp), 0, s, pdl, attr);
    switch (a.mode) {
        case GEMV_PLAIN: check_launch(cudaLaunchKernelEx(&cfg, rows_linear_kernel<GEMV_PLAIN>, a)); break;
        case GEMV_RESID: check_launch(cudaLaunchKernelEx(&cfg, rows_linear_kernel<GEMV_RESID>, a)); break;
        case GEMV_GATEUP: check_launch(cudaLaunchKernelEx(&cfg, rows_linear_kernel<GEMV_GATEUP>, a)); break;
        default: throw std::invalid_argument("rows_linear: unsupported mode");
    }
}

void launch_rmsnorm_rows(const float* x, int ldx, const __half* g, float eps, int K, int M,
                         float* out, int ldo, StreamCtl* ctl, int skip_if_stopped, cudaStream_t s,
                         bool pdl) {
    cudaLaunchAttribute attr[1];
    cudaLaunchConfig_t cfg = make_cfg(dim3(M), dim3(256), 0, s, pdl, attr);
    check_launch(cudaLaunchKernelEx(&cfg, rmsnorm_rows_kernel, x, ldx, g, eps, K, out, ldo, ctl, skip_if_stopped));
}

void launch_qkv_rows_post(float* qkv, int M, int q_heads, int kv_heads, int d, int past,
                          int pos_mod, const float* rope_cos, const float* rope_sin,
                          float* k_cache, float* v_cache, int cap, StreamCtl* ctl,
                          cudaStream_t s, bool pdl) {
    cudaLaunchAttribute attr[1];
    cudaLaunchConfig_t cfg = make_cfg(dim3(M), dim3(256), 0, s, pdl, attr);
    check_launch(cudaLaunchKernelEx(&cfg, qkv_rows_post_kernel, qkv, q_heads, kv_heads, d, past, pos_mod,
                                    rope_cos, rope_sin, k_cache, v_cache, cap, ctl));
}

void launch_attn_rows_cache(const float* qkv, int M, int q_heads, int kv_heads, int d, int past,
                            const float* k_cache, const float* v_cache, int cap, float scale,
                            float* out, cudaStream_t s, bool pdl) {
    if (past + M > cap) throw std::invalid_argument("prefill attention: rows beyond the cache capacity");
    if (d != 64 || kv_heads <= 0 || q_heads % kv_heads != 0 || q_heads / kv_heads > kPfMaxGroup ||
        (reinterpret_cast<uintptr_t>(k_cache) & 15) || (reinterpret_cast<uintptr_t>(v_cache) & 15))
        throw std::invalid_argument("prefill attention: head_dim 64, at most 16 query heads per KV head");
    const int G = q_heads / kv_heads;
    const int rb = std::max(1, kPfVectors / G);  // query rows per CTA
    cudaLaunchAttribute attr[1];
    cudaLaunchConfig_t cfg = make_cfg(dim3(kv_heads, (M + rb - 1) / rb), dim3(kPfThreads), 0, s, pdl, attr);
    check_launch(cudaLaunchKernelEx(&cfg, attn_prefill_kernel, qkv, M, q_heads, kv_heads, past, k_cache, v_cache, cap,
                                    scale, out, rb));
}


void launch_rmsnorm_rows_split(const float* x, int ldx, const __half* g, float eps, int K, int M, __half* xb,
                               StreamCtl* ctl, cudaStream_t s, bool pdl, int lo) {
    if (M > lo) throw std::invalid_argument("rmsnorm_split: more rows than the operand's row block");
    if (K % 4 != 0 || K > 4 * kNormThreads * kNormBatch || ldx % 4 != 0 || (reinterpret_cast<uintptr_t>(x) & 15) ||
        (reinterpret_cast<uintptr_t>(g) & 7))
        throw std::invalid_argument("rmsnorm_split: row length or alignment unsupported");
    cudaLaunchAttribute attr[1];
    cudaLaunchConfig_t cfg = make_cfg(dim3(M), dim3(kNormThreads), 0, s, pdl, attr);
    check_launch(cudaLaunchKernelEx(&cfg, rmsnorm_rows_split_kernel, x, ldx, g, eps, K, xb, ctl, lo));
}

void launch_dit_attention_split(const float* qkv, int nseq, int seq, int q_heads, int kv_heads, int d,
                                const float* rope_cos, const float* rope_sin, float scale, __half* xb,
                                StreamCtl* ctl, cudaStream_t s, bool pdl, int lo) {
    if (d != 64 || seq > kDitMaxSeq || nseq * seq > lo ||
        (reinterpret_cast<uintptr_t>(qkv) & 15) || (reinterpret_cast<uintptr_t>(rope_cos) & 15) ||
        (reinterpret_cast<uintptr_t>(rope_sin) & 15))
        throw std::invalid_argument("dit attention: unsupported shape");
    cudaLaunchAttribute attr[1];
    cudaLaunchConfig_t cfg = make_cfg(dim3(q_heads, nseq), dim3(kDitThreads), 0, s, pdl, attr);
    check_launch(cudaLaunchKernelEx(&cfg, dit_attention_split_kernel, qkv, seq, q_heads, kv_heads, rope_cos, rope_sin,
                                    scale, xb, ctl, lo));
}

void launch_embed_gather(const __half* table, const int32_t* ids, int M, int H, float scale,
                         float* out, cudaStream_t s) {
    embed_gather_kernel<<<M, 256, 0, s>>>(table, ids, H, scale, out);
    check_launch(cudaGetLastError());
}

void launch_dit_embed(const DitEmbedArgs& a, cudaStream_t s, bool pdl) {
    cudaLaunchAttribute attr[1];
    const size_t smem = static_cast<size_t>(kEmbedFeatures * (2 * a.D + 1) + 4 * a.D * a.P) * sizeof(float);
    if (smem > 200 * 1024) throw std::invalid_argument("dit_embed: patch too large");
    if (a.members < 0 || a.members > kGroupMembers) throw std::invalid_argument("dit_embed: 0 to 8 members");
    cudaLaunchConfig_t cfg = make_cfg(dim3((a.Hd + kEmbedFeatures - 1) / kEmbedFeatures, a.members > 0 ? a.members : 1),
                                      dim3(kEmbedThreads), smem,
                                      s, pdl, attr);
    check_launch(cudaLaunchKernelEx(&cfg, dit_embed_kernel, a));
}

void launch_vec_add(const float* a, const float* b, float* out, int n, cudaStream_t s) {
    vec_add_kernel<<<(n + 255) / 256, 256, 0, s>>>(a, b, out, n);
    check_launch(cudaGetLastError());
}

void launch_timestep_embedding(const float* t_rows, float t_val, int rows, const float* freq, int half_dim,
                               float* out, StreamCtl* ctl, cudaStream_t s, bool pdl) {
    if (rows <= 0 || half_dim <= 0 || !freq || !out) throw std::invalid_argument("timestep embedding: bad shape");
    cudaLaunchAttribute attr[1];
    const int blocks = std::min(148, (rows * half_dim + 255) / 256);
    cudaLaunchConfig_t cfg = make_cfg(dim3(blocks), dim3(256), 0, s, pdl, attr);
    check_launch(cudaLaunchKernelEx(&cfg, timestep_embedding_kernel, t_rows, t_val, rows, freq, half_dim, out, ctl));
}

void launch_dit_out(const DitOutArgs& a, cudaStream_t s, bool pdl) {
    if (!a.est_buf || !a.counter) throw std::invalid_argument("dit_out: scratch buffers missing");
    const size_t smem = static_cast<size_t>(2 * a.P + kOutFeatures) * a.Hd * sizeof(float);
    if (smem > 200 * 1024) throw std::invalid_argument("dit_out: hidden too large");
    cudaLaunchAttribute attr[1];
    if (a.members < 0 || a.members > kGroupMembers) throw std::invalid_argument("dit_out: 0 to 8 members");
    cudaLaunchConfig_t cfg = make_cfg(dim3((a.D + kOutFeatures - 1) / kOutFeatures, a.members > 0 ? a.members : 1),
                                      dim3(kOutThreads), smem, s, pdl,
                                      attr);
    check_launch(cudaLaunchKernelEx(&cfg, dit_out_kernel, a));
}

void launch_stop_decide(const __half* head_w, const float* mid, int H, StreamCtl* ctl,
                        float* logits_out, cudaStream_t s, bool pdl) {
    cudaLaunchAttribute attr[1];
    cudaLaunchConfig_t cfg = make_cfg(dim3(1), dim3(64), 0, s, pdl, attr);
    check_launch(cudaLaunchKernelEx(&cfg, stop_decide_kernel, head_w, mid, H, ctl, logits_out));
}

void launch_patch_begin(const float* noise_table, const float* latents, const float* init_cond,
                        int per_patch, float* x, float* cond, StreamCtl* ctl, cudaStream_t s, bool pdl) {
    cudaLaunchAttribute attr[1];
    cudaLaunchConfig_t cfg = make_cfg(dim3(1), dim3(256), 0, s, pdl, attr);
    check_launch(cudaLaunchKernelEx(&cfg, patch_begin_kernel, noise_table, latents, init_cond, per_patch, x,
                                    cond, ctl));
}

void launch_patch_end(const float* x, float* latents, int per_patch, StreamCtl* ctl,
                      cudaStream_t s, bool pdl) {
    cudaLaunchAttribute attr[1];
    cudaLaunchConfig_t cfg = make_cfg(dim3(1), dim3(256), 0, s, pdl, attr);
    check_launch(cudaLaunchKernelEx(&cfg, patch_end_kernel, x, latents, per_patch, ctl));
}

void launch_sdpa_rows_f32(const float* q, int heads, int src, int d, const float* k,
                          const float* v, int groups, int cur, int dv, const float* mask,
                          int mask_c, const float* past_k, const float* past_v, int past,
                          float scale, float* out, cudaStream_t s) {
    const size_t smem = static_cast<size_t>(past + cur) * sizeof(float);
    if (smem > 200 * 1024) throw std::invalid_argument("sdpa: key sequence too long");
    sdpa_rows_f32_kernel<<<dim3(heads, src), dim3(128), smem, s>>>(q, heads, src, d, k, v, groups, cur, dv,
                                                                   mask, mask_c, past_k, past_v, past,
                                                                   scale, out);
    check_launch(cudaGetLastError());
}

void launch_concat_kv(const float* past, const float* cur, int groups, int past_len, int cur_len,
                      int d, float* out, cudaStream_t s) {
    const size_t n = static_cast<size_t>(past_len + cur_len) * d;
    const int blocks = static_cast<int>(std::min<size_t>((n + 255) / 256, 1024));
    concat_kv_kernel<<<dim3(blocks, groups), 256, 0, s>>>(past, cur, past_len, cur_len, d, out);
    check_launch(cudaGetLastError());
}

}  // namespace vxc
