// Batch-1 decoder kernels: GEMV family and split-K flash-decode attention.
//
// The KV-cache decode step of base_decoder_kv / residual_decoder_kv
// (tools/export_components.py:496-550, run by src/kvcache.cpp:232-279) is a
// chain of matrix-vector products over fp16 weights. Each GEMV streams its
// weight rows into registers with 16-byte no-allocate loads BEFORE waiting on
// the previous kernel (programmatic dependent launch), so weight streaming of
// kernel i+1 overlaps kernel i; only the small fp32 input vector is read after
// the dependency resolves. RMSNorm is folded into the GEMV prologue, RoPE and
// the KV append into the q/k/v epilogue. The KV cache is fp32, as the
// reference's HostDecoderKvCache (src/kvcache.cpp:86-93): at the loop's
// lengths it is under 2% of a decode step's bytes.
#include <algorithm>
#include <cfloat>
#include <stdexcept>

#include "kernels.cuh"
#include "tc_common.cuh"

namespace vxc {
namespace {

constexpr int kGemvWarps = 4;
constexpr int kGemvThreads = kGemvWarps * kWarp;

__device__ __forceinline__ float gemv_input(const GemvArgs& a, int k) {
    if (a.in_mode == IN_CONCAT) return k < a.k1 ? a.x[k] : a.x2[k - a.k1];
    if (a.in_mode == IN_LATENT_T) {
        // make_feat_encoder_input: frame-major value[p * D + d] = latent[d * P + p]
        const int p = k / a.lat_d, d = k - p * a.lat_d;
        return a.x[d * a.lat_p + p];
    }
    return a.x[k];
}

// Epilogue of one GEMV output unit (lane 0 of its warp): bias / activation,
// residual update, SiLU(gate) * up, or RoPE + KV append for q/k/v.
template <int MODE, int RPW>
__device__ __forceinline__ void gemv_store(const GemvArgs& a, int item, const int* row, const float* acc) {
    if constexpr (MODE == GEMV_PLAIN) {
#pragma unroll
        for (int r = 0; r < RPW; ++r) {
            float v = acc[r] + (a.bias ? __half2float(a.bias[row[r]]) : 0.f);
            if (a.act == ACT_SILU) v = silu(v);
            else if (a.act == ACT_FSQ) v = rintf(tanhf(v) * a.act_scale) / a.act_scale;
            a.y[row[r]] = v;
            if (a.y2) a.y2[row[r]] = v;
        }
    } else if constexpr (MODE == GEMV_RESID) {
#pragma unroll
        for (int r = 0; r < RPW; ++r) {
            const float v = a.resid[row[r]] + (a.rscale == 1.f ? acc[r] : acc[r] * a.rscale);
            a.resid[row[r]] = v;
        }
    } else if constexpr (MODE == GEMV_GATEUP) {
        a.y[item] = silu(acc[0]) * acc[1];
    } else {  // GEMV_QKV
        const int d = a.head_dim, half = d >> 1;
        const int hh = item / half, j = item - hh * half;
        const int pos = a.ctl->kv_len[a.which];
        float o0 = acc[0], o1 = acc[1];
        const bool is_v = hh >= a.q_heads + a.kv_heads;
        if (!is_v && a.rope_cos && pos < a.cap) {
            // apply_rotary_pos_emb with rotate_half: x*cos + rotate_half(x)*sin; a one-row
            // call at pos takes the long-factor table when pos + 1 > original_max
            const bool lng = a.rope_cos_long && pos + 1 > a.rope_long_from;
            const float* c = (lng ? a.rope_cos_long : a.rope_cos) + static_cast<size_t>(pos) * d;
            const float* s = (lng ? a.rope_sin_long : a.rope_sin) + static_cast<size_t>(pos) * d;
            o0 = acc[0] * c[j] + (-acc[1]) * s[j];
            o1 = acc[1] * c[j + half] + acc[0] * s[j + half];
        }
        if (hh < a.q_heads) {
            a.y[hh * d + j] = o0;
            a.y[hh * d + j + half] = o1;
        } else if (pos >= a.cap) {
            a.ctl->error = 1;  // KV capacity exceeded: the host checks before launch
        } else {
            const int kvh = is_v ? hh - a.q_heads - a.kv_heads : hh - a.q_heads;
            float* dst = (is_v ? a.v_cache : a.k_cache) + (static_cast<size_t>(kvh) * a.cap + pos) * d;
            dst[j] = o0;
            dst[j + half] = o1;
        }
    }
}

template <int MODE, int MAXCH, int RPW>
__global__ void __launch_bounds__(kGemvThreads) gemv_kernel(const GemvArgs a) {
    extern __shared__ float xs[];
    __shared__ float red[kGemvWarps];
    pdl_launch_dependents();

    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int item = blockIdx.x * kGemvWarps + warp;
    const bool active = item < a.rows;
    const int K = a.K;

    // rows owned by this warp
    int row[RPW];
    if constexpr (MODE == GEMV_GATEUP) {
        row[0] = item;
        row[1] = item + a.rows;
    } else if constexpr (MODE == GEMV_QKV) {
        const int half = a.head_dim >> 1;
        const int hh = item / half, j = item - hh * half;
        row[0] = hh * a.head_dim + j;
        row[1] = row[0] + half;
    } else {
#pragma unroll
        for (int r = 0; r < RPW; ++r) row[r] = item * RPW + r;
    }

    // 1) stream this warp's weight rows into registers (independent of inputs)
    uint4 wr[RPW][MAXCH];
#pragma unroll
    for (int r = 0; r < RPW; ++r) {
        const __half* wrow = a.w + static_cast<size_t>(row[r]) * K;
#pragma unroll
        for (int c = 0; c < MAXCH; ++c) {
            const int e = (c * kWarp + lane) * 8;
            wr[r][c] = (active && e < K) ? ld_stream(wrow + e) : make_uint4(0, 0, 0, 0);
        }
    }

    // 2) wait for the producer of the input vector. The stop flag is read together
    // with the input (one L2 round trip, not two) and acted on once the input is
    // staged; nothing is written to global memory before the check.
    pdl_wait();
    const bool stop = a.skip_if_stopped && a.ctl && a.ctl->stopped;

    // 3) stage the (optionally RMS-normalised) input in shared memory. A plain
    // input is read as float4 (and its gain as 4 x fp16), every load of the thread
    // issued before any is used: one L2 round trip instead of a chain of them.
    float ss = 0.f;
    const bool vec = a.in_mode == IN_PLAIN && (K & 3) == 0 && (reinterpret_cast<uintptr_t>(a.x) & 15) == 0 &&
                     (reinterpret_cast<uintptr_t>(a.norm_g) & 7) == 0;
    if (vec) {
        constexpr int kV = MAXCH >= 2 ? MAXCH / 2 : 1;  // float4 per thread: K <= 256 MAXCH
        const int n4 = K >> 2;
        float4 xv[kV];
        uint2 gv[kV];
#pragma unroll
        for (int j = 0; j < kV; ++j) {
            const int i = threadIdx.x + j * kGemvThreads;
            xv[j] = i < n4 ? reinterpret_cast<const float4*>(a.x)[i] : make_float4(0.f, 0.f, 0.f, 0.f);
            gv[j] = (a.norm_g && i < n4) ? reinterpret_cast<const uint2*>(a.norm_g)[i] : make_uint2(0u, 0u);
        }
#pragma unroll
        for (int j = 0; j < kV; ++j) {
            const int i = threadIdx.x + j * kGemvThreads;
            if (i < n4) {
                float4 v = xv[j];
                ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
                if (a.norm_g) {
                    const float2 g01 = __half22float2(*reinterpret_cast<const __half2*>(&gv[j].x));
                    const float2 g23 = __half22float2(*reinterpret_cast<const __half2*>(&gv[j].y));
                    v = make_float4(v.x * g01.x, v.y * g01.y, v.z * g23.x, v.w * g23.y);
                }
                reinterpret_cast<float4*>(xs)[i] = v;
            }
        }
    } else {
        for (int k = threadIdx.x; k < K; k += kGemvThreads) {
            const float v = gemv_input(a, k);
            ss += v * v;
            xs[k] = a.norm_g ? v * __half2float(a.norm_g[k]) : v;
        }
    }
    float inv_rms = 1.f;
    if (a.norm_g) {
        ss = warp_sum(ss);
        if (lane == 0) red[warp] = ss;
        __syncthreads();
        float t = 0.f;
#pragma unroll
        for (int w = 0; w < kGemvWarps; ++w) t += red[w];
        inv_rms = rsqrtf(t / static_cast<float>(K) + a.eps);
    } else {
        __syncthreads();
    }
    if (stop || !active) return;

    // 4) dot products
    float acc[RPW];
#pragma unroll
    for (int r = 0; r < RPW; ++r) acc[r] = 0.f;
#pragma unroll
    for (int c = 0; c < MAXCH; ++c) {
        const int e = (c * kWarp + lane) * 8;
        if (e < K) {
            const float4 x0 = *reinterpret_cast<const float4*>(&xs[e]);
            const float4 x1 = *reinterpret_cast<const float4*>(&xs[e + 4]);
#pragma unroll
            for (int r = 0; r < RPW; ++r) acc[r] = dot8(wr[r][c], x0, x1, acc[r]);
        }
    }
#pragma unroll
    for (int r = 0; r < RPW; ++r) acc[r] = warp_sum(acc[r]) * inv_rms;
    if (lane != 0) return;

    // 5) epilogue
    gemv_store<MODE, RPW>(a, item, row, acc);
}

// The register-streaming GEMV for up to kGemvBatch members (streams of a group):
// each warp's weight rows are loaded once into registers, every member's input is
// staged (and RMS-normalised) in shared memory, and the warp forms one dot product
// per member; lane m stores member m. IN_PLAIN inputs only. W warps per CTA: a
// CTA stages all members' inputs once for its W weight rows (16 warps for 8-member
// batches, whose staged inputs are up to 128 KB). The inputs arrive by cp.async,
// every member's in one batch (one L2 round trip), with the stop flags beside them.
__device__ __forceinline__ void cp_async16(void* smem_dst, const void* gsrc) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(static_cast<uint32_t>(__cvta_generic_to_shared(
                     smem_dst))),
                 "l"(gsrc)
                 : "memory");
}

template <int MODE, int MAXCH, int RPW, int NB, int W>
__global__ void __launch_bounds__(W * 32, (W > 4 && MAXCH <= 8) ? 2 : 1)
    gemv_batch_kernel(const GemvArgs a, const GemvBatch b) {
    static_assert(NB <= kGemvBatch && NB <= kWarp, "lane m stores member m");
    constexpr int T = W * 32;
    constexpr int kV = (MAXCH * 64 + T - 1) / T;  // float4 of one member's input per thread (K <= 256 MAXCH)
    extern __shared__ float xs[];                 // [nb][K]
    __shared__ float red[NB][W];
    pdl_launch_dependents();
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int item = blockIdx.x * W + warp;
    const bool active = item < a.rows;
    const int K = a.K;
    int row[RPW];
    if constexpr (MODE == GEMV_GATEUP) {
        row[0] = item;
        row[1] = item + a.rows;
    } else if constexpr (MODE == GEMV_QKV) {
        const int half = a.head_dim >> 1;
        const int hh = item / half, j = item - hh * half;
        row[0] = hh * a.head_dim + j;
        row[1] = row[0] + half;
    } else {
#pragma unroll
        for (int r = 0; r < RPW; ++r) row[r] = item * RPW + r;
    }
    uint4 wr[RPW][MAXCH];
#pragma unroll
    for (int r = 0; r < RPW; ++r) {
        const __half* wrow = a.w + static_cast<size_t>(row[r]) * K;
#pragma unroll
        for (int c = 0; c < MAXCH; ++c) {
            const int e = (c * kWarp + lane) * 8;
            wr[r][c] = (active && e < K) ? ld_stream(wrow + e) : make_uint4(0, 0, 0, 0);
        }
    }
    const int n4 = K >> 2;
    uint2 gv[kV];  // the RMSNorm gain: a weight, read before the dependency wait
#pragma unroll
    for (int j = 0; j < kV; ++j) {
        const int i = threadIdx.x + j * T;
        gv[j] = (a.norm_g && i < n4) ? reinterpret_cast<const uint2*>(a.norm_g)[i] : make_uint2(0u, 0u);
    }
    pdl_wait();
    // every member's input and stop flag in one batch (a stopped member's input is still
    // valid memory; its results are simply not stored)
#pragma unroll
    for (int m = 0; m < NB; ++m) {
        if (m >= b.n) break;
#pragma unroll
        for (int j = 0; j < kV; ++j) {
            const int i = threadIdx.x + j * T;
            if (i < n4) cp_async16(xs + static_cast<size_t>(m) * K + 4 * i, b.x[m] + 4 * i);
        }
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
    bool live[NB];
    bool any = false;
#pragma unroll
    for (int m = 0; m < NB; ++m) {
        live[m] = m < b.n && !(a.skip_if_stopped && b.ctl[m] && b.ctl[m]->stopped);
        any = any || live[m];
    }
    asm volatile("cp.async.wait_group 0;" ::: "memory");
    if (!any) return;
    // each thread normalises the float4 it staged (its own copies: no barrier needed)
#pragma unroll
    for (int m = 0; m < NB; ++m) {
        if (!live[m]) continue;
        float ss = 0.f;
#pragma unroll
        for (int j = 0; j < kV; ++j) {
            const int i = threadIdx.x + j * T;
            if (i < n4) {
                float4* p4 = reinterpret_cast<float4*>(xs + static_cast<size_t>(m) * K) + i;
                float4 v = *p4;
                ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
                if (a.norm_g) {
                    const float2 g01 = __half22float2(*reinterpret_cast<const __half2*>(&gv[j].x));
                    const float2 g23 = __half22float2(*reinterpret_cast<const __half2*>(&gv[j].y));
                    v = make_float4(v.x * g01.x, v.y * g01.y, v.z * g23.x, v.w * g23.y);
                    *p4 = v;
                }
            }
        }
        if (a.norm_g) {
            ss = warp_sum(ss);
            if (lane == 0) red[m][warp] = ss;
        }
    }
    __syncthreads();
    float inv_rms[NB];
#pragma unroll
    for (int m = 0; m < NB; ++m) {
        inv_rms[m] = 1.f;
        if (a.norm_g && live[m]) {
            float t = 0.f;
#pragma unroll
            for (int w = 0; w < W; ++w) t += red[m][w];
            inv_rms[m] = rsqrtf(t / static_cast<float>(K) + a.eps);
        }
    }
    if (!active) return;
    float acc[NB][RPW];
#pragma unroll
    for (int m = 0; m < NB; ++m)
#pragma unroll
        for (int r = 0; r < RPW; ++r) acc[m][r] = 0.f;
#pragma unroll
    for (int c = 0; c < MAXCH; ++c) {
        const int e = (c * kWarp + lane) * 8;
        if (e < K) {
#pragma unroll
            for (int m = 0; m < NB; ++m) {
                if (!live[m]) continue;
                const float* xm = xs + static_cast<size_t>(m) * K;
                const float4 x0 = *reinterpret_cast<const float4*>(&xm[e]);
                const float4 x1 = *reinterpret_cast<const float4*>(&xm[e + 4]);
#pragma unroll
                for (int r = 0; r < RPW; ++r) acc[m][r] = dot8(wr[r][c], x0, x1, acc[m][r]);
            }
        }
    }
#pragma unroll
    for (int m = 0; m < NB; ++m) {
        if (!live[m]) continue;
#pragma unroll
        for (int r = 0; r < RPW; ++r) acc[m][r] = warp_sum(acc[m][r]) * inv_rms[m];
    }
#pragma unroll
    for (int m = 0; m < NB; ++m) {
        if (lane != m || !live[m]) continue;
        GemvArgs am = a;
        am.x = b.x[m];
        am.y = b.y[m];
        am.resid = b.resid[m];
        am.k_cache = b.k_cache[m];
        am.v_cache = b.v_cache[m];
        am.ctl = b.ctl[m];
        gemv_store<MODE, RPW>(am, item, row, acc[m]);
    }
}

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

template <int MODE, int RPW>
void dispatch_gemv(const GemvArgs& a, cudaStream_t s, bool pdl) {
    const int nch = (a.K + 255) / 256;
    const int blocks = (a.rows + kGemvWarps - 1) / kGemvWarps;
    cudaLaunchAttribute attr[1];
    cudaLaunchConfig_t cfg = make_cfg(dim3(blocks), dim3(kGemvThreads),
                                      static_cast<size_t>(((a.K + 7) / 8) * 8) * sizeof(float), s, pdl, attr);
    if (nch <= 1) check_launch(cudaLaunchKernelEx(&cfg, gemv_kernel<MODE, 1, RPW>, a));
    else if (nch <= 2) check_launch(cudaLaunchKernelEx(&cfg, gemv_kernel<MODE, 2, RPW>, a));
    else if (nch <= 4) check_launch(cudaLaunchKernelEx(&cfg, gemv_kernel<MODE, 4, RPW>, a));
    else if (nch <= 8) check_launch(cudaLaunchKernelEx(&cfg, gemv_kernel<MODE, 8, RPW>, a));
    else if (RPW == 1 && nch <= 16) check_launch(cudaLaunchKernelEx(&cfg, gemv_kernel<MODE, 16, 1>, a));
    else throw std::invalid_argument("gemv: input dimension too large");
}

// ------------------------------------------------------------ bulk GEMV ---
// A decoder-step form of the GEMV (an option; the register-streaming form is the
// default): at most one block per SM, each block's weight rows copied into shared
// memory by the bulk-copy engine (cp.async.bulk, completing on an mbarrier) BEFORE
// the dependency wait. A block holds no weights in registers, so the next kernel
// of the chain fits on the SM beside it and its copies stream while this one
// computes.
constexpr int kBulkThreads = 256;
constexpr int kBulkWarps = kBulkThreads / kWarp;
constexpr int kBulkBlocks = 148;
constexpr size_t kBulkSmemMax = 180 * 1024;

__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            static_cast<uint32_t>(__cvta_generic_to_shared(dst))),
        "l"(src), "r"(bytes), "r"(static_cast<uint32_t>(__cvta_generic_to_shared(bar)))
        : "memory");
}

// Time-bounded wait (kWaitNs) for phase 0 of a one-shot mbarrier; false on timeout.
__device__ __forceinline__ bool bulk_wait(uint64_t* bar) {
    return mbar_wait_addr(static_cast<uint32_t>(__cvta_generic_to_shared(bar)), 0);
}

// Weight rows per output unit: gate + up, or the two rows of a RoPE pair.
template <int MODE>
constexpr int bulk_rows() {
    return (MODE == GEMV_GATEUP || MODE == GEMV_QKV) ? 2 : 1;
}

// Output units [blockIdx.x * upb, + upb) of a.rows for the b.n members; IN_PLAIN input only.
template <int MODE, int NB>
__global__ void __launch_bounds__(kBulkThreads) gemv_bulk_kernel(const GemvArgs a, const GemvBatch b, int upb) {
    constexpr int R = bulk_rows<MODE>();
    extern __shared__ __align__(16) uint8_t bulk_sm[];
    __shared__ uint64_t bar;
    __shared__ float red[NB][kBulkWarps];
    pdl_launch_dependents();
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int K = a.K, nb = b.n;
    const int u0 = blockIdx.x * upb, nu = max(min(upb, a.rows - u0), 0);
    const size_t rowb = static_cast<size_t>(K) * 2;
    __half* ws = reinterpret_cast<__half*>(bulk_sm);  // [R * upb][K]
    float* xs = reinterpret_cast<float*>(bulk_sm + static_cast<size_t>(R) * upb * rowb);  // [nb][K]

    // 1) this block's weight rows into shared memory (independent of earlier kernels)
    if (tid == 0) {
        asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(static_cast<uint32_t>(__cvta_generic_to_shared(&bar)))
                     : "memory");
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        if (nu > 0) {
            asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(
                             static_cast<uint32_t>(__cvta_generic_to_shared(&bar))),
                         "r"(static_cast<uint32_t>(R * nu * rowb))
                         : "memory");
            if constexpr (MODE == GEMV_GATEUP) {
                bulk_g2s(ws, a.w + static_cast<size_t>(u0) * K, static_cast<uint32_t>(nu * rowb), &bar);
                bulk_g2s(ws + static_cast<size_t>(upb) * K, a.w + static_cast<size_t>(a.rows + u0) * K,
                         static_cast<uint32_t>(nu * rowb), &bar);
            } else if constexpr (MODE == GEMV_QKV) {
                const int half = a.head_dim >> 1;
                for (int i = 0; i < nu; ++i) {
                    const int p = u0 + i, hh = p / half, j = p - hh * half;
                    const size_t r0 = static_cast<size_t>(hh) * a.head_dim + j;
                    bulk_g2s(ws + static_cast<size_t>(2 * i) * K, a.w + r0 * K, static_cast<uint32_t>(rowb), &bar);
                    bulk_g2s(ws + static_cast<size_t>(2 * i + 1) * K, a.w + (r0 + half) * K,
                             static_cast<uint32_t>(rowb), &bar);
                }
            } else {
                bulk_g2s(ws, a.w + static_cast<size_t>(u0) * K, static_cast<uint32_t>(nu * rowb), &bar);
            }
        }
    }
    __syncthreads();  // the barrier is initialised before anyone waits on it

    // 2) wait for the producers of the input vectors
    pdl_wait();
    bool live[NB];
    bool any = false;
#pragma unroll
    for (int m = 0; m < NB; ++m) {
        live[m] = m < nb && !(a.skip_if_stopped && b.ctl[m] && b.ctl[m]->stopped);
        any = any || live[m];
    }

    // 3) each member's (optionally RMS-normalised) input: float4 loads, all issued at once
    float inv_rms[NB];
#pragma unroll
    for (int m = 0; m < NB; ++m) inv_rms[m] = 1.f;
    if (any) {
        const int n4 = K >> 2;
        constexpr int kV = 4;  // K <= 4096
        uint2 gv[kV];
#pragma unroll
        for (int j = 0; j < kV; ++j) {
            const int i = tid + j * kBulkThreads;
            gv[j] = (a.norm_g && i < n4) ? reinterpret_cast<const uint2*>(a.norm_g)[i] : make_uint2(0u, 0u);
        }
#pragma unroll
        for (int m = 0; m < NB; ++m) {
            if (!live[m]) continue;
            float4 xv[kV];
#pragma unroll
            for (int j = 0; j < kV; ++j) {
                const int i = tid + j * kBulkThreads;
                xv[j] = i < n4 ? reinterpret_cast<const float4*>(b.x[m])[i] : make_float4(0.f, 0.f, 0.f, 0.f);
            }
            float ss = 0.f;
#pragma unroll
            for (int j = 0; j < kV; ++j) {
                const int i = tid + j * kBulkThreads;
                if (i < n4) {
                    float4 v = xv[j];
                    ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
                    if (a.norm_g) {
                        const float2 g01 = __half22float2(*reinterpret_cast<const __half2*>(&gv[j].x));
                        const float2 g23 = __half22float2(*reinterpret_cast<const __half2*>(&gv[j].y));
                        v = make_float4(v.x * g01.x, v.y * g01.y, v.z * g23.x, v.w * g23.y);
                    }
                    reinterpret_cast<float4*>(xs + static_cast<size_t>(m) * K)[i] = v;
                }
            }
            if (a.norm_g) {
                ss = warp_sum(ss);
                if (lane == 0) red[m][warp] = ss;
            }
        }
        __syncthreads();
        if (a.norm_g) {
#pragma unroll
            for (int m = 0; m < NB; ++m) {
                if (!live[m]) continue;
                float t = 0.f;
#pragma unroll
                for (int w = 0; w < kBulkWarps; ++w) t += red[m][w];
                inv_rms[m] = rsqrtf(t / static_cast<float>(K) + a.eps);
            }
        }
    }

    // 4) the weights have landed (every thread waits: none may read early, and the
    // block may not exit with a copy in flight; bounded)
    const bool ok = nu == 0 || bulk_wait(&bar);
    if (!ok && tid == 0)
        for (int m = 0; m < nb; ++m)
            if (b.ctl[m]) b.ctl[m]->error = 3;
    if (!any || !ok) return;

    // 5) dot products: warp w takes units w, w + 8, ...; each weight row is read
    // once from shared memory for every member
    for (int i = warp; i < nu; i += kBulkWarps) {
        const __half* w0 = ws + static_cast<size_t>(MODE == GEMV_QKV ? 2 * i : i) * K;
        const __half* w1 = MODE == GEMV_GATEUP ? ws + static_cast<size_t>(upb + i) * K : w0 + K;
        float acc[NB][2];
#pragma unroll
        for (int m = 0; m < NB; ++m) acc[m][0] = acc[m][1] = 0.f;
        for (int e = lane * 8; e < K; e += kWarp * 8) {
            const uint4 wa = *reinterpret_cast<const uint4*>(w0 + e);
            uint4 wb = wa;
            if (R == 2) wb = *reinterpret_cast<const uint4*>(w1 + e);
#pragma unroll
            for (int m = 0; m < NB; ++m) {
                if (!live[m]) continue;
                const float* xm = xs + static_cast<size_t>(m) * K;
                const float4 x0 = *reinterpret_cast<const float4*>(&xm[e]);
                const float4 x1 = *reinterpret_cast<const float4*>(&xm[e + 4]);
                acc[m][0] = dot8(wa, x0, x1, acc[m][0]);
                if (R == 2) acc[m][1] = dot8(wb, x0, x1, acc[m][1]);
            }
        }
#pragma unroll
        for (int m = 0; m < NB; ++m) {
            if (!live[m]) continue;
#pragma unroll
            for (int r = 0; r < R; ++r) acc[m][r] = warp_sum(acc[m][r]) * inv_rms[m];
        }
        // lane m stores member m
#pragma unroll
        for (int m = 0; m < NB; ++m) {
            if (lane != m || !live[m]) continue;
            const int item = u0 + i;
            int row[2];
            if constexpr (MODE == GEMV_GATEUP) {
                row[0] = item;
                row[1] = item + a.rows;
            } else if constexpr (MODE == GEMV_QKV) {
                const int half = a.head_dim >> 1;
                const int hh = item / half, j = item - hh * half;
                row[0] = hh * a.head_dim + j;
                row[1] = row[0] + half;
            } else {
                row[0] = item;
                row[1] = item;
            }
            GemvArgs am = a;
            am.x = b.x[m];
            am.y = b.y[m];
            am.resid = b.resid[m];
            am.k_cache = b.k_cache[m];
            am.v_cache = b.v_cache[m];
            am.ctl = b.ctl[m];
            gemv_store<MODE, R>(am, item, row, acc[m]);
        }
    }
}

template <int MODE>
void dispatch_gemv_bulk(const GemvArgs& a, const GemvBatch& b, cudaStream_t s, bool pdl) {
    constexpr int R = bulk_rows<MODE>();
    const size_t rowb = static_cast<size_t>(a.K) * 2, xb = static_cast<size_t>(b.n) * a.K * 4;
    int upb = (a.rows + kBulkBlocks - 1) / kBulkBlocks;
    while (upb > 1 && R * upb * rowb + xb > kBulkSmemMax) upb = (upb + 1) / 2;
    const size_t smem = R * upb * rowb + xb;
    if (smem > kBulkSmemMax) throw std::invalid_argument("gemv_bulk: rows too long for shared memory");
    const int blocks = (a.rows + upb - 1) / upb;
    cudaLaunchAttribute attr[1];
    cudaLaunchConfig_t cfg = make_cfg(dim3(blocks), dim3(kBulkThreads), smem, s, pdl, attr);
    // a lone stream's launch unrolls one member slot (fewer registers), a group's all of them
    if (b.n == 1) check_launch(cudaLaunchKernelEx(&cfg, gemv_bulk_kernel<MODE, 1>, a, b, upb));
    else check_launch(cudaLaunchKernelEx(&cfg, gemv_bulk_kernel<MODE, kGemvBatch>, a, b, upb));
}

// NB: the member slots a launch unrolls (4 for groups of up to 4, else 8); W: warps per
// CTA, 16 for every batch (the staged inputs serve 16 weight rows; 12 groups of 4
// measured 2110 against 2018-2088 patches/s with 4 warps)
template <int NB>
constexpr int batch_warps() { return 16; }

template <int MODE, int RPW, int NB>
void dispatch_gemv_batch_nb(const GemvArgs& a, const GemvBatch& b, cudaStream_t s, bool pdl) {
    constexpr int W = batch_warps<NB>();
    const int nch = (a.K + 255) / 256;
    const int blocks = (a.rows + W - 1) / W;
    cudaLaunchAttribute attr[1];
    cudaLaunchConfig_t cfg = make_cfg(dim3(blocks), dim3(W * 32),
                                      static_cast<size_t>(b.n) * ((a.K + 7) / 8) * 8 * sizeof(float), s, pdl, attr);
    if (nch <= 1) check_launch(cudaLaunchKernelEx(&cfg, gemv_batch_kernel<MODE, 1, RPW, NB, W>, a, b));
    else if (nch <= 2) check_launch(cudaLaunchKernelEx(&cfg, gemv_batch_kernel<MODE, 2, RPW, NB, W>, a, b));
    else if (nch <= 4) check_launch(cudaLaunchKernelEx(&cfg, gemv_batch_kernel<MODE, 4, RPW, NB, W>, a, b));
    else if (nch <= 8) check_launch(cudaLaunchKernelEx(&cfg, gemv_batch_kernel<MODE, 8, RPW, NB, W>, a, b));
    else if (RPW == 1 && nch <= 16) check_launch(cudaLaunchKernelEx(&cfg, gemv_batch_kernel<MODE, 16, 1, NB, W>, a, b));
    else throw std::invalid_argument("gemv_batch: input dimension too large");
}

template <int MODE, int RPW>
void dispatch_gemv_batch(const GemvArgs& a, const GemvBatch& b, cudaStream_t s, bool pdl) {
    if (b.n <= 4) dispatch_gemv_batch_nb<MODE, RPW, 4>(a, b, s, pdl);
    else dispatch_gemv_batch_nb<MODE, RPW, kGemvBatch>(a, b, s, pdl);
}

// ------------------------------------------------------------ attention ---
constexpr int kAttnSplitThreads = 256;  // the split-K decode: more warps per scheduler to hide latency
constexpr int kMaxGroup = 16;

constexpr int kMinKeysPerSplit = 16;

// four consecutive elements of a K/V row starting at element c (c % 4 == 0;
// rows start on 16-byte boundaries, which the launcher checks)
template <typename KV>
__device__ __forceinline__ void load4(const KV* p, int c, float* r);
template <>
__device__ __forceinline__ void load4<float>(const float* p, int c, float* r) {
    const float4 v = *reinterpret_cast<const float4*>(p + c);
    r[0] = v.x;
    r[1] = v.y;
    r[2] = v.z;
    r[3] = v.w;
}
template <>
__device__ __forceinline__ void load4<__half>(const __half* p, int c, float* r) {
    const uint2 v = *reinterpret_cast<const uint2*>(p + c);
    const float2 lo = __half22float2(*reinterpret_cast<const __half2*>(&v.x));
    const float2 hi = __half22float2(*reinterpret_cast<const __half2*>(&v.y));
    r[0] = lo.x;
    r[1] = lo.y;
    r[2] = hi.x;
    r[3] = hi.y;
}

// Split-K flash decode. The number of active splits follows the current key
// count T (at least kMinKeysPerSplit keys each, at most 'splits'), so short
// caches do not pay for empty splits; inactive CTAs leave at once. Each split
// walks its keys in tiles of kKeyTile rows: the tile's K and V rows are staged
// in shared memory by one batch of parallel loads, scores for all G query heads
// of the KV group come from shared memory, and an online softmax (running max
// and sum per head) rescales the P.V accumulators. The last active CTA of a KV
// head combines the partial (max, sum, P.V) triples.
constexpr int kKeyTile = 32;
constexpr int kRowPad = 65;  // padded shared-memory row: conflict-free column reads

// Shared memory of one split's pass over its keys.
struct AttnSmem {
    float qs[kMaxGroup][kRowPad];
    float ks[kKeyTile][kRowPad];
    float vs[kKeyTile][64];
    float sc[kMaxGroup][kKeyTile];
    float m_s[kMaxGroup], l_s[kMaxGroup], alpha_s[kMaxGroup];
};

// The G query rows of KV head kvh, scaled, into S.qs (the caller's first loads
// after the dependency wait, issued beside its reads of the control block).
template <int NT>
__device__ __forceinline__ void stage_q(const AttnArgs& a, AttnSmem& S, int kvh, int G) {
    constexpr int D = 64;
    for (int i = threadIdx.x; i < G * D; i += NT) S.qs[i / D][i % D] = a.q[kvh * G * D + i] * a.scale;
}

// Keys [t0, t0 + n) of KV head kvh against the group's G query heads (rows staged
// by stage_q before the call): tiles of
// kKeyTile rows staged by one batch of loads, online softmax per head. On
// return S.m_s / S.l_s hold the running max and sum, acc[j] the P.V partial of
// head g_lo + j at column e = tid % 64 (heads split over the NT / 64 thread groups of
// the block).
template <typename KV, int D, int NT>
__device__ __forceinline__ void attend_keys(const AttnArgs& a, AttnSmem& S, int kvh, int G, int t0, int n, int len0,
                                            float* acc) {
    constexpr int kGroups = NT / D;  // thread groups the query heads are split over
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    if (tid < G) {
        S.m_s[tid] = -1e30f;
        S.l_s[tid] = 0.f;
    }
    const KV* k0 = static_cast<const KV*>(a.k0) + static_cast<size_t>(kvh) * a.stride0 * D;
    const KV* v0 = static_cast<const KV*>(a.v0) + static_cast<size_t>(kvh) * a.stride0 * D;
    const KV* k1 = a.k1 ? static_cast<const KV*>(a.k1) + static_cast<size_t>(kvh) * a.stride1 * D : nullptr;
    const KV* v1 = a.v1 ? static_cast<const KV*>(a.v1) + static_cast<size_t>(kvh) * a.stride1 * D : nullptr;
    const int e = tid & (D - 1), gh = tid / D;
    const int hg = (G + kGroups - 1) / kGroups, g_lo = gh * hg, g_hi = min(G, g_lo + hg);
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[j] = 0.f;
    for (int tb = 0; tb < n; tb += kKeyTile) {
        const int nt = min(kKeyTile, n - tb);
        __syncthreads();  // previous tile fully consumed (and q / stats initialised)
#pragma unroll 4
        for (int i = tid; i < nt * (D / 4); i += NT) {
            const int r = i / (D / 4), c = (i % (D / 4)) * 4;
            const int row = t0 + tb + r;
            const KV* kp = row < len0 ? k0 + static_cast<size_t>(row) * D : k1 + static_cast<size_t>(row - len0) * D;
            const KV* vp = row < len0 ? v0 + static_cast<size_t>(row) * D : v1 + static_cast<size_t>(row - len0) * D;
            float kr[4], vr[4];
            load4(kp, c, kr);
            load4(vp, c, vr);
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                S.ks[r][c + j] = kr[j];
                S.vs[r][c + j] = vr[j];
            }
        }
        __syncthreads();
        for (int i = tid; i < G * nt; i += NT) {
            const int g = i / nt, t = i - g * nt;
            float s = 0.f;
#pragma unroll 16
            for (int c = 0; c < D; ++c) s = fmaf(S.qs[g][c], S.ks[t][c], s);
            S.sc[g][t] = s + (a.mask ? a.mask[t0 + tb + t] : 0.f);
        }
        __syncthreads();
        for (int g = warp; g < G; g += NT / kWarp) {
            const float x = lane < nt ? S.sc[g][lane] : -1e30f;
            const float m_old = S.m_s[g];
            const float m_new = fmaxf(m_old, warp_max(x));
            const float p = lane < nt ? __expf(x - m_new) : 0.f;
            if (lane < nt) S.sc[g][lane] = p;
            const float psum = warp_sum(p);
            if (lane == 0) {
                const float alpha = __expf(m_old - m_new);
                S.alpha_s[g] = alpha;
                S.l_s[g] = S.l_s[g] * alpha + psum;
                S.m_s[g] = m_new;
            }
        }
        __syncthreads();
#pragma unroll
        for (int j = 0; j < 8; ++j)
            if (g_lo + j < g_hi) acc[j] *= S.alpha_s[g_lo + j];
        for (int t = 0; t < nt; ++t) {
            const float v = S.vs[t][e];
#pragma unroll
            for (int j = 0; j < 8; ++j)
                if (g_lo + j < g_hi) acc[j] = fmaf(S.sc[g_lo + j][t], v, acc[j]);
        }
    }
}

template <typename KV, int D>
__global__ void __launch_bounds__(kAttnSplitThreads) attn_decode_kernel(const AttnArgs a) {
    constexpr int NT = kAttnSplitThreads;
    static_assert(D == 64, "head_dim 64");
    __shared__ AttnSmem S;
    __shared__ int s_last;
    extern __shared__ float ps[];  // combine staging: [splits][G][D + 2]
    pdl_launch_dependents();
    pdl_wait();
    // the control block and the query rows are read in one batch of loads; nothing
    // is written to global memory before the stop flag is acted on
    int stop = 0, kv_len = 0;
    if (a.ctl) {
        stop = a.skip_if_stopped ? a.ctl->stopped : 0;
        kv_len = a.ctl->kv_len[a.which];
    }
    const int G = a.q_heads / a.kv_heads;
    const int split = blockIdx.x, kvh = blockIdx.y;
    const int tid = threadIdx.x;
    stage_q<NT>(a, S, kvh, G);
    if (stop) return;
    int len0 = a.len0, len1 = a.len1;
    if (a.ctl) {
        len0 = min(kv_len + 1, a.len0);  // len0 holds the capacity here
        len1 = 0;
    }
    const int T = len0 + len1;
    const int active = max(1, min(a.splits, (T + kMinKeysPerSplit - 1) / kMinKeysPerSplit));
    if (split >= active) return;
    const int chunk = (T + active - 1) / active;
    const int t0 = split * chunk;
    const int n = max(0, min(T, t0 + chunk) - t0);
    const int e = tid & (D - 1), gh = tid / D;
    const int hg = (G + NT / D - 1) / (NT / D), g_lo = gh * hg, g_hi = min(G, g_lo + hg);
    float acc[8];
    attend_keys<KV, D, NT>(a, S, kvh, G, t0, n, len0, acc);
    float* m_s = S.m_s;
    float* l_s = S.l_s;
    __syncthreads();
    // this split's partial (m, l, P.V) per head
    float* part = a.partial + (static_cast<size_t>(kvh) * a.splits + split) * G * (D + 2);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        const int g = g_lo + j;
        if (g < g_hi) part[g * (D + 2) + e] = acc[j];
    }
    if (tid < G) {
        part[tid * (D + 2) + D] = n > 0 ? m_s[tid] : -1e30f;
        part[tid * (D + 2) + D + 1] = l_s[tid];
    }
    __threadfence();
    __syncthreads();
    if (tid == 0) s_last = atomicAdd(&a.counters[kvh], 1) == active - 1;
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    // combine the active splits of this KV head, staged with up to 72 loads in flight per
    // thread: one L2 round trip for up to 72 x 128 floats (17 splits of 8 heads)
    const float* pk = a.partial + static_cast<size_t>(kvh) * a.splits * G * (D + 2);
    const int total = active * G * (D + 2);
    constexpr int kB = 72;
    for (int base = tid; base < total; base += NT * kB) {
        float v[kB];
#pragma unroll
        for (int j = 0; j < kB; ++j) {
            const int i = base + j * NT;
            v[j] = i < total ? __ldcg(pk + i) : 0.f;
        }
#pragma unroll
        for (int j = 0; j < kB; ++j) {
            const int i = base + j * NT;
            if (i < total) ps[i] = v[j];
        }
    }
    __syncthreads();
    for (int it = tid; it < G * D; it += NT) {
        const int g = it / D, c = it - g * D;
        float M = -1e30f;
        for (int sp = 0; sp < active; ++sp) M = fmaxf(M, ps[(sp * G + g) * (D + 2) + D]);
        float num = 0.f, den = 0.f;
        for (int sp = 0; sp < active; ++sp) {
            const float* pp = ps + (sp * G + g) * (D + 2);
            const float w = __expf(pp[D] - M);
            num = fmaf(w, pp[c], num);
            den = fmaf(w, pp[D + 1], den);
        }
        a.out[(kvh * G + g) * D + c] = num / den;
    }
    if (tid == 0) a.counters[kvh] = 0;
}

constexpr int kFinalNormThreads = 256, kFinalNormPer = 16;  // H <= 4096

__global__ void final_norm_kernel(const float* h, const __half* g, float eps, int H, float* out,
                                  float* out2, StreamCtl* ctl, int which, int bump, int skip) {
    __shared__ float red[kFinalNormThreads / 32];
    pdl_launch_dependents();
    const int tid = threadIdx.x;
    float gv[kFinalNormPer], hv[kFinalNormPer];
#pragma unroll
    for (int j = 0; j < kFinalNormPer; ++j) {  // the gain does not depend on the previous kernel
        const int k = tid + j * kFinalNormThreads;
        gv[j] = k < H ? __half2float(g[k]) : 0.f;
    }
    pdl_wait();
    // the stop flag and the hidden row in one batch of loads; nothing is written before the check
    const bool stop = skip && ctl && ctl->stopped;
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < kFinalNormPer; ++j) {
        const int k = tid + j * kFinalNormThreads;
        hv[j] = k < H ? h[k] : 0.f;
    }
#pragma unroll
    for (int j = 0; j < kFinalNormPer; ++j) ss += hv[j] * hv[j];
    ss = warp_sum(ss);
    if ((tid & 31) == 0) red[tid >> 5] = ss;
    __syncthreads();
    if (stop) return;
    float t = 0.f;
#pragma unroll
    for (int w = 0; w < kFinalNormThreads / 32; ++w) t += red[w];
    const float a = rsqrtf(t / static_cast<float>(H) + eps);
#pragma unroll
    for (int j = 0; j < kFinalNormPer; ++j) {
        const int k = tid + j * kFinalNormThreads;
        if (k < H) {
            const float v = hv[j] * a * gv[j];
            out[k] = v;
            if (out2) out2[k] = v;
        }
    }
    if (bump && ctl && tid == 0) ctl->kv_len[which] += bump;
}

}  // namespace

void launch_gemv_bulk_batch(const GemvArgs& a, const GemvBatch& b, cudaStream_t s, bool pdl) {
    bool aligned = true;
    for (int m = 0; m < b.n; ++m) aligned = aligned && (reinterpret_cast<uintptr_t>(b.x[m]) & 15) == 0;
    if (a.K <= 0 || a.K % 8 != 0 || a.K > 4096 || a.rows <= 0 || a.in_mode != IN_PLAIN || b.n < 1 ||
        b.n > kGemvBatch || !aligned || (reinterpret_cast<uintptr_t>(a.w) & 15) != 0 ||
        (reinterpret_cast<uintptr_t>(a.norm_g) & 7) != 0)
        throw std::invalid_argument("gemv_bulk: bad shape, batch or alignment");
    switch (a.mode) {
        case GEMV_PLAIN: dispatch_gemv_bulk<GEMV_PLAIN>(a, b, s, pdl); break;
        case GEMV_RESID: dispatch_gemv_bulk<GEMV_RESID>(a, b, s, pdl); break;
        case GEMV_GATEUP: dispatch_gemv_bulk<GEMV_GATEUP>(a, b, s, pdl); break;
        case GEMV_QKV:
            for (int m = 0; m < b.n; ++m)
                if (b.ctl[m] == nullptr) throw std::invalid_argument("gemv_bulk: q/k/v needs a control block");
            if (a.head_dim % 2 != 0) throw std::invalid_argument("gemv_bulk: bad q/k/v setup");
            dispatch_gemv_bulk<GEMV_QKV>(a, b, s, pdl);
            break;
        default: throw std::invalid_argument("gemv_bulk: unknown mode");
    }
}

void launch_gemv_bulk(const GemvArgs& a, cudaStream_t s, bool pdl) {
    GemvBatch b;
    b.n = 1;
    b.x[0] = a.x;
    b.y[0] = a.y;
    b.resid[0] = a.resid;
    b.k_cache[0] = a.k_cache;
    b.v_cache[0] = a.v_cache;
    b.ctl[0] = a.ctl;
    launch_gemv_bulk_batch(a, b, s, pdl);
}

void launch_gemv_batch(const GemvArgs& a, const GemvBatch& b, cudaStream_t s, bool pdl) {
    bool aligned = true;
    for (int m = 0; m < b.n; ++m) aligned = aligned && (reinterpret_cast<uintptr_t>(b.x[m]) & 15) == 0;
    if (a.K <= 0 || a.K % 8 != 0 || a.rows <= 0 || a.in_mode != IN_PLAIN || b.n < 1 || b.n > kGemvBatch ||
        !aligned || (reinterpret_cast<uintptr_t>(a.norm_g) & 7) != 0 ||
        static_cast<size_t>(b.n) * a.K * 4 > 160 * 1024)
        throw std::invalid_argument("gemv_batch: bad shape, batch or alignment");
    switch (a.mode) {
        case GEMV_PLAIN: dispatch_gemv_batch<GEMV_PLAIN, 1>(a, b, s, pdl); break;
        case GEMV_RESID: dispatch_gemv_batch<GEMV_RESID, 1>(a, b, s, pdl); break;
        case GEMV_GATEUP: dispatch_gemv_batch<GEMV_GATEUP, 2>(a, b, s, pdl); break;
        case GEMV_QKV:
            for (int m = 0; m < b.n; ++m)
                if (b.ctl[m] == nullptr) throw std::invalid_argument("gemv_batch: q/k/v needs a control block");
            if (a.head_dim % 2 != 0) throw std::invalid_argument("gemv_batch: bad q/k/v setup");
            dispatch_gemv_batch<GEMV_QKV, 2>(a, b, s, pdl);
            break;
        default: throw std::invalid_argument("gemv_batch: unknown mode");
    }
}

void launch_gemv(const GemvArgs& a, cudaStream_t s, bool pdl) {
    if (a.K <= 0 || a.K % 8 != 0 || a.rows <= 0) throw std::invalid_argument("gemv: bad shape");
    switch (a.mode) {
        case GEMV_PLAIN: dispatch_gemv<GEMV_PLAIN, 1>(a, s, pdl); break;
        case GEMV_RESID: dispatch_gemv<GEMV_RESID, 1>(a, s, pdl); break;
        case GEMV_GATEUP: dispatch_gemv<GEMV_GATEUP, 2>(a, s, pdl); break;
        case GEMV_QKV:
            if (a.head_dim % 2 != 0 || a.ctl == nullptr) throw std::invalid_argument("gemv: bad q/k/v setup");
            dispatch_gemv<GEMV_QKV, 2>(a, s, pdl);
            break;
        default: throw std::invalid_argument("gemv: unknown mode");
    }
}

// The same decode with the split-K combine inside a thread-block cluster: the
// cluster's CTAs take one contiguous key range each and send their (P.V, max, sum)
// for head g into CTA g's shared memory as asynchronous stores counted on CTA g's
// mbarrier; CTA g combines head g in rank order. No global scratch, no atomics, no
// remote loads.
// The cluster has 16 CTAs (a non-portable size); the key range is spread over
// max(8, ceil(T / 32)) of them, so up to 512 keys every working CTA walks one
// 32-key tile, and short rows do not pay for a 16-way combine.
constexpr int kAttnCluster = 16;
constexpr int kAttnMinActive = 8;

// One cluster CTA: 8 warps, warp w owns query heads w and w + 8 of the KV group.
// Its key range is walked in 32-key tiles staged in shared memory by cp.async (K
// rows padded to 68 floats: a quarter-warp's 16-byte reads of 8 rows hit 32
// distinct banks), two buffers so the next tile's copies are in flight while the
// current one is scored.
// Per tile and head, lane j scores key j, the online softmax runs across the lanes,
// and lane l accumulates output columns 2l and 2l + 1 (P.V with the probabilities
// broadcast by shuffles): no block barrier between the phases of a tile.
constexpr int kClThreads = 256;
constexpr int kClWarps = kClThreads / 32;
constexpr int kClKeys = 32;
constexpr int kClKRow = 68;

template <typename KV, int D>
__global__ void __launch_bounds__(kClThreads) attn_decode_cluster_kernel(const AttnArgs a0, const AttnBatch b) {
    static_assert(D == 64, "head_dim 64");
    static_assert(sizeof(KV) == 4, "fp32 key/value rows");
    __shared__ __align__(16) float ks[2][kClKeys][kClKRow];
    __shared__ __align__(16) float vs[2][kClKeys][D];
    __shared__ __align__(16) float qs[kMaxGroup][D];
    // combiner of head g = rank: every working CTA's (P.V, max, sum) for it, 66 floats each
    __shared__ __align__(16) float rbuf[kAttnCluster][D + 2];
    __shared__ uint64_t rbar;
    pdl_launch_dependents();
    if (threadIdx.x == 0) {
        tc::mbar_init(&rbar, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    AttnArgs a = a0;
    if (b.n > 0) {  // member blockIdx.z of a group (a cluster spans x only: one member per cluster)
        const int m = blockIdx.z;
        a.q = b.q[m];
        a.k0 = b.k0[m];
        a.v0 = b.v0[m];
        a.out = b.out[m];
        a.ctl = b.ctl[m];
    }
    pdl_wait();
    // the control block and the query rows are read in one batch of loads. The stop
    // flag is uniform over the grid (it cannot change while the kernel runs), so every
    // CTA of a cluster takes the same branch
    int stop = 0, kv_len = 0;
    if (a.ctl) {
        stop = a.skip_if_stopped ? a.ctl->stopped : 0;
        kv_len = a.ctl->kv_len[a.which];
    }
    const int G = a.q_heads / a.kv_heads, C = kAttnCluster;
    const int rank = blockIdx.x, kvh = blockIdx.y, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    for (int i = tid; i < G * D; i += kClThreads) qs[i / D][i % D] = a.q[kvh * G * D + i] * a.scale;
    if (stop) return;
    int len0 = a.len0, len1 = a.len1;
    if (a.ctl) {
        len0 = min(kv_len + 1, a.len0);  // len0 holds the capacity here
        len1 = 0;
    }
    const int T = len0 + len1;
    const int act = min(C, max(kAttnMinActive, (T + kKeyTile - 1) / kKeyTile));  // working CTAs
    const int chunk = (T + act - 1) / act, t0 = rank * chunk;
    const int n = rank < act ? max(0, min(T, t0 + chunk) - t0) : 0;
    // The combiner of head g (CTA g, g < G) expects act partials of 264 bytes. The
    // cluster-barrier arrival (release) orders this CTA's barrier set-up before any peer's
    // push, which waits for every arrival; the wait comes after the key tiles.
    constexpr uint32_t kPartBytes = (D + 2) * 4;
    __syncthreads();  // thread 0's barrier initialisation is done
    if (rank < G && tid == 0) tc::mbar_expect_tx(&rbar, static_cast<uint32_t>(act) * kPartBytes);
    asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
    const KV* k0 = static_cast<const KV*>(a.k0) + static_cast<size_t>(kvh) * a.stride0 * D;
    const KV* v0 = static_cast<const KV*>(a.v0) + static_cast<size_t>(kvh) * a.stride0 * D;
    const KV* k1 = a.k1 ? static_cast<const KV*>(a.k1) + static_cast<size_t>(kvh) * a.stride1 * D : nullptr;
    const KV* v1 = a.v1 ? static_cast<const KV*>(a.v1) + static_cast<size_t>(kvh) * a.stride1 * D : nullptr;
    // tile copies: 2 x 32 rows x 16 float4 over 256 threads, 4 cp.async each, one group
    auto stage = [&](int buf, int tb) {
        const int nt = min(kClKeys, n - tb);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int i = tid + j * kClThreads;  // 0 .. 1023
            const int kv = i >> 9, r = (i >> 4) & 31, c = (i & 15) * 4;
            if (r < nt) {
                const int row = t0 + tb + r;
                const KV* base = kv == 0 ? (row < len0 ? k0 : k1) : (row < len0 ? v0 : v1);
                const KV* p = base + static_cast<size_t>(row < len0 ? row : row - len0) * D + c;
                cp_async16(kv == 0 ? &ks[buf][r][c] : &vs[buf][r][c], p);
            }
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
    };
    float m_run[2] = {-1e30f, -1e30f}, l_run[2] = {0.f, 0.f};
    float acc[2][2] = {{0.f, 0.f}, {0.f, 0.f}};
    if (n > 0) stage(0, 0);
    asm volatile("cp.async.wait_group 0;" ::: "memory");
    __syncthreads();  // q rows and the first tile staged
    for (int tb = 0, buf = 0; tb < n; tb += kClKeys, buf ^= 1) {
        if (tb + kClKeys < n) stage(buf ^ 1, tb + kClKeys);  // the next tile's loads in flight
        const int nt = min(kClKeys, n - tb);
        float kr[D];  // lane j's key row
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
        const float mk = (a.mask && lane < nt) ? a.mask[t0 + tb + lane] : 0.f;
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
            const int g = warp + hh * kClWarps;
            if (g >= G) break;
            float x = -1e30f;
            if (lane < nt) {
                float s4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
                for (int c = 0; c < D; c += 4) {
                    const float4 q4 = *reinterpret_cast<const float4*>(&qs[g][c]);
                    s4[0] = fmaf(q4.x, kr[c], s4[0]);
                    s4[1] = fmaf(q4.y, kr[c + 1], s4[1]);
                    s4[2] = fmaf(q4.z, kr[c + 2], s4[2]);
                    s4[3] = fmaf(q4.w, kr[c + 3], s4[3]);
                }
                x = ((s4[0] + s4[1]) + (s4[2] + s4[3])) + mk;
            }
            const float m_new = fmaxf(m_run[hh], warp_max(x));
            const float p = lane < nt ? __expf(x - m_new) : 0.f;
            const float alpha = __expf(m_run[hh] - m_new);
            l_run[hh] = l_run[hh] * alpha + warp_sum(p);
            m_run[hh] = m_new;
            float o0 = acc[hh][0] * alpha, o1 = acc[hh][1] * alpha;
            for (int j = 0; j < nt; ++j) {
                const float pj = __shfl_sync(0xffffffffu, p, j);
                const float2 v2 = *reinterpret_cast<const float2*>(&vs[buf][j][2 * lane]);
                o0 = fmaf(pj, v2.x, o0);
                o1 = fmaf(pj, v2.y, o1);
            }
            acc[hh][0] = o0;
            acc[hh][1] = o1;
        }
        asm volatile("cp.async.wait_group 0;" ::: "memory");
        __syncthreads();  // this tile consumed, the next one staged
    }
    // Combine: CTA g (g < G) combines head g. Every working CTA (rank < act) sends its
    // (P.V, max, sum) for head g into CTA g's rbuf[rank] as asynchronous 8-byte stores that
    // complete on CTA g's barrier; a combiner waits for its own bytes only, and no CTA reads
    // another's shared memory, so none waits for the others before it exits.
    tc::cluster_wait();  // every CTA's receive barrier is set up
    if (rank < act) {
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
            const int g = warp + hh * kClWarps;
            if (g < G) {
                float* dst = &rbuf[rank][0];
                const uint32_t base = tc::peer_addr(dst, static_cast<uint32_t>(g));
                const uint32_t bar = tc::peer_addr(&rbar, static_cast<uint32_t>(g));
                tc::st_async2(base + 8u * lane, acc[hh][0], acc[hh][1], bar);
                if (lane == 0) tc::st_async2(base + 4u * D, n > 0 ? m_run[hh] : -1e30f, l_run[hh], bar);
            }
        }
    }
    if (rank < G) {
        const bool got = tc::mbar_wait_cluster(&rbar, 0);
        if (!got && tid == 0 && a.ctl) a.ctl->error = 3;
        if (got && tid < D) {
            const int g = rank;
            float mr[kAttnCluster], lr[kAttnCluster], ar[kAttnCluster];
#pragma unroll
            for (int r = 0; r < kAttnCluster; ++r) {  // ranks past 'act' hold no keys: weight 0
                mr[r] = r < act ? rbuf[r][D] : -1e30f;
                lr[r] = r < act ? rbuf[r][D + 1] : 0.f;
                ar[r] = r < act ? rbuf[r][tid] : 0.f;
            }
            float M = -1e30f;
#pragma unroll
            for (int r = 0; r < kAttnCluster; ++r) M = fmaxf(M, mr[r]);
            float num = 0.f, den = 0.f;
#pragma unroll
            for (int r = 0; r < kAttnCluster; ++r) {
                const float w = __expf(mr[r] - M);
                num = fmaf(w, ar[r], num);
                den = fmaf(w, lr[r], den);
            }
            a.out[(kvh * G + g) * D + tid] = num / den;
        }
    }
}

void launch_attn_decode_cluster_batch(const AttnArgs& a, const AttnBatch& b, cudaStream_t s, bool pdl) {
    if (a.head_dim != 64) throw std::invalid_argument("attention: head_dim must be 64");
    if (a.kv_heads <= 0 || a.q_heads % a.kv_heads != 0) throw std::invalid_argument("attention: bad head grouping");
    const int G = a.q_heads / a.kv_heads;
    if (G < 1 || G > kMaxGroup) throw std::invalid_argument("attention: more than 16 query heads per KV head");
    if (b.n < 0 || b.n > kGroupMembers) throw std::invalid_argument("attention: 1 to 8 members");
    for (const void* p : {a.k0, a.v0, a.k1, a.v1})
        if (reinterpret_cast<uintptr_t>(p) % 16 != 0)
            throw std::invalid_argument("attention: key/value rows must start on 16-byte boundaries");
    for (int m = 0; m < b.n; ++m)
        if ((reinterpret_cast<uintptr_t>(b.k0[m]) | reinterpret_cast<uintptr_t>(b.v0[m])) % 16 != 0)
            throw std::invalid_argument("attention: key/value rows must start on 16-byte boundaries");
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(kAttnCluster, a.kv_heads, b.n > 0 ? b.n : 1);
    cfg.blockDim = dim3(kClThreads);
    cfg.stream = s;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = kAttnCluster;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 2 : 1;
    check_launch(cudaLaunchKernelEx(&cfg, attn_decode_cluster_kernel<float, 64>, a, b));
}

void launch_attn_decode_cluster(const AttnArgs& a, cudaStream_t s, bool pdl) {
    launch_attn_decode_cluster_batch(a, AttnBatch{}, s, pdl);
}

void launch_attn_decode(const AttnArgs& a, bool fp16_kv, cudaStream_t s, bool pdl) {
    if (a.head_dim != 64) throw std::invalid_argument("attention: head_dim must be 64");
    if (a.kv_heads <= 0 || a.q_heads % a.kv_heads != 0 || a.splits < 1)
        throw std::invalid_argument("attention: bad head grouping");
    const int G = a.q_heads / a.kv_heads;
    if (G < 1 || G > kMaxGroup) throw std::invalid_argument("attention: more than 16 query heads per KV head");
    for (const void* p : {a.k0, a.v0, a.k1, a.v1})
        if (reinterpret_cast<uintptr_t>(p) % 16 != 0)
            throw std::invalid_argument("attention: key/value rows must start on 16-byte boundaries");
    // dynamic shared memory holds only the combine's staged partials
    const size_t smem = static_cast<size_t>(a.splits) * G * (64 + 2) * sizeof(float);
    if (smem > 200 * 1024) throw std::invalid_argument("attention: sequence too long for one split");
    cudaLaunchAttribute attr[1];
    cudaLaunchConfig_t cfg = make_cfg(dim3(a.splits, a.kv_heads), dim3(kAttnSplitThreads), smem, s, pdl, attr);
    if (fp16_kv) check_launch(cudaLaunchKernelEx(&cfg, attn_decode_kernel<__half, 64>, a));
    else check_launch(cudaLaunchKernelEx(&cfg, attn_decode_kernel<float, 64>, a));
}

void init_batched_attributes();

template <int MODE, int RPW, int NB>
void set_gemv_batch_attributes_nb() {
    constexpr int kSmem = 160 * 1024;  // up to kGemvBatch inputs of K <= 4096 (+ slack)
    constexpr int W = batch_warps<NB>();
    for (const void* f : {reinterpret_cast<const void*>(gemv_batch_kernel<MODE, 1, RPW, NB, W>),
                          reinterpret_cast<const void*>(gemv_batch_kernel<MODE, 2, RPW, NB, W>),
                          reinterpret_cast<const void*>(gemv_batch_kernel<MODE, 4, RPW, NB, W>),
                          reinterpret_cast<const void*>(gemv_batch_kernel<MODE, 8, RPW, NB, W>)})
        check_launch(cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem));
    if constexpr (RPW == 1)
        check_launch(cudaFuncSetAttribute(gemv_batch_kernel<MODE, 16, 1, NB, W>,
                                          cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem));
}
template <int MODE, int RPW>
void set_gemv_batch_attributes() {
    set_gemv_batch_attributes_nb<MODE, RPW, 4>();
    set_gemv_batch_attributes_nb<MODE, RPW, kGemvBatch>();
}

void init_kernel_attributes() {
    constexpr int kMax = 200 * 1024;
    set_gemv_batch_attributes<GEMV_PLAIN, 1>();
    set_gemv_batch_attributes<GEMV_RESID, 1>();
    set_gemv_batch_attributes<GEMV_GATEUP, 2>();
    set_gemv_batch_attributes<GEMV_QKV, 2>();
    check_launch(cudaFuncSetAttribute(attn_decode_kernel<__half, 64>, cudaFuncAttributeMaxDynamicSharedMemorySize, kMax));
    check_launch(cudaFuncSetAttribute(attn_decode_kernel<float, 64>, cudaFuncAttributeMaxDynamicSharedMemorySize, kMax));
    for (const void* f : {reinterpret_cast<const void*>(gemv_bulk_kernel<GEMV_PLAIN, 1>),
                          reinterpret_cast<const void*>(gemv_bulk_kernel<GEMV_RESID, 1>),
                          reinterpret_cast<const void*>(gemv_bulk_kernel<GEMV_GATEUP, 1>),
                          reinterpret_cast<const void*>(gemv_bulk_kernel<GEMV_QKV, 1>),
                          reinterpret_cast<const void*>(gemv_bulk_kernel<GEMV_PLAIN, kGemvBatch>),
                          reinterpret_cast<const void*>(gemv_bulk_kernel<GEMV_RESID, kGemvBatch>),
                          reinterpret_cast<const void*>(gemv_bulk_kernel<GEMV_GATEUP, kGemvBatch>),
                          reinterpret_cast<const void*>(gemv_bulk_kernel<GEMV_QKV, kGemvBatch>)})
        check_launch(cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(kBulkSmemMax)));
    check_launch(cudaFuncSetAttribute(attn_decode_cluster_kernel<float, 64>,
                                      cudaFuncAttributeNonPortableClusterSizeAllowed, 1));
    init_batched_attributes();
    init_tc_attributes();
    init_tc_rows_attributes();
    init_sdpa_op_attributes();
    init_tc_wide_attributes();
}

void launch_final_norm(const float* h, const __half* g, float eps, int H, float* out, float* out2,
                       StreamCtl* ctl, int which, int bump, int skip_if_stopped, cudaStream_t s,
                       bool pdl) {
    if (H <= 0 || H > kFinalNormThreads * kFinalNormPer) throw std::invalid_argument("final norm: hidden in [1, 4096]");
    cudaLaunchAttribute attr[1];
    cudaLaunchConfig_t cfg = make_cfg(dim3(1), dim3(kFinalNormThreads), 0, s, pdl, attr);
    check_launch(cudaLaunchKernelEx(&cfg, final_norm_kernel, h, g, eps, H, out, out2, ctl, which, bump,
                                    skip_if_stopped));
}

}  // namespace vxc
