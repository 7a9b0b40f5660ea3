// tcgen05 (5th-generation tensor core) linear layer for the DiT estimator's
// CFG-doubled token batch: Y[m][n] = sum_k X[m][k] W[n][k] for m < 22 tokens.
//
// Shape of the problem (tools/export_components.py:625-659): 2 CFG rows x 11
// tokens through q/k/v (1024 -> 3072), o (1024 -> 1024), gate/up (1024 -> 2 x
// 4096) and down (4096 -> 1024). With 22 tokens every weight is used 22 times:
// far below the B200 ridge point, so the kernel's job is to stream each weight
// byte from HBM exactly once at full bandwidth while the tensor cores do the
// arithmetic out of shared memory.
//
// Mapping: weights are the MMA A operand (M = 128 output features per tile,
// K-major, 128-byte swizzle, loaded by TMA); the activations are the B operand
// (N = 48: rows 0..23 hold fp16(x), rows 24..47 hold fp16(x - fp16(x)), so
// A * (hi + lo) reproduces the fp32 activations to ~2^-22 and the result keeps
// fp32-level accuracy; the extra N costs nothing at this arithmetic
// intensity). Accumulators live in TMEM (48 fp32 columns). K is split across
// the CTAs of a thread-block cluster; the partial tiles are reduced through
// distributed shared memory in a fixed order (deterministic), then the
// epilogue (plain store, residual add, or SiLU(gate) * up written straight
// into the next layer's split-fp16 B operand) runs on the reducing CTA.
//
// Roles: thread 0 issues TMA (weights before griddepcontrol.wait, so weight
// streaming overlaps the previous kernel), thread 32 issues tcgen05.mma, all
// four warps drain TMEM. Every mbarrier wait is bounded; on timeout the kernel
// records error 3 in the stream control block, still passes every cluster
// barrier and frees its TMEM, and the host reports the failure.
#include <cuda.h>

#include <algorithm>
#include <cfloat>
#include <stdexcept>
#include <type_traits>
#include <vector>

#include "kernels.cuh"
#include "tc_common.cuh"

namespace vxc {
namespace {

using namespace tc;

constexpr int kTcThreads = 128;
constexpr int kStageBytes = kABytes + kBBytes;    // 22 KiB, keeps 1 KiB alignment
constexpr int kMaxStages = 8;
constexpr int kRecvFloats = kTileRows * kLoOffset;  // split-K receive buffer: every partial of one tile
constexpr int kSqFloats = kTileRows * kLoOffset;    // squares of the updated rows (at most 128 x 24)

// A split launch can receive in its stage area when the area holds the partials and,
// behind them, the squares.
__host__ __device__ constexpr bool shared_recv_fits(bool b_tma, int splits, int recv_shared, size_t area_bytes) {
    return b_tma && splits > 1 && recv_shared && area_bytes >= static_cast<size_t>(kRecvFloats + kSqFloats) * 4;
}
constexpr int kTmemCols = 64;

// Zero token rows M..23 (and their residual rows) of 'cs' B tiles.
__device__ __forceinline__ void zero_pad_rows(uint8_t* smem, int cs, int M) {
    const int pad = kLoOffset - M;
    for (int u = threadIdx.x; u < cs * pad * 16; u += kTcThreads) {
        const int ch = u / (pad * 16), r = u - ch * pad * 16, m = M + r / 16, col = (r & 15) * 4;
        put_split4(smem + ch * kStageBytes + kABytes, m, col, make_float4(0.f, 0.f, 0.f, 0.f));
    }
}

// B = split-fp16 RMSNorm(x) for chunks c0 .. c0 + cs - 1 (RMSNorm as in
// rmsnorm_rows_split_kernel: x * rsqrt(mean(x^2) + eps) * g). The row sums of
// squares are the fixed-order sum of the producer's partials. Every thread
// issues its loads in batches before it uses any (each global round trip costs
// about a microsecond here).
__device__ void build_b_norm(uint8_t* smem, const TcLinearArgs& a, int c0, int cs, float* inv_s, float4* red) {
    const int tid = threadIdx.x;
    // 120 threads = 20 part groups x 6 token quads, then a fixed-order sum over the groups
    if (tid < 120) {
        const int r = tid / 6, q = tid - r * 6;
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int p0 = 0; p0 < a.ssq_parts; p0 += 160) {
            float4 v[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const int p = p0 + r + 20 * i;
                v[i] = p < a.ssq_parts ? __ldcg(reinterpret_cast<const float4*>(a.ssq_in + p * kSsqStride) + q)
                                       : make_float4(0.f, 0.f, 0.f, 0.f);
            }
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                acc.x += v[i].x;
                acc.y += v[i].y;
                acc.z += v[i].z;
                acc.w += v[i].w;
            }
        }
        red[r * 6 + q] = acc;
    }
    __syncthreads();
    if (tid < kLoOffset) {
        const float* rf = reinterpret_cast<const float*>(red);
        float t = 0.f;
        for (int r = 0; r < 20; ++r) t += rf[r * 24 + tid];
        inv_s[tid] = rsqrtf(t / static_cast<float>(a.K) + a.eps);
    }
    __syncthreads();
    const int per = cs * 16, total = a.M * per;  // float4 units per token row, in all
    constexpr int kB = 8;
    for (int base = 0; base < total; base += kTcThreads * kB) {
        float4 xv[kB];
        uint2 gw[kB];
#pragma unroll
        for (int i = 0; i < kB; ++i) {
            const int u = base + tid + kTcThreads * i;
            if (u < total) {
                const int m = u / per, q = u - m * per, k = (c0 + (q >> 4)) * kKChunk + (q & 15) * 4;
                xv[i] = __ldcg(reinterpret_cast<const float4*>(a.x + static_cast<size_t>(m) * a.ldx + k));
                gw[i] = __ldg(reinterpret_cast<const uint2*>(a.g + k));
            }
        }
#pragma unroll
        for (int i = 0; i < kB; ++i) {
            const int u = base + tid + kTcThreads * i;
            if (u < total) {
                const int m = u / per, q = u - m * per, ch = q >> 4, col = (q & 15) * 4;
                const float2 g01 = __half22float2(*reinterpret_cast<const __half2*>(&gw[i].x));
                const float2 g23 = __half22float2(*reinterpret_cast<const __half2*>(&gw[i].y));
                const float iv = inv_s[m];
                put_split4(smem + ch * kStageBytes + kABytes, m, col,
                           make_float4(xv[i].x * iv * g01.x, xv[i].y * iv * g01.y, xv[i].z * iv * g23.x,
                                       xv[i].w * iv * g23.y));
            }
        }
    }
    zero_pad_rows(smem, cs, a.M);
}

// Attention scratch per head of a round (floats): q and k [24][65], v [24][64],
// probabilities [2 sequences][12][13].
constexpr int kAttnRow = 65;
constexpr int kAttnHeadFloats = 2 * 24 * kAttnRow + 24 * 64 + 2 * 12 * 13;
constexpr size_t kSmemOptin = 232448;  // B200: opt-in shared memory per CTA (227 KB)
size_t g_dyn_limit = 0;                // kSmemOptin less the kernel's static shared memory (set once)

// B = split-fp16 attention output of heads c0 .. c0 + cs - 1 (one 64-wide head
// per K chunk), the math of dit_attention_split_kernel: RoPE (rotate_half) on q
// and k, scores * scale, softmax, P.V, both sequences, 'round' heads at a time.
__device__ void build_b_attn(uint8_t* smem, const TcLinearArgs& a, int c0, int cs, int round, float* scratch) {
    constexpr int D = 64, HALF = 32;
    const int tid = threadIdx.x, M = a.M, seq = a.seq;
    const int W = (a.q_heads + 2 * a.kv_heads) * D, grp = a.q_heads / a.kv_heads;
    float* qs = scratch;
    float* ks = qs + round * 24 * kAttnRow;
    float* vs = ks + round * 24 * kAttnRow;
    float* ps = vs + round * 24 * D;
    for (int h0 = 0; h0 < cs; h0 += round) {
        const int nh = min(round, cs - h0);
        // raw q / k / v rows of the round's heads (nh x M x 3 x 16 float4), loads in batches
        constexpr int kB = 9;
        const int total = nh * M * 48;
        for (int base = 0; base < total; base += kTcThreads * kB) {
            float4 v[kB];
#pragma unroll
            for (int i = 0; i < kB; ++i) {
                const int u = base + tid + kTcThreads * i;
                if (u < total) {
                    const int hl = u / (M * 48), r2 = u - hl * M * 48, i2 = r2 / 48, w = r2 - i2 * 48;
                    const int kind = w >> 4, e4 = (w & 15) * 4, h = c0 + h0 + hl, kvh = h / grp;
                    const int col = kind == 0 ? h * D : kind == 1 ? (a.q_heads + kvh) * D
                                                                  : (a.q_heads + a.kv_heads + kvh) * D;
                    v[i] = __ldcg(reinterpret_cast<const float4*>(a.qkv + static_cast<size_t>(i2) * W + col + e4));
                }
            }
#pragma unroll
            for (int i = 0; i < kB; ++i) {
                const int u = base + tid + kTcThreads * i;
                if (u < total) {
                    const int hl = u / (M * 48), r2 = u - hl * M * 48, i2 = r2 / 48, w = r2 - i2 * 48;
                    const int kind = w >> 4, e4 = (w & 15) * 4;
                    float* dst = kind == 0 ? qs + (hl * 24 + i2) * kAttnRow
                                           : kind == 1 ? ks + (hl * 24 + i2) * kAttnRow : vs + (hl * 24 + i2) * D;
                    dst[e4] = v[i].x;
                    dst[e4 + 1] = v[i].y;
                    dst[e4 + 2] = v[i].z;
                    dst[e4 + 3] = v[i].w;
                }
            }
        }
        __syncthreads();
        // RoPE (rotate_half) on q and k in place: each unit owns the pair (e, e + 32)
        for (int u = tid; u < nh * 2 * M * HALF; u += kTcThreads) {
            const int hl = u / (2 * M * HALF), r2 = u - hl * 2 * M * HALF, which = r2 / (M * HALF);
            const int r3 = r2 - which * M * HALF, i = r3 / HALF, e = r3 - i * HALF, pos = i % seq;
            float* row = (which == 0 ? qs : ks) + (hl * 24 + i) * kAttnRow;
            const float c1 = __ldg(a.rope_cos + pos * D + e), c2 = __ldg(a.rope_cos + pos * D + e + HALF);
            const float s1 = __ldg(a.rope_sin + pos * D + e), s2 = __ldg(a.rope_sin + pos * D + e + HALF);
            const float v1 = row[e], v2 = row[e + HALF];
            row[e] = v1 * c1 + (-v2) * s1;
            row[e + HALF] = v2 * c2 + v1 * s2;
        }
        __syncthreads();
        for (int u = tid; u < nh * 2 * seq * seq; u += kTcThreads) {
            const int hl = u / (2 * seq * seq), r = u - hl * 2 * seq * seq, b = r / (seq * seq);
            const int r2 = r - b * seq * seq, i = r2 / seq, j = r2 - i * seq;
            const float* q = qs + (hl * 24 + b * seq + i) * kAttnRow;
            const float* k = ks + (hl * 24 + b * seq + j) * kAttnRow;
            float sum = 0.f;
#pragma unroll 16
            for (int e = 0; e < D; ++e) sum = fmaf(q[e], k[e], sum);
            ps[((hl * 2 + b) * 12 + i) * 13 + j] = sum * a.scale;
        }
        __syncthreads();
        for (int u = tid; u < nh * 2 * seq; u += kTcThreads) {
            float* pr = ps + ((u / seq) * 12 + (u % seq)) * 13;  // u = (head * 2 + b) * seq + i
            float mx = -FLT_MAX;
            for (int j = 0; j < seq; ++j) mx = fmaxf(mx, pr[j]);
            float sum = 0.f;
            for (int j = 0; j < seq; ++j) {
                pr[j] = expf(pr[j] - mx);
                sum += pr[j];
            }
            for (int j = 0; j < seq; ++j) pr[j] /= sum;
        }
        __syncthreads();
        for (int u = tid; u < nh * M * 16; u += kTcThreads) {
            const int hl = u / (M * 16), r = u - hl * M * 16, m = r >> 4, col = (r & 15) * 4;
            const int b = m / seq, i = m - b * seq;
            const float* pr = ps + ((hl * 2 + b) * 12 + i) * 13;
            float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
            for (int j = 0; j < seq; ++j) {
                const float p = pr[j];
                const float* vr = vs + (hl * 24 + b * seq + j) * D + col;
                acc.x = fmaf(p, vr[0], acc.x);
                acc.y = fmaf(p, vr[1], acc.y);
                acc.z = fmaf(p, vr[2], acc.z);
                acc.w = fmaf(p, vr[3], acc.w);
            }
            put_split4(smem + (h0 + hl) * kStageBytes + kABytes, m, col, acc);
        }
        __syncthreads();  // the next head pair reuses the scratch
    }
    zero_pad_rows(smem, cs, M);
}

// The receive buffer can share the stage area when nothing else needs it there:
// TMA-fed token tiles, no K split (no remote pushes), no squares scratch.
__host__ __device__ constexpr bool recv_in_stage_area(bool b_tma, int splits, bool ssq_out) {
    return b_tma && splits == 1 && !ssq_out;
}

// BM: where the token operand comes from (TC_B_TMA / TC_B_NORM / TC_B_ATTN); one
// instantiation each, so the TMA form does not carry the builders' registers.
// S: the K split (cluster size, 1, 2, 4 or 8), a template parameter so that the
// rank-order sums of the partials unroll and their loads issue together.
template <int BM, int S>
__global__ void __launch_bounds__(kTcThreads, 1)
    tc_linear_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
                     const TcLinearArgs a) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    __shared__ uint64_t full_bar[kMaxStages], empty_bar[kMaxStages], done_bar;
    __shared__ uint32_t tmem_base_s;
    __shared__ int failed_s;
    __shared__ float inv_s[kLoOffset];
    __shared__ float4 red_s[120];

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int split = blockIdx.x, tile = blockIdx.y;
    // 1 KiB aligned, derived from smem_raw by pointer arithmetic so that the
    // compiler keeps shared-memory addressing for everything carved from it
    uint8_t* smem = smem_raw + ((1024u - (smem_addr(smem_raw) & 1023u)) & 1023u);
    constexpr bool b_tma = BM == TC_B_TMA;

    const int nch = a.K / kKChunk;
    const int c0 = split * nch / S, c1 = (split + 1) * nch / S, cs = c1 - c0;
    const int stages = min(a.max_stages, max(cs, 1));
    // the receive buffer sits after the stage area of the largest split: the same
    // offset in every CTA of the cluster, whatever its own chunk count
    const int stage_area = min(a.max_stages, max((nch + S - 1) / S, 1));

    // thread 0: barriers, then the weight loads at once (they depend on no earlier
    // kernel); warp 1 meanwhile allocates the TMEM accumulator
    const int r0 = a.gateup ? tile * 64 : tile * kTileRows;   // rows of W in this tile: two
    const int r1 = a.gateup ? a.rows + tile * 64 : tile * kTileRows + 64;  // 64-row boxes
    const int pre = min(stages, cs);
    // bytes landing on a stage's barrier: the weight tile, plus the token tile when TMA brings it
    const uint32_t stage_tx = b_tma ? kStageBytes : kABytes;
    int issued[kMaxStages];  // producer: loads issued per stage (for the drain below)
    if (tid == 0) {
        for (int i = 0; i < stages; ++i) {
            mbar_init(&full_bar[i], 1);
            mbar_init(&empty_bar[i], 1);
        }
        mbar_init(&done_bar, 1);
        failed_s = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&map_a)) : "memory");
        if (b_tma) asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&map_b)) : "memory");
#pragma unroll
        for (int i = 0; i < kMaxStages; ++i) issued[i] = 0;
        for (int i = 0; i < pre; ++i) {
            uint8_t* st = smem + i * kStageBytes;
            mbar_expect_tx(&full_bar[i], stage_tx);
            tma_load_2d(st, &map_a, (c0 + i) * kKChunk, r0, &full_bar[i]);
            tma_load_2d(st + kABytes / 2, &map_a, (c0 + i) * kKChunk, r1, &full_bar[i]);
            issued[i] = 1;
        }
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                         smem_addr(&tmem_base_s)), "r"(kTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem_d = tmem_base_s;
    pdl_launch_dependents();

    // tensor-core issue: thread 32, one 128 x 48 x 16 MMA per 16 fp16 of K
    auto mma_loop = [&] {
        const uint32_t idesc = umma_idesc(kTileRows, kBRows);
        for (int i = 0; i < cs; ++i) {
            const int s = i % stages;
            if (!mbar_wait(&full_bar[s], (i / stages) & 1)) {
                failed_s = 1;
                break;
            }
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            const uint32_t sa = smem_addr(smem + s * kStageBytes), sb = sa + kABytes;
#pragma unroll
            for (int kk = 0; kk < kKChunk / 16; ++kk)  // 16 fp16 (32 B) per MMA step along K
                umma_f16(tmem_d, umma_desc(sa + kk * 32), umma_desc(sb + kk * 32), idesc, (i | kk) != 0);
            umma_commit(&empty_bar[s]);  // frees the stage once these MMAs have read it
        }
        umma_commit(&done_bar);  // arrives when every MMA issued above has completed
    };

    if constexpr (b_tma) {
        if (tid == 0) {
            pdl_wait();
            for (int i = 0; i < pre; ++i)
                tma_load_2d(smem + i * kStageBytes + kABytes, &map_b, (c0 + i) * kKChunk, 0, &full_bar[i]);
            for (int i = pre; i < cs; ++i) {
                const int s = i % stages;
                if (!mbar_wait(&empty_bar[s], ((i / stages) - 1) & 1)) {
                    failed_s = 1;
                    break;
                }
                uint8_t* st = smem + s * kStageBytes;
                mbar_expect_tx(&full_bar[s], kStageBytes);
                tma_load_2d(st, &map_a, (c0 + i) * kKChunk, r0, &full_bar[s]);
                tma_load_2d(st + kABytes / 2, &map_a, (c0 + i) * kKChunk, r1, &full_bar[s]);
                tma_load_2d(st + kABytes, &map_b, (c0 + i) * kKChunk, 0, &full_bar[s]);
                issued[s] += 1;
            }
        } else if (tid == 32) {
            pdl_wait();
            mma_loop();
        } else {
            pdl_wait();
        }
    } else {
        // all chunks have their own stage (cs <= stages, checked by the launcher):
        // every thread builds the token tiles next to the weight tiles in flight
        pdl_wait();
        if constexpr (BM == TC_B_NORM) {
            build_b_norm(smem, a, c0, cs, inv_s, red_s);
        } else {
            float* scratch = reinterpret_cast<float*>(smem + static_cast<size_t>(stage_area) * kStageBytes) +
                             kRecvFloats;
            build_b_attn(smem, a, c0, cs, a.attn_round, scratch);
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // generic-proxy writes -> tensor core
        __syncthreads();
        if (tid == 32) mma_loop();
    }

    // row_scale: each token row's 1 / rms from the producer's sums of squares (warp 2,
    // idle until the epilogue; parts summed in order)
    if (a.row_scale && warp == 2) {
        if (lane < a.M) {
            float t = 0.f;
#pragma unroll 8
            for (int p = 0; p < a.ssq_parts; ++p) t += __ldcg(a.ssq_in + p * kSsqStride + lane);
            inv_s[lane] = rsqrtf(t / static_cast<float>(a.K) + a.eps);
        }
    }

    // drain the accumulator: warp w owns TMEM lanes (tile rows) 32w .. 32w + 31
    const bool ok = mbar_wait(&done_bar, 0);
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    if (!ok) failed_s = 1;
    // Output units of the tile: 128 rows, or 64 gate/up pairs; CTA p of the cluster
    // owns units [p nu, (p + 1) nu). Each thread holds one accumulator row
    // (tile row tid): v[m] = hi + lo columns of token m.
    const int units = a.gateup ? 64 : kTileRows, halves = a.gateup ? 2 : 1;
    const int nu = units / S;
    float v[kLoOffset];
    {
        float d[kBRows];
        if (ok) {
            const uint32_t t = tmem_d + (static_cast<uint32_t>(warp * 32) << 16);
            tmem_ld16(t + 0, d);
            tmem_ld16(t + 16, d + 16);
            tmem_ld16(t + 32, d + 32);
            asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
        } else {
#pragma unroll
            for (int i = 0; i < kBRows; ++i) d[i] = 0.f;
        }
#pragma unroll
        for (int m = 0; m < kLoOffset; ++m) v[m] = d[m] + d[kLoOffset + m];
    }
    if (tid == 0) {
        // no copy may still be landing in this CTA's shared memory when it is reused
        // or the CTA exits (a no-op when every stage was consumed; bounded when something failed)
        for (int i = 0; i < stages; ++i)
            if (issued[i] > 0 && !mbar_wait(&full_bar[i], (issued[i] - 1) & 1)) failed_s = 1;
    }
    if (a.row_scale) __syncthreads();  // inv_s is complete
    if (S == 1 && !a.gateup && !a.ssq_out) {
        // no split: straight from registers, coalesced across the warp
        if (a.row_scale) {
#pragma unroll
            for (int m = 0; m < kLoOffset; ++m) v[m] *= inv_s[m];
        }
        float* yc = a.y + tile * kTileRows + tid;
        float r[kLoOffset];
#pragma unroll
        for (int m = 0; m < kLoOffset; ++m) r[m] = (a.resid && m < a.M) ? yc[static_cast<size_t>(m) * a.ldy] : 0.f;
#pragma unroll
        for (int m = 0; m < kLoOffset; ++m)
            if (m < a.M)
                yc[static_cast<size_t>(m) * a.ldy] = a.resid ? r[m] + (a.rscale == 1.f ? v[m] : v[m] * a.rscale) : v[m];
        __syncthreads();
    } else {
        // Split-K exchange by push: each CTA stores its partials straight into the
        // receive buffer of the CTA that owns them (non-blocking remote stores),
        // token-major so that a warp's store is one contiguous run; one cluster
        // barrier; then owners sum the splits in rank order (deterministic).
        // recv[((p * halves + half) * M + m) * nu + lu]. Without a K split it lives in
        // the (then idle) stage area, so more CTAs of concurrent streams fit on an SM.
        const bool shared = shared_recv_fits(b_tma, S, a.recv_shared, static_cast<size_t>(stage_area) * kStageBytes);
        const bool recv_in_stages = recv_in_stage_area(b_tma, S, a.ssq_out != nullptr) || shared;
        float* recv =
            reinterpret_cast<float*>(recv_in_stages ? smem : smem + static_cast<size_t>(stage_area) * kStageBytes);
        __syncthreads();  // the stage area is idle
        if (shared) cluster_sync();  // ... in every CTA of the cluster: partials may land in it
        {
            const int u = a.gateup ? (tid & 63) : tid, half = a.gateup ? (tid >> 6) : 0;
            const int owner = u / nu, lu = u - owner * nu;
            float* dst = recv + static_cast<size_t>((split * halves + half) * a.M) * nu + lu;
            if (owner == split) {
#pragma unroll
                for (int m = 0; m < kLoOffset; ++m)
                    if (m < a.M) dst[m * nu] = v[m];
            } else {
                const uint32_t remote = peer_addr(dst, owner);
#pragma unroll
                for (int m = 0; m < kLoOffset; ++m)
                    if (m < a.M) st_peer(remote + 4u * m * nu, v[m]);
            }
        }
        asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
        if (S > 1) cluster_sync();  // every partial has landed in its owner's buffer
        else __syncthreads();
        // this CTA's units: thread -> (unit lu, token rows m0, m0 + per, ...);
        // each batch issues all its loads before any of its stores
        const int per = kTcThreads / nu, lu = tid % nu, m0 = tid / nu;
        const int col = split * nu + lu;
        // the stage area is idle now: squares of updated rows (behind the partials when those share it)
        float* sq = reinterpret_cast<float*>(smem) + (shared ? kRecvFloats : 0);
        if (a.gateup) {
            constexpr int kBatch = 4;
            for (int mb = m0; mb < a.M; mb += per * kBatch) {
                float g[kBatch][S], up[kBatch][S];
#pragma unroll
                for (int j = 0; j < kBatch; ++j) {
                    const int mc = min(mb + j * per, a.M - 1);
#pragma unroll
                    for (int p = 0; p < S; ++p) {
                        g[j][p] = recv[static_cast<size_t>((p * 2 + 0) * a.M + mc) * nu + lu];
                        up[j][p] = recv[static_cast<size_t>((p * 2 + 1) * a.M + mc) * nu + lu];
                    }
                }
#pragma unroll
                for (int j = 0; j < kBatch; ++j) {
                    const int m = mb + j * per;
                    if (m < a.M) {
                        float gs = 0.f, us = 0.f;
#pragma unroll
                        for (int p = 0; p < S; ++p) {
                            gs += g[j][p];
                            us += up[j][p];
                        }
                        if (a.row_scale) {
                            gs *= inv_s[m];
                            us *= inv_s[m];
                        }
                        store_split(a.yb, a.ldyb, m, tile * 64 + col, silu(gs) * us);
                    }
                }
            }
        } else {
            constexpr int kBatch = 8;
            float* yc = a.y + tile * kTileRows + col;
            const float gn = a.next_b ? __half2float(a.next_g[tile * kTileRows + col]) : 0.f;
            for (int mb = m0; mb < a.M; mb += per * kBatch) {
                float part[kBatch][S], r[kBatch];
#pragma unroll
                for (int j = 0; j < kBatch; ++j) {
                    const int m = mb + j * per;
                    const int mc = min(m, a.M - 1);
#pragma unroll
                    for (int p = 0; p < S; ++p) part[j][p] = recv[static_cast<size_t>(p * a.M + mc) * nu + lu];
                    r[j] = (a.resid && m < a.M) ? yc[static_cast<size_t>(m) * a.ldy] : 0.f;
                }
#pragma unroll
                for (int j = 0; j < kBatch; ++j) {
                    const int m = mb + j * per;
                    if (m < a.M) {
                        float sum = 0.f;
#pragma unroll
                        for (int p = 0; p < S; ++p) sum += part[j][p];
                        if (a.row_scale) sum *= inv_s[m];
                        const float nv = a.resid ? r[j] + (a.rscale == 1.f ? sum : sum * a.rscale) : sum;
                        yc[static_cast<size_t>(m) * a.ldy] = nv;
                        if (a.ssq_out) sq[m * nu + lu] = nv * nv;
                        if (a.next_b) store_split(a.next_b, a.ldnb, m, tile * kTileRows + col, nv * gn);
                    }
                }
            }
        }
        __syncthreads();
        if (a.ssq_out && tid < a.M) {  // this owner's part of each row's sum of squares, fixed order
            float t = 0.f;
            for (int l = 0; l < nu; ++l) t += sq[tid * nu + l];
            a.ssq_out[(tile * S + split) * kSsqStride + tid] = t;
        }
    }
    if (tid == 0 && failed_s && a.ctl) a.ctl->error = 3;
    if (warp == 1)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_d), "r"(kTmemCols)
                     : "memory");
}

}  // namespace

size_t tc_linear_smem_bytes(int K, int splits, int bmode, int attn_round, int max_stages, bool ssq_out,
                            bool recv_shared) {
    const int nch = K / kKChunk;
    const int cs = (nch + splits - 1) / splits;
    const int stages = std::min(std::min(max_stages, kMaxStages), std::max(cs, 1));
    const size_t stage_bytes = static_cast<size_t>(stages) * kStageBytes;
    if (recv_in_stage_area(bmode == TC_B_TMA, splits, ssq_out) ||
        shared_recv_fits(bmode == TC_B_TMA, splits, recv_shared, stage_bytes))
        return stage_bytes + 1024;  // + alignment slack
    const size_t recv_bytes = static_cast<size_t>(kRecvFloats) * sizeof(float);
    const size_t scratch = bmode == TC_B_ATTN ? static_cast<size_t>(attn_round) * kAttnHeadFloats * sizeof(float) : 0;
    return stage_bytes + recv_bytes + scratch + 1024;  // + alignment slack
}

template <int BM>
cudaError_t launch_split(cudaLaunchConfig_t& cfg, const CUtensorMap& map_a, const CUtensorMap& map_b,
                         const TcLinearArgs& a) {
    switch (a.splits) {
        case 1: return cudaLaunchKernelEx(&cfg, tc_linear_kernel<BM, 1>, map_a, map_b, a);
        case 2: return cudaLaunchKernelEx(&cfg, tc_linear_kernel<BM, 2>, map_a, map_b, a);
        case 4: return cudaLaunchKernelEx(&cfg, tc_linear_kernel<BM, 4>, map_a, map_b, a);
        default: return cudaLaunchKernelEx(&cfg, tc_linear_kernel<BM, 8>, map_a, map_b, a);
    }
}

// every instantiation (token-operand mode x split)
std::vector<const void*> tc_linear_kernels() {
    std::vector<const void*> k;
    auto add = [&k](auto bm) {
        constexpr int B = decltype(bm)::value;
        k.push_back(reinterpret_cast<const void*>(tc_linear_kernel<B, 1>));
        k.push_back(reinterpret_cast<const void*>(tc_linear_kernel<B, 2>));
        k.push_back(reinterpret_cast<const void*>(tc_linear_kernel<B, 4>));
        k.push_back(reinterpret_cast<const void*>(tc_linear_kernel<B, 8>));
    };
    add(std::integral_constant<int, TC_B_TMA>{});
    add(std::integral_constant<int, TC_B_NORM>{});
    add(std::integral_constant<int, TC_B_ATTN>{});
    return k;
}

size_t dyn_limit() {
    if (!g_dyn_limit) {
        size_t most = 0;
        for (const void* f : tc_linear_kernels()) {
            cudaFuncAttributes fa{};
            const cudaError_t e = cudaFuncGetAttributes(&fa, f);
            if (e != cudaSuccess) throw std::runtime_error(std::string("tc_linear attributes: ") + cudaGetErrorString(e));
            most = std::max(most, fa.sharedSizeBytes);
        }
        g_dyn_limit = kSmemOptin - most;
    }
    return g_dyn_limit;
}

int tc_attn_round(int K, int splits, int max_stages) {
    return tc_linear_smem_bytes(K, splits, TC_B_ATTN, 2, max_stages) <= dyn_limit() ? 2 : 1;
}

void launch_tc_linear(const CUtensorMap& map_a, const CUtensorMap& map_b, const TcLinearArgs& a, cudaStream_t s,
                      bool pdl) {
    if (a.K % kKChunk != 0 || a.K <= 0) throw std::invalid_argument("tc_linear: K must be a multiple of 64");
    if (a.M <= 0 || a.M > kLoOffset) throw std::invalid_argument("tc_linear: at most 24 token rows");
    if ((a.splits != 1 && a.splits != 2 && a.splits != 4 && a.splits != 8) || a.splits > a.K / kKChunk)
        throw std::invalid_argument("tc_linear: splits must be 1, 2, 4 or 8 and at most K / 64");
    const int n_tiles = a.gateup ? a.rows / 64 : a.rows / kTileRows;
    if ((a.gateup ? a.rows % 64 : a.rows % kTileRows) != 0) throw std::invalid_argument("tc_linear: rows");
    if (a.bmode != TC_B_TMA) {
        const int nch = a.K / kKChunk;
        if ((nch + a.splits - 1) / a.splits > a.max_stages)
            throw std::invalid_argument("tc_linear: a fused token tile needs a stage per K chunk of the CTA");
    }
    if (a.bmode == TC_B_NORM && (!a.x || !a.g || !a.ssq_in || a.ssq_parts <= 0 || a.ldx % 4 != 0 ||
                                 (reinterpret_cast<uintptr_t>(a.x) & 15) != 0 ||
                                 (reinterpret_cast<uintptr_t>(a.g) & 7) != 0))
        throw std::invalid_argument("tc_linear: bad RMSNorm operand");
    if (a.bmode == TC_B_ATTN &&
        (!a.qkv || !a.rope_cos || !a.rope_sin || a.kv_heads <= 0 || a.q_heads % a.kv_heads != 0 ||
         a.K != a.q_heads * 64 || a.seq <= 0 || a.seq > 12 || a.M != 2 * a.seq || a.attn_round < 1))
        throw std::invalid_argument("tc_linear: bad attention operand");
    if (a.ssq_out && (a.gateup || a.M > kSsqStride)) throw std::invalid_argument("tc_linear: bad ssq_out");
    if (a.next_b && (!a.ssq_out || !a.next_g || !a.resid || a.ldnb < a.rows))
        throw std::invalid_argument("tc_linear: next_b needs a residual launch with ssq_out and next_g");
    if (a.row_scale && (!a.ssq_in || a.ssq_parts <= 0 || a.bmode != TC_B_TMA))
        throw std::invalid_argument("tc_linear: row_scale needs ssq_in parts and a TMA-fed operand");
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(a.splits, n_tiles);
    cfg.blockDim = dim3(kTcThreads);
    if (a.max_stages < 1 || a.max_stages > kMaxStages) throw std::invalid_argument("tc_linear: max_stages in [1, 8]");
    cfg.dynamicSmemBytes = tc_linear_smem_bytes(a.K, a.splits, a.bmode, a.attn_round, a.max_stages, a.ssq_out != nullptr,
                                                a.recv_shared != 0);
    if (cfg.dynamicSmemBytes > dyn_limit()) throw std::invalid_argument("tc_linear: shared memory over 227 KB");
    cfg.stream = s;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = a.splits;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 2 : 1;
    const cudaError_t e = a.bmode == TC_B_TMA    ? launch_split<TC_B_TMA>(cfg, map_a, map_b, a)
                          : a.bmode == TC_B_NORM ? launch_split<TC_B_NORM>(cfg, map_a, map_b, a)
                                                 : launch_split<TC_B_ATTN>(cfg, map_a, map_b, a);
    if (e != cudaSuccess) throw std::runtime_error(std::string("tc_linear launch: ") + cudaGetErrorString(e));
}

void init_tc_attributes() {
    // every launch checks its own need against this limit
    for (const void* f : tc_linear_kernels()) {
        const cudaError_t e = cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                   static_cast<int>(dyn_limit()));
        if (e != cudaSuccess) throw std::runtime_error(std::string("tc_linear attribute: ") + cudaGetErrorString(e));
    }
}

// ------------------------------------------------------------ tensor maps ---
namespace {
using EncodeTiled = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                 const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                 CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiled encode_fn() {
    static EncodeTiled fn = nullptr;
    if (!fn) {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        const cudaError_t e = cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q);
        if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || !p)
            throw std::runtime_error("cuTensorMapEncodeTiled is not available");
        fn = reinterpret_cast<EncodeTiled>(p);
    }
    return fn;
}
}  // namespace

// 2-D fp16 row-major tensor [rows][cols], box [box_rows][64], 128-byte swizzle.
CUtensorMap make_tensor_map_f16(const void* base, int rows, int cols, int box_rows) {
    if ((reinterpret_cast<uintptr_t>(base) & 15) != 0 || cols % 8 != 0)
        throw std::invalid_argument("tensor map: base must be 16-byte aligned and rows a multiple of 16 bytes");
    CUtensorMap m;
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(cols) * 2};
    const cuuint32_t box[2] = {static_cast<cuuint32_t>(kKChunk), static_cast<cuuint32_t>(box_rows)};
    const cuuint32_t estr[2] = {1, 1};
    const CUresult r = encode_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides, box,
                                   estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) throw std::runtime_error("cuTensorMapEncodeTiled failed");
    return m;
}

}  // namespace vxc
