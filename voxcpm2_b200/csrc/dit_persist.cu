// Persistent DiT decoder: every layer of one estimator evaluation
// (DitEstimator.decoder, tools/export_components.py:625-659) in a single
// cooperative launch with one CTA per SM.
//
// Why: at 2 x 11 tokens the decoder is a chain of 48 small linears per
// evaluation. As separate kernels each costs ~10 us of serial latency (launch
// edge, late-starting CTAs, reduction, epilogue) against ~1-3 us of weight
// traffic. Here the weight stream never stops: a producer warp walks the whole
// evaluation's weight tiles in consumption order and keeps a ring of shared
// memory slots full with TMA loads, across layer and phase boundaries (weights
// depend on no activation), while the other warps wait only for activations.
//
// Work split. Each linear ("phase") is a set of chunk-tiles (one 128-row weight
// tile x one 64-wide K chunk); CTA c takes the contiguous range
// [c N / G, (c + 1) N / G) in tile-major order, so a CTA holds partial sums of at
// most a few output tiles ("pieces"), each accumulated in TMEM on two
// alternating chains (halves the dependent MMA chain). Partials go to global
// memory (L2) as [128 rows][24 tokens] fp32 tiles, then:
//   q/k/v, gate/up: the CTA whose arrival on a tile's counter is the last sums
//     the tile's pieces in K order (deterministic) and writes q/k/v fp32 or
//     SiLU(gate) * up as the down projection's split-fp16 operand;
//   o, down (few tiles, long K): after a grid barrier every CTA reduces a slice
//     of output features: dh += rscale * sum, plus that slice's per-token sum of
//     squares for the next RMSNorm.
// Token operands (B) are built in shared memory by the compute warps: RMSNorm of
// dh (sums of squares from the previous phase's slices), the attention of the
// CTA's heads (RoPE, softmax, P.V), or a copy of the gate/up output.
// Grid barriers: after q/k/v, o, o-reduce, gate/up, down, down-reduce (6 per layer).
//
// Roles (192 threads): warps 0-3 build operands, drain TMEM (warp w owns TMEM
// lanes 32w..32w+31) and run epilogues; warp 4 lane 0 issues TMA; warp 5 lane 0
// issues tcgen05.mma (warp 5 also owns the TMEM allocation). Every wait is
// bounded: on timeout the CTA records error 3 in the stream control block and
// winds down; no wait is unbounded.
#include <cuda.h>

#include <algorithm>
#include <cfloat>
#include <stdexcept>
#include <string>

#include "kernels.cuh"
#include "tc_common.cuh"

namespace vxc {
namespace {

using namespace tc;

constexpr int kThreads = 192;
constexpr int kCompute = 128;     // warps 0-3
constexpr int kRing = 9;          // weight-tile slots, 16 KiB each
constexpr int kMaxB = 8;          // token tiles (6 KiB each) of one phase
constexpr int kMaxPieces = 4;     // output tiles one CTA touches in one phase
constexpr int kTmemCols = 512;    // kMaxPieces x 2 chains x 64 columns
constexpr int kPartFloats = kTileRows * 24;
constexpr int kAttnRow = 65;
// attention scratch: q, k [24][65], v [24][64], probabilities [2][12][13]; reduce
// phases reuse it for squares [24][<= 64 features]
constexpr int kScratchFloats = 2 * 24 * kAttnRow + 24 * 64 + 2 * 12 * 13;
constexpr int kMaxTiles = 96;     // tile counters in the sync block
constexpr int kMaxList = 64;      // pieces of one tile
constexpr int kMaxSlice = 16;     // output features one CTA reduces in the o / down phases
constexpr int kRopeFloats = 2 * 12 * 64;
constexpr size_t kSmemBytes = 1024 + static_cast<size_t>(kRing) * kABytes + static_cast<size_t>(kMaxB) * kBBytes +
                              (kScratchFloats + kRopeFloats) * 4;

enum { PH_QKV = 0, PH_O = 1, PH_GU = 2, PH_DOWN = 3 };

void check_launch(cudaError_t e) {
    if (e != cudaSuccess) throw std::runtime_error(std::string("dit_layers: ") + cudaGetErrorString(e));
}

struct Shape {
    int tiles, nch;
};

__device__ __forceinline__ Shape phase_shape(const DitLayersArgs& a, int p) {
    const int W = (a.hq + 2 * a.hkv) * 64;
    if (p == PH_QKV) return {W / kTileRows, a.Hd / kKChunk};
    if (p == PH_O) return {a.Hd / kTileRows, a.hq};
    if (p == PH_GU) return {a.F / 64, a.Hd / kKChunk};
    return {a.Hd / kTileRows, a.F / kKChunk};
}

// chunk-tile range of CTA c over N chunk-tiles: [lo(c), lo(c + 1))
__device__ __forceinline__ int range_lo(int c, int N, int G) {
    return static_cast<int>(static_cast<long long>(c) * N / G);
}
// the CTA whose range holds chunk-tile q
__device__ __forceinline__ int owner_of(int q, int N, int G) {
    return static_cast<int>((static_cast<long long>(q + 1) * G - 1) / N);
}

__device__ __forceinline__ void named_sync() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

__device__ __forceinline__ unsigned ld_acquire(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void red_release(unsigned* p, unsigned v) {
    asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

struct Ctx {
    const DitLayersArgs& a;
    int G, c;
    uint8_t* bt;      // token tiles
    float* scratch;   // kScratchFloats
    float* rope_s;    // [2][12][64] cos, sin
    float* inv_s;     // [24]
    int* plist;       // [kMaxPieces][kMaxList] piece lists: cta << 8 | piece index
    int* pcount;      // [kMaxPieces]
    int* flag_s;      // [0] failure seen by any role (written asynchronously), [1..kMaxPieces] finisher flags
    int* cfail_s;     // compute warps' failure flag: written by thread 0 between two named barriers only,
                      // so all 128 compute threads always take the same path through the named barriers
    unsigned target;  // grid barrier arrivals expected so far
};

// All compute threads; false when this CTA is winding down (a wait timed out here or in another role).
__device__ bool grid_sync(Ctx& x) {
    __threadfence();
    named_sync();
    x.target += static_cast<unsigned>(x.G);
    if (threadIdx.x == 0) {
        if (x.flag_s[0]) *x.cfail_s = 1;
        if (!*x.cfail_s) {
            unsigned* ctr = x.a.sync;
            red_release(ctr, 1u);
            uint32_t i = 0;
            while (ld_acquire(ctr) < x.target)
                if (++i > kWaitLimit) {
                    *x.cfail_s = 1;
                    x.flag_s[0] = 1;
                    break;
                }
        }
    }
    named_sync();
    return !*x.cfail_s;
}

// Pieces of tile t (the non-empty CTA ranges that intersect it, in K order) into
// list slot 'which'; called by one thread, published by the caller's barrier.
__device__ void list_pieces(Ctx& x, int which, int t, int nch, int N) {
    const int G = x.G;
    const int c0 = owner_of(t * nch, N, G), c1 = owner_of((t + 1) * nch - 1, N, G);
    int n = 0;
    for (int cc = c0; cc <= c1 && n < kMaxList; ++cc) {
        const int l0 = range_lo(cc, N, G);
        if (range_lo(cc + 1, N, G) == l0) continue;  // empty range
        x.plist[which * kMaxList + n++] = (cc << 8) | (t - l0 / nch);
    }
    x.pcount[which] = n;
}

__device__ __forceinline__ const float* part_row(const DitLayersArgs& a, int entry, int row) {
    const int cta = entry >> 8, piece = entry & 255;
    return a.part + (static_cast<size_t>(cta) * kMaxPieces + piece) * kPartFloats + row * 24;
}

__device__ __forceinline__ void zero_pads(uint8_t* tile, int M) {
    for (int u = threadIdx.x; u < (kLoOffset - M) * 16; u += kCompute) {
        const int m = M + u / 16, col = (u & 15) * 4;
        put_split4(tile, m, col, make_float4(0.f, 0.f, 0.f, 0.f));
    }
}

// Row sums of squares from 'parts' slices [part][24] -> inv_s[m] = rsqrt(mean + eps).
// 120 threads = 20 part groups x 6 token quads, each loading its parts at once;
// then a fixed-order sum over the groups (deterministic).
__device__ void norm_scales(Ctx& x, int parts) {
    const DitLayersArgs& a = x.a;
    const int tid = threadIdx.x;
    float4* red = reinterpret_cast<float4*>(x.scratch);  // [20][6]
    if (tid < 120) {
        const int r = tid / 6, q = tid - r * 6;
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int p0 = 0; p0 < parts; p0 += 160) {
            float4 v[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const int p = p0 + r + 20 * i;
                v[i] = p < parts ? __ldcg(reinterpret_cast<const float4*>(a.ssq + p * kSsqStride) + q)
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
    named_sync();
    if (tid < 24) {
        const float* rf = x.scratch;
        float t = 0.f;
        for (int r = 0; r < 20; ++r) t += rf[(r * 6) * 4 + tid];
        x.inv_s[tid] = rsqrtf(t / static_cast<float>(a.Hd) + a.eps);
    }
    named_sync();
}

// token tiles j < nb = RMSNorm(dh) for chunk (lo + j) % nch (RMSNorm as in
// rmsnorm_rows_split_kernel: x * rsqrt(mean(x^2) + eps) * g)
__device__ void build_norm(Ctx& x, const __half* g, int parts, int lo, int nb, int nch) {
    const DitLayersArgs& a = x.a;
    const int tid = threadIdx.x;
    norm_scales(x, parts);
    const int per = nb * 16, total = a.M * per;
    constexpr int kB = 8;
    for (int base = 0; base < total; base += kCompute * kB) {
        float4 xv[kB];
        uint2 gw[kB];
#pragma unroll
        for (int i = 0; i < kB; ++i) {
            const int u = base + tid + kCompute * i;
            if (u < total) {
                const int m = u / per, r = u - m * per, j = r >> 4, col = (r & 15) * 4;
                const int k = ((lo + j) % nch) * kKChunk + col;
                xv[i] = __ldcg(reinterpret_cast<const float4*>(a.dh + static_cast<size_t>(m) * a.Hd + k));
                gw[i] = __ldg(reinterpret_cast<const uint2*>(g + k));
            }
        }
#pragma unroll
        for (int i = 0; i < kB; ++i) {
            const int u = base + tid + kCompute * i;
            if (u < total) {
                const int m = u / per, r = u - m * per, j = r >> 4, col = (r & 15) * 4;
                const float2 g01 = __half22float2(*reinterpret_cast<const __half2*>(&gw[i].x));
                const float2 g23 = __half22float2(*reinterpret_cast<const __half2*>(&gw[i].y));
                const float iv = x.inv_s[m];
                put_split4(x.bt + j * kBBytes, m, col,
                           make_float4(xv[i].x * iv * g01.x, xv[i].y * iv * g01.y, xv[i].z * iv * g23.x,
                                       xv[i].w * iv * g23.y));
            }
        }
    }
    for (int j = 0; j < nb; ++j) zero_pads(x.bt + j * kBBytes, a.M);
}

// token tile j = attention output of head h (RoPE on q and k, scores * scale,
// softmax, P.V; both sequences), as in dit_attention_split_kernel
__device__ void build_attention(Ctx& x, int h, int j) {
    constexpr int D = 64, HALF = 32;
    const DitLayersArgs& a = x.a;
    const int tid = threadIdx.x, M = a.M, seq = a.seq;
    const int W = (a.hq + 2 * a.hkv) * D, kvh = h / (a.hq / a.hkv);
    float* qs = x.scratch;
    float* ks = qs + 24 * kAttnRow;
    float* vs = ks + 24 * kAttnRow;
    float* ps = vs + 24 * D;
    // raw q / k / v rows of the head: M x 3 x 16 float4, all loads in flight at once
    {
        constexpr int kB = 9;
        const int total = M * 48;
        for (int base = 0; base < total; base += kCompute * kB) {
            float4 v[kB];
#pragma unroll
            for (int i = 0; i < kB; ++i) {
                const int u = base + tid + kCompute * i;
                if (u < total) {
                    const int r = u / 48, w = u - r * 48, kind = w >> 4, e4 = (w & 15) * 4;
                    const int col = kind == 0 ? h * D : kind == 1 ? (a.hq + kvh) * D : (a.hq + a.hkv + kvh) * D;
                    v[i] = __ldcg(reinterpret_cast<const float4*>(a.qkv + static_cast<size_t>(r) * W + col + e4));
                }
            }
#pragma unroll
            for (int i = 0; i < kB; ++i) {
                const int u = base + tid + kCompute * i;
                if (u < total) {
                    const int r = u / 48, w = u - r * 48, kind = w >> 4, e4 = (w & 15) * 4;
                    float* dst = kind == 0 ? qs + r * kAttnRow : kind == 1 ? ks + r * kAttnRow : vs + r * D;
                    dst[e4] = v[i].x;
                    dst[e4 + 1] = v[i].y;
                    dst[e4 + 2] = v[i].z;
                    dst[e4 + 3] = v[i].w;
                }
            }
        }
    }
    named_sync();
    // RoPE (rotate_half) on q and k in place: each unit owns the pair (e, e + 32)
    for (int u = tid; u < 2 * M * HALF; u += kCompute) {
        const int which = u / (M * HALF), r = u - which * M * HALF, i = r / HALF, e = r - i * HALF, pos = i % seq;
        float* row = (which == 0 ? qs : ks) + i * kAttnRow;
        const float c1 = x.rope_s[pos * D + e], c2 = x.rope_s[pos * D + e + HALF];
        const float s1 = x.rope_s[12 * D + pos * D + e], s2 = x.rope_s[12 * D + pos * D + e + HALF];
        const float v1 = row[e], v2 = row[e + HALF];
        row[e] = v1 * c1 + (-v2) * s1;
        row[e + HALF] = v2 * c2 + v1 * s2;
    }
    named_sync();
    for (int u = tid; u < 2 * seq * seq; u += kCompute) {
        const int b = u / (seq * seq), r = u - b * seq * seq, i = r / seq, jj = r - i * seq;
        const float* q = qs + (b * seq + i) * kAttnRow;
        const float* k = ks + (b * seq + jj) * kAttnRow;
        float sum = 0.f;
#pragma unroll 16
        for (int e = 0; e < D; ++e) sum = fmaf(q[e], k[e], sum);
        ps[(b * 12 + i) * 13 + jj] = sum * a.scale;
    }
    named_sync();
    for (int u = tid; u < 2 * seq; u += kCompute) {
        float* pr = ps + ((u / seq) * 12 + (u % seq)) * 13;
        float mx = -FLT_MAX;
        for (int jj = 0; jj < seq; ++jj) mx = fmaxf(mx, pr[jj]);
        float sum = 0.f;
        for (int jj = 0; jj < seq; ++jj) {
            pr[jj] = expf(pr[jj] - mx);
            sum += pr[jj];
        }
        for (int jj = 0; jj < seq; ++jj) pr[jj] /= sum;
    }
    named_sync();
    uint8_t* tile = x.bt + j * kBBytes;
    for (int u = tid; u < M * 16; u += kCompute) {
        const int m = u >> 4, col = (u & 15) * 4, b = m / seq, i = m - b * seq;
        const float* pr = ps + (b * 12 + i) * 13;
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int jj = 0; jj < seq; ++jj) {
            const float p = pr[jj];
            const float* vr = vs + (b * seq + jj) * D + col;
            acc.x = fmaf(p, vr[0], acc.x);
            acc.y = fmaf(p, vr[1], acc.y);
            acc.z = fmaf(p, vr[2], acc.z);
            acc.w = fmaf(p, vr[3], acc.w);
        }
        put_split4(tile, m, col, acc);
    }
    zero_pads(tile, M);
    named_sync();  // the scratch is reused by the next head
}

// token tiles j < nb = chunks (lo + j) % nch of the split-fp16 gate/up output [48][F]
__device__ void build_copy(Ctx& x, int lo, int nb, int nch) {
    const DitLayersArgs& a = x.a;
    constexpr int kB = 12;
    const int total = nb * kBRows * 8;
    for (int base = 0; base < total; base += kCompute * kB) {
        uint4 v[kB];
#pragma unroll
        for (int i = 0; i < kB; ++i) {
            const int u = base + threadIdx.x + kCompute * i;
            if (u < total) {
                const int j = u / (kBRows * 8), r = (u / 8) % kBRows, q = u & 7;
                const int k = ((lo + j) % nch) * kKChunk + q * 8;
                v[i] = __ldcg(reinterpret_cast<const uint4*>(a.act + static_cast<size_t>(r) * a.F + k));
            }
        }
#pragma unroll
        for (int i = 0; i < kB; ++i) {
            const int u = base + threadIdx.x + kCompute * i;
            if (u < total) {
                const int j = u / (kBRows * 8), r = (u / 8) % kBRows, q = u & 7;
                *reinterpret_cast<uint4*>(x.bt + j * kBBytes + r * 128 + ((q ^ (r & 7)) << 4)) = v[i];
            }
        }
    }
}

__device__ __forceinline__ float* part_ptr(const DitLayersArgs& a, int cta, int piece, int row) {
    return a.part + (static_cast<size_t>(cta) * kMaxPieces + piece) * kPartFloats + row * 24;
}

// Sum of the pieces (list slot 'which') of tokens [m0, m0 + 4 NQ) of tile row
// 'row', in list order, with the loads of several pieces in flight at once.
template <int NQ>
__device__ __forceinline__ void sum_pieces(const Ctx& x, int which, int row, int m0, float* out) {
    constexpr int kB = 12 / NQ;  // 12 float4 loads in flight per thread
#pragma unroll
    for (int i = 0; i < 4 * NQ; ++i) out[i] = 0.f;
    const int n = x.pcount[which];
    for (int k0 = 0; k0 < n; k0 += kB) {
        float4 v[kB][NQ];
#pragma unroll
        for (int k = 0; k < kB; ++k)
#pragma unroll
            for (int q = 0; q < NQ; ++q)
                v[k][q] = k0 + k < n
                              ? __ldcg(reinterpret_cast<const float4*>(part_row(x.a, x.plist[which * kMaxList + k0 + k], row) + m0) + q)
                              : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int k = 0; k < kB; ++k)
#pragma unroll
            for (int q = 0; q < NQ; ++q) {
                out[4 * q] += v[k][q].x;
                out[4 * q + 1] += v[k][q].y;
                out[4 * q + 2] += v[k][q].z;
                out[4 * q + 3] += v[k][q].w;
            }
    }
}

// o / down: dh += rscale * (sum of the pieces) over this CTA's feature slice,
// then the slice's per-token sum of squares (part c of the next RMSNorm). The
// pieces' rows are staged in shared memory by one batch of loads, then summed in
// list order.
__device__ void reduce_resid(Ctx& x, int nch, int N) {
    const DitLayersArgs& a = x.a;
    const int tid = threadIdx.x;
    const int f0 = static_cast<int>(static_cast<long long>(x.c) * a.Hd / x.G);
    const int nf = static_cast<int>(static_cast<long long>(x.c + 1) * a.Hd / x.G) - f0;
    const int t_first = f0 / kTileRows;
    if (tid == 0 && nf > 0) {
        list_pieces(x, 0, t_first, nch, N);
        if ((f0 + nf - 1) / kTileRows != t_first) list_pieces(x, 1, t_first + 1, nch, N);
    }
    named_sync();
    float* stage = x.scratch;  // [feature group][piece][24]
    __shared__ float sqs[24][kMaxSlice + 1];
    const int np_max = nf > 0 ? max(x.pcount[0], (f0 + nf - 1) / kTileRows != t_first ? x.pcount[1] : 0) : 1;
    const int group = max(1, min(nf, kScratchFloats / (np_max * 24)));
    for (int g0 = 0; g0 < nf; g0 += group) {
        const int ng = min(group, nf - g0);
        const int total = ng * np_max * 6;
        constexpr int kB = 8;
        for (int base = 0; base < total; base += kCompute * kB) {
            float4 v[kB];
#pragma unroll
            for (int i = 0; i < kB; ++i) {
                const int u = base + tid + kCompute * i;
                v[i] = make_float4(0.f, 0.f, 0.f, 0.f);
                if (u < total) {
                    const int fi = u / (np_max * 6), r = u - fi * np_max * 6, k = r / 6, q = r - k * 6;
                    const int f = f0 + g0 + fi, which = f / kTileRows - t_first;
                    if (k < x.pcount[which])
                        v[i] = __ldcg(reinterpret_cast<const float4*>(
                                          part_row(a, x.plist[which * kMaxList + k], f % kTileRows)) + q);
                }
            }
#pragma unroll
            for (int i = 0; i < kB; ++i) {
                const int u = base + tid + kCompute * i;
                if (u < total) reinterpret_cast<float4*>(stage)[u] = v[i];
            }
        }
        named_sync();
        for (int u = tid; u < ng * 24; u += kCompute) {
            const int fi = u / 24, m = u - fi * 24, f = f0 + g0 + fi;
            const int which = f / kTileRows - t_first;
            float v = 0.f;
            for (int k = 0; k < x.pcount[which]; ++k) v += stage[(fi * np_max + k) * 24 + m];
            if (m < a.M) {
                float* y = a.dh + static_cast<size_t>(m) * a.Hd + f;
                const float nv = __ldcg(y) + (a.rscale == 1.f ? v : v * a.rscale);
                *y = nv;
                sqs[m][g0 + fi] = nv * nv;
            }
        }
        named_sync();
    }
    if (tid < 24) {
        float t = 0.f;
        if (tid < a.M)
            for (int fi = 0; fi < nf; ++fi) t += sqs[tid][fi];
        a.ssq[x.c * kSsqStride + tid] = t;
    }
}

__global__ void __launch_bounds__(kThreads, 1) dit_layers_kernel(const DitLayersArgs a) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    __shared__ uint64_t full_bar[kRing], empty_bar[kRing], b_ready, acc_ready, fin_bar;
    __shared__ uint32_t tmem_base_s;
    __shared__ int flag_s[1 + kMaxPieces];
    __shared__ int cfail_s;
    __shared__ float inv_s[24];
    __shared__ int plist_s[kMaxPieces * kMaxList], pcount_s[kMaxPieces];

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int G = gridDim.x, c = blockIdx.x;
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* ring = smem;
    uint8_t* bt = smem + kRing * kABytes;
    float* scratch = reinterpret_cast<float*>(bt + kMaxB * kBBytes);
    float* rope_s = scratch + kScratchFloats;

    if (tid == 0) {
        for (int i = 0; i < kRing; ++i) {
            mbar_init(&full_bar[i], 1);
            mbar_init(&empty_bar[i], 1);
        }
        mbar_init(&b_ready, 1);
        mbar_init(&acc_ready, 1);
        mbar_init(&fin_bar, 1);
        for (int i = 0; i <= kMaxPieces; ++i) flag_s[i] = 0;
        cfail_s = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 5) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                         smem_addr(&tmem_base_s)), "r"(kTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = tmem_base_s;

    if (warp == 4) {
        // ---------------------------------------------------------- TMA producer
        if (lane == 0) {
            int slot = 0;
            long long n = 0;
            for (int l = 0; l < a.layers && !flag_s[0]; ++l)
                for (int p = 0; p < 4 && !flag_s[0]; ++p) {
                    const Shape sh = phase_shape(a, p);
                    const int N = sh.tiles * sh.nch, lo = range_lo(c, N, G), hi = range_lo(c + 1, N, G);
                    const CUtensorMap* map = a.maps + l * 4 + p;
                    for (int q = lo; q < hi; ++q) {
                        if (n >= kRing && !mbar_wait(&empty_bar[slot], ((n / kRing) - 1) & 1)) {
                            flag_s[0] = 1;
                            break;
                        }
                        const int t = q / sh.nch, ch = q % sh.nch;
                        const int r0 = p == PH_GU ? t * 64 : t * kTileRows;
                        const int r1 = p == PH_GU ? a.F + t * 64 : t * kTileRows + 64;
                        uint8_t* dst = ring + slot * kABytes;
                        mbar_expect_tx(&full_bar[slot], kABytes);
                        tma_load_2d(dst, map, ch * kKChunk, r0, &full_bar[slot]);
                        tma_load_2d(dst + kABytes / 2, map, ch * kKChunk, r1, &full_bar[slot]);
                        slot = slot + 1 == kRing ? 0 : slot + 1;
                        ++n;
                    }
                }
            // no load may still be landing when the CTA exits
            for (long long i = std::max(0LL, n - kRing); i < n; ++i)
                if (!mbar_wait(&full_bar[i % kRing], (i / kRing) & 1)) flag_s[0] = 1;
        }
    } else if (warp == 5) {
        // ---------------------------------------------------------- MMA issuer
        if (lane == 0) {
            const uint32_t idesc = umma_idesc(kTileRows, kBRows);
            int slot = 0, kph = 0;
            long long n = 0;
            bool ok = true;
            for (int l = 0; l < a.layers && ok; ++l)
                for (int p = 0; p < 4 && ok; ++p) {
                    const Shape sh = phase_shape(a, p);
                    const int N = sh.tiles * sh.nch, lo = range_lo(c, N, G), hi = range_lo(c + 1, N, G);
                    if (hi == lo) continue;
                    if (!mbar_wait(&b_ready, kph & 1)) {
                        ok = false;
                        break;
                    }
                    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                    const int t0 = lo / sh.nch;
                    uint32_t started = 0;
                    for (int q = lo; q < hi; ++q) {
                        const int j = q - lo, piece = q / sh.nch - t0, chain = j & 1, acc = piece * 2 + chain;
                        if (!mbar_wait(&full_bar[slot], (n / kRing) & 1)) {
                            ok = false;
                            break;
                        }
                        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                        const uint32_t sa = smem_addr(ring + slot * kABytes), sb = smem_addr(bt + j * kBBytes);
                        const uint32_t d = tmem + static_cast<uint32_t>(acc * 64);
#pragma unroll
                        for (int kk = 0; kk < kKChunk / 16; ++kk)
                            umma_f16(d, umma_desc(sa + kk * 32), umma_desc(sb + kk * 32), idesc,
                                     ((started >> acc) & 1) || kk > 0);
                        started |= 1u << acc;
                        umma_commit(&empty_bar[slot]);
                        slot = slot + 1 == kRing ? 0 : slot + 1;
                        ++n;
                    }
                    umma_commit(&acc_ready);
                    ++kph;
                }
            if (!ok) flag_s[0] = 1;
            // every MMA issued above has finished before TMEM is released
            umma_commit(&fin_bar);
            if (!mbar_wait(&fin_bar, 0)) flag_s[0] = 1;
        }
    } else {
        // ---------------------------------------------------------- compute warps
        Ctx x{a, G, c, bt, scratch, rope_s, inv_s, plist_s, pcount_s, flag_s, &cfail_s, 0u};
        int kph = 0;
        const int row = warp * 32 + lane;  // TMEM lane = tile row
        for (int i = tid; i < a.seq * 64; i += kCompute) {  // RoPE tables of the sequence positions
            rope_s[i] = a.rope_cos[i];
            rope_s[12 * 64 + i] = a.rope_sin[i];
        }
        named_sync();
        for (int l = 0; l < a.layers; ++l) {
            for (int p = 0; p < 4; ++p) {
                if (cfail_s) break;  // uniform: written only between named barriers
                const Shape sh = phase_shape(a, p);
                const int N = sh.tiles * sh.nch, lo = range_lo(c, N, G), hi = range_lo(c + 1, N, G);
                const int nb = hi - lo;
                int npieces = 0;
                if (nb > 0) {
                    const int t0 = lo / sh.nch;
                    npieces = (hi - 1) / sh.nch - t0 + 1;
                    // 1. token operand
                    if (p == PH_QKV) build_norm(x, a.norms[2 * l], l == 0 ? a.embed_parts : G, lo, nb, sh.nch);
                    else if (p == PH_GU) build_norm(x, a.norms[2 * l + 1], G, lo, nb, sh.nch);
                    else if (p == PH_O) for (int j = 0; j < nb; ++j) build_attention(x, (lo + j) % sh.nch, j);
                    else build_copy(x, lo, nb, sh.nch);
                    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                    named_sync();
                    if (tid == 0) mbar_arrive(&b_ready);
                    // 2. accumulators (one thread waits, the barrier publishes the outcome)
                    if (tid == 0 && !mbar_wait(&acc_ready, kph & 1)) {
                        cfail_s = 1;
                        flag_s[0] = 1;
                    }
                    ++kph;
                    named_sync();
                    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                    const bool ok = !cfail_s;
                    // 3. partial rows to global memory: piece P = chunks [a0, a1) of the range
                    for (int P = 0; P < npieces && ok; ++P) {
                        const int a0 = std::max(lo, (t0 + P) * sh.nch) - lo;
                        const int a1 = std::min(hi, (t0 + P + 1) * sh.nch) - lo;
                        float v[24];
#pragma unroll
                        for (int m = 0; m < 24; ++m) v[m] = 0.f;
                        for (int chain = 0; chain < 2; ++chain) {
                            const bool used = (a1 - a0 >= 2) || ((a0 & 1) == chain);
                            if (!used) continue;
                            float d[kBRows];
                            const uint32_t ta = tmem + (static_cast<uint32_t>(warp * 32) << 16) +
                                                static_cast<uint32_t>((P * 2 + chain) * 64);
                            tmem_ld16(ta, d);
                            tmem_ld16(ta + 16, d + 16);
                            tmem_ld16(ta + 32, d + 32);
                            asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
                            for (int m = 0; m < 24; ++m) v[m] += d[m] + d[kLoOffset + m];
                        }
                        float4* dst = reinterpret_cast<float4*>(part_ptr(a, c, P, row));
#pragma unroll
                        for (int q4 = 0; q4 < 6; ++q4)
                            dst[q4] = make_float4(v[4 * q4], v[4 * q4 + 1], v[4 * q4 + 2], v[4 * q4 + 3]);
                    }
                    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
                }
                // 4. q/k/v and gate/up: the last CTA to deliver a piece of a tile finishes it
                if (p == PH_QKV || p == PH_GU) {
                    __threadfence();
                    named_sync();
                    if (tid == 0)
                        for (int P = 0; P < npieces; ++P) {
                            const int t = lo / sh.nch + P;
                            list_pieces(x, P, t, sh.nch, N);
                            const unsigned old = atomicAdd(a.sync + 2 + t, 1u);
                            __threadfence();
                            flag_s[1 + P] = old == static_cast<unsigned>(pcount_s[P] - 1);
                            if (flag_s[1 + P]) a.sync[2 + t] = 0;  // ready for the next layer
                        }
                    named_sync();
                    for (int P = 0; P < npieces; ++P) {
                        if (!flag_s[1 + P]) continue;
                        const int t = lo / sh.nch + P;
                        if (p == PH_QKV) {
                            float v[24];
                            sum_pieces<6>(x, P, row, 0, v);
                            const int W = (a.hq + 2 * a.hkv) * 64;
                            for (int m = 0; m < a.M; ++m) a.qkv[static_cast<size_t>(m) * W + t * kTileRows + row] = v[m];
                        } else {
                            // thread r < 64: pair r, tokens 0..11; r >= 64: pair r - 64, tokens 12..23
                            const int pr = row & 63, m0 = row < 64 ? 0 : 12;
                            float gv[12], uv[12];
                            sum_pieces<3>(x, P, pr, m0, gv);
                            sum_pieces<3>(x, P, 64 + pr, m0, uv);
#pragma unroll
                            for (int m = 0; m < 12; ++m)
                                if (m0 + m < a.M) store_split(a.act, a.F, m0 + m, t * 64 + pr, silu(gv[m]) * uv[m]);
                        }
                    }
                }
                if (!grid_sync(x)) break;
                // 5. o / down: distributed residual reduction
                if (p == PH_O || p == PH_DOWN) {
                    reduce_resid(x, sh.nch, N);
                    if (!grid_sync(x)) break;
                }
            }
            if (cfail_s) break;
        }
    }

    __syncthreads();
    if (tid == 0 && flag_s[0] && a.ctl) a.ctl->error = 3;
    if (warp == 5) {
        __syncwarp();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
    }
}

}  // namespace

int dit_layers_grid() {
    int dev = 0, sms = 0, per_sm = 0;
    check_launch(cudaGetDevice(&dev));
    check_launch(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    check_launch(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, dit_layers_kernel, kThreads, kSmemBytes));
    if (per_sm < 1) throw std::runtime_error("dit_layers: one CTA per SM does not fit");
    return sms;
}

size_t dit_layers_part_floats(int grid) { return static_cast<size_t>(grid) * kMaxPieces * kPartFloats; }
int dit_layers_sync_words() { return 2 + kMaxTiles; }

void check_dit_layers(const DitLayersArgs& a, int grid) {
    if (grid < 1) throw std::invalid_argument("dit_layers: empty grid");
    if (a.M > 24 || a.seq > 12 || a.M != 2 * a.seq || a.Hd % kTileRows != 0 || a.F % kTileRows != 0 ||
        a.hkv <= 0 || a.hq % a.hkv != 0 || a.Hd != a.hq * 64)
        throw std::invalid_argument("dit_layers: unsupported shape");
    const int W = (a.hq + 2 * a.hkv) * 64;
    const int tiles[4] = {W / kTileRows, a.Hd / kTileRows, a.F / 64, a.Hd / kTileRows};
    const int nch[4] = {a.Hd / kKChunk, a.hq, a.Hd / kKChunk, a.F / kKChunk};
    for (int p = 0; p < 4; ++p) {
        const int N = tiles[p] * nch[p];
        const int most = (N + grid - 1) / grid;  // chunk-tiles of the largest range
        if (most > kMaxB || most > nch[p] || tiles[p] + 2 > kMaxTiles)
            throw std::invalid_argument("dit_layers: a CTA's range exceeds the token-tile buffer");
        if ((most + nch[p] - 1) / nch[p] + 1 > kMaxPieces) throw std::invalid_argument("dit_layers: too many pieces");
    }
    if ((a.Hd + grid - 1) / grid > kMaxSlice) throw std::invalid_argument("dit_layers: feature slice too wide");
}

void launch_dit_layers(const DitLayersArgs& a, int grid, cudaStream_t s) {
    check_dit_layers(a, grid);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = kSmemBytes;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    check_launch(cudaLaunchKernelEx(&cfg, dit_layers_kernel, a));
}

void init_dit_layers_attributes() {
    check_launch(cudaFuncSetAttribute(dit_layers_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      static_cast<int>(kSmemBytes)));
}

}  // namespace vxc
