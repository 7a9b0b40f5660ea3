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
// the CTAs of a thread-block cluster: each CTA sends the partial rows another CTA
// owns into that CTA's shared memory as asynchronous stores counted on its
// mbarrier, the owner sums the partials in a fixed order (deterministic), then
// the epilogue (plain store, residual add, or SiLU(gate) * up written straight
// into the next layer's split-fp16 B operand) runs on the owning CTA.
//
// Roles: thread 0 issues TMA (weights before griddepcontrol.wait, so weight
// streaming overlaps the previous kernel), thread 32 issues tcgen05.mma, all
// four warps drain TMEM. Every mbarrier wait gives up after one second of
// %globaltimer time; the failure path is written to record error 3 in the
// stream control block, keep to its cluster barriers and free its TMEM, but it
// has not been exercised on a GPU (no injected failure runs there). The TMEM
// allocation itself has no time bound: it relies on the kernels' shared-memory
// sizes keeping every co-resident mix within the SM's 512 columns.
#include <cuda.h>

#include <algorithm>
#include <stdexcept>
#include <vector>

#include "kernels.cuh"
#include "tc_common.cuh"

namespace vxc {
namespace {

using namespace tc;

constexpr int kTcThreads = 128;
constexpr int kStageBytes = kABytes + kBBytes;    // 22 KiB, keeps 1 KiB alignment
constexpr int kMaxStages = 8;
// split-K receive buffer: every partial of one tile, [part][unit][token] with the token
// run of a unit padded from 24 to 28 floats (16-byte stores; two- to four-way bank
// conflicts on the owner's reads instead of eight)
constexpr int kRecvStride = 28;
constexpr int kRecvFloats = kTileRows * kRecvStride;
constexpr int kMaxSsqParts = 128;  // sums-of-squares parts read in one batch (more: a serial loop)
// parts held in static shared memory; a launch reading more (a 16-way split producer)
// gets them behind its dynamic area, so the common launch keeps its smaller footprint
// (static shared memory counts against every CTA's residency)
constexpr int kStaticSsqParts = 64;

// Dynamic shared memory behind the stage area and the receive buffer for the row
// scale's parts, when there are more than kStaticSsqParts (at most kMaxSsqParts).
__host__ __device__ constexpr size_t ssq_tail_bytes(int row_scale, int parts) {
    return row_scale && parts > kStaticSsqParts && parts <= kMaxSsqParts
               ? static_cast<size_t>(parts) * kSsqStride * sizeof(float) : 0;
}
constexpr int kSqFloats = kTileRows * kLoOffset;    // squares of the updated rows (at most 128 x 24)

// A split launch can receive in its stage area when the area holds the partials and,
// behind them, the squares.
__host__ __device__ constexpr bool shared_recv_fits(bool b_tma, int splits, int recv_shared, size_t area_bytes) {
    return b_tma && splits > 1 && recv_shared && area_bytes >= static_cast<size_t>(kRecvFloats + kSqFloats) * 4;
}
constexpr int kTmemCols = 64;

constexpr size_t kSmemOptin = 232448;  // B200: opt-in shared memory per CTA (227 KB)
size_t g_dyn_limit = 0;                // kSmemOptin less the kernel's static shared memory (set once)

// The receive buffer can share the stage area when nothing else needs it there:
// TMA-fed token tiles, no K split (no remote pushes), no squares scratch.
__host__ __device__ constexpr bool recv_in_stage_area(bool b_tma, int splits, bool ssq_out) {
    return b_tma && splits == 1 && !ssq_out;
}

// S: the K split (cluster size, 1, 2, 4, 8, or 16 for a non-gate/up linear: a
// non-portable cluster), a template parameter so that the
// rank-order sums of the partials unroll and their loads issue together.
template <int S>
__global__ void __launch_bounds__(kTcThreads, 1)
    tc_linear_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
                     const TcLinearArgs a) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    __shared__ uint64_t full_bar[kMaxStages], empty_bar[kMaxStages], done_bar;
    __shared__ uint64_t recv_bar;  // split-K: the peers' partials for this CTA have landed
    __shared__ uint32_t tmem_base_s;
    __shared__ int failed_s;
    __shared__ float inv_s[kLoOffset];
    __shared__ __align__(16) float ssq_static[kStaticSsqParts * kSsqStride];

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int split = blockIdx.x, tile = blockIdx.y;
    // 1 KiB aligned, derived from smem_raw by pointer arithmetic so that the
    // compiler keeps shared-memory addressing for everything carved from it
    uint8_t* smem = smem_raw + ((1024u - (smem_addr(smem_raw) & 1023u)) & 1023u);
    constexpr bool b_tma = true;  // the token tiles arrive by TMA beside the weight tiles

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
        if (S > 1) mbar_init(&recv_bar, 1);
        failed_s = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        // the peers' partials: kTcThreads / S accumulator rows from each of the S - 1 peers,
        // kLoOffset floats each
        if (S > 1) mbar_expect_tx(&recv_bar, (S - 1) * (kTcThreads / S) * kLoOffset * 4);
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
    // split-K: announce that this CTA's barriers are initialised (after thread 0's
    // fence.mbarrier_init, ordered by the block barrier above); the matching wait comes
    // right before the first push into a peer, long after every CTA has arrived
    if (S > 1) cluster_arrive_relaxed();
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

    {
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
    }

    // Epilogue operands that do not wait for the MMAs, read now in one batch per
    // thread: the residual rows this thread updates and (weights) the next operand's
    // gain. Every thread has passed griddepcontrol.wait above.
    // Thread -> output unit lu of this CTA and token rows m0, m0 + per, ... (split path),
    // or accumulator row tid and every token row (direct path).
    const bool direct = S == 1 && !a.gateup && !a.ssq_out;
    const int units = a.gateup ? 64 : kTileRows, halves = a.gateup ? 2 : 1;
    const int nu = units / S;
    const int per = kTcThreads / nu, lu = tid % nu, m0 = tid / nu;  // per == S (== 2 S for gate/up)
    const int col = split * nu + lu;
    constexpr int kRows = (kLoOffset + S - 1) / S;  // token rows per thread, residual split path
    float rres[kRows];
    float rdir[kLoOffset];
    float gn = 0.f;
    if (direct) {
        if (a.resid) {
            const float* yc = a.y + tile * kTileRows + tid;
#pragma unroll
            for (int m = 0; m < kLoOffset; ++m) rdir[m] = m < a.M ? yc[static_cast<size_t>(m) * a.ldy] : 0.f;
        }
    } else if (!a.gateup) {
        const float* yc = a.y + tile * kTileRows + col;
        if (a.next_b) gn = __half2float(a.next_g[tile * kTileRows + col]);
#pragma unroll
        for (int j = 0; j < kRows; ++j) {
            const int m = m0 + j * S;
            rres[j] = (a.resid && m < a.M) ? yc[static_cast<size_t>(m) * a.ldy] : 0.f;
        }
    }

    // row_scale: each token row's 1 / rms from the producer's sums of squares. Warps 2
    // and 3 (idle until the epilogue) read all parts in one batch of 16-byte loads into
    // shared memory; lane m of warp 2 then sums row m's parts in order.
    if (a.row_scale && warp >= 2) {
        if (a.ssq_parts <= kMaxSsqParts) {
            float* ssq_s = ssq_static;
            if (a.ssq_parts > kStaticSsqParts) {  // behind the stage area and the receive buffer
                const bool rin = recv_in_stage_area(b_tma, S, a.ssq_out != nullptr) ||
                                 shared_recv_fits(b_tma, S, a.recv_shared, static_cast<size_t>(stage_area) * kStageBytes);
                ssq_s = reinterpret_cast<float*>(smem + static_cast<size_t>(stage_area) * kStageBytes +
                                                 (rin ? 0 : static_cast<size_t>(kRecvFloats) * sizeof(float)));
            }
            const int n4 = a.ssq_parts * kSsqStride / 4, t = tid - 64;
            const float4* src = reinterpret_cast<const float4*>(a.ssq_in);
            constexpr int kL = kMaxSsqParts * kSsqStride / 4 / 64;
            float4 q4[kL];
#pragma unroll
            for (int j = 0; j < kL; ++j) q4[j] = t + 64 * j < n4 ? __ldcg(src + t + 64 * j) : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
            for (int j = 0; j < kL; ++j)
                if (t + 64 * j < n4) reinterpret_cast<float4*>(ssq_s)[t + 64 * j] = q4[j];
            asm volatile("bar.sync 1, 64;" ::: "memory");  // warps 2 and 3 only
            if (warp == 2 && lane < a.M) {
                float tsum = 0.f;
                for (int p = 0; p < a.ssq_parts; ++p) tsum += ssq_s[p * kSsqStride + lane];
                inv_s[lane] = rsqrtf(tsum / static_cast<float>(a.K) + a.eps);
            }
        } else if (warp == 2 && lane < a.M) {
            float tsum = 0.f;
#pragma unroll 8
            for (int p = 0; p < a.ssq_parts; ++p) tsum += __ldcg(a.ssq_in + p * kSsqStride + lane);
            inv_s[lane] = rsqrtf(tsum / static_cast<float>(a.K) + a.eps);
        }
    }

    // drain the accumulator: warp w owns TMEM lanes (tile rows) 32w .. 32w + 31
    const bool ok = mbar_wait(&done_bar, 0);
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    if (!ok) failed_s = 1;
    // Output units of the tile: 128 rows, or 64 gate/up pairs; CTA p of the cluster
    // owns units [p nu, (p + 1) nu). Each thread holds one accumulator row
    // (tile row tid): v[m] = hi + lo columns of token m.
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
    if (direct) {
        // no split: straight from registers, coalesced across the warp
        if (a.row_scale) {
#pragma unroll
            for (int m = 0; m < kLoOffset; ++m) v[m] *= inv_s[m];
        }
        float* yc = a.y + tile * kTileRows + tid;
#pragma unroll
        for (int m = 0; m < kLoOffset; ++m)
            if (m < a.M)
                yc[static_cast<size_t>(m) * a.ldy] =
                    a.resid ? rdir[m] + (a.rscale == 1.f ? v[m] : v[m] * a.rscale) : v[m];
        __syncthreads();
    } else {
        // Split-K exchange by push: each CTA stores its accumulator rows straight into
        // the receive buffer of the CTA that owns them, as 16-byte remote stores (a
        // thread's kLoOffset tokens are one contiguous run, recv[part][unit][token]
        // with a padded token stride); one cluster barrier; then owners sum the splits
        // in rank order (deterministic). Without a K split it lives in the (then idle)
        // stage area, so more CTAs of concurrent streams fit on an SM.
        // 'shared' and S depend only on launch arguments, never on this CTA's data or on a
        // failed wait, so every CTA of the cluster passes the same cluster barriers
        const bool shared = shared_recv_fits(b_tma, S, a.recv_shared, static_cast<size_t>(stage_area) * kStageBytes);
        const bool recv_in_stages = recv_in_stage_area(b_tma, S, a.ssq_out != nullptr) || shared;
        float* recv =
            reinterpret_cast<float*>(recv_in_stages ? smem : smem + static_cast<size_t>(stage_area) * kStageBytes);
        __syncthreads();  // the stage area is idle
        if (S > 1) cluster_wait();   // every peer's receive barrier is initialised
        if (shared) cluster_sync();  // ... in every CTA of the cluster: partials may land in it
        {
            const int u = a.gateup ? (tid & 63) : tid, half = a.gateup ? (tid >> 6) : 0;
            const int owner = u / nu, ou = u - owner * nu;
            float* dst = recv + static_cast<size_t>((split * halves + half) * nu + ou) * kRecvStride;
            if (owner == split) {
#pragma unroll
                for (int c = 0; c < kLoOffset / 4; ++c)
                    reinterpret_cast<float4*>(dst)[c] = make_float4(v[4 * c], v[4 * c + 1], v[4 * c + 2], v[4 * c + 3]);
            } else {
                const uint32_t remote = peer_addr(dst, owner), rbar = peer_addr(&recv_bar, owner);
#pragma unroll
                for (int c = 0; c < kLoOffset / 4; ++c)
                    st_async4(remote + 16u * c, v[4 * c], v[4 * c + 1], v[4 * c + 2], v[4 * c + 3], rbar);
            }
        }
        asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
        __syncthreads();  // this CTA's own partials are in place
        // the peers' partials: every byte counted on the receive barrier. After the wait no
        // peer writes into this CTA's shared memory again, so it may exit without a cluster
        // barrier; its own asynchronous stores complete at peers that wait for them.
        if (S > 1 && !mbar_wait_cluster(&recv_bar, 0)) failed_s = 1;
        // this CTA's units: thread -> (unit lu, token rows m0, m0 + per, ...); all of a
        // thread's partials are read before any result is stored
        // the stage area is idle now: squares of updated rows (behind the partials when those share it)
        float* sq = reinterpret_cast<float*>(smem) + (shared ? kRecvFloats : 0);
        if (a.gateup) {
            if constexpr (S <= 8) {  // the host gives gate/up at most an 8-way split
                constexpr int kBatch = 4;
                for (int mb = m0; mb < a.M; mb += per * kBatch) {
                    float g[kBatch][S], up[kBatch][S];
#pragma unroll
                    for (int j = 0; j < kBatch; ++j) {
                        const int mc = min(mb + j * per, a.M - 1);
#pragma unroll
                        for (int p = 0; p < S; ++p) {
                            g[j][p] = recv[static_cast<size_t>((p * 2 + 0) * nu + lu) * kRecvStride + mc];
                            up[j][p] = recv[static_cast<size_t>((p * 2 + 1) * nu + lu) * kRecvStride + mc];
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
            }
        } else {
            float* yc = a.y + tile * kTileRows + col;
            float part[kRows][S];
#pragma unroll
            for (int j = 0; j < kRows; ++j) {
                const int mc = min(m0 + j * S, a.M - 1);
#pragma unroll
                for (int p = 0; p < S; ++p) part[j][p] = recv[static_cast<size_t>(p * nu + lu) * kRecvStride + mc];
            }
#pragma unroll
            for (int j = 0; j < kRows; ++j) {
                const int m = m0 + j * S;
                if (m < a.M) {
                    float sum = 0.f;
#pragma unroll
                    for (int p = 0; p < S; ++p) sum += part[j][p];
                    if (a.row_scale) sum *= inv_s[m];
                    const float nv = a.resid ? rres[j] + (a.rscale == 1.f ? sum : sum * a.rscale) : sum;
                    yc[static_cast<size_t>(m) * a.ldy] = nv;
                    if (a.ssq_out) sq[m * nu + lu] = nv * nv;
                    if (a.next_b) store_split(a.next_b, a.ldnb, m, tile * kTileRows + col, nv * gn);
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

size_t tc_linear_smem_bytes(int K, int splits, int max_stages, bool ssq_out, bool recv_shared, int row_scale_parts) {
    const int nch = K / kKChunk;
    const int cs = (nch + splits - 1) / splits;
    const int stages = std::min(std::min(max_stages, kMaxStages), std::max(cs, 1));
    const size_t stage_bytes = static_cast<size_t>(stages) * kStageBytes;
    const size_t tail = ssq_tail_bytes(row_scale_parts > 0, row_scale_parts);
    if (recv_in_stage_area(true, splits, ssq_out) || shared_recv_fits(true, splits, recv_shared, stage_bytes))
        return stage_bytes + tail + 1024;  // + alignment slack
    const size_t recv_bytes = static_cast<size_t>(kRecvFloats) * sizeof(float);
    return stage_bytes + recv_bytes + tail + 1024;  // + alignment slack
}

cudaError_t launch_split(cudaLaunchConfig_t& cfg, const CUtensorMap& map_a, const CUtensorMap& map_b,
                         const TcLinearArgs& a) {
    switch (a.splits) {
        case 1: return cudaLaunchKernelEx(&cfg, tc_linear_kernel<1>, map_a, map_b, a);
        case 2: return cudaLaunchKernelEx(&cfg, tc_linear_kernel<2>, map_a, map_b, a);
        case 4: return cudaLaunchKernelEx(&cfg, tc_linear_kernel<4>, map_a, map_b, a);
        case 8: return cudaLaunchKernelEx(&cfg, tc_linear_kernel<8>, map_a, map_b, a);
        default: return cudaLaunchKernelEx(&cfg, tc_linear_kernel<16>, map_a, map_b, a);
    }
}

// every instantiation (one per K split)
std::vector<const void*> tc_linear_kernels() {
    return {reinterpret_cast<const void*>(tc_linear_kernel<1>), reinterpret_cast<const void*>(tc_linear_kernel<2>),
            reinterpret_cast<const void*>(tc_linear_kernel<4>), reinterpret_cast<const void*>(tc_linear_kernel<8>),
            reinterpret_cast<const void*>(tc_linear_kernel<16>)};
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

void launch_tc_linear(const CUtensorMap& map_a, const CUtensorMap& map_b, const TcLinearArgs& a, cudaStream_t s,
                      bool pdl) {
    if (a.K % kKChunk != 0 || a.K <= 0) throw std::invalid_argument("tc_linear: K must be a multiple of 64");
    if (a.M <= 0 || a.M > kLoOffset) throw std::invalid_argument("tc_linear: at most 24 token rows");
    if ((a.splits != 1 && a.splits != 2 && a.splits != 4 && a.splits != 8 && a.splits != 16) ||
        a.splits > a.K / kKChunk || (a.gateup && a.splits > 8))
        throw std::invalid_argument("tc_linear: splits must be 1, 2, 4, 8 or 16 (gate/up: at most 8) and at most K / 64");
    const int n_tiles = a.gateup ? a.rows / 64 : a.rows / kTileRows;
    if ((a.gateup ? a.rows % 64 : a.rows % kTileRows) != 0) throw std::invalid_argument("tc_linear: rows");
    if (a.ssq_out && (a.gateup || a.M > kSsqStride)) throw std::invalid_argument("tc_linear: bad ssq_out");
    if (a.next_b && (!a.ssq_out || !a.next_g || !a.resid || a.ldnb < a.rows))
        throw std::invalid_argument("tc_linear: next_b needs a residual launch with ssq_out and next_g");
    if (a.row_scale && (!a.ssq_in || a.ssq_parts <= 0 || (reinterpret_cast<uintptr_t>(a.ssq_in) & 15) != 0))
        throw std::invalid_argument("tc_linear: row_scale needs 16-byte aligned ssq_in parts");
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(a.splits, n_tiles);
    cfg.blockDim = dim3(kTcThreads);
    if (a.max_stages < 1 || a.max_stages > kMaxStages) throw std::invalid_argument("tc_linear: max_stages in [1, 8]");
    cfg.dynamicSmemBytes = std::max(tc_linear_smem_bytes(a.K, a.splits, a.max_stages, a.ssq_out != nullptr,
                                                         a.recv_shared != 0, a.row_scale ? a.ssq_parts : 0),
                                    tmem_smem_floor(kTmemCols));
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
    const cudaError_t e = launch_split(cfg, map_a, map_b, a);
    if (e != cudaSuccess) throw std::runtime_error(std::string("tc_linear launch: ") + cudaGetErrorString(e));
}

void init_tc_attributes() {
    // every launch checks its own need against this limit
    for (const void* f : tc_linear_kernels()) {
        const cudaError_t e = cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                   static_cast<int>(dyn_limit()));
        if (e != cudaSuccess) throw std::runtime_error(std::string("tc_linear attribute: ") + cudaGetErrorString(e));
    }
    // the 16-way K split is a cluster of 16 CTAs, beyond the portable 8
    const cudaError_t e = cudaFuncSetAttribute(reinterpret_cast<const void*>(tc_linear_kernel<16>),
                                               cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    if (e != cudaSuccess) throw std::runtime_error(std::string("tc_linear cluster attribute: ") + cudaGetErrorString(e));
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
