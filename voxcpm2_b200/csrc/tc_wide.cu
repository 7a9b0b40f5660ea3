// tcgen05 linear over a wide token block: up to kWideTokens = 176 rows, for the
// DiT estimator of a group of up to 8 streams evaluated together
// (DitEstimator.decoder, tools/export_components.py:625-659, over 22 rows per
// stream).
//
// The weight tile is the MMA A operand (128 output features, K-major, 128-byte
// swizzle, TMA); the token rows are the B operand. The operand buffer holds a
// row block of 'lo' rows (a multiple of 16, at least M): fp16(x) in rows
// 0..lo-1 and fp16(x - fp16(x)) in rows lo..2 lo-1. A K chunk brings both halves
// with two TMA copies of one lo-row box; both accumulate into the same lo fp32
// TMEM columns (two N = lo MMAs per K step), so the accumulator already holds
// W (x_hi + x_lo). K is split across a thread-block cluster of 1, 2, 4 or 8 CTAs:
// after the MMAs each CTA sends its partial rows, one contiguous token run per
// output feature, to the CTA that owns those features as 16-byte asynchronous
// stores counted on the owner's mbarrier; the owner waits for its bytes, sums the
// partials in rank order and writes the epilogue: plain, residual
// (y += rscale * v), or SiLU(gate) * up into the next linear's split operand
// (residual half at row offset lo). The accumulator is read from TMEM 32 token
// columns at a time.
//
// TMEM: 128 columns for lo <= 128, else 256. Shared memory never drops below
// tmem_smem_floor of that count (and kFloor), so the SM's 512 TMEM columns are
// never oversubscribed by co-resident CTAs and a cluster CTA never waits for
// TMEM. Every mbarrier wait is time-bounded; on timeout the kernel records
// error 3, still passes the cluster barriers, drains its loads and frees its TMEM
// (this failure path has not been exercised on a GPU).
#include <cuda.h>

#include <algorithm>
#include <stdexcept>
#include <string>

#include "kernels.cuh"
#include "tc_common.cuh"

namespace vxc {
namespace {

using namespace tc;

constexpr int kThreads = 128;
constexpr int kMaxRing = 4;
constexpr size_t kFloor = 92 * 1024;
// dynamic shared memory a launch may ask for: the 227 KiB opt-in limit covers the
// static barriers too, so 1 KiB is left for them
constexpr size_t kSmemMax = 226 * 1024;

void check_launch(cudaError_t e) {
    if (e != cudaSuccess) throw std::runtime_error(std::string("tc_wide: ") + cudaGetErrorString(e));
}

__device__ __forceinline__ void cluster_barrier() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// Shared-memory layout of a launch, the same on the host and in every CTA.
__host__ __device__ constexpr int stage_bytes(int lo) { return kABytes + lo * kKChunk * 2 * 2; }
// the receive buffer: every (split, half, unit) of a tile, a token run of lo + 4 floats each
__host__ __device__ constexpr int recv_stride(int lo) { return lo + 4; }
__host__ __device__ constexpr size_t recv_bytes(int lo) { return static_cast<size_t>(kTileRows) * recv_stride(lo) * 4; }
__host__ __device__ constexpr int tmem_cols(int lo) { return lo <= 128 ? 128 : 256; }
// The receive buffer lives in the (then idle) stage area when the CTA has no
// K split and the stage area is large enough for it.
__host__ __device__ constexpr bool recv_in_stages(int splits, int stages, int lo) {
    return splits == 1 && static_cast<size_t>(stages) * stage_bytes(lo) >= recv_bytes(lo);
}

// S = K split (cluster size): a template parameter so the partial sums unroll.
template <int S>
__global__ void __launch_bounds__(kThreads, 1)
    tc_wide_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
                   const TcWideArgs a) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    __shared__ uint64_t full_bar[kMaxRing], empty_bar[kMaxRing], done_bar;
    __shared__ uint64_t recv_bar;  // split-K: the peers' partials for this CTA have landed
    __shared__ uint32_t tmem_base_s;
    __shared__ int failed_s;

    const int tid = threadIdx.x, warp = tid >> 5;
    const int split = blockIdx.x, tile = blockIdx.y, M = a.M, lo = a.lo;
    const int kstage = stage_bytes(lo), tcols = tmem_cols(lo);
    const uint32_t lo_bytes = static_cast<uint32_t>(lo) * kKChunk * 2;  // offset of the lo rows in a B tile
    // 1 KiB aligned, derived from smem_raw by pointer arithmetic so that the
    // compiler keeps shared-memory addressing for everything carved from it
    uint8_t* smem = smem_raw + ((1024u - (smem_addr(smem_raw) & 1023u)) & 1023u);
    const int nch = a.K / kKChunk;
    const int c0 = split * nch / S, c1 = (split + 1) * nch / S, cs = c1 - c0;
    const int stages = min(a.stages, max(cs, 1));
    // the receive buffer offset is the same in every CTA of the cluster
    const int stage_area = min(a.stages, max((nch + S - 1) / S, 1));
    const int r0 = a.gateup ? tile * 64 : tile * kTileRows;
    const int r1 = a.gateup ? a.rows + tile * 64 : tile * kTileRows + 64;
    const int pre = min(stages, cs);
    int issued[kMaxRing];

    if (tid == 0) {
        for (int i = 0; i < stages; ++i) {
            mbar_init(&full_bar[i], 1);
            mbar_init(&empty_bar[i], 1);
        }
        mbar_init(&done_bar, 1);
        if (S > 1) mbar_init(&recv_bar, 1);
        failed_s = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        // the peers' partials: kThreads / S accumulator rows from each of the S - 1 peers,
        // ceil(M / 4) 16-byte stores each
        if (S > 1) mbar_expect_tx(&recv_bar, (S - 1) * (kThreads / S) * 16 * ((M + 3) / 4));
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&map_a)) : "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&map_b)) : "memory");
#pragma unroll
        for (int i = 0; i < kMaxRing; ++i) issued[i] = 0;
        // weights first: they depend on no earlier kernel
        for (int i = 0; i < pre; ++i) {
            uint8_t* st = smem + i * kstage;
            mbar_expect_tx(&full_bar[i], kstage);
            tma_load_2d(st, &map_a, (c0 + i) * kKChunk, r0, &full_bar[i]);
            tma_load_2d(st + kABytes / 2, &map_a, (c0 + i) * kKChunk, r1, &full_bar[i]);
            issued[i] = 1;
        }
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                         smem_addr(&tmem_base_s)), "r"(tcols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = tmem_base_s;
    // split-K: this CTA's receive barrier is set up (thread 0's init and expect_tx, ordered by
    // the block barrier above); the matching wait comes right before the first push
    if (S > 1) asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
    pdl_launch_dependents();

    if (tid == 0) {
        pdl_wait();
        for (int i = 0; i < pre; ++i) {
            uint8_t* sb = smem + i * kstage + kABytes;
            tma_load_2d(sb, &map_b, (c0 + i) * kKChunk, 0, &full_bar[i]);
            tma_load_2d(sb + lo_bytes, &map_b, (c0 + i) * kKChunk, lo, &full_bar[i]);
        }
        for (int i = pre; i < cs; ++i) {
            const int s = i % stages;
            if (!mbar_wait(&empty_bar[s], ((i / stages) - 1) & 1)) {
                failed_s = 1;
                break;
            }
            uint8_t* st = smem + s * kstage;
            mbar_expect_tx(&full_bar[s], kstage);
            tma_load_2d(st, &map_a, (c0 + i) * kKChunk, r0, &full_bar[s]);
            tma_load_2d(st + kABytes / 2, &map_a, (c0 + i) * kKChunk, r1, &full_bar[s]);
            tma_load_2d(st + kABytes, &map_b, (c0 + i) * kKChunk, 0, &full_bar[s]);
            tma_load_2d(st + kABytes + lo_bytes, &map_b, (c0 + i) * kKChunk, lo, &full_bar[s]);
            issued[s] += 1;
        }
    } else if (tid == 32) {
        pdl_wait();
        const uint32_t idesc = umma_idesc(kTileRows, lo);
        for (int i = 0; i < cs; ++i) {
            const int s = i % stages;
            if (!mbar_wait(&full_bar[s], (i / stages) & 1)) {
                failed_s = 1;
                break;
            }
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            const uint32_t sa = smem_addr(smem + s * kstage), sb = sa + kABytes;
#pragma unroll
            for (int kk = 0; kk < kKChunk / 16; ++kk) {
                umma_f16(tmem, umma_desc(sa + kk * 32), umma_desc(sb + kk * 32), idesc, (i | kk) != 0);
                umma_f16(tmem, umma_desc(sa + kk * 32), umma_desc(sb + lo_bytes + kk * 32), idesc, 1);
            }
            umma_commit(&empty_bar[s]);
        }
        umma_commit(&done_bar);
    } else {
        pdl_wait();
    }

    // output features of the tile: 128 (or 64 gate + 64 up); CTA p of the
    // cluster owns features [p nu, (p + 1) nu) of each half. After the exchange, thread ->
    // (feature lu, token chunks q0, q0 + per, ... of four rows each).
    const int units = a.gateup ? 64 : kTileRows, halves = a.gateup ? 2 : 1;
    const int nu = units / S;
    const int per = kThreads / nu, lu = tid % nu, q0 = tid / nu;
    const int col = split * nu + lu;
    const int nq = (M + 3) / 4;
    // A residual launch split 4 or 8 ways reads this thread's residual rows now, in one
    // batch, instead of after the exchange (at most 11 chunks of four rows per thread).
    constexpr int kPreQ = S >= 4 ? (kWideTokens / 4 + S - 1) / S : 1;
    float rpre[kPreQ][4];
    if constexpr (S >= 4) {
        if (!a.gateup && a.resid) {
            const float* yc = a.y + tile * kTileRows + col;
#pragma unroll
            for (int jj = 0; jj < kPreQ; ++jj)
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const int m = 4 * (q0 + jj * per) + i;
                    rpre[jj][i] = m < M ? yc[static_cast<size_t>(m) * a.ldy] : 0.f;
                }
        }
    }

    const bool ok = mbar_wait(&done_bar, 0);
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    if (!ok) failed_s = 1;
    // tcgen05.ld is warp-collective: read the accumulator only if the whole warp saw it complete
    const bool wok = __all_sync(0xffffffffu, ok);
    // split launches may receive in the stage area too, once every CTA of the cluster is done with its own
    const bool shared_recv = S > 1 && a.recv_shared && static_cast<size_t>(stage_area) * kstage >= recv_bytes(lo);
    const bool local_recv = recv_in_stages(S, stages, lo) || shared_recv;
    if (tid == 0) {
        // no copy may still be landing in this CTA's shared memory (bounded when something failed)
        for (int i = 0; i < stages; ++i)
            if (issued[i] > 0 && !mbar_wait(&full_bar[i], (issued[i] - 1) & 1)) failed_s = 1;
    }
    __syncthreads();
    // this thread's accumulator row (output feature tid), token columns mb .. mb + 31
    const uint32_t lanes = tmem + (static_cast<uint32_t>(warp * 32) << 16);
    auto acc32 = [&](int mb, float* v) {
        if (wok) {
            tmem_ld16(lanes + mb, v);
            if (mb + 16 < M) tmem_ld16(lanes + mb + 16, v + 16);
            asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
        } else {
#pragma unroll
            for (int i = 0; i < 32; ++i) v[i] = 0.f;
        }
    };
    if (S == 1 && !a.gateup) {
        // no split, one feature per thread: straight from TMEM, coalesced across
        // the warp (consecutive features of one token row)
        float* yc = a.y + tile * kTileRows + tid;
        for (int mb = 0; mb < M; mb += 32) {
            float v[32];
            acc32(mb, v);
#pragma unroll
            for (int h = 0; h < 32; h += 16) {
                float r[16];
#pragma unroll
                for (int j = 0; j < 16; ++j) {
                    const int m = mb + h + j;
                    r[j] = (a.resid && m < M) ? yc[static_cast<size_t>(m) * a.ldy] : 0.f;
                }
#pragma unroll
                for (int j = 0; j < 16; ++j) {
                    const int m = mb + h + j;
                    if (m < M)
                        yc[static_cast<size_t>(m) * a.ldy] =
                            a.resid ? r[j] + (a.rscale == 1.f ? v[h + j] : v[h + j] * a.rscale) : v[h + j];
                }
            }
        }
    } else {
        // partials, one contiguous token run per (split, half, unit):
        // recv[((p * halves + half) * nu + lu) * rs + m], rs = lo + 4. Pushes are 16-byte
        // stores, and the owner reads four token rows per 16-byte load (row stride of 4
        // banks modulo 32: each quarter-warp phase touches all 32 banks once).
        const int rs = recv_stride(lo);
        float* recv = reinterpret_cast<float*>(local_recv ? smem : smem + static_cast<size_t>(stage_area) * kstage);
        if (S > 1) cluster_wait();           // every peer's receive barrier is set up
        if (shared_recv) cluster_barrier();  // every CTA's loads have landed: the stage areas are free
        {
            const int u = a.gateup ? (tid & 63) : tid, half = a.gateup ? (tid >> 6) : 0;
            const int owner = u / nu, ou = u - owner * nu;
            float* dst = recv + static_cast<size_t>((split * halves + half) * nu + ou) * rs;
            const uint32_t remote = owner == split ? 0u : peer_addr(dst, static_cast<uint32_t>(owner));
            const uint32_t rbar = owner == split ? 0u : peer_addr(&recv_bar, static_cast<uint32_t>(owner));
            for (int mb = 0; mb < M; mb += 32) {
                float v[32];
                acc32(mb, v);
#pragma unroll
                for (int c = 0; c < 8; ++c) {
                    if (mb + 4 * c >= M) break;
                    if (owner == split)
                        *reinterpret_cast<float4*>(dst + mb + 4 * c) =
                            make_float4(v[4 * c], v[4 * c + 1], v[4 * c + 2], v[4 * c + 3]);
                    else
                        st_async4(remote + 4u * static_cast<uint32_t>(mb + 4 * c), v[4 * c], v[4 * c + 1],
                                  v[4 * c + 2], v[4 * c + 3], rbar);
                }
            }
        }
        asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
        __syncthreads();  // this CTA's own partials are in place
        // the peers' partials: every byte counted on the receive barrier; after the wait no peer
        // writes into this CTA's shared memory again, so it may exit without a cluster barrier
        if (S > 1 && !mbar_wait_cluster(&recv_bar, 0)) failed_s = 1;
        // this CTA's features; each batch issues all its loads (partials and residual rows) first
        if (a.gateup) {
            constexpr int kBatch = S >= 4 ? 1 : 4 / S;
            const size_t ocol = static_cast<size_t>(tile) * 64 + col;
            for (int qb = q0; qb < nq; qb += per * kBatch) {
                float4 g[kBatch][S], up[kBatch][S];
#pragma unroll
                for (int j = 0; j < kBatch; ++j) {
                    const int q = min(qb + j * per, nq - 1);
#pragma unroll
                    for (int p = 0; p < S; ++p) {
                        g[j][p] = *reinterpret_cast<const float4*>(recv + static_cast<size_t>((p * 2 + 0) * nu + lu) * rs + 4 * q);
                        up[j][p] = *reinterpret_cast<const float4*>(recv + static_cast<size_t>((p * 2 + 1) * nu + lu) * rs + 4 * q);
                    }
                }
#pragma unroll
                for (int j = 0; j < kBatch; ++j) {
                    const int q = qb + j * per;
                    if (q >= nq) break;
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        const int m = 4 * q + i;
                        if (m >= M) break;
                        float gs = 0.f, us = 0.f;
#pragma unroll
                        for (int p = 0; p < S; ++p) {
                            gs += reinterpret_cast<const float*>(&g[j][p])[i];
                            us += reinterpret_cast<const float*>(&up[j][p])[i];
                        }
                        const float o = silu(gs) * us;
                        const __half h = __float2half_rn(o);
                        a.yb[static_cast<size_t>(m) * a.ldyb + ocol] = h;
                        a.yb[static_cast<size_t>(lo + m) * a.ldyb + ocol] = __float2half_rn(o - __half2float(h));
                    }
                }
            }
        } else if constexpr (S >= 4) {
            // residual rows already in registers: partials summed straight from shared memory
            float* yc = a.y + tile * kTileRows + col;
#pragma unroll
            for (int jj = 0; jj < kPreQ; ++jj) {
                const int q = q0 + jj * per;
                if (q >= nq) break;
                float4 sum4 = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
                for (int p = 0; p < S; ++p) {
                    const float4 v = *reinterpret_cast<const float4*>(recv + static_cast<size_t>(p * nu + lu) * rs + 4 * q);
                    sum4.x += v.x;
                    sum4.y += v.y;
                    sum4.z += v.z;
                    sum4.w += v.w;
                }
                const float sm[4] = {sum4.x, sum4.y, sum4.z, sum4.w};
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const int m = 4 * q + i;
                    if (m >= M) break;
                    yc[static_cast<size_t>(m) * a.ldy] =
                        a.resid ? rpre[jj][i] + (a.rscale == 1.f ? sm[i] : sm[i] * a.rscale) : sm[i];
                }
            }
        } else {
            constexpr int kBatch = 4;
            float* yc = a.y + tile * kTileRows + col;
            for (int qb = q0; qb < nq; qb += per * kBatch) {
                float4 part[kBatch][S];
                float r[kBatch][4];
#pragma unroll
                for (int j = 0; j < kBatch; ++j) {
                    const int q = qb + j * per, qc = min(q, nq - 1);
#pragma unroll
                    for (int p = 0; p < S; ++p)
                        part[j][p] = *reinterpret_cast<const float4*>(recv + static_cast<size_t>(p * nu + lu) * rs + 4 * qc);
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        const int m = 4 * q + i;
                        r[j][i] = (a.resid && q < nq && m < M) ? yc[static_cast<size_t>(m) * a.ldy] : 0.f;
                    }
                }
#pragma unroll
                for (int j = 0; j < kBatch; ++j) {
                    const int q = qb + j * per;
                    if (q >= nq) break;
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        const int m = 4 * q + i;
                        if (m >= M) break;
                        float sum = 0.f;
#pragma unroll
                        for (int p = 0; p < S; ++p) sum += reinterpret_cast<const float*>(&part[j][p])[i];
                        yc[static_cast<size_t>(m) * a.ldy] =
                            a.resid ? r[j][i] + (a.rscale == 1.f ? sum : sum * a.rscale) : sum;
                    }
                }
            }
        }
    }
    __syncthreads();
    if (tid == 0 && failed_s && a.ctl) a.ctl->error = 3;
    if (warp == 1)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(tcols) : "memory");
}

}  // namespace
}  // namespace vxc

namespace vxc {
namespace {

// The launch's ring depth, receive placement and dynamic shared memory: the
// deepest ring (up to a.stages) whose layout fits; a split launch whose separate
// receive buffer would not fit beside its ring receives in the stage area.
struct WidePlan {
    int stages = 1;
    int recv_shared = 0;
    size_t bytes = 0;
};

WidePlan plan_smem(const TcWideArgs& a) {
    const int nch = a.K / kKChunk, S = a.splits, lo = a.lo;
    const size_t kstage = static_cast<size_t>(stage_bytes(lo)), recv = recv_bytes(lo);
    const bool needs_recv = S > 1 || a.gateup;  // an unsplit plain / residual launch writes from TMEM
    for (int st = a.stages; st >= 1; --st) {
        const size_t area = static_cast<size_t>(std::min(st, std::max((nch + S - 1) / S, 1))) * kstage;
        int rs = a.recv_shared;
        if (S > 1 && !rs && area + recv + 1024 > kSmemMax && area >= recv) rs = 1;
        const bool in_stages = (S == 1 && area >= recv) || (S > 1 && rs && area >= recv);
        const size_t bytes = area + 1024 + ((needs_recv && !in_stages) ? recv : 0);
        if (bytes <= kSmemMax) {
            WidePlan p;
            p.stages = st;
            p.recv_shared = rs;
            p.bytes = std::max({bytes, kFloor, tmem_smem_floor(tmem_cols(lo))});
            return p;
        }
    }
    throw std::invalid_argument("tc_wide: the token block does not fit in shared memory");
}

}  // namespace

void launch_tc_wide(const CUtensorMap& map_a, const CUtensorMap& map_b, const TcWideArgs& args, cudaStream_t s,
                    bool pdl) {
    if (args.K % kKChunk != 0 || args.K <= 0) throw std::invalid_argument("tc_wide: K must be a multiple of 64");
    if (args.lo < 16 || args.lo > kWideTokens || args.lo % 16 != 0)
        throw std::invalid_argument("tc_wide: the row block must be a multiple of 16 in [16, 176]");
    if (args.M <= 0 || args.M > args.lo) throw std::invalid_argument("tc_wide: 1 to lo token rows");
    if ((args.splits != 1 && args.splits != 2 && args.splits != 4 && args.splits != 8) ||
        args.splits > args.K / kKChunk)
        throw std::invalid_argument("tc_wide: splits must be 1, 2, 4 or 8 and at most K / 64");
    if (args.stages < 1 || args.stages > kMaxRing) throw std::invalid_argument("tc_wide: stages in [1, 4]");
    if ((args.gateup ? args.rows % 64 : args.rows % kTileRows) != 0) throw std::invalid_argument("tc_wide: rows");
    const WidePlan p = plan_smem(args);
    TcWideArgs a = args;
    a.stages = p.stages;
    a.recv_shared = p.recv_shared;
    const int n_tiles = a.gateup ? a.rows / 64 : a.rows / kTileRows;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(a.splits, n_tiles);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = p.bytes;
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
    switch (a.splits) {
        case 1: check_launch(cudaLaunchKernelEx(&cfg, tc_wide_kernel<1>, map_a, map_b, a)); break;
        case 2: check_launch(cudaLaunchKernelEx(&cfg, tc_wide_kernel<2>, map_a, map_b, a)); break;
        case 4: check_launch(cudaLaunchKernelEx(&cfg, tc_wide_kernel<4>, map_a, map_b, a)); break;
        default: check_launch(cudaLaunchKernelEx(&cfg, tc_wide_kernel<8>, map_a, map_b, a)); break;
    }
}

void init_tc_wide_attributes() {
    for (const void* f : {reinterpret_cast<const void*>(tc_wide_kernel<1>), reinterpret_cast<const void*>(tc_wide_kernel<2>),
                          reinterpret_cast<const void*>(tc_wide_kernel<4>), reinterpret_cast<const void*>(tc_wide_kernel<8>)})
        check_launch(cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(kSmemMax)));
}

}  // namespace vxc
