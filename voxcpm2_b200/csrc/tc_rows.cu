// tcgen05 linear over a block of up to 128 token rows, for the decoders' prefill
// (Synthesizer::Impl::generate prefix pass, synthesizer.cpp:403-535, through
// DecoderKv.forward, tools/export_components.py:496-550).
//
// Y[m][r] = sum_k X[m][k] W[r][k] for m < M <= 128 rows. Weights are the MMA A
// operand (128 output features per tile, K-major, 128-byte swizzle, TMA); the
// rows are the B operand, N = 256: fp16(x) in rows 0..127 and fp16(x - fp16(x))
// in rows 128..255 (fp32-level accuracy, as in the patch loop's linears). A CTA
// streams its share of K for one output tile through a ring of shared-memory
// stages; the fp32 accumulator is 256 TMEM columns. Without a K split the epilogue
// writes the outputs directly: plain, residual (y += rscale * v) or SiLU(gate) * up
// as the next linear's split operand. The narrow linears (q/k/v, o, down: 8-10
// tiles) split K over up to 8 CTAs per tile: each writes its fp32 partial tile to a
// scratch buffer, and rows_reduce_kernel sums the partials in order and applies the
// same epilogue. Roles: thread 0 issues TMA, thread 32 the MMAs,
// all four warps drain TMEM (warp w owns tile rows 32w .. 32w + 31). Every wait is
// bounded; on timeout the kernel records error 3 and still frees its TMEM.
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
constexpr int kRowsN = 2 * kRowBlock;              // MMA N: hi rows then lo rows
constexpr int kBTile = kRowsN * kKChunk * 2;       // 32 KiB
constexpr int kStage = kABytes + kBTile;           // 48 KiB (1 KiB aligned)
constexpr int kMaxRing = 4;
constexpr int kTmem = 256;

void check_launch(cudaError_t e) {
    if (e != cudaSuccess) throw std::runtime_error(std::string("tc_rows: ") + cudaGetErrorString(e));
}

__global__ void __launch_bounds__(kThreads, 1)
    tc_rows_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
                   const TcRowsArgs a) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    __shared__ uint64_t full_bar[kMaxRing], empty_bar[kMaxRing], done_bar;
    __shared__ uint32_t tmem_base_s;
    __shared__ int failed_s;
    __shared__ float up_s[64][17];  // gate/up epilogue: the up rows of one 16-column block

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int tile = blockIdx.x, split = blockIdx.y, S = gridDim.y;
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int nk = a.K / kKChunk;
    const int k0 = split * nk / S, nch = (split + 1) * nk / S - k0;  // this CTA's K chunks
    const int stages = min(a.stages, nch);
    const int r0 = a.gateup ? tile * 64 : tile * kTileRows;
    const int r1 = a.gateup ? a.rows + tile * 64 : tile * kTileRows + 64;
    int issued[kMaxRing];

    if (tid == 0) {
        for (int i = 0; i < stages; ++i) {
            mbar_init(&full_bar[i], 1);
            mbar_init(&empty_bar[i], 1);
        }
        mbar_init(&done_bar, 1);
        failed_s = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
#pragma unroll
        for (int i = 0; i < kMaxRing; ++i) issued[i] = 0;
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                         smem_addr(&tmem_base_s)), "r"(kTmem)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = tmem_base_s;

    if (tid == 0) {
        for (int i = 0; i < nch; ++i) {
            const int s = i % stages;
            if (i >= stages && !mbar_wait(&empty_bar[s], ((i / stages) - 1) & 1)) {
                failed_s = 1;
                break;
            }
            uint8_t* st = smem + s * kStage;
            mbar_expect_tx(&full_bar[s], kStage);
            tma_load_2d(st, &map_a, (k0 + i) * kKChunk, r0, &full_bar[s]);
            tma_load_2d(st + kABytes / 2, &map_a, (k0 + i) * kKChunk, r1, &full_bar[s]);
            tma_load_2d(st + kABytes, &map_b, (k0 + i) * kKChunk, 0, &full_bar[s]);
            issued[s] += 1;
        }
    } else if (tid == 32) {
        const uint32_t idesc = umma_idesc(kTileRows, kRowsN);
        for (int i = 0; i < nch; ++i) {
            const int s = i % stages;
            if (!mbar_wait(&full_bar[s], (i / stages) & 1)) {
                failed_s = 1;
                break;
            }
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            const uint32_t sa = smem_addr(smem + s * kStage), sb = sa + kABytes;
#pragma unroll
            for (int kk = 0; kk < kKChunk / 16; ++kk)
                umma_f16(tmem, umma_desc(sa + kk * 32), umma_desc(sb + kk * 32), idesc, (i | kk) != 0);
            umma_commit(&empty_bar[s]);
        }
        umma_commit(&done_bar);
    }

    const bool ok = mbar_wait(&done_bar, 0);
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    if (!ok) failed_s = 1;
    const int row = warp * 32 + lane;
    const uint32_t lane_base = tmem + (static_cast<uint32_t>(warp * 32) << 16);
    for (int c0 = 0; c0 < a.M; c0 += 16) {
        float hi[16], lo[16], v[16];
        if (ok) {
            tmem_ld16(lane_base + c0, hi);
            tmem_ld16(lane_base + kRowBlock + c0, lo);
            asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
        } else {
#pragma unroll
            for (int j = 0; j < 16; ++j) hi[j] = lo[j] = 0.f;
        }
#pragma unroll
        for (int j = 0; j < 16; ++j) v[j] = hi[j] + lo[j];
        if (a.part) {
            // this split's partial of feature f (gate/up: the gate features, then the up ones)
            const int prow = a.gateup ? 2 * a.rows : a.rows;
            const int f = a.gateup ? (row < 64 ? tile * 64 + row : a.rows + tile * 64 + row - 64) : tile * kTileRows + row;
            float* pp = a.part + static_cast<size_t>(split) * a.M * prow + f;
#pragma unroll
            for (int j = 0; j < 16; ++j) {
                const int m = c0 + j;
                if (m < a.M) pp[static_cast<size_t>(m) * prow] = v[j];
            }
        } else if (a.gateup) {
            if (row >= 64)
#pragma unroll
                for (int j = 0; j < 16; ++j) up_s[row - 64][j] = v[j];
            __syncthreads();
            if (row < 64)
#pragma unroll
                for (int j = 0; j < 16; ++j) {
                    const int m = c0 + j;
                    if (m < a.M) {
                        const float o = silu(v[j]) * up_s[row][j];
                        const __half h = __float2half_rn(o);
                        const size_t col = static_cast<size_t>(tile) * 64 + row;
                        a.yb[static_cast<size_t>(m) * a.ldyb + col] = h;
                        a.yb[static_cast<size_t>(kRowBlock + m) * a.ldyb + col] = __float2half_rn(o - __half2float(h));
                    }
                }
            __syncthreads();
        } else {
#pragma unroll
            for (int j = 0; j < 16; ++j) {
                const int m = c0 + j;
                if (m < a.M) {
                    float* y = a.y + static_cast<size_t>(m) * a.ldy + tile * kTileRows + row;
                    *y = a.resid ? *y + (a.rscale == 1.f ? v[j] : v[j] * a.rscale) : v[j];
                }
            }
        }
    }
    if (tid == 0) {
        // no copy may still be landing in this CTA's shared memory when it exits
        for (int i = 0; i < stages; ++i)
            if (issued[i] > 0 && !mbar_wait(&full_bar[i], (issued[i] - 1) & 1)) failed_s = 1;
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (tid == 0 && failed_s && a.ctl) a.ctl->error = 3;
    if (warp == 1)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmem) : "memory");
}

size_t smem_bytes(int stages) { return static_cast<size_t>(stages) * kStage + 1024; }

// The split launches' second step: thread -> four consecutive features of token row
// blockIdx.y; the partials are summed in split order, then the epilogue of the
// unsplit kernel (plain, residual, or SiLU(gate) * up as the next split operand).
constexpr int kReduceThreads = 256;
__global__ void __launch_bounds__(kReduceThreads) rows_reduce_kernel(const TcRowsArgs a) {
    const int m = blockIdx.y, f4 = blockIdx.x * kReduceThreads + threadIdx.x;
    if (f4 >= a.rows / 4) return;
    const int prow = a.gateup ? 2 * a.rows : a.rows;
    const float* p0 = a.part + static_cast<size_t>(m) * prow + 4 * f4;
    const size_t pstride = static_cast<size_t>(a.M) * prow;
    float4 g[8], u[8];
#pragma unroll
    for (int p = 0; p < 8; ++p) {
        if (p < a.splits) {
            g[p] = *reinterpret_cast<const float4*>(p0 + p * pstride);
            if (a.gateup) u[p] = *reinterpret_cast<const float4*>(p0 + p * pstride + a.rows);
        }
    }
    float gs[4] = {0.f, 0.f, 0.f, 0.f}, us[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int p = 0; p < 8; ++p) {
        if (p < a.splits) {
            gs[0] += g[p].x; gs[1] += g[p].y; gs[2] += g[p].z; gs[3] += g[p].w;
            if (a.gateup) { us[0] += u[p].x; us[1] += u[p].y; us[2] += u[p].z; us[3] += u[p].w; }
        }
    }
    const int f = 4 * f4;
    if (a.gateup) {
        float o[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) o[i] = silu(gs[i]) * us[i];
        const __half2 h01 = __floats2half2_rn(o[0], o[1]), h23 = __floats2half2_rn(o[2], o[3]);
        const float2 f01 = __half22float2(h01), f23 = __half22float2(h23);
        __half* hi = a.yb + static_cast<size_t>(m) * a.ldyb + f;
        __half* lo = a.yb + static_cast<size_t>(kRowBlock + m) * a.ldyb + f;
        reinterpret_cast<__half2*>(hi)[0] = h01;
        reinterpret_cast<__half2*>(hi)[1] = h23;
        reinterpret_cast<__half2*>(lo)[0] = __floats2half2_rn(o[0] - f01.x, o[1] - f01.y);
        reinterpret_cast<__half2*>(lo)[1] = __floats2half2_rn(o[2] - f23.x, o[3] - f23.y);
    } else {
        float4* y = reinterpret_cast<float4*>(a.y + static_cast<size_t>(m) * a.ldy + f);
        float4 v = make_float4(gs[0], gs[1], gs[2], gs[3]);
        if (a.resid) {
            const float4 r = *y;
            if (a.rscale == 1.f) v = make_float4(r.x + v.x, r.y + v.y, r.z + v.z, r.w + v.w);
            else v = make_float4(r.x + v.x * a.rscale, r.y + v.y * a.rscale, r.z + v.z * a.rscale, r.w + v.w * a.rscale);
        }
        *y = v;
    }
}

}  // namespace

int tc_rows_splits(int rows, int gateup, int K) {
    const int n_tiles = gateup ? rows / 64 : rows / kTileRows;
    const int want = std::max(1, std::min({8, K / kKChunk, 128 / std::max(1, n_tiles)}));
    return want >= 8 ? 8 : want >= 4 ? 4 : want >= 2 ? 2 : 1;
}

void launch_tc_rows(const CUtensorMap& map_a, const CUtensorMap& map_b, const TcRowsArgs& a, cudaStream_t s) {
    if (a.K % kKChunk != 0 || a.K <= 0) throw std::invalid_argument("tc_rows: K must be a multiple of 64");
    if (a.M <= 0 || a.M > kRowBlock) throw std::invalid_argument("tc_rows: 1..128 token rows per launch");
    if (a.stages < 1 || a.stages > kMaxRing) throw std::invalid_argument("tc_rows: stages in [1, 4]");
    if ((a.gateup ? a.rows % 64 : a.rows % kTileRows) != 0) throw std::invalid_argument("tc_rows: rows");
    if (a.splits < 1 || a.splits > 8 || a.splits > a.K / kKChunk) throw std::invalid_argument("tc_rows: splits in [1, 8]");
    if (a.splits > 1 && (!a.part || (reinterpret_cast<uintptr_t>(a.part) & 15) != 0 || a.rows % 4 != 0 ||
                         (!a.gateup && (a.ldy % 4 != 0 || (reinterpret_cast<uintptr_t>(a.y) & 15) != 0))))
        throw std::invalid_argument("tc_rows: a split launch needs a 16-byte aligned partial buffer and outputs");
    const int n_tiles = a.gateup ? a.rows / 64 : a.rows / kTileRows;
    const int nk = a.K / kKChunk;
    const int stages = std::min(a.stages, (nk + a.splits - 1) / a.splits);
    TcRowsArgs k = a;
    if (a.splits == 1) k.part = nullptr;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(n_tiles, a.splits);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = std::max(smem_bytes(stages), tmem_smem_floor(kTmem));
    cfg.stream = s;
    check_launch(cudaLaunchKernelEx(&cfg, tc_rows_kernel, map_a, map_b, k));
    if (a.splits > 1) {
        cudaLaunchConfig_t rc = {};
        rc.gridDim = dim3((a.rows / 4 + kReduceThreads - 1) / kReduceThreads, a.M);
        rc.blockDim = dim3(kReduceThreads);
        rc.stream = s;
        check_launch(cudaLaunchKernelEx(&rc, rows_reduce_kernel, k));
    }
}

void init_tc_rows_attributes() {
    check_launch(cudaFuncSetAttribute(tc_rows_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      static_cast<int>(smem_bytes(kMaxRing))));
}

}  // namespace vxc
