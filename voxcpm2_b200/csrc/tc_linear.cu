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
#include <stdexcept>

#include "kernels.cuh"

namespace vxc {
namespace {

constexpr int kTcThreads = 128;
constexpr int kTileRows = 128;      // MMA M (output features per tile)
constexpr int kKChunk = 64;         // fp16 elements per 128-byte swizzle row
constexpr int kBRows = 48;          // MMA N (hi tokens 0..23, lo tokens 24..47)
constexpr int kLoOffset = 24;
constexpr int kABytes = kTileRows * kKChunk * 2;  // 16 KiB
constexpr int kBBytes = kBRows * kKChunk * 2;     // 6 KiB
constexpr int kStageBytes = kABytes + kBBytes;    // 22 KiB, keeps 1 KiB alignment
constexpr int kMaxStages = 8;
constexpr int kRowFloats = 25;      // exchange-buffer row stride: 24 tokens + 1 (odd: conflict-free reads)
constexpr int kTmemCols = 64;
constexpr uint32_t kWaitLimit = 1u << 22;

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes)
                 : "memory");
}

// Bounded wait for phase 'parity' of an mbarrier; false on timeout.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
    const uint32_t addr = smem_addr(bar);
    for (uint32_t i = 0; i < kWaitLimit; ++i) {
        uint32_t done;
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
            "selp.u32 %0, 1, 0, p;\n\t}"
            : "=r"(done)
            : "r"(addr), "r"(parity)
            : "memory");
        if (done) return true;
    }
    return false;
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
        ::"r"(smem_addr(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_addr(bar))
        : "memory");
}

// K-major, 128-byte-swizzle UMMA shared-memory descriptor: start address >> 4,
// leading offset 1 (unused for swizzled K-major), stride offset 1024 B between
// 8-row groups, descriptor version 1, layout type 2 (SWIZZLE_128B).
__device__ __forceinline__ uint64_t umma_desc(uint32_t saddr) {
    return static_cast<uint64_t>((saddr >> 4) & 0x3FFFu) | (1ull << 16) | (64ull << 32) | (1ull << 46) |
           (2ull << 61);
}

// kind::f16 instruction descriptor: fp32 accumulate, fp16 A and B, both K-major.
__host__ __device__ constexpr uint32_t umma_idesc(int m, int n) {
    return (1u << 4) | (static_cast<uint32_t>(n >> 3) << 17) | (static_cast<uint32_t>(m >> 4) << 24);
}

__device__ __forceinline__ void umma_f16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                         uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
        ::"r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

__device__ __forceinline__ void umma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     smem_addr(bar))
                 : "memory");
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float* v) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void cluster_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// Address of 'local' in the shared memory of cluster CTA 'rank'.
__device__ __forceinline__ uint32_t peer_addr(const void* local, uint32_t rank) {
    uint32_t remote;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(smem_addr(local)), "r"(rank));
    return remote;
}
__device__ __forceinline__ void st_peer(uint32_t remote, float v) {  // fire and forget
    asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(remote), "f"(v) : "memory");
}

__device__ __forceinline__ void store_split(__half* yb, int ld, int m, int col, float v) {
    const __half hi = __float2half_rn(v);
    yb[static_cast<size_t>(m) * ld + col] = hi;
    yb[static_cast<size_t>(kLoOffset + m) * ld + col] = __float2half_rn(v - __half2float(hi));
}

__global__ void __launch_bounds__(kTcThreads, 1)
    tc_linear_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
                     const TcLinearArgs a) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    __shared__ uint64_t full_bar[kMaxStages], empty_bar[kMaxStages], done_bar;
    __shared__ uint32_t tmem_base_s;
    __shared__ int failed_s;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int split = blockIdx.x, tile = blockIdx.y;
    const int S = a.splits;
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));

    const int nch = a.K / kKChunk;
    const int c0 = split * nch / S, c1 = (split + 1) * nch / S, cs = c1 - c0;
    const int stages = min(kMaxStages, max(cs, 1));
    // the receive buffer sits after the stage area of the largest split: the same
    // offset in every CTA of the cluster, whatever its own chunk count
    const int stage_area = min(kMaxStages, max((nch + S - 1) / S, 1));

    // thread 0: barriers, then the weight loads at once (they depend on no earlier
    // kernel); warp 1 meanwhile allocates the TMEM accumulator
    const int r0 = a.gateup ? tile * 64 : tile * kTileRows;   // rows of W in this tile: two
    const int r1 = a.gateup ? a.rows + tile * 64 : tile * kTileRows + 64;  // 64-row boxes
    const int pre = min(stages, cs);
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
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&map_b)) : "memory");
#pragma unroll
        for (int i = 0; i < kMaxStages; ++i) issued[i] = 0;
        for (int i = 0; i < pre; ++i) {
            uint8_t* st = smem + i * kStageBytes;
            mbar_expect_tx(&full_bar[i], kStageBytes);
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
    } else {
        pdl_wait();
    }

    // drain the accumulator: warp w owns TMEM lanes (tile rows) 32w .. 32w + 31
    const bool ok = mbar_wait(&done_bar, 0);
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    if (!ok) failed_s = 1;
    // Split-K exchange by push: each CTA stores its partial rows straight into the
    // receive buffer of the CTA that owns them (non-blocking remote stores), one
    // cluster barrier, then owners sum the splits in rank order (deterministic).
    // Owner slices: tile units (rows, or gate/up pairs) [o * units / S, (o+1) * units / S).
    const int units = a.gateup ? 64 : kTileRows;
    const int slice = (units + S - 1) / S;
    const int halves = a.gateup ? 2 : 1;
    float* recv = reinterpret_cast<float*>(smem + static_cast<size_t>(stage_area) * kStageBytes);
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
        const int row = warp * 32 + lane;
        const int u = a.gateup ? (row & 63) : row, half = a.gateup ? (row >> 6) : 0;
        int owner = 0;
        while (owner + 1 < S && u >= (owner + 1) * units / S) ++owner;
        const int lu = u - owner * units / S;
        float* dst = recv + ((split * slice + lu) * halves + half) * kRowFloats;
        if (S == 1) {
#pragma unroll
            for (int m = 0; m < kLoOffset; ++m)
                if (m < a.M) dst[m] = d[m] + d[kLoOffset + m];
        } else {
            const uint32_t remote = peer_addr(dst, owner);
#pragma unroll
            for (int m = 0; m < kLoOffset; ++m)
                if (m < a.M) st_peer(remote + 4 * m, d[m] + d[kLoOffset + m]);
        }
    }
    if (tid == 0) {
        // no copy may still be landing in this CTA's shared memory when it moves on
        // (a no-op when every stage was consumed; bounded when something failed)
        for (int i = 0; i < stages; ++i)
            if (issued[i] > 0 && !mbar_wait(&full_bar[i], (issued[i] - 1) & 1)) failed_s = 1;
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    if (S > 1) cluster_sync();  // every partial has landed in its owner's buffer
    else __syncthreads();
    const int u0 = split * units / S, nu = (split + 1) * units / S - u0;
    for (int it = tid; it < nu * a.M; it += kTcThreads) {
        const int m = it / nu, lu = it - m * nu;
        if (a.gateup) {
            float g = 0.f, up = 0.f;
            for (int p = 0; p < S; ++p) {
                g += recv[((p * slice + lu) * 2 + 0) * kRowFloats + m];
                up += recv[((p * slice + lu) * 2 + 1) * kRowFloats + m];
            }
            store_split(a.yb, a.ldyb, m, tile * 64 + u0 + lu, silu(g) * up);
        } else {
            float v = 0.f;
            for (int p = 0; p < S; ++p) v += recv[(p * slice + lu) * kRowFloats + m];
            float* y = a.y + static_cast<size_t>(m) * a.ldy + tile * kTileRows + u0 + lu;
            if (a.resid) *y = *y + (a.rscale == 1.f ? v : v * a.rscale);
            else *y = v;
        }
    }
    __syncthreads();
    if (tid == 0 && failed_s && a.ctl) a.ctl->error = 3;
    if (warp == 1)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_d), "r"(kTmemCols)
                     : "memory");
}

}  // namespace

size_t tc_linear_smem_bytes(int K, int splits) {
    const int nch = K / kKChunk;
    const int cs = (nch + splits - 1) / splits;
    const int stages = std::min(kMaxStages, std::max(cs, 1));
    const size_t stage_bytes = static_cast<size_t>(stages) * kStageBytes;
    // receive buffer: per source split, an owner slice of rows (or of gate/up pairs, 2 rows each)
    const size_t slice_rows = std::max((128 + splits - 1) / splits, 2 * ((64 + splits - 1) / splits));
    const size_t recv_bytes = static_cast<size_t>(splits) * slice_rows * kRowFloats * sizeof(float);
    return stage_bytes + recv_bytes + 1024;  // + alignment slack
}

void launch_tc_linear(const CUtensorMap& map_a, const CUtensorMap& map_b, const TcLinearArgs& a, cudaStream_t s,
                      bool pdl) {
    if (a.K % kKChunk != 0 || a.K <= 0) throw std::invalid_argument("tc_linear: K must be a multiple of 64");
    if (a.M <= 0 || a.M > kLoOffset) throw std::invalid_argument("tc_linear: at most 24 token rows");
    if (a.splits < 1 || a.splits > 8 || a.splits > a.K / kKChunk || a.M > kRowFloats)
        throw std::invalid_argument("tc_linear: splits must be in [1, 8] and at most K / 64");
    const int n_tiles = a.gateup ? a.rows / 64 : a.rows / kTileRows;
    if ((a.gateup ? a.rows % 64 : a.rows % kTileRows) != 0) throw std::invalid_argument("tc_linear: rows");
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(a.splits, n_tiles);
    cfg.blockDim = dim3(kTcThreads);
    cfg.dynamicSmemBytes = tc_linear_smem_bytes(a.K, a.splits);
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
    const cudaError_t e = cudaLaunchKernelEx(&cfg, tc_linear_kernel, map_a, map_b, a);
    if (e != cudaSuccess) throw std::runtime_error(std::string("tc_linear launch: ") + cudaGetErrorString(e));
}

void init_tc_attributes() {
    size_t most = 0;  // the largest launch: 8 stages plus the largest receive buffer over split counts
    for (int sp = 1; sp <= 8; ++sp) most = std::max(most, tc_linear_smem_bytes(64 * 8 * sp, sp));
    const cudaError_t e = cudaFuncSetAttribute(tc_linear_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               static_cast<int>(most));
    if (e != cudaSuccess) throw std::runtime_error(std::string("tc_linear attribute: ") + cudaGetErrorString(e));
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
