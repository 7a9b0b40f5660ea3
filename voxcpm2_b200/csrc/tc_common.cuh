// tcgen05 / TMA / mbarrier primitives shared by the tensor-core kernels.
//
// Operand conventions (both kernels): the weight tile is the MMA A operand
// (M = 128 output features, K-major, 128-byte swizzle, loaded by TMA); the
// token rows are the B operand (N = 48: fp16(x) in rows 0..23 and the residual
// fp16(x - fp16(x)) in rows 24..47, so A * (hi + lo) keeps fp32-level accuracy);
// accumulators are fp32 in TMEM.
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>

#include <cstdint>

#include "common.cuh"

namespace vxc {
namespace tc {

constexpr int kTileRows = 128;      // MMA M (output features per tile)
constexpr int kKChunk = 64;         // fp16 elements per 128-byte swizzle row
constexpr int kBRows = 48;          // MMA N (hi tokens 0..23, lo tokens 24..47)
constexpr int kLoOffset = 24;
constexpr int kABytes = kTileRows * kKChunk * 2;  // 16 KiB
constexpr int kBBytes = kBRows * kKChunk * 2;     // 6 KiB

// TMEM budget. An SM has 512 TMEM columns and 233,472 bytes of shared memory,
// 1 KiB of which every resident CTA reserves. A CTA that allocates 'cols' columns
// asks for at least cols * 456 bytes of shared memory in all (dynamic + static +
// the reserved 1 KiB): then the CTAs that fit on an SM by shared memory, from any
// mix of these kernels and launches, hold at most 512 columns together, so
// tcgen05.alloc never waits for another CTA to free columns (such a wait, with
// CTAs of split-K clusters on both sides, could otherwise close a cycle across SMs).
constexpr size_t kSmBytesPerTmemCol = (233472 + 511) / 512;  // 456
inline size_t tmem_smem_floor(int cols) { return static_cast<size_t>(cols) * kSmBytesPerTmemCol - 1024; }

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

// Time-bounded wait for phase 'parity' of an mbarrier (kWaitNs); false on timeout.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
    return mbar_wait_addr(smem_addr(bar), parity);
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
// Four floats to a 16-byte aligned address in a cluster peer's shared memory, as an
// asynchronous store that completes 16 bytes of transaction count on the peer's
// mbarrier 'remote_bar' (both addresses from peer_addr): the peer learns of the data
// by waiting on its own barrier, with no cluster-wide barrier.
__device__ __forceinline__ void st_async4(uint32_t remote, float a, float b, float c, float d, uint32_t remote_bar) {
    asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.v4.f32 [%0], {%1, %2, %3, %4}, [%5];" ::"r"(
                     remote),
                 "f"(a), "f"(b), "f"(c), "f"(d), "r"(remote_bar)
                 : "memory");
}

// Two floats, the same way (an 8-byte aligned address; 8 bytes of transaction count).
__device__ __forceinline__ void st_async2(uint32_t remote, float a, float b, uint32_t remote_bar) {
    asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.v2.f32 [%0], {%1, %2}, [%3];" ::"r"(remote),
                 "f"(a), "f"(b), "r"(remote_bar)
                 : "memory");
}

// Time-bounded wait (kWaitNs) for phase 'parity' of a local mbarrier whose
// transactions come from other CTAs of the cluster: acquire at cluster scope.
__device__ __forceinline__ bool mbar_wait_cluster(uint64_t* bar, uint32_t parity) {
    const uint32_t addr = smem_addr(bar);
    uint64_t start = 0;
    for (uint32_t i = 0;; ++i) {
        uint32_t done;
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
            "selp.u32 %0, 1, 0, p;\n\t}"
            : "=r"(done)
            : "r"(addr), "r"(parity)
            : "memory");
        if (done) return true;
        const uint64_t now = global_ns();
        if (i == 0) start = now;
        else if (now - start > kWaitNs) return false;
    }
}

// The two halves of a cluster barrier, for a barrier whose wait can come long after
// its arrival (relaxed: orders nothing by itself; see its callers).
__device__ __forceinline__ void cluster_arrive_relaxed() {
    asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() { asm volatile("barrier.cluster.wait.aligned;" ::: "memory"); }

// four floats to a 16-byte aligned address in a cluster peer's shared memory
__device__ __forceinline__ void st_peer4(uint32_t remote, float a, float b, float c, float d) {
    asm volatile("st.shared::cluster.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(remote), "f"(a), "f"(b), "f"(c), "f"(d)
                 : "memory");
}

__device__ __forceinline__ void store_split(__half* yb, int ld, int m, int col, float v) {
    const __half hi = __float2half_rn(v);
    yb[static_cast<size_t>(m) * ld + col] = hi;
    yb[static_cast<size_t>(kLoOffset + m) * ld + col] = __float2half_rn(v - __half2float(hi));
}

// Byte offset of element (row, col) of a [rows][64] fp16 tile in the 128-byte
// swizzle layout TMA writes (and the UMMA descriptor reads): the 16-byte chunk
// index of each 128-byte row is XORed with the row index modulo 8. The tile
// base is 1024-byte aligned.
__device__ __forceinline__ uint32_t swz(int row, int col) {
    return static_cast<uint32_t>(row * 128 + ((((col >> 3) ^ (row & 7)) << 4) | ((col & 7) * 2)));
}

__device__ __forceinline__ uint32_t h2_bits(__half2 h) { return *reinterpret_cast<uint32_t*>(&h); }

// Four consecutive values (col % 4 == 0) of token row m into a B tile: fp16(v)
// in row m, fp16(v - fp16(v)) in row 24 + m.
__device__ __forceinline__ void put_split4(uint8_t* bt, int m, int col, float4 v) {
    const __half2 h01 = __floats2half2_rn(v.x, v.y), h23 = __floats2half2_rn(v.z, v.w);
    const float2 f01 = __half22float2(h01), f23 = __half22float2(h23);
    const __half2 l01 = __floats2half2_rn(v.x - f01.x, v.y - f01.y);
    const __half2 l23 = __floats2half2_rn(v.z - f23.x, v.w - f23.y);
    *reinterpret_cast<uint2*>(bt + swz(m, col)) = make_uint2(h2_bits(h01), h2_bits(h23));
    *reinterpret_cast<uint2*>(bt + swz(kLoOffset + m, col)) = make_uint2(h2_bits(l01), h2_bits(l23));
}

}  // namespace tc
}  // namespace vxc
