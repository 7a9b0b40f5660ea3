// Device helpers shared by the sm_100a kernels of libvoxcpm2_cuda.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace vxc {

constexpr int kWarp = 32;

// Programmatic dependent launch (PDL). A kernel calls pdl_launch_dependents()
// first so the next kernel in the stream can be scheduled early and stream its
// weights while this one runs; it calls pdl_wait() before touching anything a
// preceding kernel wrote. Both are no-ops when the launch carries no PDL edge.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// Every mbarrier wait in these kernels gives up after this much wall time
// (%globaltimer, nanoseconds) and reports failure instead of waiting on: a pipeline
// wait normally completes within microseconds, so a wait that outlives one second
// means a copy or MMA that never arrives.
constexpr uint64_t kWaitNs = 1000000000ull;
__device__ __forceinline__ uint64_t global_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Wait for phase 'parity' of the shared-memory mbarrier at 'addr' (a shared-window
// address); false if kWaitNs passed first. mbarrier.try_wait itself suspends the
// thread for a hardware-chosen time before it returns false, so the clock is read
// only between unsuccessful tries.
__device__ __forceinline__ bool mbar_wait_addr(uint32_t addr, uint32_t parity) {
    uint64_t start = 0;
    for (uint32_t i = 0;; ++i) {
        uint32_t done;
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
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

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// Streaming 16-byte load of weights: read once per step, keep out of L1.
__device__ __forceinline__ uint4 ld_stream(const void* p) {
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
    return r;
}

// dot of 8 fp16 weights with 8 fp32 activations, fp32 accumulate
__device__ __forceinline__ float dot8(const uint4 w, const float4 a, const float4 b, float acc) {
    const __half2* h = reinterpret_cast<const __half2*>(&w);
    const float2 f0 = __half22float2(h[0]);
    const float2 f1 = __half22float2(h[1]);
    const float2 f2 = __half22float2(h[2]);
    const float2 f3 = __half22float2(h[3]);
    acc = fmaf(f0.x, a.x, acc);
    acc = fmaf(f0.y, a.y, acc);
    acc = fmaf(f1.x, a.z, acc);
    acc = fmaf(f1.y, a.w, acc);
    acc = fmaf(f2.x, b.x, acc);
    acc = fmaf(f2.y, b.y, acc);
    acc = fmaf(f3.x, b.z, acc);
    acc = fmaf(f3.y, b.w, acc);
    return acc;
}

__device__ __forceinline__ float silu(float v) { return v / (1.0f + expf(-v)); }

// Per-stream device control block. Kernels read positions from here so one
// captured CUDA graph is replayed for every patch.
struct StreamCtl {
    int kv_len[2];      // tokens in the base / residual KV caches
    int patch;          // patches generated so far (index into the noise table)
    int step;           // loop step of the current patch
    int min_patches;    // stop rule: step > min_patches && l1 > l0
    int stopped;        // set by the stop head; later kernels of the patch return early
    int error;          // non-zero: a device-side check failed (code), host reports it
    int pad;
    float stop_logits[2];
};

}  // namespace vxc
