// Single-query SDPA that never allocates device memory.
//
// vxc_sdpa's split-K decode path (one query row over more than 512 keys) keeps its
// split partials in a scratch buffer it allocates on first use. Some callers cannot let a library allocate: plugin
// hosts that hand a layer pre-allocated tensors and a stream and forbid
// allocation inside the enqueue call (cudaMalloc synchronises the device and
// can fail against a budget the host manages), or real-time audio threads that
// cannot afford cudaMalloc/cudaFree's implicit device synchronisation. For
// them this file keeps the scratch in a fixed file-scope device array, present
// on every GPU that loads the library until the process exits.
#include <algorithm>
#include <cmath>
#include <mutex>
#include <stdexcept>
#include <string>

#include "../../include/voxcpm2_cuda.h"
#include "kernels.cuh"

void vxc_internal_set_error(const char* msg);

namespace {

constexpr int kMaxHeads = 64;   // query heads per call
constexpr int kMaxSplits = 32;  // split-K partitions (the op never uses more)
constexpr int kCounterSlots = 64;
constexpr size_t kPartialFloats = static_cast<size_t>(kMaxHeads) * kMaxSplits * (64 + 2);
constexpr size_t kScratchFloats = kCounterSlots + kPartialFloats;  // 135,232 floats = 528.3 KiB

// [0, 64): per-KV-head arrival counters (int); then the split partials.
static __device__ __align__(256) float g_sdpa_scratch[kScratchFloats];

constexpr int kMaxDevices = 64;
std::mutex g_setup_mu;
float* g_scratch_addr[kMaxDevices] = {};

// Once per device, with that device current: resolve the array's device address
// (in host code its name is only a host-side stand-in) and raise the kernels'
// shared-memory limits. Neither step allocates.
float* scratch_for_current_device() {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) throw std::runtime_error(std::string("cudaGetDevice: ") + cudaGetErrorString(e));
    if (dev < 0 || dev >= kMaxDevices) throw std::runtime_error("device index beyond the supported range");
    std::lock_guard<std::mutex> lk(g_setup_mu);
    if (!g_scratch_addr[dev]) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_sdpa_scratch);
        if (e != cudaSuccess || p == nullptr)
            throw std::runtime_error(std::string("cudaGetSymbolAddress: ") + cudaGetErrorString(e));
        vxc::init_kernel_attributes();
        g_scratch_addr[dev] = static_cast<float*>(p);
    }
    return g_scratch_addr[dev];
}

}  // namespace

extern "C" VXC_API int32_t vxc_sdpa_decode_noalloc(const float* q, int32_t heads, int32_t d, const float* k,
                                                   const float* v, int32_t groups, int32_t cur, const float* mask,
                                                   const float* past_k, const float* past_v, int32_t past,
                                                   float scale, float* out, float* out_k, float* out_v,
                                                   void* cuda_stream) {
    try {
        if (!q || !k || !v || !out) throw std::invalid_argument("null argument");
        if (d != 64) throw std::invalid_argument("vxc_sdpa_decode_noalloc: head dim must be 64");
        if (heads <= 0 || groups <= 0 || heads % groups != 0 || heads / groups > 16)
            throw std::invalid_argument("vxc_sdpa_decode_noalloc: heads must be a multiple of groups (<= 16 per group)");
        if (heads > kMaxHeads)
            throw std::invalid_argument("vxc_sdpa_decode_noalloc: more than 64 query heads exceed the fixed scratch");
        if (cur <= 0 || past < 0 || (past > 0 && (!past_k || !past_v)))
            throw std::invalid_argument("vxc_sdpa_decode_noalloc: bad key/value lengths");
        cudaStream_t cs = static_cast<cudaStream_t>(cuda_stream);
        float* scratch = scratch_for_current_device();
        int* counters = reinterpret_cast<int*>(scratch);
        const int T = past + cur;
        const int splits = std::min(kMaxSplits, std::max(1, (T + 31) / 32));
        // the array keeps the previous call's contents: the counters must start at zero
        cudaError_t e = cudaMemsetAsync(counters, 0, sizeof(int) * kCounterSlots, cs);
        if (e != cudaSuccess) throw std::runtime_error(std::string("cudaMemsetAsync: ") + cudaGetErrorString(e));
        vxc::AttnArgs a;
        a.q = q;
        a.k0 = past > 0 ? past_k : k;
        a.v0 = past > 0 ? past_v : v;
        a.len0 = past > 0 ? past : cur;
        a.stride0 = past > 0 ? past : cur;
        a.k1 = past > 0 ? k : nullptr;
        a.v1 = past > 0 ? v : nullptr;
        a.len1 = past > 0 ? cur : 0;
        a.stride1 = cur;
        a.mask = mask;
        a.q_heads = heads;
        a.kv_heads = groups;
        a.head_dim = d;
        a.scale = scale == 0.f ? 1.f / std::sqrt(static_cast<float>(d)) : scale;
        a.splits = splits;
        a.partial = scratch + kCounterSlots;
        a.counters = counters;
        a.out = out;
        vxc::launch_attn_decode(a, false, cs, false);
        if (out_k) vxc::launch_concat_kv(past_k, k, groups, past, cur, d, out_k, cs);
        if (out_v) vxc::launch_concat_kv(past_v, v, groups, past, cur, d, out_v, cs);
        return VXC_STATUS_OK;
    } catch (const std::invalid_argument& ex) {
        vxc_internal_set_error(ex.what());
        return VXC_STATUS_INVALID_ARGUMENT;
    } catch (const std::exception& ex) {
        vxc_internal_set_error(ex.what());
        return VXC_STATUS_RUNTIME_ERROR;
    } catch (...) {
        vxc_internal_set_error("unknown native exception");
        return VXC_STATUS_RUNTIME_ERROR;
    }
}
