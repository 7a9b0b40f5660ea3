// The VoxCPM2SDPA layer's single-query decode (src/ncnn_layers/sdpa/voxcpm2_sdpa.cpp:115-260:
// one query row over [past | cur] keys, GQA, scale, additive mask, softmax, P.V) as one
// latency-lean launch for up to 512 keys, fp32 rows as the layer receives them.
//
// One 8-CTA cluster per KV head, 256 threads per CTA, each CTA a contiguous slice of at
// most 64 keys. Every thread issues all of its key, value and query loads before it uses
// any (one memory round trip per launch), the scores reduce across the 8 lanes of a key
// with a transposed butterfly (one head per lane at the end), and the slices' (max, sum,
// P.V) are combined in rank 0's shared memory after one cluster barrier. Sums run in a
// fixed order: results are bit-reproducible.
#include <algorithm>
#include <stdexcept>
#include <string>

#include "kernels.cuh"

namespace vxc {
namespace {

constexpr int kThreads = 256;
constexpr int kCluster = 8;
constexpr int kKeys = 64;        // keys per CTA
constexpr int kD = 64;
constexpr int kMaxHeads = 16;    // query heads per KV head
constexpr int kRow = kD + 4;     // padded shared-memory rows (16-byte aligned)

struct OpSmem {
    float ks[kKeys][kRow];
    float vs[kKeys][kRow];
    float qs[kMaxHeads][kD];
    float sc[kMaxHeads][kKeys + 4];
    float accq[2][kMaxHeads][kD];     // P.V of the two key halves
    float ml[2][kMaxHeads];           // this CTA's max and sum per head
    float mk[kKeys];                  // additive mask of this slice's keys
    float comb[kCluster][kMaxHeads][kD + 2];  // rank 0: every CTA's (m, l, P.V)
};

void check(cudaError_t e) {
    if (e != cudaSuccess) throw std::runtime_error(std::string("sdpa op: ") + cudaGetErrorString(e));
}

__device__ __forceinline__ void st_cluster(float* local, uint32_t rank, float v) {
    uint32_t addr;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;"
                 : "=r"(addr)
                 : "r"(static_cast<uint32_t>(__cvta_generic_to_shared(local))), "r"(rank));
    asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(addr), "f"(v) : "memory");
}

__global__ void __launch_bounds__(kThreads) sdpa_op_kernel(const AttnArgs a) {
    extern __shared__ __align__(16) uint8_t smem_raw[];
    OpSmem& S = *reinterpret_cast<OpSmem*>(smem_raw);
    pdl_launch_dependents();
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int rank = blockIdx.x, kvh = blockIdx.y;
    const int G = a.q_heads / a.kv_heads;
    const int T = a.len0 + a.len1;
    const int t0 = rank * kKeys, n = max(0, min(T, t0 + kKeys) - t0);
    const float* k0 = static_cast<const float*>(a.k0) + static_cast<size_t>(kvh) * a.stride0 * kD;
    const float* v0 = static_cast<const float*>(a.v0) + static_cast<size_t>(kvh) * a.stride0 * kD;
    const float* k1 = a.k1 ? static_cast<const float*>(a.k1) + static_cast<size_t>(kvh) * a.stride1 * kD : nullptr;
    const float* v1 = a.v1 ? static_cast<const float*>(a.v1) + static_cast<size_t>(kvh) * a.stride1 * kD : nullptr;
    pdl_wait();

    // ---- every load in flight at once: 4 K + 4 V float4 per thread (64 keys x 16), q, mask
    {
        float4 kr[4], vr[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int i = tid + j * kThreads, r = i >> 4, c = (i & 15) * 4;
            if (r < n) {
                const int row = t0 + r;
                const float* kp = row < a.len0 ? k0 + static_cast<size_t>(row) * kD : k1 + static_cast<size_t>(row - a.len0) * kD;
                const float* vp = row < a.len0 ? v0 + static_cast<size_t>(row) * kD : v1 + static_cast<size_t>(row - a.len0) * kD;
                kr[j] = __ldg(reinterpret_cast<const float4*>(kp + c));
                vr[j] = __ldg(reinterpret_cast<const float4*>(vp + c));
            } else {
                kr[j] = make_float4(0.f, 0.f, 0.f, 0.f);
                vr[j] = kr[j];
            }
        }
        float4 qv[2];
#pragma unroll
        for (int j = 0; j < 2; ++j) {
            const int i = tid + j * kThreads;  // float4 index into the G x 64 query rows
            qv[j] = i < G * (kD / 4) ? __ldg(reinterpret_cast<const float4*>(a.q + static_cast<size_t>(kvh) * G * kD) + i)
                                     : make_float4(0.f, 0.f, 0.f, 0.f);
        }
        const float mk = (a.mask && tid < n) ? __ldg(a.mask + t0 + tid) : 0.f;
        if (tid < kKeys) S.mk[tid] = mk;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int i = tid + j * kThreads, r = i >> 4, c = (i & 15) * 4;
            *reinterpret_cast<float4*>(&S.ks[r][c]) = kr[j];
            *reinterpret_cast<float4*>(&S.vs[r][c]) = vr[j];
        }
#pragma unroll
        for (int j = 0; j < 2; ++j) {
            const int i = tid + j * kThreads;
            if (i < G * (kD / 4)) {
                const float4 q = qv[j];
                *reinterpret_cast<float4*>(&S.qs[i / 16][(i & 15) * 4]) =
                    make_float4(q.x * a.scale, q.y * a.scale, q.z * a.scale, q.w * a.scale);
            }
        }
        __syncthreads();
        // ---- scores: 8 lanes per key (8 dims each), 4 keys per warp, 8 heads a pass
        const int l8 = lane & 7, kk = lane >> 3;
        for (int h0 = 0; h0 < G; h0 += 8) {
            float qr[8][8];
#pragma unroll
            for (int h = 0; h < 8; ++h)
#pragma unroll
                for (int i = 0; i < 8; ++i) qr[h][i] = h0 + h < G ? S.qs[h0 + h][l8 * 8 + i] : 0.f;
            for (int tb = warp * 4; tb < kKeys; tb += (kThreads / 32) * 4) {
                const int t = tb + kk;
                const float4 x0 = *reinterpret_cast<const float4*>(&S.ks[t][l8 * 8]);
                const float4 x1 = *reinterpret_cast<const float4*>(&S.ks[t][l8 * 8 + 4]);
                const float kv[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
                float dv[8];
#pragma unroll
                for (int h = 0; h < 8; ++h) {
                    float d = 0.f;
#pragma unroll
                    for (int i = 0; i < 8; ++i) d = fmaf(qr[h][i], kv[i], d);
                    dv[h] = d;
                }
                // transposed butterfly over the key's 8 lanes: lane l8 ends with head l8's sum
                const bool b2 = (l8 & 4) != 0, b1 = (l8 & 2) != 0, b0 = (l8 & 1) != 0;
                float s4[4];
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const float keep = b2 ? dv[4 + j] : dv[j], give = b2 ? dv[j] : dv[4 + j];
                    s4[j] = keep + __shfl_xor_sync(0xffffffffu, give, 4);
                }
                float s2[2];
#pragma unroll
                for (int j = 0; j < 2; ++j) {
                    const float keep = b1 ? s4[2 + j] : s4[j], give = b1 ? s4[j] : s4[2 + j];
                    s2[j] = keep + __shfl_xor_sync(0xffffffffu, give, 2);
                }
                const float keep = b0 ? s2[1] : s2[0], give = b0 ? s2[0] : s2[1];
                const float s1 = keep + __shfl_xor_sync(0xffffffffu, give, 1);
                const int h = h0 + l8;
                if (t < n && h < G) S.sc[h][t] = s1 + S.mk[t];
            }
        }
    }
    __syncthreads();
    // ---- softmax of this slice: warp h (heads h, h + 8)
    for (int h = warp; h < G; h += kThreads / 32) {
        const float x0 = lane < n ? S.sc[h][lane] : -1e30f;
        const float x1 = lane + 32 < n ? S.sc[h][lane + 32] : -1e30f;
        const float m = warp_max(fmaxf(x0, x1));
        const float p0 = lane < n ? expf(x0 - m) : 0.f;
        const float p1 = lane + 32 < n ? expf(x1 - m) : 0.f;
        if (lane < n) S.sc[h][lane] = p0;
        if (lane + 32 < n) S.sc[h][lane + 32] = p1;
        const float l = warp_sum(p0 + p1);
        if (lane == 0) {
            S.ml[0][h] = n > 0 ? m : -1e30f;
            S.ml[1][h] = l;
        }
    }
    __syncthreads();
    // ---- P.V: thread (key half, head, 4 dims); the halves summed in order
    {
        const int per = G * 16, groups = min(2, kThreads / per);
        const int qi = tid / per, r = tid - qi * per, h = r / 16, d4 = r - h * 16;
        if (qi < groups) {
            const int tb = qi * (kKeys / groups), te = min(n, tb + kKeys / groups);
            float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 4
            for (int t = tb; t < te; ++t) {
                const float p = S.sc[h][t];
                const float4 v = *reinterpret_cast<const float4*>(&S.vs[t][d4 * 4]);
                acc.x = fmaf(p, v.x, acc.x);
                acc.y = fmaf(p, v.y, acc.y);
                acc.z = fmaf(p, v.z, acc.z);
                acc.w = fmaf(p, v.w, acc.w);
            }
            *reinterpret_cast<float4*>(&S.accq[qi][h][d4 * 4]) = acc;
        }
        __syncthreads();
        // ---- publish (m, l, P.V) into rank 0's combine slot for this rank
        for (int i = tid; i < G * (kD + 2); i += kThreads) {
            const int h = i / (kD + 2), c = i - h * (kD + 2);
            float v;
            if (c < kD) {
                v = S.accq[0][h][c];
                for (int q = 1; q < groups; ++q) v += S.accq[q][h][c];
            } else {
                v = S.ml[c - kD][h];
            }
            st_cluster(&S.comb[rank][h][c], 0, v);
        }
    }
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
    if (rank == 0) {
        for (int i = tid; i < G * kD; i += kThreads) {
            const int h = i / kD, c = i - h * kD;
            float M = -1e30f;
#pragma unroll
            for (int r = 0; r < kCluster; ++r) M = fmaxf(M, S.comb[r][h][kD]);
            float num = 0.f, den = 0.f;
#pragma unroll
            for (int r = 0; r < kCluster; ++r) {
                const float w = expf(S.comb[r][h][kD] - M);
                num = fmaf(w, S.comb[r][h][c], num);
                den = fmaf(w, S.comb[r][h][kD + 1], den);
            }
            a.out[(static_cast<size_t>(kvh) * G + h) * kD + c] = num / den;
        }
    }
}

}  // namespace

bool sdpa_op_supported(const AttnArgs& a) {
    return a.head_dim == kD && a.kv_heads > 0 && a.q_heads % a.kv_heads == 0 && a.q_heads / a.kv_heads <= kMaxHeads &&
           a.len0 + a.len1 <= kCluster * kKeys && a.len0 + a.len1 > 0 && !a.ctl;
}

void launch_sdpa_op(const AttnArgs& a, cudaStream_t s, bool pdl) {
    if (!sdpa_op_supported(a)) throw std::invalid_argument("sdpa op: unsupported shape");
    for (const void* p : {static_cast<const void*>(a.q), a.k0, a.v0, a.k1, a.v1})
        if (reinterpret_cast<uintptr_t>(p) % 16 != 0)
            throw std::invalid_argument("sdpa op: rows must start on 16-byte boundaries");
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(kCluster, a.kv_heads);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = sizeof(OpSmem);
    cfg.stream = s;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = kCluster;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 2 : 1;
    check(cudaLaunchKernelEx(&cfg, sdpa_op_kernel, a));
}

void init_sdpa_op_attributes() {
    check(cudaFuncSetAttribute(sdpa_op_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(sizeof(OpSmem))));
}

}  // namespace vxc
