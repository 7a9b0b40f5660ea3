// Persistent batch-1 decoder step: every layer of one KV-cache decode step of
// base_decoder_kv / residual_decoder_kv (tools/export_components.py:496-550, run
// by src/kvcache.cpp:232-279) in ONE cooperative launch, one CTA per SM.
//
// Why: a decode step is a chain of dependent matrix-vector products. As separate
// kernels each link pays a launch ramp, an L2 round trip for its input and a
// reduction tail (~1 us per dependent kernel on this part), so 121 kernels hold a
// 717 MB step near 0.2 of the HBM roofline. Here the weights never wait on the
// chain: every CTA owns a fixed slice of every layer's four matrices, and the
// bulk-copy engine streams the NEXT layer's slice of a matrix into shared memory
// as soon as the CTA is done with the current one, so at each phase the weights
// are already on chip and only the small activation vector moves.
//
// Phases of layer l (CTA b of NB; A = kv_heads x kSplits attention CTAs, the rest
// G = NB - A also run gate/up):
//   1  h -> RMSNorm -> its q/k/v rows (RoPE pairs), RoPE; the new K/V row is
//      appended to the fp32 cache at position pos (= ctl->kv_len[which])
//   2  attention CTAs: keys [split] of one KV head (cached rows prefetched into
//      shared memory, the new row from phase 1), online softmax, partial P.V
//   3  softmax combine of the partials -> attention vector -> its o rows, residual
//   4  h' -> RMSNorm -> its gate/up rows -> SiLU(gate) * up
//   5  its down rows over the whole SiLU*up vector, residual
// Vectors pass between phases through global memory as 64-bit words holding the
// fp32 value and a 32-bit tag unique to (invocation, layer, phase); a reader
// spins on each word until its tag appears. A word is written by one 64-bit
// store and read by one 64-bit load (single-copy atomic), so value and tag always
// arrive together: no fences, no grid barriers, one round trip per hand-off.
// Every spin gives up after about a second (2^31 SM cycles; the bulk-copy waits after
// kWaitNs of %globaltimer) or as soon as another CTA has reported a failure; the kernel
// then records error 4 and runs to its end.
//
// Sums are in a fixed order (warp butterflies, fixed part orders), so results
// are bit-reproducible from run to run.
#include <algorithm>
#include <cstdint>
#include <stdexcept>
#include <string>

#include "kernels.cuh"

namespace vxc {
namespace {

using u64 = unsigned long long;

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / kWarp;
constexpr int kSplits = 4;      // attention CTAs per KV head
constexpr int kKvRows = 128;    // cached keys per attention sub-chunk in shared memory
constexpr int kMaxG = 8;        // query heads per KV head
constexpr int kMaxChunks = 4;   // 256-element chunks of a lane's slice (K <= 1024 per dot)
constexpr int kHd = 64;         // head_dim
constexpr int kScStride = kKvRows + 4;
// a hand-off spin gives up after 2^31 SM cycles (about a second at the B200's clocks)
constexpr long long kSpinCycles = 1ll << 31;

void check_launch(cudaError_t e) {
    if (e != cudaSuccess) throw std::runtime_error(std::string("decode step: ") + cudaGetErrorString(e));
}

struct StepPlan {
    int nb = 0, na = 0, ng = 0;       // CTAs, attention CTAs, gate/up CTAs
    int units = 0;                    // q/k/v RoPE-pair units ((hq + 2 hkv) * hd / 2)
    int nq = 0, no = 0, ngu = 0;      // most units / rows a CTA owns: q/k/v units, o (= down) rows, gate/up units
    int kp = 0, np = 0;               // down: K part length (multiple of 256, <= 1024) and parts
    // exchange word offsets
    int x_qkv = 0, x_part = 0, x_hm = 0, x_act = 0, x_h = 0, x_words = 0;
    // shared-memory byte offsets
    int s_wq = 0, s_wo = 0, s_wd = 0, s_xs = 0, s_hs = 0, s_red = 0, s_red2 = 0, s_dpart = 0, s_u = 0;
    int s_gin = 0, s_gpost = 0, s_rope = 0;  // input-norm gain, post-norm gains [2][H] (by layer parity), RoPE row
    // attention CTAs, inside the U region
    int s_kb = 0, s_vb = 0, s_qs = 0, s_kn = 0, s_vn = 0, s_sc = 0, s_accq = 0, s_accr = 0, s_ml = 0, s_act = 0;
    int smem = 0;
};

__device__ __forceinline__ void xput(u64* p, float v, uint32_t tag) {
    const u64 w = (static_cast<u64>(tag) << 32) | __float_as_uint(v);
    asm volatile("st.relaxed.gpu.global.b64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}
__device__ __forceinline__ u64 xld(const u64* p) {
    u64 w;
    asm volatile("ld.relaxed.gpu.global.b64 %0, [%1];" : "=l"(w) : "l"(p) : "memory");
    return w;
}

// Failure state shared by the CTAs of one invocation: seq[1] == inv + 1 means
// some CTA gave up.
struct Abort {
    unsigned* word;
    unsigned id;
    __device__ bool raised() const { return *reinterpret_cast<volatile unsigned*>(word) == id; }
    __device__ void raise() const { *reinterpret_cast<volatile unsigned*>(word) = id; }
};

// Reads the words ptr[k] (k < cnt <= N) into v[k], all loads in flight at once,
// spinning on the ones whose tag has not arrived. False on timeout or abort.
template <int N>
__device__ bool xgather(const u64* const (&ptr)[N], int cnt, uint32_t tag, float (&v)[N], const Abort& ab) {
    uint32_t pending = 0;
#pragma unroll
    for (int k = 0; k < N; ++k)
        if (k < cnt) pending |= 1u << k;
    long long start = 0;
    bool timing = false;
    while (pending) {
        u64 w[N];
#pragma unroll
        for (int k = 0; k < N; ++k)
            if ((pending >> k) & 1u) w[k] = xld(ptr[k]);
#pragma unroll
        for (int k = 0; k < N; ++k)
            if (((pending >> k) & 1u) && static_cast<uint32_t>(w[k] >> 32) == tag) {
                v[k] = __uint_as_float(static_cast<uint32_t>(w[k]));
                pending &= ~(1u << k);
            }
        if (pending) {
            // the SM cycle counter (cheap to read, unlike %globaltimer) bounds the spin
            const long long now = clock64();
            if (!timing) {
                start = now;
                timing = true;
            } else if (now - start > kSpinCycles || ab.raised()) {
                ab.raise();
                return false;
            }
        }
    }
    return true;
}

// The same for words base[idx[k]] (offsets instead of pointers: fewer registers).
template <int N>
__device__ bool xgather_at(const u64* base, const int (&idx)[N], int cnt, uint32_t tag, float (&v)[N], const Abort& ab) {
    uint32_t pending = 0;
#pragma unroll
    for (int k = 0; k < N; ++k)
        if (k < cnt) pending |= 1u << k;
    long long start = 0;
    bool timing = false;
    while (pending) {
        u64 w[N];
#pragma unroll
        for (int k = 0; k < N; ++k)
            if ((pending >> k) & 1u) w[k] = xld(base + idx[k]);
#pragma unroll
        for (int k = 0; k < N; ++k)
            if (((pending >> k) & 1u) && static_cast<uint32_t>(w[k] >> 32) == tag) {
                v[k] = __uint_as_float(static_cast<uint32_t>(w[k]));
                pending &= ~(1u << k);
            }
        if (pending) {
            // the SM cycle counter (cheap to read, unlike %globaltimer) bounds the spin
            const long long now = clock64();
            if (!timing) {
                start = now;
                timing = true;
            } else if (now - start > kSpinCycles || ab.raised()) {
                ab.raise();
                return false;
            }
        }
    }
    return true;
}

// dst[i] = word i of the concatenation of up to three word ranges (s0, n0),
// (s1, n1), (s2, n2); the CTA's threads take words tid, tid + kThreads, ..., eight at
// a time with their loads in flight together.
__device__ bool xget(const u64* s0, int n0, const u64* s1, int n1, const u64* s2, int n2, uint32_t tag, float* dst,
                     const Abort& ab) {
    constexpr int kB = 8;
    const int n = n0 + n1 + n2;
    bool ok = true;
    for (int base = threadIdx.x; base < n && ok; base += kThreads * kB) {
        const u64* ptr[kB];
        float v[kB];
        int cnt = 0;
#pragma unroll
        for (int k = 0; k < kB; ++k) {
            const int i = base + k * kThreads;
            ptr[k] = s0;
            if (i < n) {
                ptr[k] = i < n0 ? s0 + i : i < n0 + n1 ? s1 + (i - n0) : s2 + (i - n0 - n1);
                cnt = k + 1;
            }
        }
        ok = xgather<kB>(ptr, cnt, tag, v, ab);
#pragma unroll
        for (int k = 0; k < kB; ++k)
            if (k < cnt) dst[base + k * kThreads] = v[k];
    }
    return ok;
}

__device__ __forceinline__ bool xget1(const u64* s, int n, uint32_t tag, float* dst, const Abort& ab) {
    return xget(s, n, nullptr, 0, nullptr, 0, tag, dst, ab);
}

__device__ __forceinline__ void bulk_copy(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            static_cast<uint32_t>(__cvta_generic_to_shared(dst))),
        "l"(src), "r"(bytes), "r"(static_cast<uint32_t>(__cvta_generic_to_shared(bar)))
        : "memory");
}
__device__ __forceinline__ void bar_expect(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(
                     static_cast<uint32_t>(__cvta_generic_to_shared(bar))),
                 "r"(bytes)
                 : "memory");
}

// The lane's slice of a K-vector in shared memory: xr[c][i] = src[(c * 32 + lane) * 8 + i].
__device__ __forceinline__ void load_slice(const float* src, int nc, int lane, float (&xr)[kMaxChunks][8]) {
#pragma unroll
    for (int c = 0; c < kMaxChunks; ++c) {
        if (c < nc) {
            const float4 a = *reinterpret_cast<const float4*>(src + (c * 32 + lane) * 8);
            const float4 b = *reinterpret_cast<const float4*>(src + (c * 32 + lane) * 8 + 4);
            xr[c][0] = a.x; xr[c][1] = a.y; xr[c][2] = a.z; xr[c][3] = a.w;
            xr[c][4] = b.x; xr[c][5] = b.y; xr[c][6] = b.z; xr[c][7] = b.w;
        } else {
#pragma unroll
            for (int i = 0; i < 8; ++i) xr[c][i] = 0.f;
        }
    }
}

// n <= R weight rows (fp16 in shared memory, w[r]) . the lane's slice, each summed over
// the warp: every load of all rows issued first, one FMA chain per (row, chunk), and
// the rows' butterflies interleaved, so the warp waits on one latency, not R x 4.
template <int R>
__device__ __forceinline__ void rows_dot(const __half* const (&w)[R], int n, const float (&xr)[kMaxChunks][8], int nc,
                                         int lane, float (&out)[R]) {
    uint4 wv[R][kMaxChunks];
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
        for (int c = 0; c < kMaxChunks; ++c)
            wv[r][c] = (r < n && c < nc) ? *reinterpret_cast<const uint4*>(w[r] + (c * 32 + lane) * 8)
                                         : make_uint4(0u, 0u, 0u, 0u);
#pragma unroll
    for (int r = 0; r < R; ++r) {
        float part[kMaxChunks];
#pragma unroll
        for (int c = 0; c < kMaxChunks; ++c)
            part[c] = dot8(wv[r][c], make_float4(xr[c][0], xr[c][1], xr[c][2], xr[c][3]),
                           make_float4(xr[c][4], xr[c][5], xr[c][6], xr[c][7]), 0.f);
        float acc = part[0];
#pragma unroll
        for (int c = 1; c < kMaxChunks; ++c) acc += part[c];
        out[r] = acc;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
#pragma unroll
        for (int r = 0; r < R; ++r) out[r] += __shfl_xor_sync(0xffffffffu, out[r], o);
}

// Sum over the CTA in a fixed order; every thread gets the total. red: kWarps floats.
__device__ __forceinline__ float block_sum(float v, float* red) {
    v = warp_sum(v);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
    __syncthreads();
    float t = 0.f;
    for (int i = 0; i < kWarps; ++i) t += red[i];
    __syncthreads();
    return t;
}

__global__ void __launch_bounds__(kThreads, 1) decode_step_kernel(const DecodeStepArgs a, const StepPlan p) {
    extern __shared__ __align__(128) uint8_t sm[];
    __shared__ uint64_t bar[4];  // fills of: q/k/v slice, o slice, U region (gate/up slice or keys), down slice
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, b = blockIdx.x;
    StreamCtl* ctl = a.ctl;
    if (a.skip_if_stopped && ctl->stopped) return;  // every CTA reads the same flag
    const int pos = ctl->kv_len[a.which];           // rows already in the cache = the new row's index
    if (pos >= a.cap) {
        if (b == 0 && tid == 0) ctl->error = 1;
        return;
    }
    const unsigned inv = *reinterpret_cast<volatile unsigned*>(a.seq);
    const Abort ab{a.seq + 1, inv + 1};
    const int L = a.layers, H = a.H, F = a.F, hq = a.hq, hkv = a.hkv, G = hq / hkv, Ko = hq * kHd;
    auto tag = [&](int l, int ph) -> uint32_t { return ((inv * static_cast<uint32_t>(L) + l) << 3) + ph + 1; };
    u64* X = a.xbuf;

    // this CTA's slices
    const bool attn = b >= p.ng;
    const int ai = b - p.ng, kvh = attn ? ai / kSplits : 0, sp = attn ? ai % kSplits : 0;
    const int u0 = static_cast<int>(static_cast<long>(b) * p.units / p.nb);
    const int u1 = static_cast<int>(static_cast<long>(b + 1) * p.units / p.nb);
    const int o0 = static_cast<int>(static_cast<long>(b) * H / p.nb), o1 = static_cast<int>(static_cast<long>(b + 1) * H / p.nb);
    const int g0 = attn ? 0 : static_cast<int>(static_cast<long>(b) * F / p.ng);
    const int g1 = attn ? 0 : static_cast<int>(static_cast<long>(b + 1) * F / p.ng);
    const int nq = u1 - u0, no = o1 - o0, ngu = g1 - g0;
    const int T = pos + 1, chunk = (T + kSplits - 1) / kSplits;
    const int k0 = attn ? min(T, sp * chunk) : 0, k1 = attn ? min(T, k0 + chunk) : 0;

    __half* wq = reinterpret_cast<__half*>(sm + p.s_wq);
    __half* wo = reinterpret_cast<__half*>(sm + p.s_wo);
    __half* wd = reinterpret_cast<__half*>(sm + p.s_wd);
    __half* wu = reinterpret_cast<__half*>(sm + p.s_u);
    float* xs = reinterpret_cast<float*>(sm + p.s_xs);
    float* hs = reinterpret_cast<float*>(sm + p.s_hs);
    float* red = reinterpret_cast<float*>(sm + p.s_red);
    float* red2 = reinterpret_cast<float*>(sm + p.s_red2);
    float* dpart = reinterpret_cast<float*>(sm + p.s_dpart);
    float* kb = reinterpret_cast<float*>(sm + p.s_kb);
    float* vb = reinterpret_cast<float*>(sm + p.s_vb);
    float* qs = reinterpret_cast<float*>(sm + p.s_qs);
    float* kn = reinterpret_cast<float*>(sm + p.s_kn);
    float* vn = reinterpret_cast<float*>(sm + p.s_vn);
    float* sc = reinterpret_cast<float*>(sm + p.s_sc);
    float* accq = reinterpret_cast<float*>(sm + p.s_accq);
    float* accr = reinterpret_cast<float*>(sm + p.s_accr);
    float* ml = reinterpret_cast<float*>(sm + p.s_ml);
    // SiLU * up: gate/up CTAs reuse their (then consumed) gate/up slice
    float* act = reinterpret_cast<float*>(sm + (attn ? p.s_act : p.s_u));

    const size_t plane = static_cast<size_t>(hkv) * a.cap * kHd;
    auto kcache = [&](int l) { return a.k_cache + static_cast<size_t>(l) * plane + static_cast<size_t>(kvh) * a.cap * kHd; };
    auto vcache = [&](int l) { return a.v_cache + static_cast<size_t>(l) * plane + static_cast<size_t>(kvh) * a.cap * kHd; };

    // ---- fills (thread 0): one mbarrier phase per fill, bytes == 0 arrives plainly
    auto finish_fill = [&](int k, uint32_t bytes) {
        if (bytes == 0)
            asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(
                             static_cast<uint32_t>(__cvta_generic_to_shared(&bar[k])))
                         : "memory");
    };
    auto fill_q = [&](int l) {  // q/k/v rows, and layer l's two RMSNorm gains
        const __half* w = a.lw[l * 6 + 0];
        const uint32_t rowb = static_cast<uint32_t>(H) * 2, bytes = 2u * nq * rowb + 2u * rowb;
        bar_expect(&bar[0], bytes);
        bulk_copy(sm + p.s_gin, a.lw[l * 6 + 4], rowb, &bar[0]);
        bulk_copy(sm + p.s_gpost + (l & 1) * rowb, a.lw[l * 6 + 5], rowb, &bar[0]);
        for (int i = 0; i < nq; ++i) {
            const int u = u0 + i, hh = u / (kHd / 2), j = u - hh * (kHd / 2);
            const size_t r0 = static_cast<size_t>(hh) * kHd + j;
            bulk_copy(wq + static_cast<size_t>(2 * i) * H, w + r0 * H, rowb, &bar[0]);
            bulk_copy(wq + static_cast<size_t>(2 * i + 1) * H, w + (r0 + kHd / 2) * H, rowb, &bar[0]);
        }
        finish_fill(0, bytes);
    };
    auto fill_o = [&](int l) {
        const uint32_t bytes = static_cast<uint32_t>(no) * Ko * 2;
        if (bytes) {
            bar_expect(&bar[1], bytes);
            bulk_copy(wo, a.lw[l * 6 + 1] + static_cast<size_t>(o0) * Ko, bytes, &bar[1]);
        }
        finish_fill(1, bytes);
    };
    auto fill_u = [&](int l, int s0) {  // gate/up slice, or cached keys [s0, ...) of this split
        uint32_t bytes = 0;
        if (!attn) {
            const uint32_t part = static_cast<uint32_t>(ngu) * H * 2;
            bytes = 2 * part;
            if (bytes) {
                const __half* w = a.lw[l * 6 + 2];
                bar_expect(&bar[2], bytes);
                bulk_copy(wu, w + static_cast<size_t>(g0) * H, part, &bar[2]);
                bulk_copy(wu + static_cast<size_t>(ngu) * H, w + static_cast<size_t>(F + g0) * H, part, &bar[2]);
            }
        } else {
            const int c1 = min(min(k1, pos), s0 + kKvRows);
            const uint32_t part = c1 > s0 ? static_cast<uint32_t>(c1 - s0) * kHd * 4 : 0u;
            bytes = 2 * part;
            if (bytes) {
                bar_expect(&bar[2], bytes);
                bulk_copy(kb, kcache(l) + static_cast<size_t>(s0) * kHd, part, &bar[2]);
                bulk_copy(vb, vcache(l) + static_cast<size_t>(s0) * kHd, part, &bar[2]);
            }
        }
        finish_fill(2, bytes);
    };
    auto fill_d = [&](int l) {
        const uint32_t bytes = static_cast<uint32_t>(no) * F * 2;
        if (bytes) {
            bar_expect(&bar[3], bytes);
            bulk_copy(wd, a.lw[l * 6 + 3] + static_cast<size_t>(o0) * F, bytes, &bar[3]);
        }
        finish_fill(3, bytes);
    };
    uint32_t phase[4] = {0, 0, 0, 0};  // completed waits per buffer (uniform over the CTA)
    bool ok = true;
    auto wait_fill = [&](int k) {
        if (!mbar_wait_addr(static_cast<uint32_t>(__cvta_generic_to_shared(&bar[k])), phase[k] & 1u)) {
            ab.raise();
            ok = false;
        }
        ++phase[k];
    };

    if (tid == 0) {
        for (int k = 0; k < 4; ++k)
            asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(
                             static_cast<uint32_t>(__cvta_generic_to_shared(&bar[k])))
                         : "memory");
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        fill_q(0);
        fill_o(0);
        fill_u(0, k0);
        fill_d(0);
    }
    __syncthreads();

    const int nch = H / 256, ncho = Ko / 256;
    float* rope_s = reinterpret_cast<float*>(sm + p.s_rope);  // cos [64] | sin [64] of position pos
    if (a.rope_cos && tid < 2 * kHd) {
        const bool lng = a.rope_cos_long && pos + 1 > a.rope_long_from;  // make_rope_cache's rule for one row
        const float* c = (lng ? a.rope_cos_long : a.rope_cos) + static_cast<size_t>(pos) * kHd;
        const float* sn = (lng ? a.rope_sin_long : a.rope_sin) + static_cast<size_t>(pos) * kHd;
        rope_s[tid] = tid < kHd ? c[tid] : sn[tid - kHd];
    }
    const __half* gin = reinterpret_cast<const __half*>(sm + p.s_gin);
    for (int l = 0; l < L; ++l) {
        const __half* post_norm = reinterpret_cast<const __half*>(sm + p.s_gpost) + (l & 1) * H;
        const bool last = l + 1 == L;

        // ---------------- phase 1: RMSNorm(h) -> q/k/v rows, RoPE, KV append
        if (l == 0) {
            for (int i = tid; i < H; i += kThreads) hs[i] = a.h[i];
        } else {
            ok &= xget1(X + p.x_h, H, tag(l - 1, 4), hs, ab);
        }
        wait_fill(0);
        __syncthreads();
        {
            float ss = 0.f;
            for (int i = tid; i < H; i += kThreads) ss += hs[i] * hs[i];
            const float inv_rms = rsqrtf(block_sum(ss, red) / static_cast<float>(H) + a.eps);
            for (int i = tid; i < H; i += kThreads) xs[i] = hs[i] * inv_rms * __half2float(gin[i]);
        }
        __syncthreads();
        {
            float xr[kMaxChunks][8];
            load_slice(xs, nch, lane, xr);
            for (int r0 = warp * 2; r0 < 2 * nq; r0 += kWarps * 2) {
                const __half* w2[2] = {wq + static_cast<size_t>(r0) * H, wq + static_cast<size_t>(r0 + 1) * H};
                float d2[2];
                rows_dot<2>(w2, min(2, 2 * nq - r0), xr, nch, lane, d2);
                if (lane == 0) {
                    red2[r0] = d2[0];
                    if (r0 + 1 < 2 * nq) red2[r0 + 1] = d2[1];
                }
            }
        }
        __syncthreads();
        if (tid < nq) {
            const int half = kHd / 2, u = u0 + tid, hh = u / half, j = u - hh * half;
            const float a0 = red2[2 * tid], a1 = red2[2 * tid + 1];
            float v0 = a0, v1 = a1;
            const bool is_v = hh >= hq + hkv;
            if (!is_v && a.rope_cos) {  // apply_rotary_pos_emb (rotate_half) at position pos
                const float* c = rope_s;
                const float* s = rope_s + kHd;
                v0 = a0 * c[j] + (-a1) * s[j];
                v1 = a1 * c[j + half] + a0 * s[j + half];
            }
            const uint32_t tg = tag(l, 0);
            xput(X + p.x_qkv + hh * kHd + j, v0, tg);
            xput(X + p.x_qkv + hh * kHd + j + half, v1, tg);
            if (hh >= hq) {
                const int kh = is_v ? hh - hq - hkv : hh - hq;
                float* dst = (is_v ? a.v_cache : a.k_cache) + static_cast<size_t>(l) * plane +
                             (static_cast<size_t>(kh) * a.cap + pos) * kHd;
                dst[j] = v0;
                dst[j + half] = v1;
            }
        }
        __syncthreads();
        if (tid == 0) {
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            if (!last) fill_q(l + 1);
            if (l > 0) {
                // this layer's down and gate/up slices: issued only now, after the hand-off at the
                // layer's start, so their bursts do not queue that hand-off's loads
                fill_d(l);
                if (!attn) fill_u(l, 0);
            }
        }

        // ---------------- phase 2: attention over this split's keys (attention CTAs)
        if (attn) {
            const uint32_t tg = tag(l, 0);
            ok &= xget(X + p.x_qkv + kvh * G * kHd, G * kHd, X + p.x_qkv + (hq + kvh) * kHd, kHd,
                       X + p.x_qkv + (hq + hkv + kvh) * kHd, kHd, tg, qs, ab);  // qs | kn | vn are contiguous
            for (int i = tid; i < G * kHd; i += kThreads) accr[i] = 0.f;
            if (tid < G) {
                ml[tid] = -1e30f;  // running max
                ml[G + tid] = 0.f; // running sum
            }
            wait_fill(2);  // the first sub-chunk's cached rows (prefetched)
            __syncthreads();
            const int l8 = lane & 7, kk = lane >> 3;
            for (int s0 = k0; s0 < k1; s0 += kKvRows) {
                const int s1 = min(k1, s0 + kKvRows), n = s1 - s0;
                if (s0 != k0) {  // a further sub-chunk (splits over 128 keys): load it now
                    __syncthreads();
                    if (tid == 0) {
                        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                        fill_u(l, s0);
                    }
                    wait_fill(2);
                }
                if (s1 > pos && tid < kHd) {  // the new key / value row, from phase 1
                    kb[(pos - s0) * kHd + tid] = kn[tid];
                    vb[(pos - s0) * kHd + tid] = vn[tid];
                }
                __syncthreads();
                // scores: 8 lanes per key (8 dims each), 4 keys per warp, 4 heads at a time
                for (int hg0 = 0; hg0 < G; hg0 += 4) {
                    float qr[4][8];
#pragma unroll
                    for (int h = 0; h < 4; ++h)
#pragma unroll
                        for (int i = 0; i < 8; ++i)
                            qr[h][i] = hg0 + h < G ? qs[(hg0 + h) * kHd + l8 * 8 + i] * a.scale : 0.f;
#pragma unroll 2
                    for (int tb = warp * 4; tb < n; tb += kWarps * 4) {
                        const int t = tb + kk;
                        const bool valid = t < n;
                        float kv[8];
                        if (valid) {
                            const float4 x0 = *reinterpret_cast<const float4*>(kb + t * kHd + l8 * 8);
                            const float4 x1 = *reinterpret_cast<const float4*>(kb + t * kHd + l8 * 8 + 4);
                            kv[0] = x0.x; kv[1] = x0.y; kv[2] = x0.z; kv[3] = x0.w;
                            kv[4] = x1.x; kv[5] = x1.y; kv[6] = x1.z; kv[7] = x1.w;
                        } else {
#pragma unroll
                            for (int i = 0; i < 8; ++i) kv[i] = 0.f;
                        }
                        float dv[4];
#pragma unroll
                        for (int h = 0; h < 4; ++h) {
                            float d = 0.f;
#pragma unroll
                            for (int i = 0; i < 8; ++i) d = fmaf(qr[h][i], kv[i], d);
                            dv[h] = d;
                        }
                        // transposed butterfly over the key's 8 lanes: 4 shuffles for 4 heads;
                        // lanes 2h' and 2h' + 1 of each half end with head (hi ? 2 : 0) + b1
                        const bool hi = (lane & 4) != 0, b1 = (lane & 2) != 0;
                        float s0 = hi ? dv[2] : dv[0], s1 = hi ? dv[3] : dv[1];
                        const float o0 = hi ? dv[0] : dv[2], o1 = hi ? dv[1] : dv[3];
                        s0 += __shfl_xor_sync(0xffffffffu, o0, 4);
                        s1 += __shfl_xor_sync(0xffffffffu, o1, 4);
                        float tsum = b1 ? s1 : s0;
                        tsum += __shfl_xor_sync(0xffffffffu, b1 ? s0 : s1, 2);
                        tsum += __shfl_xor_sync(0xffffffffu, tsum, 1);
                        const int hh = hg0 + (hi ? 2 : 0) + (b1 ? 1 : 0);
                        if (valid && (lane & 1) == 0 && hh < G) sc[hh * kScStride + t] = tsum;
                    }
                }
                __syncthreads();
                // online softmax: warp h updates head h's running max / sum
                if (warp < G) {
                    const int h = warp;
                    float mx = -1e30f;
                    for (int t = lane; t < n; t += 32) mx = fmaxf(mx, sc[h * kScStride + t]);
                    mx = warp_max(mx);
                    const float m_old = ml[h], m_new = fmaxf(m_old, mx);
                    float sum = 0.f;
                    for (int t = lane; t < n; t += 32) {
                        const float e = expf(sc[h * kScStride + t] - m_new);
                        sc[h * kScStride + t] = e;
                        sum += e;
                    }
                    sum = warp_sum(sum);
                    __syncwarp();
                    if (lane == 0) {
                        const float corr = expf(m_old - m_new);
                        ml[h] = m_new;
                        ml[G + h] = ml[G + h] * corr + sum;
                        ml[2 * G + h] = corr;
                    }
                }
                __syncthreads();
                // P.V: thread (key group qi, head h, 4 dims d4); groups summed in order below
                {
                    const int per = G * 16, groups = kThreads / per;
                    const int qi = tid / per, r = tid - qi * per, h = r / 16, d4 = r - h * 16;
                    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
                    if (qi < groups)
#pragma unroll 4
                        for (int t = qi; t < n; t += groups) {
                            const float pr = sc[h * kScStride + t];
                            const float4 v = *reinterpret_cast<const float4*>(vb + t * kHd + d4 * 4);
                            acc.x = fmaf(pr, v.x, acc.x);
                            acc.y = fmaf(pr, v.y, acc.y);
                            acc.z = fmaf(pr, v.z, acc.z);
                            acc.w = fmaf(pr, v.w, acc.w);
                        }
                    if (qi < groups)
                        *reinterpret_cast<float4*>(accq + (static_cast<size_t>(qi) * G + h) * kHd + d4 * 4) = acc;
                    __syncthreads();
                    for (int e = tid; e < G * kHd; e += kThreads) {
                        float s = 0.f;
                        for (int q = 0; q < groups; ++q) s += accq[static_cast<size_t>(q) * G * kHd + e];
                        accr[e] = accr[e] * ml[2 * G + e / kHd] + s;
                    }
                }
                __syncthreads();
            }
            // partial (m, l, unnormalised P.V) of this split
            const uint32_t tp = tag(l, 1);
            u64* part = X + p.x_part + static_cast<size_t>(ai) * G * (kHd + 2);
            for (int e = tid; e < G * (kHd + 2); e += kThreads)
                xput(part + e, e < G ? ml[e] : e < 2 * G ? ml[e] : accr[e - 2 * G], tp);
            __syncthreads();
            if (tid == 0 && !last) {
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                fill_u(l + 1, k0);
            }
        }

        // ---------------- phase 3: combine the splits -> attention vector -> o rows + residual
        // thread: elements e .. e + 3 of one head, e = 4 tid (+ 4 kThreads i): per split its m,
        // l and the four P.V values, one gather with all loads in flight
        for (int e = 4 * tid; e < Ko; e += 4 * kThreads) {
            const uint32_t tp = tag(l, 1);
            const int h = e / kHd, d = e - h * kHd, kh = h / G, hg = h - kh * G;
            int idx[6 * kSplits];
            float v[6 * kSplits];
#pragma unroll
            for (int sp2 = 0; sp2 < kSplits; ++sp2) {
                const int base = (kh * kSplits + sp2) * G * (kHd + 2);
                idx[6 * sp2] = base + hg;
                idx[6 * sp2 + 1] = base + G + hg;
#pragma unroll
                for (int j = 0; j < 4; ++j) idx[6 * sp2 + 2 + j] = base + 2 * G + hg * kHd + d + j;
            }
            ok &= xgather_at<6 * kSplits>(X + p.x_part, idx, 6 * kSplits, tp, v, ab);
            float M = -1e30f;
#pragma unroll
            for (int sp2 = 0; sp2 < kSplits; ++sp2) M = fmaxf(M, v[6 * sp2]);
            float den = 0.f, num[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
            for (int sp2 = 0; sp2 < kSplits; ++sp2) {
                const float c = expf(v[6 * sp2] - M);
                den = fmaf(c, v[6 * sp2 + 1], den);
#pragma unroll
                for (int j = 0; j < 4; ++j) num[j] = fmaf(c, v[6 * sp2 + 2 + j], num[j]);
            }
#pragma unroll
            for (int j = 0; j < 4; ++j) xs[e + j] = num[j] / den;
        }
        __syncthreads();
        wait_fill(1);
        {
            float xr[kMaxChunks][8];
            load_slice(xs, ncho, lane, xr);
            const uint32_t tg = tag(l, 2);
            for (int r = warp; r < no; r += kWarps) {
                const __half* w1[1] = {wo + static_cast<size_t>(r) * Ko};
                float d1[1];
                rows_dot<1>(w1, 1, xr, ncho, lane, d1);
                if (lane == 0) xput(X + p.x_hm + o0 + r, hs[o0 + r] + (a.rscale == 1.f ? d1[0] : d1[0] * a.rscale), tg);
            }
        }
        __syncthreads();
        if (tid == 0 && !last) {
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            fill_o(l + 1);
        }

        // ---------------- phase 4: RMSNorm(h') -> gate/up rows -> SiLU(gate) * up
        ok &= xget1(X + p.x_hm, H, tag(l, 2), hs, ab);
        __syncthreads();
        if (!attn) {
            float ss = 0.f;
            for (int i = tid; i < H; i += kThreads) ss += hs[i] * hs[i];
            const float inv_rms = rsqrtf(block_sum(ss, red) / static_cast<float>(H) + a.eps);
            for (int i = tid; i < H; i += kThreads) xs[i] = hs[i] * inv_rms * __half2float(post_norm[i]);
            __syncthreads();
            wait_fill(2);
            float xr[kMaxChunks][8];
            load_slice(xs, nch, lane, xr);
            const uint32_t tg = tag(l, 3);
            for (int i = warp * 2; i < ngu; i += kWarps * 2) {
                const int i1 = min(i + 1, ngu - 1);
                const __half* w4[4] = {wu + static_cast<size_t>(i) * H, wu + static_cast<size_t>(ngu + i) * H,
                                       wu + static_cast<size_t>(i1) * H, wu + static_cast<size_t>(ngu + i1) * H};
                float d4[4];
                rows_dot<4>(w4, i + 1 < ngu ? 4 : 2, xr, nch, lane, d4);
                if (lane == 0) {
                    xput(X + p.x_act + g0 + i, silu(d4[0]) * d4[1], tg);
                    if (i + 1 < ngu) xput(X + p.x_act + g0 + i + 1, silu(d4[2]) * d4[3], tg);
                }
            }
        }
        __syncthreads();  // gate/up CTAs: the slice is consumed; 'act' may overwrite it

        // ---------------- phase 5: down rows over SiLU * up, residual
        ok &= xget1(X + p.x_act, F, tag(l, 3), act, ab);
        __syncthreads();
        wait_fill(3);
        {
            // task t = (row t / np, K part t % np); a warp takes tasks warp, warp + 8, ...
            const int tasks = no * p.np, kc = p.kp / 256;
            float xr[kMaxChunks][8];
            int loaded = -1;
            for (int t0 = warp; t0 < tasks;) {
                const int q = t0 % p.np;
                // this warp's next tasks of the same K part (up to 4), one batch
                int tk[4], n = 0;
                int t = t0;
                for (; t < tasks && n < 4; t += kWarps) {
                    if (t % p.np != q) break;
                    tk[n++] = t;
                }
                for (int k = n; k < 4; ++k) tk[k] = tk[0];
                if (q != loaded) {
                    load_slice(act + q * p.kp, kc, lane, xr);
                    loaded = q;
                }
                const __half* w4[4];
#pragma unroll
                for (int k = 0; k < 4; ++k) w4[k] = wd + static_cast<size_t>(tk[k] / p.np) * F + q * p.kp;
                float d4[4];
                rows_dot<4>(w4, n, xr, kc, lane, d4);
                if (lane == 0)
                    for (int k = 0; k < n; ++k) dpart[tk[k]] = d4[k];
                t0 = t;
            }
        }
        __syncthreads();
        if (tid < no) {
            float s = 0.f;
            for (int q = 0; q < p.np; ++q) s += dpart[tid * p.np + q];
            const float hn = hs[o0 + tid] + (a.rscale == 1.f ? s : s * a.rscale);
            xput(X + p.x_h + o0 + tid, hn, tag(l, 4));
            if (last) a.h[o0 + tid] = hn;
        }
        __syncthreads();  // the down and gate/up slices (and act) are consumed: layer l + 1 refills them
    }

    // ---------------- final RMSNorm of the CTA's rows
    ok &= xget1(X + p.x_h, H, tag(L - 1, 4), hs, ab);
    __syncthreads();
    {
        float ss = 0.f;
        for (int i = tid; i < H; i += kThreads) ss += hs[i] * hs[i];
        const float inv_rms = rsqrtf(block_sum(ss, red) / static_cast<float>(H) + a.eps);
        for (int r = o0 + tid; r < o1; r += kThreads) {
            const float v = hs[r] * inv_rms * __half2float(a.final_norm[r]);
            a.out[r] = v;
            if (a.out2) a.out2[r] = v;
        }
    }
    if (!ok) ctl->error = 4;
    if (b == 0 && tid == 0) {
        // every CTA has read pos and the invocation id (this CTA read all of their last outputs)
        if (a.advance) ctl->kv_len[a.which] = pos + 1;
        *reinterpret_cast<volatile unsigned*>(a.seq) = inv + 1;
    }
}

int g_grid = 0;

StepPlan make_plan(const DecodeStepArgs& a, int nb) {
    StepPlan p;
    const int H = a.H, F = a.F, G = a.hkv > 0 ? a.hq / a.hkv : 0, Ko = a.hq * kHd;
    p.nb = nb;
    p.na = a.hkv * kSplits;
    p.ng = nb - p.na;
    p.units = (a.hq + 2 * a.hkv) * kHd / 2;
    p.nq = (p.units + nb - 1) / nb;
    p.no = (H + nb - 1) / nb;
    p.ngu = p.ng > 0 ? (F + p.ng - 1) / p.ng : 0;
    p.kp = 0;
    for (int kp = 1024; kp >= 256; kp -= 256)
        if (F % kp == 0) {
            p.kp = kp;
            break;
        }
    p.np = p.kp ? F / p.kp : 0;
    // exchange words
    p.x_qkv = 0;
    p.x_part = p.x_qkv + (a.hq + 2 * a.hkv) * kHd;
    p.x_hm = p.x_part + p.na * G * (kHd + 2);
    p.x_act = p.x_hm + H;
    p.x_h = p.x_act + F;
    p.x_words = p.x_h + H;
    // shared memory
    int off = 0;
    auto take = [&](int bytes) {
        const int at = off;
        off += (bytes + 127) / 128 * 128;
        return at;
    };
    p.s_wq = take(2 * p.nq * H * 2);
    p.s_wo = take(p.no * Ko * 2);
    p.s_wd = take(p.no * F * 2);
    p.s_xs = take(std::max(H, Ko) * 4);
    p.s_hs = take(H * 4);
    p.s_red = take(kWarps * 4);
    p.s_red2 = take(2 * p.nq * 4);
    p.s_dpart = take(std::max(1, p.no * p.np) * 4);
    p.s_gin = take(H * 2);
    p.s_gpost = take(2 * H * 2);
    p.s_rope = take(2 * kHd * 4);
    p.s_u = off;
    // the U region: gate/up slice (and SiLU * up after it), or the attention CTAs' buffers
    int u = 0;
    auto utake = [&](int bytes) {
        const int at = p.s_u + u;
        u += (bytes + 127) / 128 * 128;
        return at;
    };
    p.s_kb = utake((kKvRows + 1) * kHd * 4);
    p.s_vb = utake((kKvRows + 1) * kHd * 4);
    p.s_qs = utake(G * kHd * 4);  // qs, kn, vn contiguous: one xget fills all three
    p.s_kn = p.s_qs + G * kHd * 4;
    p.s_vn = p.s_kn + kHd * 4;
    u += 2 * kHd * 4;
    p.s_sc = utake(G * kScStride * 4);
    p.s_accq = utake(kThreads * 4 * 4);
    p.s_accr = utake(G * kHd * 4);
    p.s_ml = utake(3 * G * 4);
    p.s_act = utake(F * 4);
    const int attn_bytes = u;
    const int gu_bytes = std::max(2 * p.ngu * H * 2, F * 4);
    p.smem = p.s_u + std::max(attn_bytes, (gu_bytes + 127) / 128 * 128);
    return p;
}

void check_plan(const DecodeStepArgs& a, const StepPlan& p, bool pointers) {
    auto bad = [](const char* m) { throw std::invalid_argument(std::string("persistent decoder step: ") + m); };
    if (a.hd != kHd) bad("head_dim must be 64");
    if (a.hkv <= 0 || a.hq % a.hkv != 0 || a.hq / a.hkv > kMaxG) bad("at most 8 query heads per KV head");
    if (a.H % 256 != 0 || a.H > 1024 || a.H <= 0) bad("hidden must be a multiple of 256, at most 1024");
    if ((a.hq * kHd) % 256 != 0 || a.hq * kHd > 1024) bad("q_heads x 64 must be a multiple of 256, at most 1024");
    if (a.F % 256 != 0 || a.F <= 0 || p.kp == 0) bad("ffn must be a multiple of 256");
    if (p.ng < 1 || p.nb < p.na + 1) bad("too few SMs for the attention CTAs");
    if (2 * p.nq > kThreads || p.no > kThreads || p.no * p.np > 4096) bad("too few SMs for the model's rows");
    if (p.smem > 232448 - 1024) bad("the per-CTA slices exceed shared memory");
    if (!pointers) return;
    if (!a.lw || !a.final_norm || !a.h || !a.out || !a.k_cache || !a.v_cache || !a.ctl || !a.xbuf || !a.seq)
        bad("null argument");
    if (a.cap <= 0 || (reinterpret_cast<uintptr_t>(a.k_cache) & 15) || (reinterpret_cast<uintptr_t>(a.v_cache) & 15))
        bad("KV caches must be 16-byte aligned");
}

}  // namespace

int decode_step_grid() {
    if (!g_grid) {
        int dev = 0, n = 0;
        check_launch(cudaGetDevice(&dev));
        check_launch(cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev));
        g_grid = n;
    }
    return g_grid;
}

size_t decode_step_words(const DecodeStepArgs& a) { return static_cast<size_t>(make_plan(a, decode_step_grid()).x_words); }

void check_decode_step(const DecodeStepArgs& a) { check_plan(a, make_plan(a, decode_step_grid()), false); }

void launch_decode_step(const DecodeStepArgs& a, cudaStream_t s) {
    const StepPlan p = make_plan(a, decode_step_grid());
    check_plan(a, p, true);
    int per_sm = 0;
    check_launch(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, decode_step_kernel, kThreads,
                                                               static_cast<size_t>(p.smem)));
    if (per_sm < 1) throw std::runtime_error("persistent decoder step: one CTA per SM does not fit");
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(p.nb);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = static_cast<size_t>(p.smem);
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;  // every CTA resident at once: they wait on one another
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    check_launch(cudaLaunchKernelEx(&cfg, decode_step_kernel, a, p));
}

void init_decode_step_attributes() {
    check_launch(cudaFuncSetAttribute(decode_step_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 232448 - 1024));
}

}  // namespace vxc
