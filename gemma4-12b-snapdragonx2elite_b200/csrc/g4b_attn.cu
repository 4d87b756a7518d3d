// g4b_attn.cu -- decode attention over the f16 KV cache: the engine's prepkv and
// attn dispatches (vk/prepkv.comp, vk/attn.comp), recorded per layer between the
// q|k|v and o GEMVs (src/vk_engine.py:281-282).
//
//   prepkv  one CTA per KV head: k = RoPE(rmsnorm(k, knw)), v = v * rsqrt(mean(v^2) + eps),
//           both stored as f16 at the token's cache slot (a ring of `window` slots for
//           sliding layers).
//   decode  flash decoding: grid (splits, KV heads).  A CTA normalises and rotates the
//           query heads that share its KV head (GQA), then its 8 warps stream their
//           share of the split's keys -- each K and V row is read once for all those
//           heads, 16-byte loads per lane -- with an online softmax per warp; the warps'
//           partials merge in shared memory, and a split's (max, sum, weighted V) goes
//           to the workspace for a second kernel to combine.  HBM-bound on the cache:
//           T * hd * 2 bytes of K and of V per KV head.
//
// The token position is read from device memory, so one captured graph serves every
// token; the split count is fixed on the host from the cache's capacity, and splits
// beyond the live keys finish at once.
#include <algorithm>

#include "g4b_common.cuh"

namespace g4b {

constexpr int kAttnThreads = 256;
constexpr int kAttnWarps = kAttnThreads / 32;
constexpr float kAttnEps = 1e-6f;     // vk/attn.comp:25, vk/prepkv.comp:21
constexpr float kNegInit = -1e30f;    // the shaders' running-max start (vk/attn.comp:29)

// n consecutive values (n = 4, 8, 16) of an f32 or f16 vector as f32
template <int N, bool F32>
__device__ __forceinline__ void loadn(const void* base, size_t at, float (&v)[N]) {
    if constexpr (F32) {
        const float4* p = reinterpret_cast<const float4*>(reinterpret_cast<const float*>(base) + at);
        #pragma unroll
        for (int j = 0; j < N / 4; j++) {
            const float4 a = __ldg(p + j);
            v[4 * j] = a.x; v[4 * j + 1] = a.y; v[4 * j + 2] = a.z; v[4 * j + 3] = a.w;
        }
    } else {
        const uint2* p = reinterpret_cast<const uint2*>(reinterpret_cast<const __half*>(base) + at);
        #pragma unroll
        for (int j = 0; j < N / 4; j++) {
            const uint2 u = __ldg(p + j);
            v[4 * j] = h_lo(u.x); v[4 * j + 1] = h_hi(u.x); v[4 * j + 2] = h_lo(u.y); v[4 * j + 3] = h_hi(u.y);
        }
    }
}

// the cache rows: n f16 values as f32 (L2 reads: the cache is streamed, not reused within a CTA)
template <int N>
__device__ __forceinline__ void load_f16n(const uint16_t* p, float (&v)[N]) {
    #pragma unroll
    for (int j = 0; j < N / 8; j++) {
        const uint4 u = __ldcs(reinterpret_cast<const uint4*>(p) + j);
        v[8 * j] = h_lo(u.x); v[8 * j + 1] = h_hi(u.x); v[8 * j + 2] = h_lo(u.y); v[8 * j + 3] = h_hi(u.y);
        v[8 * j + 4] = h_lo(u.z); v[8 * j + 5] = h_hi(u.z); v[8 * j + 6] = h_lo(u.w); v[8 * j + 7] = h_hi(u.w);
    }
    if constexpr (N % 8) {
        const uint2 u = __ldcs(reinterpret_cast<const uint2*>(p + (N / 8) * 8));
        v[N - 4] = h_lo(u.x); v[N - 3] = h_hi(u.x); v[N - 2] = h_lo(u.y); v[N - 1] = h_hi(u.y);
    }
}

__device__ __forceinline__ float warp_sum(float v) {
    #pragma unroll
    for (int m = 16; m >= 1; m >>= 1) v += __shfl_xor_sync(0xffffffffu, v, m);
    return v;
}

// ------------------------------------------------------------------ prepkv
// One CTA per KV head; thread t owns elements t and t + 256 (hd <= 512).
template <bool XF32>
__global__ void __launch_bounds__(kAttnThreads) attn_prepkv_kernel(const void* __restrict__ qkv,
                                                                  const float* __restrict__ knw,
                                                                  const float* __restrict__ cos_t,
                                                                  const float* __restrict__ sin_t, uint16_t* kc,
                                                                  uint16_t* vc, int hd, int koff, int voff,
                                                                  int stride, int window,
                                                                  const int* __restrict__ pos_dev) {
    __shared__ float hv[512];
    __shared__ float wsum[kAttnWarps];
    const int h = blockIdx.x, t = threadIdx.x, lane = t & 31, warp = t >> 5, hf = hd / 2;
    const int pos = __ldg(pos_dev);
    const int slot = window > 0 ? pos % window : pos;
    auto elem = [&](int off, int i) -> float {
        return XF32 ? __ldg(reinterpret_cast<const float*>(qkv) + off + (size_t)h * hd + i)
                    : __half2float(__ldg(reinterpret_cast<const __half*>(qkv) + off + (size_t)h * hd + i));
    };
    auto inv_rms = [&](float s) {
        s = warp_sum(s);
        if (lane == 0) wsum[warp] = s;
        __syncthreads();
        float tot = 0.f;
        #pragma unroll
        for (int w = 0; w < kAttnWarps; w++) tot += wsum[w];
        __syncthreads();
        return rsqrtf(tot / (float)hd + kAttnEps);
    };
    // k: rmsnorm with knw, then RoPE (vk/prepkv.comp:18-24)
    float s = 0.f;
    for (int i = t; i < hd; i += kAttnThreads) {
        const float v = elem(koff, i);
        hv[i] = v;
        s += v * v;
    }
    const float ik = inv_rms(s);
    for (int i = t; i < hd; i += kAttnThreads) hv[i] = hv[i] * ik * __ldg(knw + i);
    __syncthreads();
    uint16_t* krow = kc + ((size_t)h * stride + slot) * hd;
    for (int i = t; i < hd; i += kAttnThreads) {
        const float rh = i < hf ? -hv[i + hf] : hv[i - hf];
        krow[i] = __half_as_ushort(__float2half_rn(hv[i] * __ldg(cos_t + i) + rh * __ldg(sin_t + i)));
    }
    // v: rmsnorm without a weight (vk/prepkv.comp:25-29); with keqv the caller passes voff = koff
    s = 0.f;
    float vv[2] = {0.f, 0.f};
    for (int i = t, n = 0; i < hd; i += kAttnThreads, n++) {
        vv[n] = elem(voff, i);
        s += vv[n] * vv[n];
    }
    const float iv = inv_rms(s);
    uint16_t* vrow = vc + ((size_t)h * stride + slot) * hd;
    for (int i = t, n = 0; i < hd; i += kAttnThreads, n++) vrow[i] = __half_as_ushort(__float2half_rn(vv[n] * iv));
}

// ------------------------------------------------------------------ decode
struct AttnArgs {
    const void* qkv;
    const float* qnw;
    const float* cos_t;
    const float* sin_t;
    const uint16_t* kc;
    const uint16_t* vc;
    void* out;           // S == 1: [nH, hd] output
    float* part;         // S > 1: [nH][S][hd] weighted V sums
    float* pml;          // S > 1: [nH][S][2] (running max, sum)
    const int* pos_dev;
    int nH, nkv, hd, qoff, stride, window, S, out_f32;
};

// D = hd / 32 values per lane, G = query heads per KV head
template <int D, int G, bool XF32>
__global__ void __launch_bounds__(kAttnThreads) attn_decode_kernel(const AttnArgs a) {
    constexpr int HD = 32 * D;
    static_assert(G * D <= 32, "query heads x values per lane held in registers");
    __shared__ float qs[G][HD];                       // the normed query heads
    __shared__ float xacc[kAttnWarps / 2][G][HD];     // partials handed down the warp merge tree
    __shared__ float xm[kAttnWarps / 2][G], xl[kAttnWarps / 2][G];
    const int s = blockIdx.x, kvh = blockIdx.y, t = threadIdx.x, lane = t & 31, warp = t >> 5;
    const int pos = __ldg(a.pos_dev);
    const int T = a.window > 0 ? min(pos + 1, a.window) : pos + 1;
    const int k0 = (int)((long long)s * T / a.S), k1 = (int)((long long)(s + 1) * T / a.S);
    // the query heads of this KV head: rmsnorm with qnw, then RoPE (vk/attn.comp:22-28)
    if (warp < G) {
        const int h = kvh * G + warp;
        float q[D];
        loadn<D, XF32>(a.qkv, (size_t)a.qoff + (size_t)h * HD + lane * D, q);
        float ss = 0.f;
        #pragma unroll
        for (int d = 0; d < D; d++) ss += q[d] * q[d];
        const float iq = rsqrtf(warp_sum(ss) / (float)HD + kAttnEps);
        #pragma unroll
        for (int d = 0; d < D; d++) qs[warp][lane * D + d] = q[d] * iq * __ldg(a.qnw + lane * D + d);
    }
    __syncthreads();
    float qr[G][D];
    #pragma unroll
    for (int g = 0; g < G; g++)
        #pragma unroll
        for (int d = 0; d < D; d++) {
            const int i = lane * D + d, hf = HD / 2;
            const float rh = i < hf ? -qs[g][i + hf] : qs[g][i - hf];
            qr[g][d] = qs[g][i] * __ldg(a.cos_t + i) + rh * __ldg(a.sin_t + i);
        }
    // this warp's keys: an online softmax per query head
    float m[G], l[G], acc[G][D];
    #pragma unroll
    for (int g = 0; g < G; g++) {
        m[g] = kNegInit;
        l[g] = 0.f;
        #pragma unroll
        for (int d = 0; d < D; d++) acc[g][d] = 0.f;
    }
    const size_t row0 = (size_t)kvh * a.stride;
    for (int j = k0 + warp; j < k1; j += kAttnWarps) {
        float kv[D], vv[D];
        load_f16n<D>(a.kc + (row0 + j) * HD + lane * D, kv);
        load_f16n<D>(a.vc + (row0 + j) * HD + lane * D, vv);
        #pragma unroll
        for (int g = 0; g < G; g++) {
            float dot = 0.f;
            #pragma unroll
            for (int d = 0; d < D; d++) dot = fmaf(qr[g][d], kv[d], dot);
            dot = warp_sum(dot);
            const float mn = fmaxf(m[g], dot);
            const float corr = __expf(m[g] - mn), p = __expf(dot - mn);
            l[g] = l[g] * corr + p;
            m[g] = mn;
            #pragma unroll
            for (int d = 0; d < D; d++) acc[g][d] = fmaf(p, vv[d], acc[g][d] * corr);
        }
    }
    // merge the warps' partials down a tree (8 -> 4 -> 2 -> 1): the upper half hands its (max, sum,
    // weighted V) to the lower half through shared memory, which rescales and adds in registers
    #pragma unroll
    for (int half = kAttnWarps / 2; half >= 1; half >>= 1) {
        if (warp >= half && warp < 2 * half) {
            #pragma unroll
            for (int g = 0; g < G; g++) {
                if (lane == 0) {
                    xm[warp - half][g] = m[g];
                    xl[warp - half][g] = l[g];
                }
                #pragma unroll
                for (int d = 0; d < D; d++) xacc[warp - half][g][lane * D + d] = acc[g][d];
            }
        }
        __syncthreads();
        if (warp < half) {
            #pragma unroll
            for (int g = 0; g < G; g++) {
                const float m2 = xm[warp][g], l2 = xl[warp][g], M = fmaxf(m[g], m2);
                const float e1 = __expf(m[g] - M), e2 = __expf(m2 - M);
                l[g] = l[g] * e1 + l2 * e2;
                m[g] = M;
                #pragma unroll
                for (int d = 0; d < D; d++) acc[g][d] = acc[g][d] * e1 + xacc[warp][g][lane * D + d] * e2;
            }
        }
        __syncthreads();
    }
    if (warp == 0) {
        #pragma unroll
        for (int g = 0; g < G; g++) {
            const int h = kvh * G + g;
            if (a.S == 1) {
                const float invl = 1.0f / l[g];
                #pragma unroll
                for (int d = 0; d < D; d++) {
                    const float o = acc[g][d] * invl;
                    const size_t at = (size_t)h * HD + lane * D + d;
                    if (a.out_f32) reinterpret_cast<float*>(a.out)[at] = o;
                    else reinterpret_cast<__half*>(a.out)[at] = __float2half_rn(o);
                }
            } else {
                #pragma unroll
                for (int d = 0; d < D; d++) a.part[((size_t)h * a.S + s) * HD + lane * D + d] = acc[g][d];
                if (lane == 0) {
                    a.pml[((size_t)h * a.S + s) * 2] = m[g];
                    a.pml[((size_t)h * a.S + s) * 2 + 1] = l[g];
                }
            }
        }
    }
}

// the splits' partials -> the output, per query head: out = sum_s v_s e^(m_s - M) / sum_s l_s e^(m_s - M)
__global__ void __launch_bounds__(kAttnThreads) attn_combine_kernel(const AttnArgs a) {
    const int h = blockIdx.x, S = a.S;
    extern __shared__ float sh_e[];                   // [S] weights e^(m_s - M)
    __shared__ float s_L;
    if (threadIdx.x < 32) {
        float M = kNegInit;
        for (int s = threadIdx.x; s < S; s += 32) M = fmaxf(M, a.pml[((size_t)h * S + s) * 2]);
        #pragma unroll
        for (int o = 16; o >= 1; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
        float L = 0.f;
        for (int s = threadIdx.x; s < S; s += 32) {
            const float e = __expf(a.pml[((size_t)h * S + s) * 2] - M);
            sh_e[s] = e;
            L = fmaf(a.pml[((size_t)h * S + s) * 2 + 1], e, L);
        }
        L = warp_sum(L);
        if (threadIdx.x == 0) s_L = L;
    }
    __syncthreads();
    const float invL = 1.0f / s_L;
    for (int i = threadIdx.x; i < a.hd; i += kAttnThreads) {
        float v = 0.f;
        for (int s = 0; s < S; s++) v = fmaf(a.part[((size_t)h * S + s) * a.hd + i], sh_e[s], v);
        const float o = v * invL;
        if (a.out_f32) reinterpret_cast<float*>(a.out)[(size_t)h * a.hd + i] = o;
        else reinterpret_cast<__half*>(a.out)[(size_t)h * a.hd + i] = __float2half_rn(o);
    }
}

// splits of the keys: about two CTAs per SM over the KV heads, at least 32 keys per split
static int attn_splits(int nkv, int max_T, int sms) {
    const int by_keys = (max_T + 31) / 32;
    const int by_sms = std::max(1, 2 * sms / std::max(nkv, 1));
    return std::max(1, std::min(by_keys, by_sms));
}

template <int D, int G>
static cudaError_t launch_decode(const AttnArgs& a, bool xf32, cudaStream_t s) {
    const dim3 grid(a.S, a.nkv);
    if (xf32) attn_decode_kernel<D, G, true><<<grid, kAttnThreads, 0, s>>>(a);
    else attn_decode_kernel<D, G, false><<<grid, kAttnThreads, 0, s>>>(a);
    return cudaGetLastError();
}

template <int D>
static cudaError_t launch_decode_g(const AttnArgs& a, int G, bool xf32, cudaStream_t s) {
    switch (G) {
        case 1: return launch_decode<D, 1>(a, xf32, s);
        case 2: return launch_decode<D, 2>(a, xf32, s);
        case 4: return launch_decode<D, (D <= 8 ? 4 : 2)>(a, xf32, s);    // G * D <= 32 (checked by the caller)
        default: return launch_decode<D, (D <= 4 ? 8 : 2)>(a, xf32, s);
    }
}

// the (hd, query heads per KV head) pairs with an instance: G * hd / 32 <= 32 values per lane
// (hd 128: G 1-8; hd 256: G 1-4; hd 512: G 1-2), G a power of two
static bool attn_shape_ok(int hd, int G) {
    const bool g_ok = G == 1 || G == 2 || G == 4 || G == 8;
    return (hd == 128 || hd == 256 || hd == 512) && g_ok && G * (hd / 32) <= 32;
}

}  // namespace g4b

using namespace g4b;

extern "C" {

int g4b_attn_prepkv(const void* qkv, int dtype, const float* knw, const float* cos_t, const float* sin_t, uint16_t* kc,
                    uint16_t* vc, int nkv, int hd, int koff, int voff, int keqv, int stride, int window,
                    const int* pos_dev, g4b_stream_t stream) {
    G4B_ENTRY("attn_prepkv");
    G4B_REQUIRE(qkv && knw && cos_t && sin_t && kc && vc && pos_dev, G4B_E_ARG, "attn_prepkv: NULL pointer");
    G4B_REQUIRE(dtype == G4B_DT_F32 || dtype == G4B_DT_F16, G4B_E_ARG, "attn_prepkv: bad dtype %d", dtype);
    G4B_REQUIRE(nkv >= 1 && (hd == 128 || hd == 256 || hd == 512) && stride >= 1 && window >= 0 &&
                    window <= stride && koff >= 0 && voff >= 0,
                G4B_E_SHAPE, "attn_prepkv: nkv=%d hd=%d (128/256/512) stride=%d window=%d koff=%d voff=%d", nkv, hd,
                stride, window, koff, voff);
    int st = check_device(nullptr);
    if (st != G4B_OK) return st;
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    const int vo = keqv ? koff : voff;
    if (dtype == G4B_DT_F32)
        attn_prepkv_kernel<true><<<nkv, kAttnThreads, 0, s>>>(qkv, knw, cos_t, sin_t, kc, vc, hd, koff, vo, stride,
                                                              window, pos_dev);
    else
        attn_prepkv_kernel<false><<<nkv, kAttnThreads, 0, s>>>(qkv, knw, cos_t, sin_t, kc, vc, hd, koff, vo, stride,
                                                               window, pos_dev);
    count_launch();
    return launch_status("attn_prepkv");
}

size_t g4b_attn_workspace_bytes(int nH, int nkv, int hd, int max_T) {
    if (nH <= 0 || nkv <= 0 || hd <= 0 || max_T <= 0) return 0;
    int sms = 148;
    if (check_device(&sms) != G4B_OK) sms = 148;
    clear_error();
    const int S = attn_splits(nkv, max_T, sms);
    if (S == 1) return 0;
    return (size_t)nH * S * (hd + 2) * sizeof(float);
}

int g4b_attn_decode(const void* qkv, int dtype, const float* qnw, const float* cos_t, const float* sin_t,
                    const uint16_t* kc, const uint16_t* vc, void* out, int out_dtype, int nH, int nkv, int hd,
                    int qoff, int stride, int window, const int* pos_dev, void* workspace, size_t ws_bytes,
                    g4b_stream_t stream) {
    G4B_ENTRY("attn_decode");
    G4B_REQUIRE(qkv && qnw && cos_t && sin_t && kc && vc && out && pos_dev, G4B_E_ARG, "attn_decode: NULL pointer");
    G4B_REQUIRE(dtype == G4B_DT_F32 || dtype == G4B_DT_F16, G4B_E_ARG, "attn_decode: bad dtype %d", dtype);
    G4B_REQUIRE(out_dtype == G4B_DT_F32 || out_dtype == G4B_DT_F16, G4B_E_ARG, "attn_decode: bad out_dtype %d",
                out_dtype);
    G4B_REQUIRE(nkv >= 1 && nH >= nkv && nH % nkv == 0 && stride >= 1 && window >= 0 && window <= stride && qoff >= 0,
                G4B_E_SHAPE, "attn_decode: nH=%d nkv=%d stride=%d window=%d", nH, nkv, stride, window);
    const int G = nH / nkv;
    G4B_REQUIRE(attn_shape_ok(hd, G), G4B_E_SHAPE,
                "attn_decode: hd=%d with %d query heads per KV head (hd 128: 1-8, hd 256: 1-4, hd 512: 1-2)", hd,
                G);
    const bool xf32 = dtype == G4B_DT_F32;
    const size_t esz = xf32 ? 4 : 2;
    G4B_REQUIRE(aligned16(kc) && aligned16(vc) && aligned16((const char*)qkv + (size_t)qoff * esz) && aligned16(out),
                G4B_E_ALIGN, "attn_decode: qkv + qoff, the caches and out must be 16-byte aligned");
    int sms = 148;
    int st = check_device(&sms);
    if (st != G4B_OK) return st;
    const int max_T = window > 0 ? window : stride;
    const int S = attn_splits(nkv, max_T, sms);
    const size_t need = S == 1 ? 0 : (size_t)nH * S * (hd + 2) * sizeof(float);
    G4B_REQUIRE(ws_bytes >= need && (need == 0 || (workspace && aligned16(workspace))), G4B_E_WORKSPACE,
                "attn_decode: needs a 16-byte aligned workspace of %zu bytes, got %zu", need, ws_bytes);
    AttnArgs a{};
    a.qkv = qkv;
    a.qnw = qnw;
    a.cos_t = cos_t;
    a.sin_t = sin_t;
    a.kc = kc;
    a.vc = vc;
    a.out = out;
    a.part = S > 1 ? reinterpret_cast<float*>(workspace) : nullptr;
    a.pml = S > 1 ? reinterpret_cast<float*>(workspace) + (size_t)nH * S * hd : nullptr;
    a.pos_dev = pos_dev;
    a.nH = nH;
    a.nkv = nkv;
    a.hd = hd;
    a.qoff = qoff;
    a.stride = stride;
    a.window = window;
    a.S = S;
    a.out_f32 = out_dtype == G4B_DT_F32;
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    cudaError_t e = hd == 128 ? launch_decode_g<4>(a, G, xf32, s)
                  : hd == 256 ? launch_decode_g<8>(a, G, xf32, s)
                              : launch_decode_g<16>(a, G, xf32, s);
    if (e != cudaSuccess) return fail(G4B_E_CUDA, "attn_decode: launch: %s", cudaGetErrorString(e));
    count_launch();
    if (S > 1) {
        attn_combine_kernel<<<nH, kAttnThreads, (size_t)S * sizeof(float), s>>>(a);
        count_launch();
    }
    return launch_status("attn_decode");
}

}  // extern "C"
