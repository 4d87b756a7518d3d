// g4b_attn.cu -- attention over the f16 KV cache: the engine's prepkv and attn
// dispatches (vk/prepkv.comp, vk/attn.comp), recorded per layer between the q|k|v and
// o GEMVs (src/vk_engine.py:281-282), and their prefill forms (vk/pre_prepkv.comp,
// vk/pre_attn.comp; src/vk_engine.py:416-417).
//
//   prepkv  one CTA per (KV head, token): k = RoPE(rmsnorm(k, knw)), v = v * rsqrt(mean(v^2)
//           + eps), both stored as f16 at the token's cache slot (a ring of `window` slots
//           for sliding layers).
//   decode  flash decoding: grid (splits, KV heads).  A CTA normalises and rotates the
//           query heads that share its KV head (GQA), then its 8 warps stream their
//           share of the split's keys -- each K and V row is read once for all those
//           heads, 16-byte loads per lane, 4 keys in flight per warp -- with an online
//           softmax per warp; the warps' partials merge in shared memory, a split's (max,
//           sum, weighted V) goes to the workspace, and the last split of a KV head to
//           finish combines them.  HBM-bound on the cache: T * hd * 2 bytes of K and of V
//           per KV head.
//
//   prefill causal attention of a chunk of M tokens, flash-attention style on the tensor
//           cores (mma.sync m16n8k16, f32 accumulate): a CTA takes 64-128 (token, query
//           head) rows of one KV head -- the heads that share a KV head share its K and V
//           tiles -- and streams the key tiles through shared memory (cp.async, double
//           buffered).  The normed, rotated q and the softmax weights p enter the MMAs as
//           f16 hi + lo pairs, so scores and weighted sums keep about 21 bits.
//
// The token position (the chunk's first, for prefill) is read from device memory, so
// one captured graph serves every token; the decode split count is fixed on the host
// from the cache's capacity, and splits beyond the live keys finish at once.
#include <algorithm>

#include "g4b_common.cuh"

namespace g4b {

constexpr int kAttnThreads = 256;
constexpr int kAttnWarps = kAttnThreads / 32;
constexpr float kAttnEps = 1e-6f;     // vk/attn.comp:25, vk/prepkv.comp:21
constexpr float kNegInit = -1e30f;    // the shaders' running-max start (vk/attn.comp:29)
constexpr int kAttnMaxSplits = 64;    // key splits per KV head (the last split combines them from shared memory)

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
// One KV head of one token, by a CTA of kAttnThreads threads (thread t owns elements t and t + 256;
// hd <= 512): k = RoPE(rmsnorm(k, knw)) and v = rmsnorm(v) as f16 into slot `slot` of kc / vc
// (vk/prepkv.comp:18-29, vk/pre_prepkv.comp:20-30).  rb is the head's offset into the kin / vin rows.
template <bool XF32>
__device__ __forceinline__ void prep_head(const void* kin, const void* vin, size_t rb, const float* __restrict__ knw,
                                          const float* __restrict__ cb, const float* __restrict__ sb, uint16_t* kc,
                                          uint16_t* vc, int h, int hd, int stride, int slot, float* hv, float* wsum) {
    const int t = threadIdx.x, lane = t & 31, warp = t >> 5, hf = hd / 2;
    auto elem = [&](const void* base, int i) -> float {
        return XF32 ? __ldg(reinterpret_cast<const float*>(base) + rb + i)
                    : __half2float(__ldg(reinterpret_cast<const __half*>(base) + rb + i));
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
    float s = 0.f;
    for (int i = t; i < hd; i += kAttnThreads) {
        const float v = elem(kin, i);
        hv[i] = v;
        s += v * v;
    }
    const float ik = inv_rms(s);
    for (int i = t; i < hd; i += kAttnThreads) hv[i] = hv[i] * ik * __ldg(knw + i);
    __syncthreads();
    uint16_t* krow = kc + ((size_t)h * stride + slot) * hd;
    for (int i = t; i < hd; i += kAttnThreads) {
        const float rh = i < hf ? -hv[i + hf] : hv[i - hf];
        krow[i] = __half_as_ushort(__float2half_rn(hv[i] * __ldg(cb + i) + rh * __ldg(sb + i)));
    }
    s = 0.f;
    float vv[2] = {0.f, 0.f};
    for (int i = t, n = 0; i < hd; i += kAttnThreads, n++) {
        vv[n] = elem(vin, i);
        s += vv[n] * vv[n];
    }
    const float iv = inv_rms(s);
    uint16_t* vrow = vc + ((size_t)h * stride + slot) * hd;
    for (int i = t, n = 0; i < hd; i += kAttnThreads, n++) vrow[i] = __half_as_ushort(__float2half_rn(vv[n] * iv));
}

// One CTA per (KV head, token m).  Token m's k and v rows are row_stride elements after token m-1's;
// its cos / sin row is cs_stride floats after (0: one shared row, the decode token); its position is
// pos_dev[0] + m.  k = v passes vin = kin.
template <bool XF32>
__global__ void __launch_bounds__(kAttnThreads) attn_prepkv_kernel(const void* __restrict__ kin,
                                                                  const void* __restrict__ vin, int row_stride,
                                                                  const float* __restrict__ knw,
                                                                  const float* __restrict__ cos_t,
                                                                  const float* __restrict__ sin_t, int cs_stride,
                                                                  uint16_t* kc, uint16_t* vc, int hd, int stride,
                                                                  int window, const int* __restrict__ pos_dev) {
    __shared__ float hv[512];
    __shared__ float wsum[kAttnWarps];
    const int h = blockIdx.x, m = blockIdx.y;
    const int pos = __ldg(pos_dev) + m;
    const int slot = window > 0 ? pos % window : pos;
    if (slot >= stride) return;   // past the cache (the host checks what it can; the position is on the device)
    // a chunk longer than the ring writes some slots twice: the later token's write is the one that stays
    if (window > 0 && m + window < (int)gridDim.y) return;
    prep_head<XF32>(kin, vin, (size_t)m * row_stride + (size_t)h * hd, knw, cos_t + (size_t)m * cs_stride,
                    sin_t + (size_t)m * cs_stride, kc, vc, h, hd, stride, slot, hv, wsum);
}

// ------------------------------------------------------------------ decode
struct AttnArgs {
    const void* qkv;
    const float* qnw;
    const float* knw;    // PREP: the k norm weight
    int koff, voff;      // PREP: k and v in qkv (voff = koff for k = v)
    const float* cos_t;
    const float* sin_t;
    const uint16_t* kc;
    const uint16_t* vc;
    void* out;           // S == 1: [nH, hd] output
    float* part;         // S > 1: [nH][S][hd] weighted V sums
    float* pml;          // S > 1: [nH][S][2] (running max, sum)
    unsigned* arrive;    // S > 1: [nkv] split arrival counters, zero between calls
    const int* pos_dev;
    int nH, nkv, hd, qoff, stride, window, S, out_f32;
};

// n f16 values of a cache row as n / 2 packed pairs (streamed: the cache is read once per token)
template <int N>
__device__ __forceinline__ void load_pairs(const uint16_t* p, uint32_t (&w)[N / 2]) {
    if constexpr (N == 4) {
        const uint2 u = __ldcs(reinterpret_cast<const uint2*>(p));
        w[0] = u.x; w[1] = u.y;
    } else {
        #pragma unroll
        for (int j = 0; j < N / 8; j++) {
            const uint4 u = __ldcs(reinterpret_cast<const uint4*>(p) + j);
            w[4 * j] = u.x; w[4 * j + 1] = u.y; w[4 * j + 2] = u.z; w[4 * j + 3] = u.w;
        }
    }
}

// D = hd / 32 values per lane, G = query heads per KV head; PREP: the CTA whose split holds this
// token's slot first writes the token's k / v there (prepkv fused in: the engine's two dispatches in
// one launch)
template <int D, int G, bool XF32, bool PREP>
__global__ void __launch_bounds__(kAttnThreads, 2) attn_decode_kernel(const AttnArgs a) {
    constexpr int HD = 32 * D;
    constexpr int KB = D >= 16 ? 2 : 4;   // keys a warp loads at once (4 KB in flight per warp at hd 256)
    constexpr int DW = D / 2;
    static_assert(G * D <= 32, "query heads x values per lane held in registers");
    __shared__ float xacc[kAttnWarps][G][HD];   // every warp's partial, merged by all threads
    __shared__ float xm[kAttnWarps][G], xl[kAttnWarps][G];
    const int s = blockIdx.x, kvh = blockIdx.y, t = threadIdx.x, lane = t & 31, warp = t >> 5;
    // launched as a programmatic dependent: scheduled while the kernel before it (the chain that wrote
    // q|k|v) finishes; nothing is read before that kernel has completed
    pdl_launch_dependents();
    pdl_wait();
    const int pos = __ldg(a.pos_dev);
    const int T = min(a.window > 0 ? min(pos + 1, a.window) : pos + 1, a.stride);   // never past the cache
    const int k0 = (int)((long long)s * T / a.S), k1 = (int)((long long)(s + 1) * T / a.S);
    const size_t row0 = (size_t)kvh * a.stride;
    if constexpr (PREP) {
        __shared__ float hv[512];
        __shared__ float wsum[kAttnWarps];
        const int slot = a.window > 0 ? pos % a.window : pos;
        if (slot >= k0 && slot < k1) {   // the same for every thread of the CTA
            const size_t esz = XF32 ? 4 : 2;
            prep_head<XF32>(reinterpret_cast<const char*>(a.qkv) + (size_t)a.koff * esz,
                            reinterpret_cast<const char*>(a.qkv) + (size_t)a.voff * esz, (size_t)kvh * HD, a.knw,
                            a.cos_t, a.sin_t, const_cast<uint16_t*>(a.kc), const_cast<uint16_t*>(a.vc), kvh, HD,
                            a.stride, slot, hv, wsum);
            __syncthreads();   // the new row is read below by other warps of this CTA
        }
    }
    // the query heads of this KV head: rmsnorm with qnw, then RoPE (vk/attn.comp:22-28); every warp
    // makes its own copy (element i's rotation partner i +- hd/2 is in lane ^ 16)
    float q[G][D];
    #pragma unroll
    for (int g = 0; g < G; g++) {
        float v[D];
        loadn<D, XF32>(a.qkv, (size_t)a.qoff + (size_t)(kvh * G + g) * HD + lane * D, v);
        float ss = 0.f;
        #pragma unroll
        for (int d = 0; d < D; d++) ss += v[d] * v[d];
        const float iq = rsqrtf(warp_sum(ss) / (float)HD + kAttnEps);
        #pragma unroll
        for (int d = 0; d < D; d++) {
            const int i = lane * D + d;
            const float nv = v[d] * iq * __ldg(a.qnw + i);
            const float pv = __shfl_xor_sync(0xffffffffu, nv, 16);
            q[g][d] = nv * __ldg(a.cos_t + i) + (lane < 16 ? -pv : pv) * __ldg(a.sin_t + i);
        }
    }
    // this warp's keys, KB at a time: an online softmax per query head
    float m[G], l[G], acc[G][D];
    #pragma unroll
    for (int g = 0; g < G; g++) {
        m[g] = kNegInit;
        l[g] = 0.f;
        #pragma unroll
        for (int d = 0; d < D; d++) acc[g][d] = 0.f;
    }
    const uint16_t* kbase = a.kc + row0 * HD + lane * D;
    const uint16_t* vbase = a.vc + row0 * HD + lane * D;
    for (int j0 = k0 + warp * KB; j0 < k1; j0 += kAttnWarps * KB) {
        uint32_t kr[KB][DW], vr[KB][DW];
        #pragma unroll
        for (int u = 0; u < KB; u++) {
            const size_t j = (size_t)min(j0 + u, k1 - 1);   // past the split: a repeat, weighted 0 below
            load_pairs<D>(kbase + j * HD, kr[u]);
            load_pairs<D>(vbase + j * HD, vr[u]);
        }
        float dot[G][KB];
        #pragma unroll
        for (int g = 0; g < G; g++)
            #pragma unroll
            for (int u = 0; u < KB; u++) {
                float x = 0.f;
                #pragma unroll
                for (int w = 0; w < DW; w++) {
                    x = fmaf(q[g][2 * w], h_lo(kr[u][w]), x);
                    x = fmaf(q[g][2 * w + 1], h_hi(kr[u][w]), x);
                }
                dot[g][u] = x;
            }
        #pragma unroll
        for (int mk = 16; mk >= 1; mk >>= 1)
            #pragma unroll
            for (int g = 0; g < G; g++)
                #pragma unroll
                for (int u = 0; u < KB; u++) dot[g][u] += __shfl_xor_sync(0xffffffffu, dot[g][u], mk);
        #pragma unroll
        for (int g = 0; g < G; g++) {
            float mx = m[g];
            #pragma unroll
            for (int u = 0; u < KB; u++)
                if (j0 + u < k1) mx = fmaxf(mx, dot[g][u]);
            const float corr = __expf(m[g] - mx);
            float p[KB], ps = 0.f;
            #pragma unroll
            for (int u = 0; u < KB; u++) {
                p[u] = j0 + u < k1 ? __expf(dot[g][u] - mx) : 0.f;
                ps += p[u];
            }
            l[g] = l[g] * corr + ps;
            m[g] = mx;
            #pragma unroll
            for (int w = 0; w < DW; w++) {
                float a0 = acc[g][2 * w] * corr, a1 = acc[g][2 * w + 1] * corr;
                #pragma unroll
                for (int u = 0; u < KB; u++) {
                    a0 = fmaf(p[u], h_lo(vr[u][w]), a0);
                    a1 = fmaf(p[u], h_hi(vr[u][w]), a1);
                }
                acc[g][2 * w] = a0;
                acc[g][2 * w + 1] = a1;
            }
        }
    }
    // merge the 8 warps' partials: each thread rescales and sums a few (head, element) values
    #pragma unroll
    for (int g = 0; g < G; g++) {
        if (lane == 0) {
            xm[warp][g] = m[g];
            xl[warp][g] = l[g];
        }
        #pragma unroll
        for (int d = 0; d < D; d++) xacc[warp][g][lane * D + d] = acc[g][d];
    }
    __syncthreads();
    for (int e = t; e < G * HD; e += kAttnThreads) {
        const int g = e / HD, i = e % HD, h = kvh * G + g;
        float M = kNegInit;
        #pragma unroll
        for (int w = 0; w < kAttnWarps; w++) M = fmaxf(M, xm[w][g]);
        float L = 0.f, V = 0.f;
        #pragma unroll
        for (int w = 0; w < kAttnWarps; w++) {
            const float ew = __expf(xm[w][g] - M);
            L = fmaf(xl[w][g], ew, L);
            V = fmaf(xacc[w][g][i], ew, V);
        }
        if (a.S == 1) {
            const float o = V / L;
            if (a.out_f32) reinterpret_cast<float*>(a.out)[(size_t)h * HD + i] = o;
            else reinterpret_cast<__half*>(a.out)[(size_t)h * HD + i] = __float2half_rn(o);
        } else {
            a.part[((size_t)h * a.S + s) * HD + i] = V;
            if (i == 0) {
                a.pml[((size_t)h * a.S + s) * 2] = M;
                a.pml[((size_t)h * a.S + s) * 2 + 1] = L;
            }
        }
    }
    if (a.S == 1) return;
    // the last split of this KV head to arrive combines all of them:
    //   out = sum_s v_s e^(m_s - M) / sum_s l_s e^(m_s - M)
    // (atomicInc wraps the counter back to zero for the next call)
    __shared__ unsigned s_last;
    __threadfence();
    __syncthreads();
    if (t == 0) s_last = atomicInc(a.arrive + kvh, (unsigned)(a.S - 1)) == (unsigned)(a.S - 1);
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    // warp g: head g's split weights e^(m_s - M) / L into shared memory (one round trip for the (m, l)s)
    __shared__ float s_w[G][kAttnMaxSplits];
    if (warp < G) {
        const float2* pm = reinterpret_cast<const float2*>(a.pml) + (size_t)(kvh * G + warp) * a.S;
        float2 v[kAttnMaxSplits / 32];
        float M = kNegInit;
        #pragma unroll
        for (int r = 0; r < kAttnMaxSplits / 32; r++) {
            const int k = lane + 32 * r;
            v[r] = k < a.S ? __ldcg(pm + k) : make_float2(kNegInit, 0.f);
            M = fmaxf(M, v[r].x);
        }
        #pragma unroll
        for (int mk = 16; mk >= 1; mk >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, mk));
        float L = 0.f;
        #pragma unroll
        for (int r = 0; r < kAttnMaxSplits / 32; r++) {
            v[r].x = __expf(v[r].x - M);
            L = fmaf(v[r].y, v[r].x, L);
        }
        const float invL = 1.0f / warp_sum(L);
        #pragma unroll
        for (int r = 0; r < kAttnMaxSplits / 32; r++)
            if (lane + 32 * r < a.S) s_w[warp][lane + 32 * r] = v[r].x * invL;
    }
    __syncthreads();
    for (int e = t; e < G * HD; e += kAttnThreads) {
        const int g = e / HD, i = e % HD, h = kvh * G + g;
        const float* pp = a.part + (size_t)h * a.S * HD + i;
        float V = 0.f;
        #pragma unroll 8
        for (int k = 0; k < a.S; k++) V = fmaf(__ldcg(pp + (size_t)k * HD), s_w[g][k], V);
        if (a.out_f32) reinterpret_cast<float*>(a.out)[(size_t)h * HD + i] = V;
        else reinterpret_cast<__half*>(a.out)[(size_t)h * HD + i] = __float2half_rn(V);
    }
}

// the workspace's arrival counters (one per KV head), ahead of the partials
static size_t attn_ws_counters(int nkv) { return ((size_t)nkv * sizeof(unsigned) + 255) / 256 * 256; }

// splits of the keys: about two CTAs per SM over the KV heads, at least 32 keys per split
static int attn_splits(int nkv, int max_T, int sms) {
    const int by_keys = (max_T + 31) / 32;
    const int by_sms = std::max(1, 2 * sms / std::max(nkv, 1));
    return std::max(1, std::min(std::min(by_keys, by_sms), kAttnMaxSplits));
}

// as a programmatic dependent of the previous kernel (the kernel waits for it before reading anything)
template <int D, int G, bool PREP>
static cudaError_t launch_decode(const AttnArgs& a, bool xf32, cudaStream_t s) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(a.S, a.nkv);
    cfg.blockDim = dim3(kAttnThreads);
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return xf32 ? cudaLaunchKernelEx(&cfg, attn_decode_kernel<D, G, true, PREP>, a)
                : cudaLaunchKernelEx(&cfg, attn_decode_kernel<D, G, false, PREP>, a);
}

template <int D, bool PREP>
static cudaError_t launch_decode_g(const AttnArgs& a, int G, bool xf32, cudaStream_t s) {
    switch (G) {
        case 1: return launch_decode<D, 1, PREP>(a, xf32, s);
        case 2: return launch_decode<D, 2, PREP>(a, xf32, s);
        case 4: return launch_decode<D, (D <= 8 ? 4 : 2), PREP>(a, xf32, s);   // G * D <= 32 (checked by the caller)
        default: return launch_decode<D, (D <= 4 ? 8 : 2), PREP>(a, xf32, s);
    }
}

template <bool PREP>
static cudaError_t launch_decode_hd(const AttnArgs& a, int G, bool xf32, cudaStream_t s) {
    return a.hd == 128 ? launch_decode_g<4, PREP>(a, G, xf32, s)
         : a.hd == 256 ? launch_decode_g<8, PREP>(a, G, xf32, s)
                       : launch_decode_g<16, PREP>(a, G, xf32, s);
}

// the (hd, query heads per KV head) pairs with an instance: G * hd / 32 <= 32 values per lane
// (hd 128: G 1-8; hd 256: G 1-4; hd 512: G 1-2), G a power of two
static bool attn_shape_ok(int hd, int G) {
    const bool g_ok = G == 1 || G == 2 || G == 4 || G == 8;
    return (hd == 128 || hd == 256 || hd == 512) && g_ok && G * (hd / 32) <= 32;
}


// ------------------------------------------------------------------ prefill attention
namespace pf {

// D = A(16x16 f16) * B(16x8 f16) + D, f32 accumulate (a register-only op, free to schedule)
__device__ __forceinline__ void mma(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void ldsm4(uint32_t addr, uint32_t (&r)[4]) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr));
}
__device__ __forceinline__ void ldsm4t(uint32_t addr, uint32_t (&r)[4]) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr));
}
// 16 bytes global -> shared; src-size 0 writes zeros (rows past the live keys)
__device__ __forceinline__ void cp16(uint32_t dst, const void* src, bool valid) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(valid ? 16 : 0)
                 : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// x, y as f16 (hi) and their remainders as f16 (lo): hi + lo carries ~21 bits of each
__device__ __forceinline__ void split2(float x, float y, uint32_t& hi, uint32_t& lo) {
    const __half xh = __float2half_rn(x), yh = __float2half_rn(y);
    hi = pack_half2(xh, yh);
    lo = pack_half2(__float2half_rn(x - __half2float(xh)), __float2half_rn(y - __half2float(yh)));
}

// HD head_dim; NRW warps of 16 rows; CS warps split the output columns (each computes the scores);
// BK keys per tile
template <int HD, int NRW, int CS, int BK>
struct Cfg {
    static constexpr int BQ = 16 * NRW;          // (token, head) rows per CTA
    static constexpr int NW = NRW * CS;
    static constexpr int THREADS = 32 * NW;
    static constexpr int OC = HD / CS;           // output columns per warp
    static constexpr int RB = HD * 2;            // bytes per shared-memory row
    static constexpr int CH = HD / 8;            // 16-byte chunks per row
    static constexpr int Q_BYTES = BQ * RB;      // the hi (or the lo) q tile
    static constexpr int KV_BYTES = BK * RB;     // one K (or V) tile
    static constexpr int SMEM = 2 * Q_BYTES + 4 * KV_BYTES;
    static_assert(HD % 64 == 0 && BK % 16 == 0 && OC % 16 == 0, "tile shapes");
};

// row r, 16-byte chunk c of a tile: chunk c of each row moves to c ^ (r % 8), so the 8 rows an ldmatrix
// reads at one logical chunk sit in 8 different bank groups
__device__ __forceinline__ uint32_t swz(int r, int c, int rb) {
    return (uint32_t)(r * rb + ((c ^ (r & 7)) << 4));
}

}  // namespace pf

struct PrefillArgs {
    const void* q;        // [M, q_stride]: head h of token m at m * q_stride + h * hd
    const float* qnw;
    const float* cosM;    // [M, hd]
    const float* sinM;
    const uint16_t* kc;   // [nkv, stride, hd]
    const uint16_t* vc;
    void* out;            // [M, out_stride]
    const int* p0_dev;    // the chunk's first position
    int M, G, hd, q_stride, out_stride, stride, window, nqt, out_f32;
};

// grid (query tiles, KV heads).  Rows are (token, query head) pairs, row = m * G + g: the G heads of
// one KV head for consecutive tokens.  pre_attn.comp's arithmetic per (h, m): q normed and rotated at
// the token's own angles, scores over the keys 0 .. T-1 (T = pos + 1, or min(pos + 1, window)), keys
// whose absolute position on a sliding ring is after the token's excluded, online softmax, out = acc / l.
template <int HD, int NRW, int CS, int BK, bool XF32>
__global__ void __launch_bounds__(32 * NRW * CS, 1) attn_prefill_kernel(const PrefillArgs a) {
    using C = pf::Cfg<HD, NRW, CS, BK>;
    extern __shared__ __align__(128) uint8_t sm[];
    const uint32_t sQh = smem_u32(sm), sQl = sQh + C::Q_BYTES, sK = sQl + C::Q_BYTES, sV = sK + 2 * C::KV_BYTES;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int rw = warp % NRW, cs = warp / NRW;
    const int qt = a.nqt - 1 - (int)blockIdx.x;   // the latest tokens (most keys) first
    const int kvh = blockIdx.y, G = a.G;
    const int p0 = __ldg(a.p0_dev);
    const int row0 = qt * C::BQ;
    const int nrows = min(C::BQ, a.M * G - row0);
    auto keys_of = [&](int pos) {
        const int T = a.window > 0 ? min(pos + 1, a.window) : pos + 1;
        return max(0, min(T, a.stride));
    };
    const int T_max = keys_of(p0 + (row0 + nrows - 1) / G);
    const int ntiles = (T_max + BK - 1) / BK;
    const size_t kv0 = (size_t)kvh * a.stride;

    auto load_kv = [&](int t, int buf) {
        for (int i = tid; i < BK * C::CH; i += C::THREADS) {
            const int r = i / C::CH, c = i % C::CH, slot = t * BK + r;
            const bool valid = slot < T_max;
            const size_t src = (kv0 + (size_t)(valid ? slot : 0)) * HD + (size_t)c * 8;
            const uint32_t off = pf::swz(r, c, C::RB) + (uint32_t)(buf * C::KV_BYTES);
            pf::cp16(sK + off, a.kc + src, valid);
            pf::cp16(sV + off, a.vc + src, valid);
        }
        pf::cp_commit();
    };
    if (ntiles > 0) load_kv(0, 0);
    if (ntiles > 1) load_kv(1, 1);

    // ---- q: rmsnorm with qnw, RoPE at the token's angles (vk/pre_attn.comp:22-28), as f16 hi + lo
    {
        constexpr int PER = HD / 32;   // lane l holds elements l * PER .. l * PER + PER - 1
        for (int r = warp; r < C::BQ; r += C::NW) {
            const bool live = r < nrows;
            const int row = row0 + r, m = live ? row / G : 0, h = kvh * G + (live ? row % G : 0);
            float v[PER];
            if (live) loadn<PER, XF32>(a.q, (size_t)m * a.q_stride + (size_t)h * HD + (size_t)lane * PER, v);
            else {
                #pragma unroll
                for (int d = 0; d < PER; d++) v[d] = 0.f;
            }
            float ss = 0.f;
            #pragma unroll
            for (int d = 0; d < PER; d++) ss += v[d] * v[d];
            const float iq = rsqrtf(warp_sum(ss) / (float)HD + kAttnEps);
            float nv[PER];
            #pragma unroll
            for (int d = 0; d < PER; d++) nv[d] = v[d] * iq * __ldg(a.qnw + lane * PER + d);
            // element i's rotation partner i +- HD/2 is held by lane ^ 16
            const float* cb = a.cosM + (size_t)m * HD;
            const float* sb = a.sinM + (size_t)m * HD;
            uint32_t hi[PER / 2], lo[PER / 2];
            #pragma unroll
            for (int d = 0; d < PER; d += 2) {
                float x[2];
                #pragma unroll
                for (int e = 0; e < 2; e++) {
                    const int i = lane * PER + d + e;
                    const float pv = __shfl_xor_sync(0xffffffffu, nv[d + e], 16);
                    const float rh = lane < 16 ? -pv : pv;
                    x[e] = live ? nv[d + e] * __ldg(cb + i) + rh * __ldg(sb + i) : 0.f;
                }
                pf::split2(x[0], x[1], hi[d / 2], lo[d / 2]);
            }
            // PER halves = PER / 8 chunks (PER = 4: half a chunk)
            if constexpr (PER >= 8) {
                #pragma unroll
                for (int cc = 0; cc < PER / 8; cc++) {
                    const uint32_t off = pf::swz(r, lane * (PER / 8) + cc, C::RB);
                    asm volatile("st.shared.v4.b32 [%0], {%1,%2,%3,%4};" ::"r"(sQh + off), "r"(hi[4 * cc]),
                                 "r"(hi[4 * cc + 1]), "r"(hi[4 * cc + 2]), "r"(hi[4 * cc + 3]));
                    asm volatile("st.shared.v4.b32 [%0], {%1,%2,%3,%4};" ::"r"(sQl + off), "r"(lo[4 * cc]),
                                 "r"(lo[4 * cc + 1]), "r"(lo[4 * cc + 2]), "r"(lo[4 * cc + 3]));
                }
            } else {
                const uint32_t off = pf::swz(r, lane >> 1, C::RB) + (uint32_t)((lane & 1) * 8);
                asm volatile("st.shared.v2.b32 [%0], {%1,%2};" ::"r"(sQh + off), "r"(hi[0]), "r"(hi[1]));
                asm volatile("st.shared.v2.b32 [%0], {%1,%2};" ::"r"(sQl + off), "r"(lo[0]), "r"(lo[1]));
            }
        }
    }

    // this lane's two rows of its warp's 16: g and g + 8
    const int g = lane >> 2, q4 = lane & 3;
    int posr[2], Tr[2];
    #pragma unroll
    for (int i = 0; i < 2; i++) {
        const int r = rw * 16 + g + 8 * i;
        const bool live = r < nrows;
        posr[i] = p0 + (live ? (row0 + r) / G : 0);
        Tr[i] = live ? keys_of(posr[i]) : 0;
    }
    const long long base = (long long)p0 + a.M - 1;   // the chunk's last position: every chunk key is written
    float o[C::OC / 8][4];
    #pragma unroll
    for (int n = 0; n < C::OC / 8; n++) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
    float mrow[2] = {kNegInit, kNegInit}, lrow[2] = {0.f, 0.f};

    for (int t = 0; t < ntiles; t++) {
        if (t + 1 < ntiles) pf::cp_wait<1>();
        else pf::cp_wait<0>();
        __syncthreads();
        const uint32_t kb = sK + (uint32_t)((t & 1) * C::KV_BYTES), vb = sV + (uint32_t)((t & 1) * C::KV_BYTES);
        // S = q K^T over the head dim (q as hi + lo)
        float s[BK / 8][4];
        #pragma unroll
        for (int n = 0; n < BK / 8; n++) s[n][0] = s[n][1] = s[n][2] = s[n][3] = 0.f;
        #pragma unroll 4
        for (int kk = 0; kk < HD / 16; kk++) {
            uint32_t ah[4], al[4];
            const int ar = rw * 16 + (lane & 7) + 8 * ((lane >> 3) & 1), ac = 2 * kk + (lane >> 4);
            pf::ldsm4(sQh + pf::swz(ar, ac, C::RB), ah);
            pf::ldsm4(sQl + pf::swz(ar, ac, C::RB), al);
            #pragma unroll
            for (int nt = 0; nt < BK / 8; nt += 2) {
                uint32_t b[4];
                const int br = nt * 8 + (lane & 7) + 8 * (lane >> 4), bc = 2 * kk + ((lane >> 3) & 1);
                pf::ldsm4(kb + pf::swz(br, bc, C::RB), b);
                pf::mma(s[nt], ah, b[0], b[1]);
                pf::mma(s[nt], al, b[0], b[1]);
                pf::mma(s[nt + 1], ah, b[2], b[3]);
                pf::mma(s[nt + 1], al, b[2], b[3]);
            }
        }
        // mask, then the online softmax (the row max over the quad's lanes).  Slots at or past the row's
        // T are not keys at all (-inf: weight 0 always); a ring slot holding a later position scores
        // -1e30 as in the shader, so a row whose every key is such a slot gets the shader's result (equal
        // weights over them) and any real key wipes them (its corr is exp(-1e30 - s) = 0)
        float mx[2] = {-INFINITY, -INFINITY};
        #pragma unroll
        for (int nt = 0; nt < BK / 8; nt++)
            #pragma unroll
            for (int e = 0; e < 4; e++) {
                const int i = e >> 1, key = t * BK + nt * 8 + 2 * q4 + (e & 1);
                if (key >= Tr[i]) {
                    s[nt][e] = -INFINITY;
                } else if (a.window > 0) {
                    const long long posn = base - ((base + a.window - key) % a.window);
                    if (posn > posr[i]) s[nt][e] = kNegInit;
                }
                mx[i] = fmaxf(mx[i], s[nt][e]);
            }
        float corr[2];
        #pragma unroll
        for (int i = 0; i < 2; i++) {
            mx[i] = fmaxf(mx[i], __shfl_xor_sync(0xffffffffu, mx[i], 1));
            mx[i] = fmaxf(mx[i], __shfl_xor_sync(0xffffffffu, mx[i], 2));
            const float mn = fmaxf(mrow[i], mx[i]);
            corr[i] = __expf(mrow[i] - mn);
            mrow[i] = mn;
        }
        float ls[2] = {0.f, 0.f};
        #pragma unroll
        for (int nt = 0; nt < BK / 8; nt++)
            #pragma unroll
            for (int e = 0; e < 4; e++) {
                const float p = __expf(s[nt][e] - mrow[e >> 1]);
                s[nt][e] = p;
                ls[e >> 1] += p;
            }
        #pragma unroll
        for (int i = 0; i < 2; i++) lrow[i] = lrow[i] * corr[i] + ls[i];   // this lane's share of the row sum
        #pragma unroll
        for (int n = 0; n < C::OC / 8; n++) {
            o[n][0] *= corr[0];
            o[n][1] *= corr[0];
            o[n][2] *= corr[1];
            o[n][3] *= corr[1];
        }
        // O += P V over this warp's columns, 16 keys at a time (p as hi + lo A fragments)
        #pragma unroll
        for (int kb16 = 0; kb16 < BK / 16; kb16++) {
            uint32_t ph[4], pl[4];
            pf::split2(s[2 * kb16][0], s[2 * kb16][1], ph[0], pl[0]);
            pf::split2(s[2 * kb16][2], s[2 * kb16][3], ph[1], pl[1]);
            pf::split2(s[2 * kb16 + 1][0], s[2 * kb16 + 1][1], ph[2], pl[2]);
            pf::split2(s[2 * kb16 + 1][2], s[2 * kb16 + 1][3], ph[3], pl[3]);
            const int vr = kb16 * 16 + (lane & 7) + 8 * ((lane >> 3) & 1);
            #pragma unroll
            for (int nt = 0; nt < C::OC / 8; nt += 2) {
                uint32_t b[4];
                pf::ldsm4t(vb + pf::swz(vr, (cs * C::OC + nt * 8) / 8 + (lane >> 4), C::RB), b);
                pf::mma(o[nt], ph, b[0], b[1]);
                pf::mma(o[nt], pl, b[0], b[1]);
                pf::mma(o[nt + 1], ph, b[2], b[3]);
                pf::mma(o[nt + 1], pl, b[2], b[3]);
            }
        }
        __syncthreads();   // every warp is done with this buffer pair
        if (t + 2 < ntiles) load_kv(t + 2, t & 1);
    }

    // out = acc / l for the live rows
    #pragma unroll
    for (int i = 0; i < 2; i++) {
        float l = lrow[i];
        l += __shfl_xor_sync(0xffffffffu, l, 1);
        l += __shfl_xor_sync(0xffffffffu, l, 2);
        const int r = rw * 16 + g + 8 * i;
        if (r >= nrows) continue;
        const int row = row0 + r, m = row / G, h = kvh * G + row % G;
        const float inv = 1.0f / l;
        const size_t ob = (size_t)m * a.out_stride + (size_t)h * HD + (size_t)cs * C::OC + 2 * q4;
        #pragma unroll
        for (int n = 0; n < C::OC / 8; n++) {
            const float x0 = o[n][2 * i] * inv, x1 = o[n][2 * i + 1] * inv;
            if (a.out_f32) *reinterpret_cast<float2*>(reinterpret_cast<float*>(a.out) + ob + n * 8) = make_float2(x0, x1);
            else *reinterpret_cast<__half2*>(reinterpret_cast<__half*>(a.out) + ob + n * 8) = __floats2half2_rn(x0, x1);
        }
    }
}

template <int HD, int NRW, int CS, int BK>
static cudaError_t launch_prefill(const PrefillArgs& a, int nkv, bool xf32, cudaStream_t s) {
    using C = pf::Cfg<HD, NRW, CS, BK>;
    auto k = xf32 ? attn_prefill_kernel<HD, NRW, CS, BK, true> : attn_prefill_kernel<HD, NRW, CS, BK, false>;
    cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
    if (e != cudaSuccess) return e;
    k<<<dim3(a.nqt, nkv), C::THREADS, C::SMEM, s>>>(a);
    return cudaGetLastError();
}

// rows per CTA for each head_dim: hd 128: 64 rows, 64-key tiles (96 KB); hd 256: 128 rows, 32-key tiles
// (192 KB); hd 512: 64 rows with the columns split over two warps per row group, 16-key tiles (192 KB)
static int prefill_rows(int hd) { return hd == 256 ? 128 : 64; }

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
    const size_t esz = dtype == G4B_DT_F32 ? 4 : 2;
    const char* kin = reinterpret_cast<const char*>(qkv) + (size_t)koff * esz;
    const char* vin = reinterpret_cast<const char*>(qkv) + (size_t)(keqv ? koff : voff) * esz;
    if (dtype == G4B_DT_F32)
        attn_prepkv_kernel<true><<<dim3(nkv, 1), kAttnThreads, 0, s>>>(kin, vin, 0, knw, cos_t, sin_t, 0, kc, vc, hd,
                                                                       stride, window, pos_dev);
    else
        attn_prepkv_kernel<false><<<dim3(nkv, 1), kAttnThreads, 0, s>>>(kin, vin, 0, knw, cos_t, sin_t, 0, kc, vc, hd,
                                                                        stride, window, pos_dev);
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
    return attn_ws_counters(nkv) + (size_t)nH * S * (hd + 2) * sizeof(float);
}

}  // extern "C"

// g4b_attn_decode and g4b_attn_decode_prepkv: the checks and the launches; knw != nullptr fuses prepkv
static int attn_decode_impl(const char* op, const void* qkv, int dtype, const float* qnw, const float* knw,
                            const float* cos_t, const float* sin_t, const uint16_t* kc, const uint16_t* vc, void* out,
                            int out_dtype, int nH, int nkv, int hd, int qoff, int koff, int voff, int keqv, int stride,
                            int window, const int* pos_dev, void* workspace, size_t ws_bytes, g4b_stream_t stream) {
    G4B_REQUIRE(qkv && qnw && cos_t && sin_t && kc && vc && out && pos_dev, G4B_E_ARG, "%s: NULL pointer", op);
    G4B_REQUIRE(dtype == G4B_DT_F32 || dtype == G4B_DT_F16, G4B_E_ARG, "%s: bad dtype %d", op, dtype);
    G4B_REQUIRE(out_dtype == G4B_DT_F32 || out_dtype == G4B_DT_F16, G4B_E_ARG, "%s: bad out_dtype %d", op,
                out_dtype);
    G4B_REQUIRE(nkv >= 1 && nH >= nkv && nH % nkv == 0 && stride >= 1 && window >= 0 && window <= stride && qoff >= 0 &&
                    koff >= 0 && voff >= 0,
                G4B_E_SHAPE, "%s: nH=%d nkv=%d stride=%d window=%d", op, nH, nkv, stride, window);
    const int G = nH / nkv;
    G4B_REQUIRE(attn_shape_ok(hd, G), G4B_E_SHAPE,
                "%s: hd=%d with %d query heads per KV head (hd 128: 1-8, hd 256: 1-4, hd 512: 1-2)", op, hd, G);
    const bool xf32 = dtype == G4B_DT_F32;
    const size_t esz = xf32 ? 4 : 2;
    G4B_REQUIRE(aligned16(kc) && aligned16(vc) && aligned16((const char*)qkv + (size_t)qoff * esz) && aligned16(out),
                G4B_E_ALIGN, "%s: qkv + qoff, the caches and out must be 16-byte aligned", op);
    int sms = 148;
    int st = check_device(&sms);
    if (st != G4B_OK) return st;
    const int max_T = window > 0 ? window : stride;
    const int S = attn_splits(nkv, max_T, sms);
    const size_t cbytes = attn_ws_counters(nkv);
    const size_t need = S == 1 ? 0 : cbytes + (size_t)nH * S * (hd + 2) * sizeof(float);
    G4B_REQUIRE(ws_bytes >= need && (need == 0 || (workspace && aligned16(workspace))), G4B_E_WORKSPACE,
                "%s: needs a 16-byte aligned, zero-initialised workspace of %zu bytes, got %zu", op, need, ws_bytes);
    AttnArgs a{};
    a.qkv = qkv;
    a.qnw = qnw;
    a.knw = knw;
    a.koff = koff;
    a.voff = keqv ? koff : voff;
    a.cos_t = cos_t;
    a.sin_t = sin_t;
    a.kc = kc;
    a.vc = vc;
    a.out = out;
    char* wsb = reinterpret_cast<char*>(workspace);
    a.arrive = S > 1 ? reinterpret_cast<unsigned*>(wsb) : nullptr;
    a.part = S > 1 ? reinterpret_cast<float*>(wsb + cbytes) : nullptr;
    a.pml = S > 1 ? reinterpret_cast<float*>(wsb + cbytes) + (size_t)nH * S * hd : nullptr;
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
    cudaError_t e = knw ? launch_decode_hd<true>(a, G, xf32, s) : launch_decode_hd<false>(a, G, xf32, s);
    if (e != cudaSuccess) return fail(G4B_E_CUDA, "%s: launch: %s", op, cudaGetErrorString(e));
    count_launch();
    return launch_status(op);
}

extern "C" {

int g4b_attn_decode(const void* qkv, int dtype, const float* qnw, const float* cos_t, const float* sin_t,
                    const uint16_t* kc, const uint16_t* vc, void* out, int out_dtype, int nH, int nkv, int hd,
                    int qoff, int stride, int window, const int* pos_dev, void* workspace, size_t ws_bytes,
                    g4b_stream_t stream) {
    G4B_ENTRY("attn_decode");
    return attn_decode_impl("attn_decode", qkv, dtype, qnw, nullptr, cos_t, sin_t, kc, vc, out, out_dtype, nH, nkv, hd,
                            qoff, 0, 0, 0, stride, window, pos_dev, workspace, ws_bytes, stream);
}

int g4b_attn_decode_prepkv(const void* qkv, int dtype, const float* qnw, const float* knw, const float* cos_t,
                           const float* sin_t, uint16_t* kc, uint16_t* vc, void* out, int out_dtype, int nH, int nkv,
                           int hd, int qoff, int koff, int voff, int keqv, int stride, int window, const int* pos_dev,
                           void* workspace, size_t ws_bytes, g4b_stream_t stream) {
    G4B_ENTRY("attn_decode_prepkv");
    G4B_REQUIRE(knw, G4B_E_ARG, "attn_decode_prepkv: NULL knw");
    return attn_decode_impl("attn_decode_prepkv", qkv, dtype, qnw, knw, cos_t, sin_t, kc, vc, out, out_dtype, nH, nkv,
                            hd, qoff, koff, voff, keqv, stride, window, pos_dev, workspace, ws_bytes, stream);
}

int g4b_attn_prefill_prepkv(const void* k, const void* v, int dtype, int row_stride, int M, const float* knw,
                            const float* cosM, const float* sinM, uint16_t* kc, uint16_t* vc, int nkv, int hd,
                            int stride, int window, const int* p0_dev, g4b_stream_t stream) {
    G4B_ENTRY("attn_prefill_prepkv");
    G4B_REQUIRE(k && v && knw && cosM && sinM && kc && vc && p0_dev, G4B_E_ARG,
                "attn_prefill_prepkv: NULL pointer");
    G4B_REQUIRE(dtype == G4B_DT_F32 || dtype == G4B_DT_F16, G4B_E_ARG, "attn_prefill_prepkv: bad dtype %d", dtype);
    G4B_REQUIRE(M >= 1 && M <= 65535 && nkv >= 1 && (hd == 128 || hd == 256 || hd == 512) && stride >= 1 &&
                    window >= 0 && window <= stride && row_stride >= nkv * hd,
                G4B_E_SHAPE, "attn_prefill_prepkv: M=%d nkv=%d hd=%d (128/256/512) stride=%d window=%d row_stride=%d",
                M, nkv, hd, stride, window, row_stride);
    int st = check_device(nullptr);
    if (st != G4B_OK) return st;
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    if (dtype == G4B_DT_F32)
        attn_prepkv_kernel<true><<<dim3(nkv, M), kAttnThreads, 0, s>>>(k, v, row_stride, knw, cosM, sinM, hd, kc, vc,
                                                                       hd, stride, window, p0_dev);
    else
        attn_prepkv_kernel<false><<<dim3(nkv, M), kAttnThreads, 0, s>>>(k, v, row_stride, knw, cosM, sinM, hd, kc, vc,
                                                                        hd, stride, window, p0_dev);
    count_launch();
    return launch_status("attn_prefill_prepkv");
}

int g4b_attn_prefill(const void* q, int dtype, int q_stride, int M, const float* qnw, const float* cosM,
                     const float* sinM, const uint16_t* kc, const uint16_t* vc, void* out, int out_dtype,
                     int out_stride, int nH, int nkv, int hd, int stride, int window, const int* p0_dev,
                     g4b_stream_t stream) {
    G4B_ENTRY("attn_prefill");
    G4B_REQUIRE(q && qnw && cosM && sinM && kc && vc && out && p0_dev, G4B_E_ARG, "attn_prefill: NULL pointer");
    G4B_REQUIRE(dtype == G4B_DT_F32 || dtype == G4B_DT_F16, G4B_E_ARG, "attn_prefill: bad dtype %d", dtype);
    G4B_REQUIRE(out_dtype == G4B_DT_F32 || out_dtype == G4B_DT_F16, G4B_E_ARG, "attn_prefill: bad out_dtype %d",
                out_dtype);
    G4B_REQUIRE(M >= 1 && nkv >= 1 && nH >= nkv && nH % nkv == 0 && (hd == 128 || hd == 256 || hd == 512) &&
                    stride >= 1 && window >= 0 && window <= stride && q_stride >= nH * hd && out_stride >= nH * hd &&
                    q_stride % 8 == 0 && out_stride % 8 == 0,
                G4B_E_SHAPE,
                "attn_prefill: M=%d nH=%d nkv=%d hd=%d (128/256/512) stride=%d window=%d q_stride=%d out_stride=%d "
                "(multiples of 8, >= nH * hd)",
                M, nH, nkv, hd, stride, window, q_stride, out_stride);
    G4B_REQUIRE(aligned16(q) && aligned16(kc) && aligned16(vc) && aligned16(out), G4B_E_ALIGN,
                "attn_prefill: q, the caches and out must be 16-byte aligned");
    const long long rows = (long long)M * (nH / nkv);
    const int br = prefill_rows(hd);
    G4B_REQUIRE((rows + br - 1) / br <= 0x7fffffffLL && nkv <= 65535, G4B_E_SHAPE, "attn_prefill: too many rows");
    int st = check_device(nullptr);
    if (st != G4B_OK) return st;
    PrefillArgs a{};
    a.q = q;
    a.qnw = qnw;
    a.cosM = cosM;
    a.sinM = sinM;
    a.kc = kc;
    a.vc = vc;
    a.out = out;
    a.p0_dev = p0_dev;
    a.M = M;
    a.G = nH / nkv;
    a.hd = hd;
    a.q_stride = q_stride;
    a.out_stride = out_stride;
    a.stride = stride;
    a.window = window;
    a.nqt = (int)((rows + br - 1) / br);
    a.out_f32 = out_dtype == G4B_DT_F32;
    const bool xf32 = dtype == G4B_DT_F32;
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    cudaError_t e = hd == 128 ? launch_prefill<128, 4, 1, 64>(a, nkv, xf32, s)
                  : hd == 256 ? launch_prefill<256, 8, 1, 32>(a, nkv, xf32, s)
                              : launch_prefill<512, 4, 2, 16>(a, nkv, xf32, s);
    if (e != cudaSuccess) return fail(G4B_E_CUDA, "attn_prefill: launch: %s", cudaGetErrorString(e));
    count_launch();
    return launch_status("attn_prefill");
}

}  // extern "C"

