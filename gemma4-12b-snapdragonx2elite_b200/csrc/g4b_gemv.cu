// g4b_gemv.cu -- int4 block-scaled decode GEMV / small-batch GEMM, the split-K
// reduce and the weight dequantiser.
//
// Replaces vk/gemv.comp:11-33, vk/gemv_fp8.comp:20-40 and vk/reduce.comp:8-12
// (recorded by gemv_ds()/gemv(), src/vk_engine.py:214-226, 270-272).
//
// B200 design (HBM-bound: 0.5625 bytes of weight+scale per weight element):
//   * A CTA (4 warps) owns a 256-column tile and one K-slice of 32-row scale
//     blocks.  Thread (g = lane/4, q = lane%4) of a warp loads, for each block,
//     rows 8q..8q+7 of columns 32g..32g+31 as 128-bit loads: a warp reads 4 rows
//     x 128 contiguous bytes per instruction.  Each warp double-buffers its
//     blocks in registers, so two blocks of loads are in flight per warp.
//   * The nibbles are turned into exact f16 values (q - 8) with the 0x6400
//     exponent trick (one LOP3 per two weights, one HSUB2/HFMA2 to remove the
//     offset) and fed to mma.sync m16n8k16 as the A operand: the tensor core
//     does the dot products over the block's 32 rows, so the ALU issue rate per
//     weight stays well under what 8 TB/s of int4 demands.  A row = output
//     column, B column = (token, hi/lo piece) of x, k = the block's rows.
//     Products are exact, accumulation f32.
//   * The per-block scale is applied in f32 to each block's dot products:
//     acc += scale * dot, so the weights are used exactly as the reference
//     uses them ((q - 8) * scale in f32, vk/gemv.comp:25-28) and only the f32
//     summation order differs.
//   * f32 activations are split exactly into f16 hi + lo pieces (two B
//     columns); f16 activations use one.
//   * K-slices write f32 partials; the last CTA of a column tile to arrive sums
//     them in slice order (deterministic), scales by inv and writes y -- the
//     reduce.comp dispatch fused into the GEMV.
#include <algorithm>

#include "g4b_common.cuh"

namespace g4b {

constexpr int kGemvWarps = 4;
constexpr int kGemvThreads = kGemvWarps * 32;
constexpr int kGemvTileN = 256;
constexpr int kGemvMaxTok = 8;

struct GemvArgs {
    const void* x;        // [M, K] f32 or f16
    const uint32_t* wp;   // [K, N/8]
    const void* scales;   // [nblk, N] f16 or e4m3
    void* y;              // [M, N]
    float* partial;       // [slices, M, N] (slices > 1)
    unsigned* counters;   // [ntiles]      (slices > 1)
    float inv;
    int M, N, K, nblk, bps, slices;
};

__device__ __forceinline__ uint32_t comp(const uint4& v, int i) {
    return i == 0 ? v.x : i == 1 ? v.y : i == 2 ? v.z : v.w;
}

__device__ __forceinline__ uint4 ld_stream_v4(const void* p) {
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "l"(p));
    return r;
}

__device__ __forceinline__ uint2 ld_stream_v2(const void* p) {
    uint2 r;
    asm volatile("ld.global.nc.L1::no_allocate.v2.u32 {%0,%1}, [%2];" : "=r"(r.x), "=r"(r.y) : "l"(p));
    return r;
}

// (q - 8) as exact f16x2 for the nibble pair selected by j from a PRMT-merged
// word P: the low 16 bits hold four nibbles of one row, the high 16 bits the
// same four columns of the next row; j picks the column (0..3).
__device__ __forceinline__ uint32_t deq_pair(uint32_t P, int j) {
    const uint32_t src = (j >= 2) ? (P >> 8) : P;
    if ((j & 1) == 0) {
        // 0x6400 | q = 1024 + q ; minus 1032 -> q - 8
        return hsub2_u(and_or(src, 0x000F000Fu, 0x64006400u), 0x64086408u);
    } else {
        // 0x6400 | (q << 4) = 1024 + 16 q ; * 1/16 - 72 -> q - 8
        return hfma2_u(and_or(src, 0x00F000F0u, 0x64006400u), 0x2C002C00u, 0xD480D480u);
    }
}

template <int SFMT>
struct ScaleRegs;
template <>
struct ScaleRegs<G4B_SCALE_F16> { uint4 v[4]; };   // 32 f16 = columns 0..31
template <>
struct ScaleRegs<G4B_SCALE_E4M3> { uint4 v[2]; };  // 32 bytes

template <bool XF32, int NT>
struct XRegs;
template <int NT>
struct XRegs<true, NT> { float4 v[NT][2]; };       // 8 f32 rows per token tile
template <int NT>
struct XRegs<false, NT> { uint4 v[NT]; };          // 8 f16 rows per token tile

template <bool XF32, int SFMT, int NT>
struct Stage {
    uint4 w[8];
    ScaleRegs<SFMT> s;
    XRegs<XF32, NT> x;
};

// Load one 32-row block b for this thread.  `nvalid` = valid words (0, 2 or 4)
// of the thread's 4-word column group; WIDE = rows are 16-byte aligned.
template <bool XF32, int SFMT, int NT, bool WIDE>
__device__ __forceinline__ void load_stage(Stage<XF32, SFMT, NT>& st, const GemvArgs& a, int b, int q,
                                           int word0, int col0, int nvalid, int g) {
    const int nb8 = a.N >> 3;
    const int row0 = b * 32 + 8 * q;
    #pragma unroll
    for (int i = 0; i < 8; i++) {
        const uint32_t* p = a.wp + (size_t)(row0 + i) * nb8 + word0;
        if constexpr (WIDE) {
            st.w[i] = nvalid ? ld_stream_v4(p) : make_uint4(0, 0, 0, 0);
        } else {
            uint2 lo = nvalid ? ld_stream_v2(p) : make_uint2(0, 0);
            uint2 hi = nvalid == 4 ? ld_stream_v2(p + 2) : make_uint2(0, 0);
            st.w[i] = make_uint4(lo.x, lo.y, hi.x, hi.y);
        }
    }
    if constexpr (SFMT == G4B_SCALE_F16) {
        const uint16_t* sp = (const uint16_t*)a.scales + (size_t)b * a.N + col0;
        #pragma unroll
        for (int i = 0; i < 4; i++)
            st.s.v[i] = (nvalid * 8 > i * 8) ? ld_stream_v4(sp + 8 * i) : make_uint4(0, 0, 0, 0);
    } else {
        const uint8_t* sp = (const uint8_t*)a.scales + (size_t)b * a.N + col0;
        #pragma unroll
        for (int i = 0; i < 2; i++)
            st.s.v[i] = (nvalid * 8 > i * 16) ? ld_stream_v4(sp + 16 * i) : make_uint4(0, 0, 0, 0);
    }
    // activations: thread supplies B column g of each token tile t
    #pragma unroll
    for (int t = 0; t < NT; t++) {
        const int tok = 4 * t + (g >> 1);
        const bool live = tok < a.M && (XF32 || (g & 1) == 0);
        if constexpr (XF32) {
            const float* xp = (const float*)a.x + (size_t)tok * a.K + row0;
            st.x.v[t][0] = live ? __ldg((const float4*)xp) : make_float4(0, 0, 0, 0);
            st.x.v[t][1] = live ? __ldg((const float4*)xp + 1) : make_float4(0, 0, 0, 0);
        } else {
            const __half* xp = (const __half*)a.x + (size_t)tok * a.K + row0;
            st.x.v[t] = live ? __ldg((const uint4*)xp) : make_uint4(0, 0, 0, 0);
        }
    }
}

// f32 -> the f16 piece this lane supplies: hi = f16(x), lo = f16(x - hi).
__device__ __forceinline__ uint32_t split_pair(float a, float b, bool lo) {
    __half ha = __float2half_rn(a), hb = __float2half_rn(b);
    if (lo) {
        ha = __float2half_rn(a - __half2float(ha));
        hb = __float2half_rn(b - __half2float(hb));
    }
    return pack_half2(ha, hb);
}

template <bool XF32, int SFMT, int NT>
__device__ __forceinline__ void compute_stage(const Stage<XF32, SFMT, NT>& st, float (&acc)[NT][16][2], int g) {
    // B fragments: b[t][h][0] = rows (4h, 4h+1), b[t][h][1] = rows (4h+2, 4h+3)
    uint32_t bf[NT][2][2];
    #pragma unroll
    for (int t = 0; t < NT; t++) {
        if constexpr (XF32) {
            const bool lo = (g & 1) != 0;
            const float4 x0 = st.x.v[t][0], x1 = st.x.v[t][1];
            bf[t][0][0] = split_pair(x0.x, x0.y, lo);
            bf[t][0][1] = split_pair(x0.z, x0.w, lo);
            bf[t][1][0] = split_pair(x1.x, x1.y, lo);
            bf[t][1][1] = split_pair(x1.z, x1.w, lo);
        } else {
            bf[t][0][0] = st.x.v[t].x;
            bf[t][0][1] = st.x.v[t].y;
            bf[t][1][0] = st.x.v[t].z;
            bf[t][1][1] = st.x.v[t].w;
        }
    }
    #pragma unroll
    for (int u = 0; u < 4; u++) {
        // scales of columns 8u..8u+7 as f32
        float sc[8];
        if constexpr (SFMT == G4B_SCALE_F16) {
            const uint4 s4 = st.s.v[u];
            #pragma unroll
            for (int k = 0; k < 4; k++) {
                const uint32_t hw = comp(s4, k);
                sc[2 * k] = h_lo(hw);
                sc[2 * k + 1] = h_hi(hw);
            }
        } else {
            const uint4 s4 = st.s.v[u >> 1];
            const uint32_t w0 = comp(s4, (u & 1) * 2), w1 = comp(s4, (u & 1) * 2 + 1);
            const uint32_t h01 = e4m3x2_to_f16x2((uint16_t)(w0 & 0xffffu));
            const uint32_t h23 = e4m3x2_to_f16x2((uint16_t)(w0 >> 16));
            const uint32_t h45 = e4m3x2_to_f16x2((uint16_t)(w1 & 0xffffu));
            const uint32_t h67 = e4m3x2_to_f16x2((uint16_t)(w1 >> 16));
            sc[0] = h_lo(h01); sc[1] = h_hi(h01); sc[2] = h_lo(h23); sc[3] = h_hi(h23);
            sc[4] = h_lo(h45); sc[5] = h_hi(h45); sc[6] = h_lo(h67); sc[7] = h_hi(h67);
        }
        uint32_t Plo[2], Phi[2], Qlo[2], Qhi[2];
        #pragma unroll
        for (int h = 0; h < 2; h++) {
            const uint32_t r0 = comp(st.w[4 * h + 0], u), r1 = comp(st.w[4 * h + 1], u);
            const uint32_t r2 = comp(st.w[4 * h + 2], u), r3 = comp(st.w[4 * h + 3], u);
            Plo[h] = prmt(r0, r1, 0x5410);  // columns 0..3 of rows (4h, 4h+1)
            Phi[h] = prmt(r0, r1, 0x7632);  // columns 4..7
            Qlo[h] = prmt(r2, r3, 0x5410);  // rows (4h+2, 4h+3)
            Qhi[h] = prmt(r2, r3, 0x7632);
        }
        #pragma unroll
        for (int j = 0; j < 4; j++) {
            float c[NT][4];
            #pragma unroll
            for (int t = 0; t < NT; t++) c[t][0] = c[t][1] = c[t][2] = c[t][3] = 0.f;
            #pragma unroll
            for (int h = 0; h < 2; h++) {
                const uint32_t a0 = deq_pair(Plo[h], j);  // A row g   = column 8u+j,   k = rows 4h, 4h+1
                const uint32_t a1 = deq_pair(Phi[h], j);  // A row g+8 = column 8u+j+4
                const uint32_t a2 = deq_pair(Qlo[h], j);  // A row g,   k = rows 4h+2, 4h+3
                const uint32_t a3 = deq_pair(Qhi[h], j);
                #pragma unroll
                for (int t = 0; t < NT; t++) mma_16816(c[t], a0, a1, a2, a3, bf[t][h][0], bf[t][h][1]);
            }
            #pragma unroll
            for (int t = 0; t < NT; t++) {
                acc[t][u * 4 + j][0] = fmaf(sc[j], c[t][0] + c[t][1], acc[t][u * 4 + j][0]);
                acc[t][u * 4 + j][1] = fmaf(sc[j + 4], c[t][2] + c[t][3], acc[t][u * 4 + j][1]);
            }
        }
    }
}

template <bool XF32, int SFMT, int NT, bool WIDE, bool YF32>
__global__ void __launch_bounds__(kGemvThreads, NT == 1 ? 3 : 2) gemv_i4_kernel(GemvArgs a) {
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int g = lane >> 2, q = lane & 3;
    const int tile = blockIdx.x, slice = blockIdx.y;
    const int col0 = tile * kGemvTileN + 32 * g;
    const int word0 = col0 >> 3;
    const int nvalid = col0 + 32 <= a.N ? 4 : (col0 + 16 <= a.N ? 2 : 0);
    const int b_begin = slice * a.bps;
    const int b_end = min(a.nblk, b_begin + a.bps);

    float acc[NT][16][2];
    #pragma unroll
    for (int t = 0; t < NT; t++)
        #pragma unroll
        for (int i = 0; i < 16; i++) acc[t][i][0] = acc[t][i][1] = 0.f;

    Stage<XF32, SFMT, NT> sa, sb;
    int b = b_begin + warp;
    if (b < b_end) {
        load_stage<XF32, SFMT, NT, WIDE>(sa, a, b, q, word0, col0, nvalid, g);
        for (;;) {
            if (b + kGemvWarps < b_end) load_stage<XF32, SFMT, NT, WIDE>(sb, a, b + kGemvWarps, q, word0, col0, nvalid, g);
            compute_stage<XF32, SFMT, NT>(sa, acc, g);
            b += kGemvWarps;
            if (b >= b_end) break;
            if (b + kGemvWarps < b_end) load_stage<XF32, SFMT, NT, WIDE>(sa, a, b + kGemvWarps, q, word0, col0, nvalid, g);
            compute_stage<XF32, SFMT, NT>(sb, acc, g);
            b += kGemvWarps;
            if (b >= b_end) break;
        }
    }

    // ---- CTA reduction over the 4 warps (padded rows: conflict-free stores)
    __shared__ float red[kGemvWarps][NT * 4][8][33];
    __shared__ unsigned s_last;
    #pragma unroll
    for (int t = 0; t < NT; t++) {
        #pragma unroll
        for (int u = 0; u < 4; u++)
            #pragma unroll
            for (int j = 0; j < 4; j++) {
                red[warp][4 * t + q][g][8 * u + j] = acc[t][u * 4 + j][0];
                red[warp][4 * t + q][g][8 * u + j + 4] = acc[t][u * 4 + j][1];
            }
    }
    __syncthreads();
    const int ntok = min(a.M, NT * 4);
    const float inv = SFMT == G4B_SCALE_E4M3 ? a.inv : 1.0f;
    for (int i = tid; i < ntok * kGemvTileN; i += kGemvThreads) {
        const int tok = i / kGemvTileN, col = i % kGemvTileN;
        const int n = tile * kGemvTileN + col;
        if (n >= a.N) continue;
        const int gg = col >> 5, cc = col & 31;
        const float v = ((red[0][tok][gg][cc] + red[1][tok][gg][cc]) + red[2][tok][gg][cc]) + red[3][tok][gg][cc];
        if (a.slices == 1) {
            const float o = v * inv;
            if (YF32) ((float*)a.y)[(size_t)tok * a.N + n] = o;
            else ((__half*)a.y)[(size_t)tok * a.N + n] = __float2half_rn(o);
        } else {
            a.partial[((size_t)slice * a.M + tok) * a.N + n] = v;
        }
    }
    if (a.slices == 1) return;

    // ---- split-K: the last CTA of this column tile sums the slices in order
    __threadfence();
    __syncthreads();
    if (tid == 0) s_last = (atomicAdd(&a.counters[tile], 1u) == (unsigned)(a.slices - 1)) ? 1u : 0u;
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    for (int i = tid; i < ntok * kGemvTileN; i += kGemvThreads) {
        const int tok = i / kGemvTileN, col = i % kGemvTileN;
        const int n = tile * kGemvTileN + col;
        if (n >= a.N) continue;
        float v = 0.f;
        for (int c = 0; c < a.slices; c++) v += __ldcg(&a.partial[((size_t)c * a.M + tok) * a.N + n]);
        const float o = v * inv;
        if (YF32) ((float*)a.y)[(size_t)tok * a.N + n] = o;
        else ((__half*)a.y)[(size_t)tok * a.N + n] = __float2half_rn(o);
    }
    if (tid == 0) a.counters[tile] = 0u;  // the workspace is ready for the next call
}

// ---------------------------------------------------------------- planning
struct GemvPlan {
    int ntiles, slices, bps, mg;   // mg = tokens per launch (<= 8)
    size_t part_bytes, ws_bytes;
};

static size_t align256(size_t v) { return (v + 255) & ~(size_t)255; }

static GemvPlan gemv_plan(int M, int N, int K, int split, int sms) {
    GemvPlan p{};
    const int nblk = K / 32;
    p.ntiles = (N + kGemvTileN - 1) / kGemvTileN;
    p.mg = std::min(M, kGemvMaxTok);
    if (split > 0) {
        p.slices = split;
        p.bps = nblk / split;
    } else {
        // enough CTAs for ~4 resident per SM, but at least one block per warp
        const int target = 4 * std::max(sms, 1);
        int s = std::max(1, (target + p.ntiles - 1) / p.ntiles);
        int bps = (nblk + s - 1) / s;
        bps = std::max(bps, std::min(kGemvWarps, nblk));
        p.bps = bps;
        p.slices = (nblk + bps - 1) / bps;
    }
    if (p.slices > 1) {
        p.part_bytes = align256((size_t)p.slices * p.mg * N * sizeof(float));
        p.ws_bytes = p.part_bytes + align256((size_t)p.ntiles * sizeof(unsigned));
    }
    return p;
}

template <bool XF32, int SFMT, int NT, bool WIDE, bool YF32>
static void launch_gemv(const GemvArgs& a, const GemvPlan& p, cudaStream_t s) {
    dim3 grid(p.ntiles, p.slices);
    gemv_i4_kernel<XF32, SFMT, NT, WIDE, YF32><<<grid, kGemvThreads, 0, s>>>(a);
}

template <bool XF32, int SFMT, int NT>
static void dispatch_wide_y(const GemvArgs& a, const GemvPlan& p, bool wide, bool yf32, cudaStream_t s) {
    if (wide) {
        if (yf32) launch_gemv<XF32, SFMT, NT, true, true>(a, p, s);
        else launch_gemv<XF32, SFMT, NT, true, false>(a, p, s);
    } else {
        if (yf32) launch_gemv<XF32, SFMT, NT, false, true>(a, p, s);
        else launch_gemv<XF32, SFMT, NT, false, false>(a, p, s);
    }
}

static void dispatch_gemv(const GemvArgs& a, const GemvPlan& p, bool xf32, int sfmt, int nt, bool wide, bool yf32,
                          cudaStream_t s) {
    if (xf32) {
        if (sfmt == G4B_SCALE_F16) {
            if (nt == 1) dispatch_wide_y<true, G4B_SCALE_F16, 1>(a, p, wide, yf32, s);
            else dispatch_wide_y<true, G4B_SCALE_F16, 2>(a, p, wide, yf32, s);
        } else {
            if (nt == 1) dispatch_wide_y<true, G4B_SCALE_E4M3, 1>(a, p, wide, yf32, s);
            else dispatch_wide_y<true, G4B_SCALE_E4M3, 2>(a, p, wide, yf32, s);
        }
    } else {
        if (sfmt == G4B_SCALE_F16) {
            if (nt == 1) dispatch_wide_y<false, G4B_SCALE_F16, 1>(a, p, wide, yf32, s);
            else dispatch_wide_y<false, G4B_SCALE_F16, 2>(a, p, wide, yf32, s);
        } else {
            if (nt == 1) dispatch_wide_y<false, G4B_SCALE_E4M3, 1>(a, p, wide, yf32, s);
            else dispatch_wide_y<false, G4B_SCALE_E4M3, 2>(a, p, wide, yf32, s);
        }
    }
}

// ------------------------------------------------------------- reduce kernel
__global__ void reduce_partials_kernel(const float* __restrict__ partial, float* __restrict__ y, int N, int split) {
    const int n4 = blockIdx.x * blockDim.x + threadIdx.x;
    if (n4 * 4 >= N) return;
    float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int c = 0; c < split; c++) {
        const float4 v = __ldg((const float4*)(partial + (size_t)c * N) + n4);
        s.x += v.x; s.y += v.y; s.z += v.z; s.w += v.w;
    }
    ((float4*)y)[n4] = s;
}

// ------------------------------------------------------------ dequant kernel
template <int SFMT, bool OUT_F32>
__global__ void dequant_i4_kernel(const uint32_t* __restrict__ wp, const void* __restrict__ scales, float inv,
                                  void* __restrict__ out, int N, int K) {
    const int nb8 = N >> 3;
    const size_t total = (size_t)K * nb8;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
        const int k = (int)(i / nb8), gw = (int)(i % nb8);
        const uint32_t w = __ldg(wp + i);
        const int b = k >> 5;
        float v[8];
        #pragma unroll
        for (int j = 0; j < 8; j++) {
            const int n = gw * 8 + j;
            const float s = SFMT == G4B_SCALE_F16
                                ? __half2float(((const __half*)scales)[(size_t)b * N + n])
                                : e4m3_decode_ref(((const uint8_t*)scales)[(size_t)b * N + n]);
            v[j] = (float)((w >> (4 * j)) & 15u) - 8.0f;
            v[j] = __fmul_rn(v[j], s);  // exact: 4-bit x 11-bit significands
            if (SFMT == G4B_SCALE_E4M3) v[j] = __fmul_rn(v[j], inv);  // a power of two: exact
        }
        if (OUT_F32) {
            float4* o = (float4*)((float*)out + (size_t)k * N + gw * 8);
            o[0] = make_float4(v[0], v[1], v[2], v[3]);
            o[1] = make_float4(v[4], v[5], v[6], v[7]);
        } else {
            uint4 o;
            o.x = pack_half2(__float2half_rn(v[0]), __float2half_rn(v[1]));
            o.y = pack_half2(__float2half_rn(v[2]), __float2half_rn(v[3]));
            o.z = pack_half2(__float2half_rn(v[4]), __float2half_rn(v[5]));
            o.w = pack_half2(__float2half_rn(v[6]), __float2half_rn(v[7]));
            *(uint4*)((__half*)out + (size_t)k * N + gw * 8) = o;
        }
    }
}

}  // namespace g4b

using namespace g4b;

extern "C" {

size_t g4b_gemv_workspace_bytes(int M, int N, int K, int split) {
    if (M <= 0 || N <= 0 || K <= 0 || K % 32) return 0;
    int sms = 148;
    if (check_device(&sms) != G4B_OK) sms = 148;
    clear_error();
    return gemv_plan(M, N, K, split, sms).ws_bytes;
}

int g4b_gemv_i4(const void* x, int x_dtype, int M, const uint32_t* wp, const void* scales, int scale_fmt,
                float inv, void* y, int y_dtype, int N, int K, int split, void* workspace, size_t ws_bytes,
                g4b_stream_t stream) {
    G4B_ENTRY("gemv_i4");
    G4B_REQUIRE(x && wp && scales && y, G4B_E_ARG, "gemv_i4: NULL pointer argument");
    G4B_REQUIRE(x_dtype == G4B_DT_F32 || x_dtype == G4B_DT_F16, G4B_E_ARG, "gemv_i4: bad x_dtype %d", x_dtype);
    G4B_REQUIRE(y_dtype == G4B_DT_F32 || y_dtype == G4B_DT_F16, G4B_E_ARG, "gemv_i4: bad y_dtype %d", y_dtype);
    G4B_REQUIRE(scale_fmt == G4B_SCALE_F16 || scale_fmt == G4B_SCALE_E4M3, G4B_E_ARG,
                "gemv_i4: bad scale_fmt %d", scale_fmt);
    G4B_REQUIRE(M >= 1 && N > 0 && K > 0, G4B_E_SHAPE, "gemv_i4: M=%d N=%d K=%d must be positive", M, N, K);
    G4B_REQUIRE(N % 16 == 0, G4B_E_SHAPE, "gemv_i4: N=%d must be a multiple of 16", N);
    G4B_REQUIRE(K % 32 == 0, G4B_E_SHAPE, "gemv_i4: K=%d must be a multiple of 32", K);
    const int nblk = K / 32;
    G4B_REQUIRE(split >= 0 && (split == 0 || nblk % split == 0), G4B_E_SHAPE,
                "gemv_i4: split=%d must divide K/32=%d (or be 0)", split, nblk);
    G4B_REQUIRE(aligned16(x) && aligned16(wp) && aligned16(scales), G4B_E_ALIGN,
                "gemv_i4: x, wp and scales must be 16-byte aligned");
    G4B_REQUIRE(((uintptr_t)y & (y_dtype == G4B_DT_F32 ? 3u : 1u)) == 0, G4B_E_ALIGN, "gemv_i4: y misaligned");
    int sms = 0;
    int st = check_device(&sms);
    if (st != G4B_OK) return st;
    const GemvPlan p = gemv_plan(M, N, K, split, sms);
    if (p.slices > 1) {
        G4B_REQUIRE(workspace != nullptr && ws_bytes >= p.ws_bytes, G4B_E_WORKSPACE,
                    "gemv_i4: needs %zu bytes of workspace, got %zu", p.ws_bytes, workspace ? ws_bytes : 0);
        G4B_REQUIRE(aligned16(workspace), G4B_E_ALIGN, "gemv_i4: workspace must be 16-byte aligned");
    }
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    const bool wide = (N % 32) == 0;
    const size_t xe = x_dtype == G4B_DT_F32 ? 4 : 2, ye = y_dtype == G4B_DT_F32 ? 4 : 2;
    for (int m0 = 0; m0 < M; m0 += kGemvMaxTok) {
        GemvArgs a{};
        a.M = std::min(kGemvMaxTok, M - m0);
        a.x = (const char*)x + (size_t)m0 * K * xe;
        a.y = (char*)y + (size_t)m0 * N * ye;
        a.wp = wp;
        a.scales = scales;
        a.inv = inv;
        a.N = N;
        a.K = K;
        a.nblk = nblk;
        a.bps = p.bps;
        a.slices = p.slices;
        if (p.slices > 1) {
            a.partial = (float*)workspace;
            a.counters = (unsigned*)((char*)workspace + p.part_bytes);
        }
        const int nt = a.M <= 4 ? 1 : 2;
        dispatch_gemv(a, p, x_dtype == G4B_DT_F32, scale_fmt, nt, wide, y_dtype == G4B_DT_F32, s);
        count_launch();
        st = launch_status("gemv_i4");
        if (st != G4B_OK) return st;
    }
    return G4B_OK;
}

int g4b_reduce_partials(const float* partial, float* y, int N, int split, g4b_stream_t stream) {
    G4B_ENTRY("reduce_partials");
    G4B_REQUIRE(partial && y, G4B_E_ARG, "reduce_partials: NULL pointer argument");
    G4B_REQUIRE(N > 0 && N % 4 == 0 && split >= 1, G4B_E_SHAPE, "reduce_partials: N=%d (multiple of 4), split=%d",
                N, split);
    G4B_REQUIRE(aligned16(partial) && aligned16(y), G4B_E_ALIGN, "reduce_partials: pointers must be 16-byte aligned");
    int st = check_device(nullptr);
    if (st != G4B_OK) return st;
    const int threads = 256, blocks = (N / 4 + threads - 1) / threads;
    reduce_partials_kernel<<<blocks, threads, 0, reinterpret_cast<cudaStream_t>(stream)>>>(partial, y, N, split);
    count_launch();
    return launch_status("reduce_partials");
}

int g4b_dequant_i4(const uint32_t* wp, const void* scales, int scale_fmt, float inv, void* out, int out_dtype, int N,
                   int K, g4b_stream_t stream) {
    G4B_ENTRY("dequant_i4");
    G4B_REQUIRE(wp && scales && out, G4B_E_ARG, "dequant_i4: NULL pointer argument");
    G4B_REQUIRE(scale_fmt == G4B_SCALE_F16 || scale_fmt == G4B_SCALE_E4M3, G4B_E_ARG, "dequant_i4: bad scale_fmt");
    G4B_REQUIRE(out_dtype == G4B_DT_F32 || out_dtype == G4B_DT_F16, G4B_E_ARG, "dequant_i4: bad out_dtype");
    G4B_REQUIRE(N > 0 && N % 16 == 0 && K > 0 && K % 32 == 0, G4B_E_SHAPE,
                "dequant_i4: N=%d (multiple of 16), K=%d (multiple of 32)", N, K);
    G4B_REQUIRE(aligned16(wp) && aligned16(scales) && aligned16(out), G4B_E_ALIGN,
                "dequant_i4: pointers must be 16-byte aligned");
    int sms = 148;
    int st = check_device(&sms);
    if (st != G4B_OK) return st;
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    const size_t total = (size_t)K * (N / 8);
    const int threads = 256;
    const int blocks = (int)std::min<size_t>((total + threads - 1) / threads, (size_t)sms * 16);
    if (scale_fmt == G4B_SCALE_F16) {
        if (out_dtype == G4B_DT_F32) dequant_i4_kernel<G4B_SCALE_F16, true><<<blocks, threads, 0, s>>>(wp, scales, inv, out, N, K);
        else dequant_i4_kernel<G4B_SCALE_F16, false><<<blocks, threads, 0, s>>>(wp, scales, inv, out, N, K);
    } else {
        if (out_dtype == G4B_DT_F32) dequant_i4_kernel<G4B_SCALE_E4M3, true><<<blocks, threads, 0, s>>>(wp, scales, inv, out, N, K);
        else dequant_i4_kernel<G4B_SCALE_E4M3, false><<<blocks, threads, 0, s>>>(wp, scales, inv, out, N, K);
    }
    count_launch();
    return launch_status("dequant_i4");
}

}  // extern "C"
