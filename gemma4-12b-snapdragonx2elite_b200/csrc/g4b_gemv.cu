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
#include <cstdlib>
#include <mutex>
#include <vector>
#include <utility>

#include "g4b_tcgen05.cuh"

namespace g4b {

// Launch flags of the current host call (set by g4b_gemv_i4_ex for its duration).
static thread_local bool t_pdl = false;
// Bytes at t_clear_ptr to zero on the launch stream right before the next
// kernel launch of the current host call (g4b_gemv_i4_noalloc's counters):
// enqueued only once every check has passed, so a rejected call launches nothing.
static thread_local void* t_clear_ptr = nullptr;
static thread_local size_t t_clear_bytes = 0;

// Launch `kern` on `s`, with programmatic dependent launch when t_pdl is set:
// the grid may then start while the previous kernel in the stream is still
// running (every kernel here waits with griddepcontrol.wait before it reads
// activations or writes outputs and workspace).
template <typename... KArgs, typename... Args>
static cudaError_t launch_k(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                            Args&&... args) {
    if (t_clear_ptr) {
        void* p = t_clear_ptr;
        t_clear_ptr = nullptr;
        const cudaError_t e = cudaMemsetAsync(p, 0, t_clear_bytes, s);
        if (e != cudaSuccess) return e;
    }
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    if (t_pdl) {
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
    }
    return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

constexpr int kGemvWarps = 4;
constexpr int kGemvThreads = kGemvWarps * 32;
constexpr int kGemvTileN = 256;
constexpr int kGemvMaxTok = 8;
// The workspace starts with a fixed region of per-tile arrival counters (so a
// call never lands its counters on another call's partials), then the partials.
constexpr int kGemvMaxTiles = 4096;
constexpr size_t kGemvCounterBytes = kGemvMaxTiles * sizeof(unsigned);

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
    pdl_wait();
    pdl_launch_dependents();
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

// ============================================================ streaming GEMV
// A persistent grid (two CTAs per SM).  A producer warp streams weight tiles of
// [128 rows (4 scale blocks) x 256 columns] into a shared-memory ring with one
// 2-D TMA load each (plus one TMA load of their 4 x 256 scales), a second
// producer warp copies the matching activation rows, and 4 consumer warps
// each run compute_stage() on one of the tile's 32-row blocks.  Work = the
// (column tile, block quad) items in tile-major order, split into equal
// contiguous ranges per CTA.  A CTA's share of a tile is reduced across its 4
// warps in shared memory (in warp order); a tile shared by several CTAs is
// summed by the last CTA to arrive (per-tile counter), in CTA order, so the
// result is deterministic.  With a caller-given split the ranges are exactly
// the reference's K-slices.
// (tile, k-chunk) of consecutive items: one division when a walk starts, none
// per item (64-bit division is a long emulated sequence on the GPU)
struct ItemCursor {
    int t, o, noct;
    __device__ ItemCursor(long long item, int noct_) : t((int)(item / noct_)), o((int)(item % noct_)), noct(noct_) {}
    __device__ __forceinline__ void next() {
        if (++o == noct) {
            o = 0;
            ++t;
        }
    }
};

constexpr int kStTN = 256;
constexpr int kStRows = 128;                         // rows per stage = 4 scale blocks
constexpr int kStWBytes = kStRows * (kStTN / 2);     // 16 KB of packed weights
constexpr int kStThreads = 192;                      // warps 0-3 consumers, 4 weights, 5 activations
constexpr int kStMaxStages = 8;

static __device__ unsigned g_gemv_status;

struct StreamArgs {
    const void* x;
    void* y;
    float* partial;      // [G * maxseg, M, kStTN]
    unsigned* counters;  // [ntiles]
    float inv;
    int M, N, K, nquad, ntiles, L, maxseg, stages, stage_bytes, s_bytes;
    long long total;
};

template <bool XF32, int SFMT, int NT, bool YF32>
__global__ void __launch_bounds__(kStThreads, 2) gemv_i4_stream_kernel(const StreamArgs a,
                                                                      const __grid_constant__ CUtensorMap wmap,
                                                                      const __grid_constant__ CUtensorMap smap) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ uint64_t bars[2 * kStMaxStages];
    __shared__ unsigned s_last;
    __shared__ int s_issued;
    __shared__ int s_abort;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    volatile int* abort_flag = &s_abort;
    const int S = a.stages;
    const uint32_t smem0 = smem_u32(smem);
    const uint32_t bar0 = smem_u32(bars);
    auto full_bar = [&](int s) { return bar0 + 8u * s; };
    auto empty_bar = [&](int s) { return bar0 + 8u * (kStMaxStages + s); };
    const long long ibeg = (long long)blockIdx.x * a.L;
    const long long iend = min(ibeg + (long long)a.L, a.total);
    constexpr int esz = XF32 ? 4 : 2;
    constexpr int ssz = SFMT == G4B_SCALE_F16 ? 2 : 1;
    // per-warp reduction area after the stages: [4 warps][NT*4 tokens][8][33] f32
    float (*red)[NT * 4][8][33] = reinterpret_cast<float (*)[NT * 4][8][33]>(smem + (size_t)S * a.stage_bytes);

    if (tid == 0) {
        for (int s = 0; s < S; s++) {
            mbar_init(full_bar(s), 1);
            mbar_init(empty_bar(s), 4);
        }
        s_abort = 0;
        s_issued = 0;
        fence_mbar_init();
    }
    __syncthreads();
    pdl_launch_dependents();

    if (warp == 4) {
        // ---------------- weight + scale producer: one TMA box of each per stage
        if (lane == 0) {
            prefetch_tensor_map(&wmap);
            prefetch_tensor_map(&smap);
            const uint64_t pol = l2_evict_first_policy();
            int i = 0;
            ItemCursor cw(ibeg, a.nquad);
            for (long long it = ibeg; it < iend; ++it, ++i, cw.next()) {
                const int s = i % S;
                if (i >= S && !mbar_wait(empty_bar(s), ((i / S) & 1) ^ 1, abort_flag, &g_gemv_status)) break;
                const int t = cw.t, qd = cw.o;
                // full boxes always land (out-of-range columns are zero-filled)
                mbar_arrive_expect_tx(full_bar(s), kStWBytes + a.s_bytes + (uint32_t)(a.M * kStRows * esz));
                const uint32_t st = smem0 + (uint32_t)s * a.stage_bytes;
                tma_load_2d(st, &wmap, t * (kStTN / 8), qd * kStRows, full_bar(s), pol);
                tma_load_2d(st + kStWBytes, &smap, t * (kStTN * ssz / 8), qd * 4, full_bar(s), pol);
            }
            s_issued = i;
        }
    } else if (warp == 5) {
        // ---------------- activation producer (waits for the previous grid)
        pdl_wait();
        int i = 0;
        ItemCursor cx(ibeg, a.nquad);
        for (long long it = ibeg; it < iend; ++it, ++i, cx.next()) {
            const int s = i % S;
            if (i >= S && !mbar_wait(empty_bar(s), ((i / S) & 1) ^ 1, abort_flag, &g_gemv_status)) break;
            const int qd = cx.o;
            if (lane < a.M)
                bulk_g2s_nohint(smem0 + (uint32_t)s * a.stage_bytes + kStWBytes + a.s_bytes + lane * kStRows * esz,
                                reinterpret_cast<const uint8_t*>(a.x) + ((size_t)lane * a.K + qd * kStRows) * esz,
                                kStRows * esz, full_bar(s));
        }
    } else {
        // ---------------- consumers: warp w takes the tile's block w
        pdl_wait();  // outputs and workspace may still be read by the previous grid
        const int g = lane >> 2, q = lane & 3, ctid = tid;
        float acc[NT][16][2];
        long long cur_t = -1;
        const float inv = SFMT == G4B_SCALE_E4M3 ? a.inv : 1.0f;

        auto flush = [&](long long t) {
            // 1. the 4 warps' sums into shared memory (padded rows: conflict-free)
            #pragma unroll
            for (int t2 = 0; t2 < NT; t2++)
                #pragma unroll
                for (int u = 0; u < 4; u++)
                    #pragma unroll
                    for (int j = 0; j < 4; j++) {
                        red[warp][4 * t2 + q][g][8 * u + j] = acc[t2][u * 4 + j][0];
                        red[warp][4 * t2 + q][g][8 * u + j + 4] = acc[t2][u * 4 + j][1];
                    }
            named_bar_sync(1, 128);
            const int c = blockIdx.x;
            const long long c_first = (t * a.nquad) / a.L, c_last = ((t + 1) * a.nquad - 1) / a.L;
            const bool single = c_first == c_last;
            const bool ok = !*abort_flag;
            const int n_base = (int)t * kStTN;
            const long long slot = (long long)c * a.maxseg + (t - ((long long)c * a.L) / a.nquad);
            // 2. warp-ordered sum, then y (tile owned by this CTA alone) or a partial
            for (int e = ctid; e < a.M * kStTN && ok; e += 128) {
                const int tok = e / kStTN, col = e % kStTN, n = n_base + col;
                const int gg = col >> 5, cc = col & 31;
                const float v = ((red[0][tok][gg][cc] + red[1][tok][gg][cc]) + red[2][tok][gg][cc]) + red[3][tok][gg][cc];
                if (single) {
                    if (n < a.N) {
                        if (YF32) ((float*)a.y)[(size_t)tok * a.N + n] = v * inv;
                        else ((__half*)a.y)[(size_t)tok * a.N + n] = __float2half_rn(v * inv);
                    }
                } else {
                    a.partial[((size_t)slot * a.M + tok) * kStTN + col] = v;
                }
            }
            if (!single) {
                __threadfence();
                named_bar_sync(1, 128);
                if (ctid == 0) s_last = ok && (atomicAdd(&a.counters[t], 1u) == (unsigned)(c_last - c_first)) ? 1u : 0u;
                named_bar_sync(1, 128);
                if (s_last) {
                    __threadfence();
                    const int nseg = (int)(c_last - c_first + 1);
                    for (int e = ctid; e < a.M * kStTN; e += 128) {
                        const int tok = e / kStTN, col = e % kStTN, n = n_base + col;
                        float v = 0.f;
                        // 8 independent loads in flight, summed in CTA order
                        for (int k0 = 0; k0 < nseg; k0 += 8) {
                            float pv[8];
                            #pragma unroll
                            for (int k = 0; k < 8; k++) {
                                const long long cc = c_first + k0 + k;
                                pv[k] = 0.f;
                                if (k0 + k < nseg) {
                                    const long long sl = cc * a.maxseg + (t - (cc * a.L) / a.nquad);
                                    pv[k] = __ldcg(&a.partial[((size_t)sl * a.M + tok) * kStTN + col]);
                                }
                            }
                            #pragma unroll
                            for (int k = 0; k < 8; k++)
                                if (k0 + k < nseg) v += pv[k];
                        }
                        if (n < a.N) {
                            if (YF32) ((float*)a.y)[(size_t)tok * a.N + n] = v * inv;
                            else ((__half*)a.y)[(size_t)tok * a.N + n] = __float2half_rn(v * inv);
                        }
                    }
                    if (ctid == 0) a.counters[t] = 0u;  // ready for the next call
                }
            }
            named_bar_sync(1, 128);  // red[] is reused by the next flush
        };

        int i = 0;
        ItemCursor cc(ibeg, a.nquad);
        for (long long it = ibeg; it < iend; ++it, ++i, cc.next()) {
            const long long t = cc.t;
            if (t != cur_t) {
                if (cur_t >= 0) flush(cur_t);
                #pragma unroll
                for (int t2 = 0; t2 < NT; t2++)
                    #pragma unroll
                    for (int k = 0; k < 16; k++) acc[t2][k][0] = acc[t2][k][1] = 0.f;
                cur_t = t;
            }
            const int s = i % S;
            if (mbar_wait(full_bar(s), (i / S) & 1, abort_flag, &g_gemv_status)) {
                const uint8_t* st = smem + (size_t)s * a.stage_bytes;
                const int row0 = 32 * warp + 8 * q;
                Stage<XF32, SFMT, NT> sg;
                #pragma unroll
                for (int r = 0; r < 8; r++)
                    sg.w[r] = *reinterpret_cast<const uint4*>(st + (row0 + r) * (kStTN / 2) + 16 * g);
                if constexpr (SFMT == G4B_SCALE_F16) {
                    #pragma unroll
                    for (int k = 0; k < 4; k++)
                        sg.s.v[k] = *reinterpret_cast<const uint4*>(st + kStWBytes + (warp * kStTN + 32 * g + 8 * k) * 2);
                } else {
                    #pragma unroll
                    for (int k = 0; k < 2; k++)
                        sg.s.v[k] = *reinterpret_cast<const uint4*>(st + kStWBytes + warp * kStTN + 32 * g + 16 * k);
                }
                const uint8_t* xs = st + kStWBytes + a.s_bytes;
                #pragma unroll
                for (int t2 = 0; t2 < NT; t2++) {
                    const int tok = 4 * t2 + (g >> 1);
                    const bool live = tok < a.M && (XF32 || (g & 1) == 0);
                    if constexpr (XF32) {
                        const float4* xp = reinterpret_cast<const float4*>(xs + (tok * kStRows + row0) * 4);
                        sg.x.v[t2][0] = live ? xp[0] : make_float4(0, 0, 0, 0);
                        sg.x.v[t2][1] = live ? xp[1] : make_float4(0, 0, 0, 0);
                    } else {
                        sg.x.v[t2] = live ? *reinterpret_cast<const uint4*>(xs + (tok * kStRows + row0) * 2)
                                          : make_uint4(0, 0, 0, 0);
                    }
                }
                compute_stage<XF32, SFMT, NT>(sg, acc, g);
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(empty_bar(s));
        }
        if (cur_t >= 0) flush(cur_t);
    }

    __syncthreads();
    if (tid == 0 && *abort_flag) {
        // drain: let every TMA load this CTA issued land before the CTA exits
        const int issued = s_issued;
        for (int i = max(0, issued - S); i < issued; i++) {
            const uint64_t t0 = global_ns();
            while (!mbar_try_wait(full_bar(i % S), (i / S) & 1) && global_ns() - t0 < kWaitLimitNs) {
            }
        }
    }
}

// ====================================================== streaming GEMV, M = 1
// The decode case (one token) gets its own consumer arithmetic and layout:
//  * nibble -> f16 with a single AND: (w & 0x000F000F) is the f16 pair
//    (q * 2^-24, q' * 2^-24) exactly (subnormals; the tensor core keeps them),
//    and (w & 0x00F000F0) is (q * 2^-20, ...).  The 2^24 / 2^20 and the -8
//    offset are applied per block in f32:  sum (q - 8) x = 2^E * C - 8 * X
//    with X = the sum of the block's x.
//  * block-diagonal B: the 8 columns of one m16n8k16 B operand hold x masked
//    to 8 different 32-row blocks (f16 x; 4 blocks x {hi, lo} pieces for f32
//    x), so every accumulator element is a useful per-block dot product and
//    the per-block scale is applied once per stage.
//  * the A fragments come straight from ldmatrix.x4.trans: for a 16-bit
//    column g (4 weight columns) it hands lane (g, q) rows 2q and 2q+1 packed
//    in one register -- the k-pair layout m16n8k16 wants -- so one
//    instruction feeds 4 mma operands.  The weight tile lands 128-byte
//    swizzled and the 8 rows of each 8x8 matrix are rotated per lane so they
//    fall on 8 different swizzle phases: conflict-free.
//  * work: a stage of [256 rows (8 blocks) x 256 columns] goes to one of 2
//    warp groups (item i -> group i % 2), each of its 8 warps taking one
//    16-byte column segment (32 columns); one ldmatrix.x4 feeds two mma
//    steps.  Each group owns 2 stages (double buffering); a barrier is only
//    ever waited on by the group that consumes it, in order, so the parity of
//    the phase it waits for can never alias an older, still-pending phase.
constexpr int kM1Rows = 256;
constexpr int kM1WBytes = kM1Rows * (kStTN / 2);  // 32 KB
constexpr int kM1Groups = 2;
constexpr int kM1PerGroup = 2;                     // private stages per group
constexpr int kM1Stages = kM1Groups * kM1PerGroup;
constexpr int kM1WarpsPerGroup = 8;
constexpr int kM1Consumers = 32 * kM1WarpsPerGroup * kM1Groups;  // 512
constexpr int kM1Threads = kM1Consumers + 64;      // + TMA producer warp + activation producer warp
constexpr int kChainThreads = kM1Threads + 32;     // the chain adds an L2 prefetch warp

// Up to three GEMVs that read the same x (the engine's q/k/v, or gate/up) run
// as one launch: their column tiles are numbered one after another ("segments"),
// and every per-tile decision (which weights to load, where y goes, which
// e4m3 inverse scale applies) looks the segment up from the tile index.
constexpr int kTcMaxSeg = 3;
constexpr int kMaxCtas = 256;  // split-K plans never use more CTAs than this (one per SM)

struct TcSeg {
    void* y;
    float inv;    // e4m3 2^-shift (1 for f16 scales)
    int N;
    int tile0;    // first tile of this segment in the launch's tile numbering
};

struct TcMaps {
    CUtensorMap w[kTcMaxSeg];
    CUtensorMap s[kTcMaxSeg];
};

template <class A>
__host__ __device__ __forceinline__ int tc_seg_of(const A& a, long long t) {
    return (int)(t >= a.seg1.tile0) + (int)(t >= a.seg2.tile0);
}
template <class A>
__host__ __device__ __forceinline__ const TcSeg& tc_seg(const A& a, int sg) {
    return sg == 0 ? a.seg0 : (sg == 1 ? a.seg1 : a.seg2);
}

// item i of a CTA -> its group, shared-memory stage and barrier phase parity
__device__ __forceinline__ int m1_group(int i) { return i % kM1Groups; }
__device__ __forceinline__ int m1_stage(int i) { return i % kM1Groups + kM1Groups * ((i / kM1Groups) % kM1PerGroup); }
__device__ __forceinline__ uint32_t m1_parity(int i) { return (uint32_t)((i / kM1Groups) / kM1PerGroup) & 1u; }

struct M1Args {
    const void* x;
    float* partial;      // [G * maxseg, kStTN]
    unsigned* counters;  // [ntiles]
    TcSeg seg0, seg1, seg2;
    int nseg, K, noct, ntiles, G, maxseg, stage_bytes, s_bytes;
    int mode;            // partition of the items over the CTAs (kM1Balanced ...)
    long long total;
};

// How an M = 1 launch splits its total = ntiles * noct items (item = tile *
// noct + k-chunk) over its G CTAs; every CTA owns one contiguous range.
//   balanced     CTA c owns [c*T/G, (c+1)*T/G): the fewest items per CTA, but
//                a CTA can straddle two shared tiles (two split-K flushes, the
//                items of one tile after the other's);
//   tile split   ntiles < G: tile t's k-chunks split evenly over n_t CTAs,
//                n_t = G/ntiles, one more for the first G%ntiles tiles;
//   whole tiles  ntiles >= G: CTA c owns tiles [c*ntiles/G, (c+1)*ntiles/G).
constexpr int kM1Balanced = 0;
constexpr int kM1TileSplit = 1;
constexpr int kM1WholeTiles = 2;

__host__ __device__ __forceinline__ void m1_range(int mode, long long total, int ntiles, int noct, int G, int c,
                                                  long long& ib, long long& ie) {
    if (mode == kM1TileSplit) {
        const int q = G / ntiles, r = G % ntiles;
        int t, k, n;
        if (c < r * (q + 1)) {
            t = c / (q + 1);
            k = c - t * (q + 1);
            n = q + 1;
        } else {
            const int c2 = c - r * (q + 1);
            t = r + c2 / q;
            k = c2 - (t - r) * q;
            n = q;
        }
        ib = (long long)t * noct + k * noct / n;
        ie = (long long)t * noct + (k + 1) * noct / n;
    } else if (mode == kM1WholeTiles) {
        ib = (long long)c * ntiles / G * noct;
        ie = (long long)(c + 1) * ntiles / G * noct;
    } else {
        ib = (long long)c * total / G;
        ie = (long long)(c + 1) * total / G;
    }
}

// The first and last CTA that own items of tile t (whole tiles: one CTA).
__host__ __device__ __forceinline__ void m1_span(int mode, long long total, int ntiles, int noct, int G, long long t,
                                                 long long& cf, long long& cl) {
    if (mode == kM1TileSplit) {
        const int q = G / ntiles, r = G % ntiles;
        cf = t < r ? t * (q + 1) : (long long)r * (q + 1) + (t - r) * q;
        cl = cf + q + (t < r ? 1 : 0) - 1;
    } else if (mode == kM1WholeTiles) {
        cf = cl = 0;  // never needed: every tile is single-owned
    } else {
        cf = ((t * noct + 1) * G - 1) / total;
        cl = (((t + 1) * noct) * G - 1) / total;
    }
}

__device__ __forceinline__ uint32_t nib_sub(uint32_t P, int j) {
    const uint32_t src = (j >= 2) ? (P >> 8) : P;
    return src & ((j & 1) ? 0x00F000F0u : 0x000F000Fu);
}

// byte offset of 32-bit word `word` (0..31) of row `row` in a 128-byte-swizzled tile
__device__ __forceinline__ int swz128(int row, int word) {
    return row * 128 + ((((word >> 2) ^ (row & 7)) << 4) | ((word & 3) << 2));
}

template <bool XF32, int SFMT, bool YF32>
__global__ void __launch_bounds__(kM1Threads, 1) gemv_i4_m1_kernel(const M1Args a,
                                                                  const __grid_constant__ TcMaps maps) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    __shared__ uint64_t bars[2 * kM1Stages];
    __shared__ float red[2][kM1Groups][kStTN];  // double-buffered: consecutive flushes never share it
    __shared__ unsigned s_last;
    __shared__ long long s_pending;              // shared tile this CTA must still reduce (-1: none)
    __shared__ int s_issued;
    __shared__ int s_abort;
    __shared__ __align__(16) uint32_t s_zero[32];  // B-fragment source for lanes that feed zeros
    __shared__ int s_ftile[kMaxCtas];              // first tile of each CTA's item range
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    volatile int* abort_flag = &s_abort;
    constexpr int esz = XF32 ? 4 : 2;
    constexpr int ssz = SFMT == G4B_SCALE_F16 ? 2 : 1;
    // the swizzle pattern repeats every 1024 bytes: align the stages to it
    const uint32_t raw0 = smem_u32(smem_raw);
    const uint32_t smem0 = (raw0 + 1023u) & ~1023u;
    uint8_t* smem = smem_raw + (smem0 - raw0);
    const uint32_t bar0 = smem_u32(bars);
    auto full_bar = [&](int s) { return bar0 + 8u * s; };
    auto empty_bar = [&](int s) { return bar0 + 8u * (kM1Stages + s); };
    // balanced contiguous item ranges: CTA c owns [c*T/G, (c+1)*T/G)
    long long ibeg, iend;
    m1_range(a.mode, a.total, a.ntiles, a.noct, a.G, blockIdx.x, ibeg, iend);
    const int pw = kM1Consumers / 32;  // first producer warp

    if (tid == 0) {
        for (int s = 0; s < kM1Stages; s++) {
            mbar_init(full_bar(s), 1);
            mbar_init(empty_bar(s), kM1WarpsPerGroup);
        }
        s_abort = 0;
        s_issued = 0;
        s_pending = -1;
        fence_mbar_init();
    }
    if (tid < 32) s_zero[tid] = 0u;
    // the split-K reduction needs every CTA's first tile: one division per CTA, here, in parallel
    for (int c = tid; c < a.G; c += blockDim.x) {
        long long ib, ie;
        m1_range(a.mode, a.total, a.ntiles, a.noct, a.G, c, ib, ie);
        s_ftile[c] = (int)(ib / a.noct);
    }
    __syncthreads();
    pdl_launch_dependents();

    if (warp == pw) {
        if (lane == 0) {
            for (int sg = 0; sg < a.nseg; sg++) {
                prefetch_tensor_map(&maps.w[sg]);
                prefetch_tensor_map(&maps.s[sg]);
            }
            const uint64_t pol = l2_evict_first_policy();
            int i = 0;
            ItemCursor cw(ibeg, a.noct);
            for (long long it = ibeg; it < iend; ++it, ++i, cw.next()) {
                const int s = m1_stage(i);
                if (i >= kM1Stages && !mbar_wait(empty_bar(s), m1_parity(i) ^ 1u, abort_flag, &g_gemv_status)) break;
                const int sg = tc_seg_of(a, cw.t);
                const int lt = cw.t - tc_seg(a, sg).tile0, o = cw.o;
                mbar_arrive_expect_tx(full_bar(s), kM1WBytes + a.s_bytes + kM1Rows * esz);
                const uint32_t st = smem0 + (uint32_t)s * a.stage_bytes;
                tma_load_2d(st, &maps.w[sg], lt * (kStTN / 8), o * kM1Rows, full_bar(s), pol);
                tma_load_2d(st + kM1WBytes, &maps.s[sg], lt * (kStTN * ssz / 8), o * 8, full_bar(s), pol);
            }
            s_issued = i;
        }
    } else if (warp == pw + 1) {
        pdl_wait();
        if (lane == 0) {
            int i = 0;
            ItemCursor cx(ibeg, a.noct);
            for (long long it = ibeg; it < iend; ++it, ++i, cx.next()) {
                const int s = m1_stage(i);
                if (i >= kM1Stages && !mbar_wait(empty_bar(s), m1_parity(i) ^ 1u, abort_flag, &g_gemv_status)) break;
                const int o = cx.o;
                bulk_g2s_nohint(smem0 + (uint32_t)s * a.stage_bytes + kM1WBytes + a.s_bytes,
                                reinterpret_cast<const uint8_t*>(a.x) + (size_t)o * kM1Rows * esz, kM1Rows * esz,
                                full_bar(s));
            }
        }
    } else {
        pdl_wait();
        const int g = lane >> 2, q = lane & 3, ctid = tid;
        const int grp = warp / kM1WarpsPerGroup, seg = warp % kM1WarpsPerGroup;  // 16-byte column segment
        const int colA = 32 * seg + 4 * g;  // this lane's columns: colA + j (j = 0, 1) and colA + 2 + j
        // ldmatrix.x4: lane L addresses row L%8 of matrix L/8; matrix m = (step p + m/2, k-pair m%2)
        const int lm = lane >> 3, lrr = lane & 7, lq = lrr >> 1, le = lrr & 1;
        const int lds = lm >> 1, lh = lm & 1;
        // y[n] of the tile's segment, scaled by its e4m3 inverse scale
        auto write_y = [&](long long t, int col, float v) {
            const TcSeg& sgm = tc_seg(a, tc_seg_of(a, t));
            const int n = ((int)t - sgm.tile0) * kStTN + col;
            const float inv = SFMT == G4B_SCALE_E4M3 ? sgm.inv : 1.0f;
            if (n < sgm.N) {
                if (YF32) ((float*)sgm.y)[n] = v * inv;
                else ((__half*)sgm.y)[n] = __float2half_rn(v * inv);
            }
        };
        constexpr int NPASS = XF32 ? 2 : 1;   // f32 x: two passes of 4 blocks
        constexpr int NSTEP = XF32 ? 8 : 16;  // mma steps per pass
        constexpr int RMUL = XF32 ? 4 : 2;    // rows advanced per step
        float acc[2][2];
        const long long t_first = ibeg / a.noct, t_last = iend > ibeg ? (iend - 1) / a.noct : t_first - 1;
        // Sum a shared tile's partials in CTA order (deterministic) and write y.
        auto reduce_tile = [&](long long t) {
            long long c_first, c_last;
            m1_span(a.mode, a.total, a.ntiles, a.noct, a.G, t, c_first, c_last);
            const int nseg = (int)(c_last - c_first + 1);
            if (ctid < kStTN) {
                const int col = ctid;
                float v = 0.f;
                for (int k0 = 0; k0 < nseg; k0 += 8) {
                    float pv[8];
                    #pragma unroll
                    for (int k = 0; k < 8; k++) {
                        pv[k] = 0.f;
                        if (k0 + k < nseg) {
                            const long long cc = c_first + k0 + k;
                            const long long sl = cc * a.maxseg + (t - s_ftile[cc]);
                            pv[k] = __ldcg(&a.partial[(size_t)sl * kStTN + col]);
                        }
                    }
                    #pragma unroll
                    for (int k = 0; k < 8; k++)
                        if (k0 + k < nseg) v += pv[k];
                }
                write_y(t, col, v);
            }
            if (ctid == 0) a.counters[t] = 0u;  // ready for the next call
        };
        int nflush = 0;

        for (long long t = t_first; t <= t_last; ++t) {
            acc[0][0] = acc[0][1] = acc[1][0] = acc[1][1] = 0.f;
            const long long tb = max(ibeg, t * a.noct), te = min(iend, (t + 1) * a.noct);
            long long it = tb + ((grp - (tb - ibeg) % kM1Groups + kM1Groups) % kM1Groups);
            for (; it < te; it += kM1Groups) {
                const int i = (int)(it - ibeg);
                const int s = m1_stage(i);
                if (!mbar_wait(full_bar(s), m1_parity(i), abort_flag, &g_gemv_status)) {
                    __syncwarp();
                    if (lane == 0) mbar_arrive(empty_bar(s));
                    continue;
                }
                const uint32_t st_u = smem0 + (uint32_t)s * a.stage_bytes;
                const uint8_t* st = smem + (size_t)s * a.stage_bytes;
                const uint8_t* sc = st + kM1WBytes;
                const uint8_t* xs = sc + a.s_bytes;
                // block sums X[b] of the stage's 8 blocks: lane l sums rows 8l..8l+7
                float xsum;
                if constexpr (XF32) {
                    const float4 v0 = *reinterpret_cast<const float4*>(xs + lane * 32);
                    const float4 v1 = *reinterpret_cast<const float4*>(xs + lane * 32 + 16);
                    xsum = ((((((v0.x + v0.y) + v0.z) + v0.w) + v1.x) + v1.y) + v1.z) + v1.w;
                } else {
                    const uint4 v = *reinterpret_cast<const uint4*>(xs + lane * 16);
                    xsum = ((((((h_lo(v.x) + h_hi(v.x)) + h_lo(v.y)) + h_hi(v.y)) + h_lo(v.z)) + h_hi(v.z)) + h_lo(v.w)) +
                           h_hi(v.w);
                }
                xsum += __shfl_xor_sync(0xffffffffu, xsum, 1);
                xsum += __shfl_xor_sync(0xffffffffu, xsum, 2);
                #pragma unroll 1
                for (int pass = 0; pass < NPASS; pass++) {
                    // ldmatrix row of this lane: block and rotated row (swizzle phase differs per lane)
                    const int lblk = XF32 ? 4 * pass + lq : lq + 4 * lh;
                    const int lrot = RMUL * lds + 2 * lq + le + ((XF32 && lh) ? 2 : 0);
                    const uint32_t lbase = st_u + (uint32_t)(lblk * 32 * 128);
                    // row offsets for the 4 step phases (steps p = 4m + d advance the row by 8m (f16) / 16m (f32))
                    uint32_t roff[4], swz[4];
                    #pragma unroll
                    for (int d = 0; d < 4; d++) {
                        const int r = (RMUL * d + lrot) & 31;
                        roff[d] = (uint32_t)(r * 128);
                        swz[d] = (uint32_t)((seg ^ (r & 7)) << 4);
                    }
                    // B-fragment sources: lanes that feed zeros read a zeroed area instead
                    uint32_t xb0, xb1, xoff;
                    if constexpr (XF32) {
                        const bool mine = (g >> 1) == q;
                        xb0 = mine ? smem_u32(xs) + (uint32_t)((4 * pass + q) * 128) : smem_u32(s_zero);
                        xb1 = xb0;
                        xoff = (uint32_t)(8 * q);
                    } else {
                        xb0 = g == q ? smem_u32(xs) + (uint32_t)(q * 64) : smem_u32(s_zero);
                        xb1 = g == q + 4 ? smem_u32(xs) + (uint32_t)((q + 4) * 64) : smem_u32(s_zero);
                        xoff = (uint32_t)(4 * q);
                    }
                    float C[2][4];
                    #pragma unroll
                    for (int k = 0; k < 2; k++) C[k][0] = C[k][1] = C[k][2] = C[k][3] = 0.f;
                    #pragma unroll
                    for (int p = 0; p < NSTEP; p += 2) {
                        const int d = p & 3, mrow = (p >> 2) * (RMUL == 2 ? 1024 : 2048);
                        const uint32_t addr = lbase + (((roff[d] + (uint32_t)mrow) & 4095u) | swz[d]);
                        uint32_t ra0, rb0, ra1, rb1;
                        ldsm_x4_trans(addr, ra0, rb0, ra1, rb1);
                        #pragma unroll
                        for (int ss = 0; ss < 2; ss++) {
                            const uint32_t RA = ss ? ra1 : ra0, RB = ss ? rb1 : rb0;
                            const int pp = p + ss;
                            uint32_t b0, b1;
                            if constexpr (XF32) {
                                const uint32_t o0 = (xoff + 16u * pp) & 127u, o1 = (xoff + 16u * pp + 8u) & 127u;
                                float2 xa, xb;
                                asm volatile("ld.shared.v2.f32 {%0,%1}, [%2];" : "=f"(xa.x), "=f"(xa.y) : "r"(xb0 + o0));
                                asm volatile("ld.shared.v2.f32 {%0,%1}, [%2];" : "=f"(xb.x), "=f"(xb.y) : "r"(xb1 + o1));
                                const bool lo = (g & 1) != 0;
                                b0 = split_pair(xa.x, xa.y, lo);
                                b1 = split_pair(xb.x, xb.y, lo);
                            } else {
                                const uint32_t o = (xoff + 4u * pp) & 63u;
                                asm volatile("ld.shared.b32 %0, [%1];" : "=r"(b0) : "r"(xb0 + o));
                                asm volatile("ld.shared.b32 %0, [%1];" : "=r"(b1) : "r"(xb1 + o));
                            }
                            const uint32_t RA8 = RA >> 8, RB8 = RB >> 8;
                            mma_16816(C[0], RA & 0x000F000Fu, RA8 & 0x000F000Fu, RB & 0x000F000Fu, RB8 & 0x000F000Fu, b0, b1);
                            mma_16816(C[1], RA & 0x00F000F0u, RA8 & 0x00F000F0u, RB & 0x00F000F0u, RB8 & 0x00F000F0u, b0, b1);
                        }
                    }
                    // per-block scale, 2^E and -8 X correction, in f32
                    int blk0, blk1;
                    if constexpr (XF32) { blk0 = 4 * pass + q; blk1 = blk0; } else { blk0 = 2 * q; blk1 = 2 * q + 1; }
                    const float X0 = __shfl_sync(0xffffffffu, xsum, 4 * blk0);
                    const float X1 = __shfl_sync(0xffffffffu, xsum, 4 * blk1);
                    // scales of columns colA .. colA+3 in blocks blk0 / blk1
                    float s0[4], s1[4];
                    if constexpr (SFMT == G4B_SCALE_F16) {
                        const uint2 u0 = *reinterpret_cast<const uint2*>(sc + (blk0 * kStTN + colA) * 2);
                        const uint2 u1 = *reinterpret_cast<const uint2*>(sc + (blk1 * kStTN + colA) * 2);
                        s0[0] = h_lo(u0.x); s0[1] = h_hi(u0.x); s0[2] = h_lo(u0.y); s0[3] = h_hi(u0.y);
                        s1[0] = h_lo(u1.x); s1[1] = h_hi(u1.x); s1[2] = h_lo(u1.y); s1[3] = h_hi(u1.y);
                    } else {
                        const uint32_t u0 = *reinterpret_cast<const uint32_t*>(sc + blk0 * kStTN + colA);
                        const uint32_t u1 = *reinterpret_cast<const uint32_t*>(sc + blk1 * kStTN + colA);
                        uint32_t h;
                        h = e4m3x2_to_f16x2((uint16_t)(u0 & 0xffffu)); s0[0] = h_lo(h); s0[1] = h_hi(h);
                        h = e4m3x2_to_f16x2((uint16_t)(u0 >> 16));     s0[2] = h_lo(h); s0[3] = h_hi(h);
                        h = e4m3x2_to_f16x2((uint16_t)(u1 & 0xffffu)); s1[0] = h_lo(h); s1[1] = h_hi(h);
                        h = e4m3x2_to_f16x2((uint16_t)(u1 >> 16));     s1[2] = h_lo(h); s1[3] = h_hi(h);
                    }
                    #pragma unroll
                    for (int j = 0; j < 2; j++) {
                        const float E = j ? 1048576.0f : 16777216.0f;  // 2^20 (high nibble) / 2^24 (low nibble)
                        // C[j][0..1]: column colA + j; C[j][2..3]: column colA + 2 + j
                        if constexpr (XF32) {
                            acc[j][0] = fmaf(s0[j], fmaf(C[j][0] + C[j][1], E, -8.0f * X0), acc[j][0]);
                            acc[j][1] = fmaf(s0[2 + j], fmaf(C[j][2] + C[j][3], E, -8.0f * X0), acc[j][1]);
                        } else {
                            acc[j][0] = fmaf(s0[j], fmaf(C[j][0], E, -8.0f * X0), acc[j][0]);
                            acc[j][0] = fmaf(s1[j], fmaf(C[j][1], E, -8.0f * X1), acc[j][0]);
                            acc[j][1] = fmaf(s0[2 + j], fmaf(C[j][2], E, -8.0f * X0), acc[j][1]);
                            acc[j][1] = fmaf(s1[2 + j], fmaf(C[j][3], E, -8.0f * X1), acc[j][1]);
                        }
                    }
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(empty_bar(s));
            }
            // ---- flush tile t: quad sum (the lanes of a quad hold different blocks), group sum, CTA share
            #pragma unroll
            for (int k = 0; k < 2; k++)
                #pragma unroll
                for (int h = 0; h < 2; h++) {
                    float v = acc[k][h];
                    v += __shfl_xor_sync(0xffffffffu, v, 1);
                    v += __shfl_xor_sync(0xffffffffu, v, 2);
                    acc[k][h] = v;
                }
            const int rb = nflush++ & 1;
            if (q == 0) {
                #pragma unroll
                for (int j = 0; j < 2; j++) {
                    red[rb][grp][colA + j] = acc[j][0];
                    red[rb][grp][colA + 2 + j] = acc[j][1];
                }
            }
            named_bar_sync(1, kM1Consumers);
            const int c = blockIdx.x;
            // a tile is this CTA's alone when the CTA owns all its k-chunks
            const bool single = ibeg <= t * a.noct && iend >= (t + 1) * a.noct;
            long long c_first = 0, c_last = 0;
            if (!single) m1_span(a.mode, a.total, a.ntiles, a.noct, a.G, t, c_first, c_last);
            const bool ok = !*abort_flag;
            const long long slot = (long long)c * a.maxseg + (t - ibeg / a.noct);
            if (ctid < kStTN && ok) {
                const int col = ctid;
                float v = red[rb][0][col];
                #pragma unroll
                for (int gg = 1; gg < kM1Groups; gg++) v += red[rb][gg][col];
                if (single) {
                    write_y(t, col, v);
                } else {
                    a.partial[(size_t)slot * kStTN + col] = v;
                }
            }
            if (!single) {
                // publish this CTA's partial: one thread arrives for the CTA (after the barrier) with an
                // acquire-release add on the tile's counter; the last of the tile's CTAs to arrive reduces it
                named_bar_sync(1, kM1Consumers);
                if (t < t_last) {
                    // not our final tile: do not stall the other consumers on the atomic; if we
                    // turn out to be the last arriver, the reduction runs after our last item
                    if (ctid == 0 && ok && atom_add_acq_rel_gpu(&a.counters[t], 1u) == (unsigned)(c_last - c_first))
                        s_pending = t;
                } else {
                    if (ctid == 0)
                        s_last = ok && atom_add_acq_rel_gpu(&a.counters[t], 1u) == (unsigned)(c_last - c_first) ? 1u : 0u;
                    named_bar_sync(1, kM1Consumers);
                    if (s_last) reduce_tile(t);
                }
            }
        }
        // the deferred reduction of an earlier tile this CTA was the last to finish
        named_bar_sync(1, kM1Consumers);
        if (s_pending >= 0 && !*abort_flag) reduce_tile(s_pending);
    }

    __syncthreads();
    if (tid == 0 && *abort_flag) {
        const int issued = s_issued;
        for (int i = max(0, issued - kM1Stages); i < issued; i++) {
            const uint64_t t0 = global_ns();
            while (!mbar_try_wait(full_bar(m1_stage(i)), m1_parity(i)) && global_ns() - t0 < kWaitLimitNs) {
            }
        }
    }
}

// ---------------------------------------------------------------- GEMV chains
// A chain of M = 1 GEMV steps run by one persistent launch (g4b_gemv_chain_*):
// the engine's recorded command buffer of gemv() dispatches with a barrier
// after each (src/vk_engine.py:254-290, bar() at :261).  Step j reads x only
// after every column tile of step j-1 has been written (a per-step count of
// written tiles) -- or, when x is step j-1's first output, each 256-row slice
// as soon as that slice's tile is (forwarded words) -- and writes only after
// steps j-2 and j-3 are complete; the weight stream runs on from one step into
// the next.
//
// Each step carries its own partition of (tile, k-chunk) items over the CTAs,
// chosen on the host: CTA c owns the contiguous items [range[c], range[c+1]).
// For the small decode GEMVs the host prefers tile-aligned ranges (no CTA
// straddles two shared tiles), so a CTA never runs its items one tile after
// another with a split-K flush and a deferred reduction in between.
struct ChainStep {
    const void* x;
    TcSeg seg0, seg1, seg2;
    const int* range;  // [G + 1]: CTA c < G owns items [range[c], range[c+1]); item = tile * noct + k-chunk
    const int* cspan;  // [ntiles][2]: first and last CTA owning items of tile t (bit 31 of the first:
                       // that CTA's range starts in an earlier tile)
    int nseg, K, noct, ntiles, G;
    // tensor parallel: yreg >= 0: every written y value of segment 0 is also pushed, tagged with the
    // run's epoch, into slot [rank] of region yreg of every rank's exchange buffer; xreg >= 0: x is
    // the rank-order sum of the world slots of region xreg (the all-reduce of the previous step's y)
    int xreg, yreg;
    // forwarded x (one GPU): yfw >= 0: every written y value of segment 0 is also stored, tagged with
    // the run's epoch, at word yfw + n of the chain's forward area; xfw >= 0: x is the previous step's
    // segment-0 output read from those words (each x slice waits only for its own words, not for the
    // whole previous step)
    int xfw, yfw;
    // the activation warp's step wait covers the counts of steps wlo .. j-1 (wlo < j-1 when the steps
    // in between read forwarded x and so never waited on a count themselves); xind: none of the chain's
    // steps writes x, so its first slice may be loaded before the wait
    int wlo, xind;
    // completion count of the step: its tiles, plus the slices of h_out its loads write (NORMADD)
    int done;
    // fused element-wise work on x (g4b_chain_xform; one rank only): kind, an RMSNORM over a vector
    // no step of the chain wrote (the activation warp sums its squares itself), and the number of
    // column tiles of the producer step (the one before) whose sums it reads
    int xf_kind, xf_self, xf_ptiles;
    float xf_scale, xf_eps;
    const void* xf_a;
    const void* xf_b;
    const float* xf_w;
    const float* xf_wpost;
    float* xf_hout;
    const float* xf_sums;      // the producer's tile sums [xf_ptiles][4]
    // producer side: each segment-0 tile written also stores {sum h^2, sum h*(y*w), sum (y*w)^2,
    // sum y^2} over its columns (h = sum_res, w = sum_wpost; both null: only sum y^2) for the next
    // step's norm
    float* sums_out;
    const float* sum_res;
    const float* sum_wpost;
};
static_assert(sizeof(ChainStep) % 8 == 0, "ChainStep is copied as 32-bit words");

struct ChainArgs {
    const ChainStep* steps;   // [nsteps], device memory
    const CUtensorMap* maps;  // [nsteps][2 * kTcMaxSeg]: weight maps, then scale maps; device memory
    unsigned* sync;           // [nsteps] tiles written per step, then the exit count and the abort word
    unsigned long long* partial;  // [2][2 * G][kStTN] {f32 bits, step tag} words: CTA c's partials of its
                                  // first and its last tile, by step parity
    unsigned long long* const* peers;  // [world] exchange buffers (this rank's own at [rank]); null if world 1
    unsigned long long* fwd;           // the forward area: {f32 bits, epoch} words of forwarded outputs
    int nsteps, stage_bytes, s_bytes, maxtiles, G, rank, world;
    int pf_items;             // L2 prefetch distance: items ahead of the TMA producer (0 = off)
};

// element-wise work fused into a chain step's activation load (G4B_XF_*)
constexpr int kXfNone = 0, kXfRmsNorm = 1, kXfNormAdd = 2, kXfGeluMul = 3;
static_assert(kXfNone == G4B_XF_NONE && kXfRmsNorm == G4B_XF_RMSNORM && kXfNormAdd == G4B_XF_NORMADD &&
                  kXfGeluMul == G4B_XF_GELU_MUL,
              "the kernel's element-wise kinds are the header's");

// elements [r0, r0 + 8) of an f32 (F32) or f16 vector as f32, through L2 (the vector may have
// been written by other SMs during the launch)
template <bool F32>
__device__ __forceinline__ void load8(const void* p, int r0, float (&v)[8]) {
    if constexpr (F32) {
        const float4* q = reinterpret_cast<const float4*>(reinterpret_cast<const float*>(p) + r0);
        const float4 a = __ldcg(q), b = __ldcg(q + 1);
        v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
        v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
    } else {
        const uint4 u = __ldcg(reinterpret_cast<const uint4*>(reinterpret_cast<const __half*>(p) + r0));
        v[0] = h_lo(u.x); v[1] = h_hi(u.x); v[2] = h_lo(u.y); v[3] = h_hi(u.y);
        v[4] = h_lo(u.z); v[5] = h_hi(u.z); v[6] = h_lo(u.w); v[7] = h_hi(u.w);
    }
}

// A chain stage's x slice, 1 KB either way, then the slice's 8 block sums (f32):
//   f16 x: 32-row block b at bytes [128 b, 128 b + 64), repeated at +64, so the consumers read a
//          block's words from any rotation without wrapping;
//   f32 x: block b at [128 b, 128 b + 128): 16 words f16x2(hi) of its row pairs, then the 16 words
//          f16x2(lo), hi = f16(x) and lo = f16(x - hi) -- the split the tensor cores take f32 x in,
//          made once here instead of by every consumer lane.
// Lane l holds rows 8l .. 8l+7 (block l/4).
constexpr int kChainXBytes = kM1Rows * 4;
constexpr int kChainXSumBytes = 32;
__device__ __forceinline__ int chain_xoff16(int lane) { return (lane >> 2) * 128 + (lane & 3) * 16; }

// a lane's 8 activations into a stage's x slice (rows 8*lane .. +8), in the chain's x dtype; for f32 x
// also the slice's block sums (a block's 32 values added in a fixed order: a lane's 8 in row order,
// then lanes l^1, l^2) for the -8 X correction -- f16 x leaves them to the consumers, which read the
// 32 values anyway
template <bool F32>
__device__ __forceinline__ void store8(uint8_t* dst, int lane, const float (&v)[8]) {
    if constexpr (F32) {
        uint4 hi, lo;
        uint32_t* hw = &hi.x;
        uint32_t* lw = &lo.x;
        #pragma unroll
        for (int k = 0; k < 4; k++) {
            const __half ha = __float2half_rn(v[2 * k]), hb = __float2half_rn(v[2 * k + 1]);
            hw[k] = pack_half2(ha, hb);
            lw[k] = pack_half2(__float2half_rn(v[2 * k] - __half2float(ha)),
                               __float2half_rn(v[2 * k + 1] - __half2float(hb)));
        }
        *reinterpret_cast<uint4*>(dst + chain_xoff16(lane)) = hi;
        *reinterpret_cast<uint4*>(dst + chain_xoff16(lane) + 64) = lo;
        float s = ((((((v[0] + v[1]) + v[2]) + v[3]) + v[4]) + v[5]) + v[6]) + v[7];
        s += __shfl_xor_sync(0xffffffffu, s, 1);
        s += __shfl_xor_sync(0xffffffffu, s, 2);
        if ((lane & 3) == 0) reinterpret_cast<float*>(dst + kChainXBytes)[lane >> 2] = s;
    } else {
        uint4 h;
        h.x = pack_half2(__float2half_rn(v[0]), __float2half_rn(v[1]));
        h.y = pack_half2(__float2half_rn(v[2]), __float2half_rn(v[3]));
        h.z = pack_half2(__float2half_rn(v[4]), __float2half_rn(v[5]));
        h.w = pack_half2(__float2half_rn(v[6]), __float2half_rn(v[7]));
        *reinterpret_cast<uint4*>(dst + chain_xoff16(lane)) = h;
        *reinterpret_cast<uint4*>(dst + chain_xoff16(lane) + 64) = h;
    }
}

// a lane's 8 consecutive activations (rows 8*lane .. +8) of an f32 or f16 slice as f32
template <bool F32>
__device__ __forceinline__ void unpack8(const uint4 (&u)[F32 ? 2 : 1], float (&v)[8]) {
    if constexpr (F32) {
        v[0] = __uint_as_float(u[0].x); v[1] = __uint_as_float(u[0].y);
        v[2] = __uint_as_float(u[0].z); v[3] = __uint_as_float(u[0].w);
        v[4] = __uint_as_float(u[1].x); v[5] = __uint_as_float(u[1].y);
        v[6] = __uint_as_float(u[1].z); v[7] = __uint_as_float(u[1].w);
    } else {
        v[0] = h_lo(u[0].x); v[1] = h_hi(u[0].x); v[2] = h_lo(u[0].y); v[3] = h_hi(u[0].y);
        v[4] = h_lo(u[0].z); v[5] = h_hi(u[0].z); v[6] = h_lo(u[0].w); v[7] = h_hi(u[0].w);
    }
}

// exchange-buffer words: {f32 bits (low), run epoch (high)}; a 64-bit aligned
// access is single-copy atomic, so a word that carries the epoch carries its value
__device__ __forceinline__ void st_relaxed_sys_u64(unsigned long long* p, unsigned long long v) {
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_relaxed_sys_u64(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void st_relaxed_gpu_u64(unsigned long long* p, unsigned long long v) {
    asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_relaxed_gpu_u64(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ unsigned ld_acquire_gpu_u32(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Bounded wait until *count >= need (acquire).  Gives up (false) on the
// CTA's or the chain's abort word, or after kWaitLimitNs (raising both).
__device__ __forceinline__ bool chain_wait_count(const unsigned* count, unsigned need, unsigned* gabort,
                                                 volatile int* abort) {
    if (ld_acquire_gpu_u32(count) >= need) return true;
    const uint64_t t0 = global_ns();
    for (int spin = 0;; spin++) {
        if (spin > 4096) __nanosleep(64);  // a step boundary normally resolves within the spin
        if (ld_acquire_gpu_u32(count) >= need) return true;
        if (*abort || *(volatile unsigned*)gabort) {
            *abort = 1;
            return false;
        }
        if (global_ns() - t0 > kWaitLimitNs) {
            *abort = 1;
            atomicOr(&g_gemv_status, kStatusTimeout);
            atomicExch(gabort, 1u);
            return false;
        }
    }
}

// One persistent grid of one CTA per SM (a cooperative launch: every CTA is
// resident, so the steps can wait on one another).  Warp roles as in
// gemv_i4_m1_kernel; the activation warp stores x with plain loads (x was
// written by other SMs during this launch) and arrives on the stage's full
// barrier itself.
template <bool XF32, int SFMT, bool YF32>
__global__ void __launch_bounds__(kChainThreads, 1) gemv_i4_chain_kernel(const __grid_constant__ ChainArgs ch) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    __shared__ uint64_t bars[2 * kM1Stages];
    __shared__ float red[2][kM1Groups][kStTN];  // double-buffered: consecutive flushes never share it
    __shared__ int s_pending;                    // shared tile this CTA must still reduce (-1: none)
    __shared__ int s_issued, s_xdone;
    __shared__ int s_prod, s_prod_done;          // items the TMA producer has issued; it has stopped
    __shared__ int s_abort;
    __shared__ __align__(16) uint32_t s_zero[32];  // B-fragment source for lanes that feed zeros
    __shared__ __align__(8) ChainStep s_step[2];   // the consumers' current and next step
    __shared__ unsigned long long* s_peers[8];
    __shared__ float4 s_tsum[2][kM1WarpsPerGroup];  // per-warp tile sums (double-buffered)
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int c = blockIdx.x;
    volatile int* abort_flag = &s_abort;
    constexpr int esz = XF32 ? 4 : 2;
    constexpr int ssz = SFMT == G4B_SCALE_F16 ? 2 : 1;
    constexpr int kStepWords = (int)(sizeof(ChainStep) / 4);
    const int nsteps = ch.nsteps, stage_bytes = ch.stage_bytes, s_bytes = ch.s_bytes;
    unsigned* const gabort = ch.sync + nsteps + 1;
    // this run's epoch (the last CTA of the previous run advanced the count)
    const unsigned epoch = *(volatile unsigned*)(ch.sync + nsteps + 2) + 1u;
    // the swizzle pattern repeats every 1024 bytes: align the stages to it
    const uint32_t raw0 = smem_u32(smem_raw);
    const uint32_t smem0 = (raw0 + 1023u) & ~1023u;
    uint8_t* smem = smem_raw + (smem0 - raw0);
    const uint32_t bar0 = smem_u32(bars);
    auto full_bar = [&](int s) { return bar0 + 8u * s; };
    auto empty_bar = [&](int s) { return bar0 + 8u * (kM1Stages + s); };
    // this CTA's items of a step
    auto my_range = [&](const ChainStep& d, int& ib, int& ie) {
        if (c < d.G) {
            ib = __ldg(d.range + c);
            ie = __ldg(d.range + c + 1);
        } else {
            ib = ie = 0;
        }
    };
    const int pw = kM1Consumers / 32;  // first producer warp

    if (tid == 0) {
        for (int s = 0; s < kM1Stages; s++) {
            mbar_init(full_bar(s), 2);  // the TMA producer's arrival (with the bytes) + the activation warp's
            mbar_init(empty_bar(s), kM1WarpsPerGroup);
        }
        s_abort = 0;
        s_issued = 0;
        s_xdone = 0;
        s_prod = 0;
        s_prod_done = 0;
        s_pending = -1;
        fence_mbar_init();
    }
    if (tid < 32) s_zero[tid] = 0u;
    if (tid < kStepWords) reinterpret_cast<uint32_t*>(&s_step[0])[tid] = __ldg(reinterpret_cast<const uint32_t*>(ch.steps) + tid);
    if (tid < ch.world && ch.peers) s_peers[tid] = ch.peers[tid];
    // a programmatic dependent launched after this chain may be scheduled now (it waits for our completion)
    pdl_launch_dependents();
    __syncthreads();

    if (warp == pw) {
        if (lane == 0) {
            const uint64_t pol = l2_evict_first_policy();
            int i = 0;  // this CTA's item number over all steps
            bool stop = false;
            for (int sg = 0; sg < 2 * kTcMaxSeg; sg++) prefetch_tensor_map(ch.maps + sg);
            for (int j = 0; j < nsteps && !stop; j++) {
                const ChainStep d = ch.steps[j];
                const CUtensorMap* wm = ch.maps + (size_t)j * 2 * kTcMaxSeg;
                const CUtensorMap* sm = wm + kTcMaxSeg;
                // the maps were copied in before the launch and never change during it
                if (j + 1 < nsteps)
                    for (int sg = 0; sg < 2 * kTcMaxSeg; sg++) prefetch_tensor_map(wm + 2 * kTcMaxSeg + sg);
                int ibeg, iend;
                my_range(d, ibeg, iend);
                int t = ibeg / d.noct, o = ibeg - t * d.noct;
                for (int it = ibeg; it < iend; ++it, ++i) {
                    const int s = m1_stage(i);
                    // after an abort the consumers release stages without reading them: issue nothing more
                    if (*abort_flag ||
                        (i >= kM1Stages && !mbar_wait(empty_bar(s), m1_parity(i) ^ 1u, abort_flag, &g_gemv_status))) {
                        stop = true;
                        break;
                    }
                    const int sg = tc_seg_of(d, t);
                    const int lt = t - tc_seg(d, sg).tile0;
                    mbar_arrive_expect_tx(full_bar(s), kM1WBytes + s_bytes);
                    const uint32_t st = smem0 + (uint32_t)s * stage_bytes;
                    tma_load_2d(st, &wm[sg], lt * (kStTN / 8), o * kM1Rows, full_bar(s), pol);
                    tma_load_2d(st + kM1WBytes, &sm[sg], lt * (kStTN * ssz / 8), o * 8, full_bar(s), pol);
                    *(volatile int*)&s_prod = i + 1;
                    if (++o == d.noct) {
                        o = 0;
                        ++t;
                    }
                }
            }
            s_issued = i;
            *(volatile int*)&s_prod_done = 1;
        }
    } else if (warp == pw + 2) {
        // L2 prefetch of the weight and scale tiles the TMA producer will load next.  A step
        // boundary holds the consumers, and with them the producer once its stages are full;
        // meanwhile HBM keeps streaming the coming items into L2, and their TMA loads then hit L2.
        // This warp stays at most pf_items items ahead of the producer, skips items the producer
        // has already issued, never holds anyone up, and stops with the producer.
        if (lane == 0 && ch.pf_items > 0) {
            int i = 0;
            bool stop = false;
            for (int j = 0; j < nsteps && !stop; j++) {
                const ChainStep d = ch.steps[j];
                const CUtensorMap* wm = ch.maps + (size_t)j * 2 * kTcMaxSeg;
                const CUtensorMap* sm = wm + kTcMaxSeg;
                int ibeg, iend;
                my_range(d, ibeg, iend);
                int t = ibeg / d.noct, o = ibeg - t * d.noct;
                for (int it = ibeg; it < iend; ++it, ++i) {
                    if (i >= *(volatile int*)&s_prod + ch.pf_items) {
                        const uint64_t t0 = global_ns();
                        while (i >= *(volatile int*)&s_prod + ch.pf_items) {
                            if (*abort_flag || *(volatile int*)&s_prod_done || global_ns() - t0 > kWaitLimitNs) {
                                stop = true;
                                break;
                            }
                            __nanosleep(256);
                        }
                        if (stop) break;
                    }
                    if (i >= *(volatile int*)&s_prod) {
                        const int sg = tc_seg_of(d, t);
                        const int lt = t - tc_seg(d, sg).tile0;
                        tma_prefetch_l2_2d(&wm[sg], lt * (kStTN / 8), o * kM1Rows);
                        tma_prefetch_l2_2d(&sm[sg], lt * (kStTN * ssz / 8), o * 8);
                        // the item's x slice too, so that its load after the step boundary hits L2 (the
                        // lines stay coherent with whatever an earlier step writes to them later)
                        if (d.x && d.xreg < 0 && d.xfw < 0 && d.xf_kind == kXfNone)
                            bulk_prefetch_l2(reinterpret_cast<const uint8_t*>(d.x) + (size_t)o * kM1Rows * esz,
                                             kM1Rows * esz);
                    }
                    if (++o == d.noct) {
                        o = 0;
                        ++t;
                    }
                }
            }
        }
    } else if (warp == pw + 1) {
        // x slices by plain loads (L2, not L1: x was written by other SMs during this launch).  Launched as a
        // programmatic dependent (G4B_CHAIN_RUN_PDL), the chain streams weights from its start, and only
        // this warp -- whose loads are the first reads of anything an earlier kernel wrote -- waits for the
        // kernel before it; every write of the chain follows these loads.
        pdl_wait();
        int i = 0;
        bool stop = false;
        for (int j = 0; j < nsteps && !stop; j++) {
            const ChainStep* dj = ch.steps + j;
            const int noct = dj->noct, K = dj->K, xreg = dj->xreg, xfw = dj->xfw;
            const uint8_t* x = reinterpret_cast<const uint8_t*>(dj->x);
            int ibeg, iend;
            my_range(*dj, ibeg, iend);
            const int xk = dj->xf_kind;
            // an x that no step writes: its first slice is loaded before the step wait, so that the
            // wait's end is followed by shared-memory stores only
            constexpr int kPreVecs = kM1Rows * esz / 512;  // 16-byte loads per lane for one slice
            uint4 pre[kPreVecs];
            const bool hoist = dj->xind && xk == kXfNone && xreg < 0 && xfw < 0 && iend > ibeg;
            if (hoist) {
                const uint4* src = reinterpret_cast<const uint4*>(x + (size_t)(ibeg % noct) * kM1Rows * esz);
                #pragma unroll
                for (int b = 0; b < kPreVecs; b++) pre[b] = __ldcg(src + kPreVecs * lane + b);
            }
            // an all-reduce input and a forwarded x carry their own readiness (the epoch in every word):
            // no step wait.  Otherwise wait for the counts of steps wlo .. j-1 at once, a lane per step.
            if (iend > ibeg && j > 0 && xreg < 0 && xfw < 0) {
                bool ok = true;
                for (int k0 = dj->wlo; k0 < j && ok; k0 += 32) {
                    const int k = k0 + lane;
                    const bool okl = k < j ? chain_wait_count(&ch.sync[k], (unsigned)ch.steps[k].done, gabort, abort_flag)
                                           : true;
                    ok = __all_sync(0xffffffffu, okl);
                }
                if (!ok) break;
            }
            // the step's norm scales, once per step: from the producer's tile sums (summed in a fixed
            // lane order) or, for a vector the chain did not write, from the vector itself.  The sums'
            // loads are issued here and only reduced after the first slice's loads are in flight, so
            // they cost no round trip of their own.
            float inv_r = 0.f, inv_h = 0.f;
            bool scales_ready = xk == kXfNone || xk == kXfGeluMul || iend <= ibeg;
            float4 S = make_float4(0.f, 0.f, 0.f, 0.f);
            if (!scales_ready) {
                if (dj->xf_self) {
                    for (int r0 = 8 * lane; r0 < K; r0 += 256) {
                        float a8[8];
                        load8<true>(dj->xf_a, r0, a8);
                        #pragma unroll
                        for (int e = 0; e < 8; e++) S.w = fmaf(a8[e], a8[e], S.w);
                    }
                } else {
                    for (int t = lane; t < dj->xf_ptiles; t += 32) {
                        const float4 v = __ldcg(reinterpret_cast<const float4*>(dj->xf_sums) + t);
                        S.x += v.x;
                        S.y += v.y;
                        S.z += v.z;
                        S.w += v.w;
                    }
                }
            }
            auto norm_scales = [&]() {
                #pragma unroll
                for (int m = 16; m >= 1; m >>= 1) {
                    S.x += __shfl_xor_sync(0xffffffffu, S.x, m);
                    S.y += __shfl_xor_sync(0xffffffffu, S.y, m);
                    S.z += __shfl_xor_sync(0xffffffffu, S.z, m);
                    S.w += __shfl_xor_sync(0xffffffffu, S.w, m);
                }
                const float invK = 1.0f / (float)K;
                if (xk == kXfRmsNorm) {
                    inv_h = rsqrtf(S.w * invK + dj->xf_eps);
                } else {
                    // h' = (h + r * inv_r * w_post) * scale, so sum h'^2 = scale^2 (sum h^2
                    // + 2 inv_r sum h (r w_post) + inv_r^2 sum (r w_post)^2)
                    inv_r = rsqrtf(S.w * invK + dj->xf_eps);
                    const float sh = dj->xf_scale * dj->xf_scale * fmaf(inv_r * inv_r, S.z, fmaf(2.0f * inv_r, S.y, S.x));
                    inv_h = rsqrtf(fmaxf(sh, 0.f) * invK + dj->xf_eps);
                }
                scales_ready = true;
            };
            int nh = 0;  // slices of h_out this warp wrote in this step
            int o = ibeg % noct;
            for (int it = ibeg; it < iend; ++it, ++i) {
                const int s = m1_stage(i);
                if (i >= kM1Stages) {
                    bool ok = true;
                    if (lane == 0) ok = mbar_wait(empty_bar(s), m1_parity(i) ^ 1u, abort_flag, &g_gemv_status);
                    if (!__shfl_sync(0xffffffffu, ok, 0)) {
                        stop = true;
                        break;
                    }
                }
                uint8_t* dst = smem + (size_t)s * stage_bytes + kM1WBytes + s_bytes;
                if (xk != kXfNone) {
                    // rows o*256 + 8*lane .. +8 through the step's element-wise work, in f32
                    const int r0 = o * kM1Rows + 8 * lane;
                    float v[8];
                    if (xk == kXfGeluMul) {
                        // vk/gelumul.comp: gelu_tanh(gate) * up
                        float g8[8], u8[8];
                        load8<YF32>(dj->xf_a, r0, g8);
                        load8<YF32>(dj->xf_b, r0, u8);
                        #pragma unroll
                        for (int e = 0; e < 8; e++) {
                            const float xg = g8[e];
                            const float gl = 0.5f * xg * (1.0f + tanhf(0.7978845608028654f * (xg + 0.044715f * xg * xg * xg)));
                            v[e] = gl * u8[e];
                        }
                    } else if (xk == kXfRmsNorm) {
                        // vk/rmsnorm.comp: x * inv * w
                        float a8[8], w8[8];
                        if (dj->xf_self) load8<true>(dj->xf_a, r0, a8);
                        else load8<YF32>(dj->xf_a, r0, a8);
                        load8<true>(dj->xf_w, r0, w8);
                        if (!scales_ready) norm_scales();
                        #pragma unroll
                        for (int e = 0; e < 8; e++) v[e] = a8[e] * inv_h * w8[e];
                    } else {
                        // vk/normadd.comp then vk/rmsnorm.comp: h' = (h + r * inv_r * w_post) * scale,
                        // x = h' * inv_h * w; the CTA holding tile 0's item of this slice stores h'
                        float r8[8], h8[8], p8[8], w8[8];
                        load8<YF32>(dj->xf_a, r0, r8);
                        load8<true>(dj->xf_b, r0, h8);
                        load8<true>(dj->xf_wpost, r0, p8);
                        load8<true>(dj->xf_w, r0, w8);
                        if (!scales_ready) norm_scales();
                        #pragma unroll
                        for (int e = 0; e < 8; e++) {
                            h8[e] = (h8[e] + r8[e] * inv_r * p8[e]) * dj->xf_scale;
                            v[e] = h8[e] * inv_h * w8[e];
                        }
                        if (it < noct) {
                            float4* ho = reinterpret_cast<float4*>(dj->xf_hout + r0);
                            ho[0] = make_float4(h8[0], h8[1], h8[2], h8[3]);
                            ho[1] = make_float4(h8[4], h8[5], h8[6], h8[7]);
                            nh++;
                        }
                    }
                    store8<XF32>(dst, lane, v);
                } else if (xfw >= 0) {
                    // rows o*256 + 8*lane .. +8 of the previous step's first output: its words, polled
                    // until they carry this run's epoch (bounded); only words still without it are
                    // loaded again
                    const unsigned long long* src = ch.fwd + xfw + (size_t)o * kM1Rows + 8 * lane;
                    unsigned long long w[8];
                    #pragma unroll
                    for (int e = 0; e < 8; e++) w[e] = ld_relaxed_gpu_u64(src + e);
                    bool ok = true;
                    uint64_t t0 = 0;
                    for (;;) {
                        bool all = true;
                        #pragma unroll
                        for (int e = 0; e < 8; e++) all = all && (unsigned)(w[e] >> 32) == epoch;
                        if (all) break;
                        if (t0 == 0) t0 = global_ns();
                        if (*abort_flag || *(volatile unsigned*)gabort) {
                            ok = false;
                            break;
                        }
                        if (global_ns() - t0 > kWaitLimitNs) {
                            atomicOr(&g_gemv_status, kStatusTimeout);
                            atomicExch(gabort, 1u);
                            ok = false;
                            break;
                        }
                        #pragma unroll
                        for (int e = 0; e < 8; e++)
                            if ((unsigned)(w[e] >> 32) != epoch) w[e] = ld_relaxed_gpu_u64(src + e);
                    }
                    if (!__all_sync(0xffffffffu, ok)) {
                        if (lane == 0) *abort_flag = 1;
                        stop = true;
                        break;
                    }
                    float v[8];
                    #pragma unroll
                    for (int e = 0; e < 8; e++) v[e] = __uint_as_float((unsigned)w[e]);
                    store8<XF32>(dst, lane, v);
                } else if (xreg < 0) {
                    const uint8_t* src = x + (size_t)o * kM1Rows * esz;
                    uint4 u[kPreVecs];
                    #pragma unroll
                    for (int b = 0; b < kPreVecs; b++)
                        u[b] = hoist && it == ibeg ? pre[b] : __ldcg(reinterpret_cast<const uint4*>(src) + kPreVecs * lane + b);
                    if constexpr (XF32) {
                        float v[8];
                        unpack8<XF32>(u, v);
                        store8<XF32>(dst, lane, v);
                    } else {
                        *reinterpret_cast<uint4*>(dst + chain_xoff16(lane)) = u[0];
                        *reinterpret_cast<uint4*>(dst + chain_xoff16(lane) + 64) = u[0];
                    }
                } else {
                    // rows o*256 + 8*lane .. +8: the world ranks' words, polled until they carry this
                    // run's epoch (bounded), summed in rank order.  A rank's 8 words are loaded at once
                    // (one round trip); only words still without the epoch are loaded again.
                    const unsigned long long* base = s_peers[ch.rank] + xreg + (size_t)o * kM1Rows + 8 * lane;
                    float v[8];
                    #pragma unroll
                    for (int e = 0; e < 8; e++) v[e] = 0.f;
                    bool ok = true;
                    uint64_t t0 = 0;
                    for (int r = 0; r < ch.world && ok; r++) {
                        const unsigned long long* src = base + (size_t)r * K;
                        unsigned long long w[8];
                        #pragma unroll
                        for (int e = 0; e < 8; e++) w[e] = ld_relaxed_sys_u64(src + e);
                        for (;;) {
                            bool all = true;
                            #pragma unroll
                            for (int e = 0; e < 8; e++) all = all && (unsigned)(w[e] >> 32) == epoch;
                            if (all) break;
                            if (t0 == 0) t0 = global_ns();
                            if (*abort_flag || *(volatile unsigned*)gabort) {
                                ok = false;
                                break;
                            }
                            if (global_ns() - t0 > kWaitLimitNs) {
                                atomicOr(&g_gemv_status, kStatusTimeout);
                                atomicExch(gabort, 1u);
                                ok = false;
                                break;
                            }
                            #pragma unroll
                            for (int e = 0; e < 8; e++)
                                if ((unsigned)(w[e] >> 32) != epoch) w[e] = ld_relaxed_sys_u64(src + e);
                        }
                        #pragma unroll
                        for (int e = 0; e < 8; e++) v[e] += __uint_as_float((unsigned)w[e]);
                    }
                    if (!__all_sync(0xffffffffu, ok)) {
                        if (lane == 0) *abort_flag = 1;
                        stop = true;
                        break;
                    }
                    store8<XF32>(dst, lane, v);
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(full_bar(s));
                if (++o == noct) o = 0;
            }
            // the h' slices this warp stored count toward the step's completion: whoever waits for
            // the step (or any later one) then sees them
            if (__any_sync(0xffffffffu, nh > 0)) {
                __threadfence();
                __syncwarp();
                if (lane == 0) red_add_release_gpu(&ch.sync[j], (unsigned)nh);
            }
        }
        if (lane == 0) s_xdone = i;
    } else {
        const int g = lane >> 2, q = lane & 3, ctid = tid;
        const int grp = warp / kM1WarpsPerGroup, seg = warp % kM1WarpsPerGroup;  // 16-byte column segment
        const int colA = 32 * seg + 4 * g;  // this lane's columns: colA + j (j = 0, 1) and colA + 2 + j
        // ldmatrix.x4: lane L addresses row L%8 of matrix L/8; matrix m = (step p + m/2, k-pair m%2)
        const int lm = lane >> 3, lrr = lane & 7, lq = lrr >> 1, le = lrr & 1;
        const int lds = lm >> 1, lh = lm & 1;
        constexpr int NPASS = XF32 ? 2 : 1;   // f32 x: two passes of 4 blocks
        constexpr int NSTEP = XF32 ? 8 : 16;  // mma steps per pass
        constexpr int RMUL = XF32 ? 4 : 2;    // rows advanced per step
        int nflush = 0;
        int nsums = 0;       // tile-sum emissions so far (picks the s_tsum buffer)
        int ibase = 0;       // this CTA's items in earlier steps
        unsigned ndone = 0;  // ctid 0: tiles of the current step whose y this CTA wrote

        for (int j = 0; j < nsteps; j++) {
            // Steps j-2 and j-3 complete (acquire, two threads at once), normally long since:
            //  - step j's partial slots are step j-2's, so every tile of step j-2 (its reductions
            //    included) is written before they are reused;
            //  - a step that reads forwarded or all-reduced x waits on no count before its loads, so
            //    this is what orders its writes after every read and write of the steps before j-1
            //    (by induction over the steps: j-2 and j-3 waited the same way) -- a later layer
            //    overwriting a buffer an earlier step still reads or writes.  The host refuses
            //    forwarded x where step j's outputs overlap what step j-1 reads or writes.
            if (j >= 2 && (ctid == 0 || (ctid == 32 && j >= 3))) {
                const int k = ctid == 0 ? j - 2 : j - 3;
                chain_wait_count(&ch.sync[k], (unsigned)ch.steps[k].done, gabort, abort_flag);
            }
            // every consumer is done with step j-1, whose descriptor slot now takes step j+1's
            named_bar_sync(1, kM1Consumers);
            if (j + 1 < nsteps && ctid < kStepWords)
                reinterpret_cast<uint32_t*>(&s_step[(j + 1) & 1])[ctid] =
                    __ldg(reinterpret_cast<const uint32_t*>(ch.steps + j + 1) + ctid);
            const ChainStep& d = s_step[j & 1];
            int ibeg, iend;
            my_range(d, ibeg, iend);
            unsigned long long* const partial = ch.partial + (size_t)(j & 1) * 2 * ch.G * kStTN;
            // this step's tag in its partial words: distinct for every (run, step), so words left by the
            // step two back (same buffer) or by an earlier run never pass for this step's
            const unsigned tag = epoch * (unsigned)nsteps + (unsigned)j + 1u;
            // y[n] of the tile's segment, scaled by its e4m3 inverse scale; a step whose y is
            // all-reduced also pushes the value to slot [rank] of every rank's exchange region
            auto write_y = [&](int t, int col, float v) {
                const TcSeg& sgm = tc_seg(d, tc_seg_of(d, t));
                const int n = (t - sgm.tile0) * kStTN + col;
                const float inv = SFMT == G4B_SCALE_E4M3 ? sgm.inv : 1.0f;
                if (n < sgm.N) {
                    const float y = v * inv;
                    if (YF32) ((float*)sgm.y)[n] = y;
                    else ((__half*)sgm.y)[n] = __float2half_rn(y);
                    if (d.yreg >= 0) {
                        const unsigned long long w = ((unsigned long long)epoch << 32) | __float_as_uint(y);
                        const size_t at = (size_t)d.yreg + (size_t)ch.rank * sgm.N + n;
                        for (int p = 0; p < ch.world; p++) st_relaxed_sys_u64(s_peers[p] + at, w);
                    }
                    // the next step reads segment 0 as forwarded words (segment 1's first tile is
                    // 1 << 30 when the step has one segment)
                    if (d.yfw >= 0 && t < d.seg1.tile0)
                        st_relaxed_gpu_u64(ch.fwd + d.yfw + n, ((unsigned long long)epoch << 32) | __float_as_uint(y));
                }
            };
            // the tile sums a segment-0 tile of this step hands to the next step's norm: every thread
            // ctid < kStTN calls this for the tile (valid = it holds a finished value v), whatever
            // the abort state, so the named barrier below is always complete
            auto emit_sums = [&](int t, float v, bool valid) {
                const int n = t * kStTN + ctid;
                float4 S = make_float4(0.f, 0.f, 0.f, 0.f);
                if (valid && n < d.seg0.N) {
                    const float inv = SFMT == G4B_SCALE_E4M3 ? d.seg0.inv : 1.0f;
                    float yv = v * inv;
                    if (!YF32) yv = __half2float(__float2half_rn(yv));  // the value the next step reads
                    S.w = yv * yv;
                    if (d.sum_res) {
                        const float hr = __ldcg(d.sum_res + n), yw = yv * __ldg(d.sum_wpost + n);
                        S.x = hr * hr;
                        S.y = hr * yw;
                        S.z = yw * yw;
                    }
                }
                #pragma unroll
                for (int m = 16; m >= 1; m >>= 1) {
                    S.x += __shfl_xor_sync(0xffffffffu, S.x, m);
                    S.y += __shfl_xor_sync(0xffffffffu, S.y, m);
                    S.z += __shfl_xor_sync(0xffffffffu, S.z, m);
                    S.w += __shfl_xor_sync(0xffffffffu, S.w, m);
                }
                const int sb = nsums & 1;
                if (lane == 0) s_tsum[sb][warp] = S;
                named_bar_sync(2, kStTN);
                if (ctid == 0) {
                    float4 T = s_tsum[sb][0];
                    #pragma unroll
                    for (int w = 1; w < kStTN / 32; w++) {
                        const float4 u = s_tsum[sb][w];
                        T.x += u.x;
                        T.y += u.y;
                        T.z += u.z;
                        T.w += u.w;
                    }
                    reinterpret_cast<float4*>(d.sums_out)[t] = T;
                }
                nsums++;
            };
            const bool emits = d.sums_out != nullptr;
            const int seg0_tiles = d.nseg > 1 ? d.seg1.tile0 : d.ntiles;
            float acc[2][2];
            const int t_first = ibeg / d.noct, t_last = iend > ibeg ? (iend - 1) / d.noct : t_first - 1;
            // Sum a shared tile's partials in CTA order (deterministic) and write y.  The tile's
            // reducer is the CTA holding its last k-chunk; each sharer stores its partial as {f32,
            // tag} words and moves on, and the reducer polls the words until every one carries this
            // step's tag (bounded) -- no fence, no atomic round trip.  CTA cc keeps its share of its
            // first tile in slot 2cc and of its last in 2cc + 1; only the tile's first CTA can have
            // started in an earlier tile (bit 31 of cspan[2t]), every later one starts in t.
            auto reduce_tile = [&](int t) {
                const unsigned f = (unsigned)__ldg(d.cspan + 2 * t);
                const int c_first = (int)(f & 0x7fffffffu), c_last = __ldg(d.cspan + 2 * t + 1);
                if (ctid < kStTN) {
                    const int col = ctid;
                    float v = 0.f;
                    bool ok = true;
                    uint64_t t0 = 0;
                    // up to 16 sharers' words in flight at once (one round trip for the decode shapes)
                    constexpr int kPoll = 16;
                    for (int k0 = c_first; k0 <= c_last && ok; k0 += kPoll) {
                        unsigned long long w[kPoll];
                        #pragma unroll
                        for (int k = 0; k < kPoll; k++) {
                            const int cc = k0 + k;
                            const int sl = 2 * cc + (cc == c_first ? (int)(f >> 31) : 0);
                            w[k] = cc <= c_last ? ld_relaxed_gpu_u64(&partial[(size_t)sl * kStTN + col])
                                                : ((unsigned long long)tag << 32);
                        }
                        for (;;) {
                            bool all = true;
                            #pragma unroll
                            for (int k = 0; k < kPoll; k++) all = all && (unsigned)(w[k] >> 32) == tag;
                            if (all) break;
                            if (t0 == 0) t0 = global_ns();
                            if (*abort_flag || *(volatile unsigned*)gabort) {
                                ok = false;
                                break;
                            }
                            if (global_ns() - t0 > kWaitLimitNs) {
                                atomicOr(&g_gemv_status, kStatusTimeout);
                                atomicExch(gabort, 1u);
                                *abort_flag = 1;
                                ok = false;
                                break;
                            }
                            #pragma unroll
                            for (int k = 0; k < kPoll; k++) {
                                const int cc = k0 + k;
                                const int sl = 2 * cc + (cc == c_first ? (int)(f >> 31) : 0);
                                if ((unsigned)(w[k] >> 32) != tag)
                                    w[k] = ld_relaxed_gpu_u64(&partial[(size_t)sl * kStTN + col]);
                            }
                        }
                        #pragma unroll
                        for (int k = 0; k < kPoll; k++)
                            if (k0 + k <= c_last) v += __uint_as_float((unsigned)w[k]);
                    }
                    if (ok) write_y(t, col, v);
                    if (emits && t < seg0_tiles) emit_sums(t, v, ok);
                }
            };

            for (int t = t_first; t <= t_last; ++t) {
                acc[0][0] = acc[0][1] = acc[1][0] = acc[1][1] = 0.f;
                const int tb = max(ibeg, t * d.noct), te = min(iend, (t + 1) * d.noct);
                int it = tb + ((grp - (ibase + tb - ibeg) % kM1Groups + kM1Groups) % kM1Groups);
                for (; it < te; it += kM1Groups) {
                    const int i = ibase + (it - ibeg);
                    const int s = m1_stage(i);
                    if (!mbar_wait(full_bar(s), m1_parity(i), abort_flag, &g_gemv_status)) {
                        __syncwarp();
                        if (lane == 0) mbar_arrive(empty_bar(s));
                        continue;
                    }
                    const uint32_t st_u = smem0 + (uint32_t)s * stage_bytes;
                    const uint8_t* st = smem + (size_t)s * stage_bytes;
                    const uint8_t* sc = st + kM1WBytes;
                    const uint8_t* xs = sc + s_bytes;
                    // block sums X[b] of the slice: stored with it by the activation warp (f32 x), or
                    // summed here, lane l over rows 8l..8l+7 (f16 x)
                    const float* xss = reinterpret_cast<const float*>(xs + kChainXBytes);
                    float xsum = 0.f;
                    if constexpr (!XF32) {
                        const uint4 v = *reinterpret_cast<const uint4*>(xs + chain_xoff16(lane));
                        xsum = ((((((h_lo(v.x) + h_hi(v.x)) + h_lo(v.y)) + h_hi(v.y)) + h_lo(v.z)) + h_hi(v.z)) + h_lo(v.w)) +
                               h_hi(v.w);
                        xsum += __shfl_xor_sync(0xffffffffu, xsum, 1);
                        xsum += __shfl_xor_sync(0xffffffffu, xsum, 2);
                    }
                    #pragma unroll 1
                    for (int pass = 0; pass < NPASS; pass++) {
                        // ldmatrix row of this lane: block and rotated row (swizzle phase differs per lane)
                        const int lblk = XF32 ? 4 * pass + lq : lq + 4 * lh;
                        const int lrot = RMUL * lds + 2 * lq + le + ((XF32 && lh) ? 2 : 0);
                        const uint32_t lbase = st_u + (uint32_t)(lblk * 32 * 128);
                        // the ldmatrix offset of each step pair p (p = 4m + d advances the row by 8m (f16) / 16m
                        // (f32)), rotated and swizzled once here so the loop adds only the stage base
                        uint32_t aoff[NSTEP / 2];
                        #pragma unroll
                        for (int p = 0; p < NSTEP; p += 2) {
                            const int d = p & 3, mrow = (p >> 2) * (RMUL == 2 ? 1024 : 2048);
                            const int r = (RMUL * d + lrot) & 31;
                            aoff[p / 2] = ((uint32_t)(r * 128 + mrow) & 4095u) | (uint32_t)((seg ^ (r & 7)) << 4);
                        }
                        // B-fragment sources: lanes that feed zeros read a zeroed area instead
                        uint32_t xb0, xb1, xoff;
                        if constexpr (XF32) {
                            const bool mine = (g >> 1) == q;
                            xb0 = (mine ? smem_u32(xs) + (uint32_t)((4 * pass + q) * 128) : smem_u32(s_zero)) +
                                  ((g & 1) ? 64u : 0u);
                            xb1 = xb0;
                            xoff = (uint32_t)(4 * q);
                        } else {
                            // each 32-row block of x sits twice in a row (128 bytes), so the rotated
                            // word (q + pp) is read at a constant offset from here: no wrap to compute
                            xb0 = (g == q ? smem_u32(xs) + (uint32_t)(q * 128) : smem_u32(s_zero)) + (uint32_t)(4 * q);
                            xb1 = (g == q + 4 ? smem_u32(xs) + (uint32_t)((q + 4) * 128) : smem_u32(s_zero)) +
                                  (uint32_t)(4 * q);
                            xoff = 0u;
                        }
                        float C[2][4];
                        #pragma unroll
                        for (int k = 0; k < 2; k++) C[k][0] = C[k][1] = C[k][2] = C[k][3] = 0.f;
                        #pragma unroll
                        for (int p = 0; p < NSTEP; p += 2) {
                            const uint32_t addr = lbase + aoff[p / 2];
                            uint32_t ra0, rb0, ra1, rb1;
                            ldsm_x4_trans(addr, ra0, rb0, ra1, rb1);
                            #pragma unroll
                            for (int ss = 0; ss < 2; ss++) {
                                const uint32_t RA = ss ? ra1 : ra0, RB = ss ? rb1 : rb0;
                                const int pp = p + ss;
                                uint32_t b0, b1;
                                if constexpr (XF32) {
                                    // the pre-split f16 words of row pairs (q + 2pp) and (q + 2pp + 1) mod 16
                                    // of the block: hi words for even g, lo words (at +64) for odd g
                                    asm volatile("ld.shared.b32 %0, [%1];" : "=r"(b0) : "r"(xb0 + ((xoff + 8u * pp) & 63u)));
                                    asm volatile("ld.shared.b32 %0, [%1];" : "=r"(b1) : "r"(xb1 + ((xoff + 8u * pp + 4u) & 63u)));
                                } else {
                                    asm volatile("ld.shared.b32 %0, [%1];" : "=r"(b0) : "r"(xb0 + 4u * pp));
                                    asm volatile("ld.shared.b32 %0, [%1];" : "=r"(b1) : "r"(xb1 + 4u * pp));
                                }
                                const uint32_t RA8 = RA >> 8, RB8 = RB >> 8;
                                mma_16816(C[0], RA & 0x000F000Fu, RA8 & 0x000F000Fu, RB & 0x000F000Fu, RB8 & 0x000F000Fu, b0, b1);
                                mma_16816(C[1], RA & 0x00F000F0u, RA8 & 0x00F000F0u, RB & 0x00F000F0u, RB8 & 0x00F000F0u, b0, b1);
                            }
                        }
                        // per-block scale, 2^E and -8 X correction, in f32
                        int blk0, blk1;
                        if constexpr (XF32) { blk0 = 4 * pass + q; blk1 = blk0; } else { blk0 = 2 * q; blk1 = 2 * q + 1; }
                        float X0, X1;
                        if constexpr (XF32) {
                            X0 = xss[blk0];
                            X1 = xss[blk1];
                        } else {
                            X0 = __shfl_sync(0xffffffffu, xsum, 4 * blk0);
                            X1 = __shfl_sync(0xffffffffu, xsum, 4 * blk1);
                        }
                        // scales of columns colA .. colA+3 in blocks blk0 / blk1
                        float s0[4], s1[4];
                        if constexpr (SFMT == G4B_SCALE_F16) {
                            const uint2 u0 = *reinterpret_cast<const uint2*>(sc + (blk0 * kStTN + colA) * 2);
                            const uint2 u1 = *reinterpret_cast<const uint2*>(sc + (blk1 * kStTN + colA) * 2);
                            s0[0] = h_lo(u0.x); s0[1] = h_hi(u0.x); s0[2] = h_lo(u0.y); s0[3] = h_hi(u0.y);
                            s1[0] = h_lo(u1.x); s1[1] = h_hi(u1.x); s1[2] = h_lo(u1.y); s1[3] = h_hi(u1.y);
                        } else {
                            const uint32_t u0 = *reinterpret_cast<const uint32_t*>(sc + blk0 * kStTN + colA);
                            const uint32_t u1 = *reinterpret_cast<const uint32_t*>(sc + blk1 * kStTN + colA);
                            uint32_t h;
                            h = e4m3x2_to_f16x2((uint16_t)(u0 & 0xffffu)); s0[0] = h_lo(h); s0[1] = h_hi(h);
                            h = e4m3x2_to_f16x2((uint16_t)(u0 >> 16));     s0[2] = h_lo(h); s0[3] = h_hi(h);
                            h = e4m3x2_to_f16x2((uint16_t)(u1 & 0xffffu)); s1[0] = h_lo(h); s1[1] = h_hi(h);
                            h = e4m3x2_to_f16x2((uint16_t)(u1 >> 16));     s1[2] = h_lo(h); s1[3] = h_hi(h);
                        }
                        #pragma unroll
                        for (int j = 0; j < 2; j++) {
                            const float E = j ? 1048576.0f : 16777216.0f;  // 2^20 (high nibble) / 2^24 (low nibble)
                            // C[j][0..1]: column colA + j; C[j][2..3]: column colA + 2 + j
                            if constexpr (XF32) {
                                acc[j][0] = fmaf(s0[j], fmaf(C[j][0] + C[j][1], E, -8.0f * X0), acc[j][0]);
                                acc[j][1] = fmaf(s0[2 + j], fmaf(C[j][2] + C[j][3], E, -8.0f * X0), acc[j][1]);
                            } else {
                                acc[j][0] = fmaf(s0[j], fmaf(C[j][0], E, -8.0f * X0), acc[j][0]);
                                acc[j][0] = fmaf(s1[j], fmaf(C[j][1], E, -8.0f * X1), acc[j][0]);
                                acc[j][1] = fmaf(s0[2 + j], fmaf(C[j][2], E, -8.0f * X0), acc[j][1]);
                                acc[j][1] = fmaf(s1[2 + j], fmaf(C[j][3], E, -8.0f * X1), acc[j][1]);
                            }
                        }
                    }
                    __syncwarp();
                    if (lane == 0) mbar_arrive(empty_bar(s));
                }
                // ---- flush tile t: quad sum (the lanes of a quad hold different blocks), group sum, CTA share
                #pragma unroll
                for (int k = 0; k < 2; k++)
                    #pragma unroll
                    for (int h = 0; h < 2; h++) {
                        float v = acc[k][h];
                        v += __shfl_xor_sync(0xffffffffu, v, 1);
                        v += __shfl_xor_sync(0xffffffffu, v, 2);
                        acc[k][h] = v;
                    }
                const int rb = nflush++ & 1;
                if (q == 0) {
                    #pragma unroll
                    for (int jj = 0; jj < 2; jj++) {
                        red[rb][grp][colA + jj] = acc[jj][0];
                        red[rb][grp][colA + 2 + jj] = acc[jj][1];
                    }
                }
                named_bar_sync(1, kM1Consumers);
                // the tile is this CTA's alone when the CTA owns all its k-chunks
                const bool single = ibeg <= t * d.noct && iend >= (t + 1) * d.noct;
                const bool ok = !*abort_flag;
                if (ctid < kStTN) {
                    const int col = ctid;
                    float v = red[rb][0][col];
                    #pragma unroll
                    for (int gg = 1; gg < kM1Groups; gg++) v += red[rb][gg][col];
                    if (ok) {
                        if (single) write_y(t, col, v);
                        else
                            st_relaxed_gpu_u64(&partial[(size_t)(2 * c + (t == t_first ? 0 : 1)) * kStTN + col],
                                               ((unsigned long long)tag << 32) | __float_as_uint(v));
                    }
                    if (single && emits && t < seg0_tiles) emit_sums(t, v, ok);
                }
                if (single) {
                    if (ctid == 0 && ok) ndone++;
                } else if (__ldg(d.cspan + 2 * t + 1) == c) {
                    // this CTA holds the tile's last k-chunk: it reduces the tile, now if this is its final
                    // tile, otherwise after its last item (the other consumers keep going meanwhile); after
                    // an abort the reduction gives up at once, but every thread still takes this path
                    if (t < t_last) {
                        if (ctid == 0) s_pending = t;
                    } else {
                        reduce_tile(t);
                        if (ctid == 0 && !*abort_flag) ndone++;
                    }
                }
            }
            // the deferred reduction of an earlier tile this CTA was the last to finish
            named_bar_sync(1, kM1Consumers);
            if (s_pending >= 0) {
                reduce_tile(s_pending);
                if (ctid == 0 && !*abort_flag) ndone++;
            }
            // every y this CTA wrote in step j is stored: count its tiles as written
            named_bar_sync(1, kM1Consumers);
            if (ctid == 0) {
                s_pending = -1;
                if (ndone) red_add_release_gpu(&ch.sync[j], ndone);
                ndone = 0;
                if (*abort_flag) atomicExch(gabort, 1u);
            }
            ibase += iend - ibeg;
        }
    }

    __syncthreads();
    if (tid == 0 && *abort_flag) {
        // wait (bounded) for the copies still in flight into this CTA's shared memory; an item
        // whose x the activation warp never stored still needs that warp's arrival
        const int issued = s_issued;
        for (int i = max(0, issued - kM1Stages); i < issued; i++) {
            if (i >= s_xdone) mbar_arrive(full_bar(m1_stage(i)));
            const uint64_t t0 = global_ns();
            while (!mbar_try_wait(full_bar(m1_stage(i)), m1_parity(i)) && global_ns() - t0 < kWaitLimitNs) {
            }
        }
    }
    if (tid == 0) {
        if (*abort_flag) atomicExch(gabort, 1u);
        __threadfence();
        if (atomicAdd(&ch.sync[nsteps], 1u) == gridDim.x - 1u) {
            // the last CTA out: every CTA is past all its waits, so the chain's counts can be
            // cleared for the next launch (partial words need no clearing: their tags name the run)
            __threadfence();
            for (int j = 0; j < nsteps; j++) ch.sync[j] = 0u;
            *gabort = 0u;
            ch.sync[nsteps + 2] = epoch;  // the next run's epoch is one more
            ch.sync[nsteps] = 0u;
        }
    }
}

struct M1Plan {
    int ntiles, noct, G, maxseg, stage_bytes, s_bytes, mode;
    long long total;
    size_t smem, ws_bytes;
};

static M1Plan m1_plan(int nseg, const int* Ns, int K, int sms, bool xf32, int sfmt) {
    M1Plan p{};
    p.noct = K / 256;
    p.ntiles = 0;
    for (int i = 0; i < nseg; i++) p.ntiles += (Ns[i] + kStTN - 1) / kStTN;
    p.total = (long long)p.ntiles * p.noct;
    p.G = (int)std::max<long long>(1, std::min<long long>(std::min(std::max(sms, 1), kMaxCtas), p.total));
    p.s_bytes = 8 * kStTN * (sfmt == G4B_SCALE_F16 ? 2 : 1);
    p.stage_bytes = (kM1WBytes + p.s_bytes + kM1Rows * (xf32 ? 4 : 2) + 1023) & ~1023;  // swizzle atoms stay aligned
    p.smem = (size_t)kM1Stages * p.stage_bytes + 1024;                                     // + base alignment slack
    // the tile-aligned partition unless it costs more than one item over the balanced one's longest range
    // plus a straddle (a CTA running two shared tiles one after the other)
    const long long max_bal = (p.total + p.G - 1) / p.G;
    bool straddle = false;
    for (int c = 0; c < p.G && !straddle; c++) {
        const long long ib = (long long)c * p.total / p.G, ie = (long long)(c + 1) * p.total / p.G;
        if ((ie - 1) / p.noct > ib / p.noct && (ib % p.noct || ie % p.noct)) straddle = true;
    }
    const int ta_mode = p.ntiles >= p.G ? kM1WholeTiles : kM1TileSplit;
    long long max_ta = 0;
    for (int c = 0; c < p.G; c++) {
        long long ib, ie;
        m1_range(ta_mode, p.total, p.ntiles, p.noct, p.G, c, ib, ie);
        max_ta = std::max(max_ta, ie - ib);
    }
    p.mode = max_ta <= max_bal + (straddle ? 1 : 0) ? ta_mode : kM1Balanced;
    // partial slots per CTA: the most tiles a CTA's range touches, plus one (balanced ranges)
    p.maxseg = p.mode == kM1Balanced ? (int)((max_bal + p.noct - 1) / p.noct + 1) : 1;
    // a tile is split across CTAs unless every CTA boundary falls on a tile boundary
    bool multi = false;
    for (int c = 0; c < p.G && !multi; c++) {
        long long ib, ie;
        m1_range(p.mode, p.total, p.ntiles, p.noct, p.G, c, ib, ie);
        if (ib % p.noct || ie % p.noct) multi = true;
    }
    if (multi) p.ws_bytes = kGemvCounterBytes + (((size_t)p.G * p.maxseg * kStTN * sizeof(float) + 255) & ~(size_t)255);
    return p;
}

static bool m1_ok(int M, int N, int K, int split) { return M == 1 && split == 0 && N % 32 == 0 && K % 256 == 0; }

template <bool XF32, int SFMT, bool YF32>
static int launch_m1(const M1Args& a, const M1Plan& p, const uint32_t* const* wps, const void* const* scales,
                     cudaStream_t s) {
    TcMaps maps;
    constexpr int ssz = SFMT == G4B_SCALE_F16 ? 2 : 1;
    for (int i = 0; i < kTcMaxSeg; i++) {
        const int k = i < a.nseg ? i : 0;  // unused slots repeat segment 0's maps
        const int N = tc_seg(a, k).N;
        int st = tensor_map_2d(&maps.w[i], CU_TENSOR_MAP_DATA_TYPE_UINT32, wps[k], (uint64_t)N / 8, (uint64_t)a.K,
                               (uint64_t)N / 2, kStTN / 8, kM1Rows, CU_TENSOR_MAP_SWIZZLE_128B,
                               CU_TENSOR_MAP_L2_PROMOTION_L2_128B);
        if (st != G4B_OK) return st;
        st = tensor_map_2d(&maps.s[i], CU_TENSOR_MAP_DATA_TYPE_UINT64, scales[k], (uint64_t)N * ssz / 8,
                           (uint64_t)a.K / 32, (uint64_t)N * ssz, kStTN * ssz / 8, 8, CU_TENSOR_MAP_SWIZZLE_NONE);
        if (st != G4B_OK) return st;
    }
    auto kern = gemv_i4_m1_kernel<XF32, SFMT, YF32>;
    static int attr_set_mask = 0;
    int dev = 0;
    cudaGetDevice(&dev);
    if (!(attr_set_mask & (1 << (dev & 31)))) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
        if (e != cudaSuccess) return fail(G4B_E_CUDA, "gemv_i4: cudaFuncSetAttribute: %s", cudaGetErrorString(e));
        attr_set_mask |= 1 << (dev & 31);
    }
    cudaError_t e = launch_k(kern, dim3(p.G), dim3(kM1Threads), p.smem, s, a, maps);
    if (e != cudaSuccess) return fail(G4B_E_CUDA, "gemv_i4: launch: %s", cudaGetErrorString(e));
    return G4B_OK;
}

static int dispatch_m1(const M1Args& a, const M1Plan& p, const uint32_t* const* wp, const void* const* sc, bool xf32,
                       int sfmt, bool yf32, cudaStream_t s) {
    if (xf32) {
        if (sfmt == G4B_SCALE_F16) return yf32 ? launch_m1<true, G4B_SCALE_F16, true>(a, p, wp, sc, s) : launch_m1<true, G4B_SCALE_F16, false>(a, p, wp, sc, s);
        return yf32 ? launch_m1<true, G4B_SCALE_E4M3, true>(a, p, wp, sc, s) : launch_m1<true, G4B_SCALE_E4M3, false>(a, p, wp, sc, s);
    }
    if (sfmt == G4B_SCALE_F16) return yf32 ? launch_m1<false, G4B_SCALE_F16, true>(a, p, wp, sc, s) : launch_m1<false, G4B_SCALE_F16, false>(a, p, wp, sc, s);
    return yf32 ? launch_m1<false, G4B_SCALE_E4M3, true>(a, p, wp, sc, s) : launch_m1<false, G4B_SCALE_E4M3, false>(a, p, wp, sc, s);
}

// ------------------------------------------------------- M = 1 on tcgen05
// gemv_tc_kernel: the decode GEMV (M = 1) with the dot products on the
// tcgen05 tensor core, so that no SM pipe but HBM limits it.
//
//  * item = 64 rows (two scale blocks) x 256 columns of packed words (8 KB);
//    a CTA walks a contiguous, balanced range of items, tile-major, and the
//    split-K partials of a tile shared by several CTAs are reduced by the last
//    one to arrive, in CTA order (deterministic), as in gemv_i4_m1_kernel.
//  * dequantisation is one shift and one AND per 32-bit word, no nibble
//    gather: TMEM lane 4g+p holds, for every row k, the f16 pair
//    (q[k][8g+p], q[k][8g+p+4]) as exact subnormals (q * 2^-24 or q * 2^-20,
//    nibble positions p even / odd), i.e. the row's word shifted right by
//    8*(p/2) and masked with 0x000F000F or 0x00F000F0.  Four warps write a
//    64-row item as 64 TMEM columns: the A operand of eight M=128, N=16, K=16
//    MMAs.
//  * the B operand is x spread over a sparse [16 x 16] tile per 8 rows: the
//    low element of a pair meets column 2b, the high element column 2b+1,
//    where b is the row's scale block within the item; f32 x uses a second
//    pair of columns for its f16 low part.  The accumulator therefore holds,
//    per lane, one dot product per (block, column), and the block scales are
//    applied in f32 afterwards: acc += s * (2^E * dot - 8 * sum(x over block)).
//    The non-zero positions of the sparse tiles never change, so the tiles are
//    zeroed once and each item only writes its x values.
//  * footprint <= half an SM (256 threads, <= 106 KB shared memory, 256 TMEM
//    columns), so with programmatic dependent launch the next GEMV's CTA
//    lives beside this one and streams its weights while this one finishes.
// Warps: 0 TMA producer (packed words and scales at once, each item's slice of
// x once the previous grid has completed), 1 MMA issuer (and TMEM owner),
// 2-3 x -> B tiles (alternate items), 4-7 dequant + epilogue (TMEM lane
// quarters 0-3).
constexpr int kTcRows = 64;
constexpr int kTcTN = 256;
constexpr int kTcWBytes = kTcRows * (kTcTN / 2);  // 8 KB of packed words per item
constexpr int kTcThreads = 256;
constexpr int kTcDq0 = 4;                          // first dequant warp
constexpr uint32_t kTcACol = 0;                    // 2 A stages x 64 columns
constexpr uint32_t kTcDCol = 128;                  // 2 accumulators x 16 columns

template <bool XF32, int SFMT>
struct TcCfg {
    static constexpr int kBTile = 16 * 16 * 2;                   // one [N=16 x K=16] f16 tile
    static constexpr int kBBytes = (kTcRows / 8) * kBTile;       // 4 KB
    static constexpr int kSBytes = 2 * kTcTN * (SFMT == G4B_SCALE_F16 ? 2 : 1);
    static constexpr int kXBytes = kTcRows * (XF32 ? 4 : 2);    // the item's slice of x
    static constexpr int kStageBytes = kTcWBytes + kBBytes + kSBytes + kXBytes;
    static constexpr int kStages = 8;
    static constexpr size_t kSmem = (size_t)kStages * kStageBytes + 128;
};


struct TcArgs {
    const void* x;
    float* partial;      // [G * maxseg, 256]
    unsigned* counters;  // [ntiles]
    TcSeg seg0, seg1, seg2;
    int nseg, K, noct, ntiles, G, maxseg;
    long long total;
};



// byte offset of element (n, kk) in a K-major, unswizzled [16 x 16] f16 tile
// (core matrices of 8 rows x 8 elements: K groups 128 B apart, row groups 256 B)
__device__ __forceinline__ uint32_t btile_off(int n, int kk) {
    return (uint32_t)((n >> 3) * 256 + (kk >> 3) * 128 + (n & 7) * 16 + (kk & 7) * 2);
}

template <bool XF32, int SFMT, bool YF32>
__global__ void __launch_bounds__(kTcThreads, 2) gemv_tc_kernel(const TcArgs a, const __grid_constant__ TcMaps maps) {
    using Cfg = TcCfg<XF32, SFMT>;
    constexpr int S = Cfg::kStages;
    constexpr int ssz = SFMT == G4B_SCALE_F16 ? 2 : 1;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    __shared__ uint64_t bars[5 * S + 9];
    __shared__ int s_ftile[kMaxCtas];  // first tile of each CTA's item range
    __shared__ float s_xb[S][2];
    __shared__ uint32_t s_tmem;
    __shared__ int s_abort;
    __shared__ int s_issued;
    __shared__ int s_xissued;
    __shared__ long long s_pending;
    __shared__ unsigned s_last;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    volatile int* abort_flag = &s_abort;
    const uint32_t raw0 = smem_u32(smem_raw);
    const uint32_t sm0 = (raw0 + 127u) & ~127u;
    uint8_t* smem = smem_raw + (sm0 - raw0);
    const uint32_t bar0 = smem_u32(bars);
    auto full_bar = [&](int s) { return bar0 + 8u * s; };               // TMA landed (1 + tx)
    auto bfull_bar = [&](int s) { return bar0 + 8u * (S + s); };        // B tiles + block sums written (1)
    auto wempty_bar = [&](int s) { return bar0 + 8u * (2 * S + s); };   // words + scales consumed (4)
    auto bempty_bar = [&](int s) { return bar0 + 8u * (3 * S + s); };   // MMAs done with the B tiles (commit)
    auto afull_bar = [&](int i) { return bar0 + 8u * (4 * S + i); };    // A stage written (4)
    auto aempty_bar = [&](int i) { return bar0 + 8u * (4 * S + 2 + i); };  // MMAs done with the A stage
    auto dfull_bar = [&](int i) { return bar0 + 8u * (4 * S + 4 + i); };   // accumulator ready
    auto dempty_bar = [&](int i) { return bar0 + 8u * (4 * S + 6 + i); };  // accumulator read (4)
    const uint32_t drain_bar = bar0 + 8u * (4 * S + 8);
    auto xfull_bar = [&](int s) { return bar0 + 8u * (4 * S + 9 + s); };  // x slice landed (1 + tx)
    const long long ibeg = (long long)blockIdx.x * a.total / a.G;
    const long long iend = (long long)(blockIdx.x + 1) * a.total / a.G;
    const int n_items = (int)(iend - ibeg);

    if (tid == 0) {
        for (int s = 0; s < S; s++) {
            mbar_init(full_bar(s), 1);
            mbar_init(bfull_bar(s), 1);
            mbar_init(wempty_bar(s), 4 + 1);  // 4 dequant warps (words, scales) + the builder (x)
            mbar_init(bempty_bar(s), 1);
            mbar_init(xfull_bar(s), 1);
        }
        for (int i = 0; i < 2; i++) {
            mbar_init(afull_bar(i), 4);
            mbar_init(aempty_bar(i), 1);
            mbar_init(dfull_bar(i), 1);
            mbar_init(dempty_bar(i), 4);
        }
        mbar_init(drain_bar, 1);
        s_abort = 0;
        s_issued = 0;
        s_xissued = 0;
        s_pending = -1;
        fence_mbar_init();
    }
    for (int c = tid; c < a.G; c += kTcThreads) s_ftile[c] = (int)(((long long)c * a.total / a.G) / a.noct);
    // the sparse B tiles: zero once, only their fixed non-zero positions are rewritten
    for (int s = 0; s < S; s++) {
        uint4* b = reinterpret_cast<uint4*>(smem + (size_t)s * Cfg::kStageBytes + kTcWBytes);
        for (int v = tid; v < Cfg::kBBytes / 16; v += kTcThreads) b[v] = make_uint4(0u, 0u, 0u, 0u);
    }
    tc::fence_proxy_async_smem();
    if (warp == 1) {
        tc::tmem_alloc(smem_u32(&s_tmem), 256);
        tc::tmem_relinquish();
    }
    tc::fence_before();
    __syncthreads();
    tc::fence_after();
    const uint32_t tmem = s_tmem;
    pdl_launch_dependents();

    if (warp == 0) {
        // ------------------------------------------------------- TMA producer
        if (lane == 0) {
            for (int sg = 0; sg < a.nseg; sg++) {
                prefetch_tensor_map(&maps.w[sg]);
                prefetch_tensor_map(&maps.s[sg]);
            }
            const uint64_t pol = l2_evict_first_policy();
            auto issue_w = [&](int i, int t, int o) {  // packed words + scales of item i = (tile t, chunk o)
                const int s = i % S;
                const int sg = tc_seg_of(a, t);
                const int lt = t - tc_seg(a, sg).tile0;  // tile within its segment
                const uint32_t st = sm0 + (uint32_t)(s * Cfg::kStageBytes);
                mbar_arrive_expect_tx(full_bar(s), kTcWBytes + Cfg::kSBytes);
                tma_load_2d(st, &maps.w[sg], lt * (kTcTN / 8), o * kTcRows, full_bar(s), pol);
                tma_load_2d(st + kTcWBytes + Cfg::kBBytes, &maps.s[sg], lt * (kTcTN * ssz / 8), o * 2, full_bar(s), pol);
            };
            auto issue_x = [&](int i, int o) {  // the item's slice of x (only after the previous grid is done)
                const int s = i % S;
                const uint32_t st = sm0 + (uint32_t)(s * Cfg::kStageBytes);
                mbar_arrive_expect_tx(xfull_bar(s), Cfg::kXBytes);
                bulk_g2s_nohint(st + kTcWBytes + Cfg::kBBytes + Cfg::kSBytes,
                                reinterpret_cast<const uint8_t*>(a.x) + (size_t)o * Cfg::kXBytes, Cfg::kXBytes,
                                xfull_bar(s));
            };
            // weights do not depend on the previous kernel: fill every stage before waiting for it
            const int npre = n_items < S ? n_items : S;
            ItemCursor cw(ibeg, a.noct), cx(ibeg, a.noct);
            for (int i = 0; i < npre; i++, cw.next()) issue_w(i, cw.t, cw.o);
            pdl_wait();
            for (int i = 0; i < npre; i++, cx.next()) issue_x(i, cx.o);
            int i = npre, xi = npre;
            for (; i < n_items; i++, cw.next()) {
                const int s = i % S;
                if (!mbar_wait(wempty_bar(s), ((i / S) & 1) ^ 1, abort_flag, &g_gemv_status)) break;
                issue_w(i, cw.t, cw.o);
                issue_x(i, cw.o);
                xi = i + 1;
            }
            s_issued = i;
            s_xissued = xi;
        }
    } else if (warp == 1) {
        // ------------------------------------------------------- MMA issuer
        if (lane == 0) {
            constexpr uint32_t idesc = tc::idesc(1, 0, 0, 0, 0, 16, 128);
            bool ok = true;
            for (int i = 0; ok && i < n_items; i++) {
                const int s = i % S, ab = i & 1;
                const uint32_t ph = (uint32_t)(i >> 1) & 1u;
                if (!mbar_wait(dempty_bar(ab), ph ^ 1u, abort_flag, &g_gemv_status) ||
                    !mbar_wait(afull_bar(ab), ph, abort_flag, &g_gemv_status) ||
                    !mbar_wait(bfull_bar(s), (uint32_t)(i / S) & 1u, abort_flag, &g_gemv_status)) {
                    ok = false;
                    break;
                }
                tc::fence_after();
                // the B tiles of a stage are kBTile apart: step the descriptor's start-address field
                const uint64_t bdesc = tc::sdesc_noswz(sm0 + (uint32_t)(s * Cfg::kStageBytes + kTcWBytes), 128, 256);
                const uint32_t dcol = tmem + kTcDCol + 16u * ab, acol = tmem + kTcACol + 64u * ab;
#pragma unroll
                for (int j = 0; j < kTcRows / 8; j++)
                    tc::mma_f16_ts(dcol, acol + 8u * j, bdesc + (uint64_t)(j * (Cfg::kBTile >> 4)), idesc, j != 0);
                tc::commit(aempty_bar(ab));
                tc::commit(bempty_bar(s));
                tc::commit(dfull_bar(ab));
            }
            tc::commit(drain_bar);
            mbar_wait_drain(drain_bar, 0, &g_gemv_status);
        }
    } else if (warp == 2 || warp == 3) {
        // ------------------------------------------------------- x -> sparse B tiles
        // two warps, alternating items; x is already in the stage (bulk-copied by warp 0)
        for (int i = warp - 2; i < n_items; i += 2) {
            const int s = i % S;
            const uint32_t ps = (uint32_t)(i / S) & 1u;
            const bool good = mbar_wait(xfull_bar(s), ps, abort_flag, &g_gemv_status) &&
                              (i < S || mbar_wait(bempty_bar(s), ps ^ 1u, abort_flag, &g_gemv_status));
            if (!__all_sync(0xffffffffu, good)) break;  // warp-uniform exit
            uint8_t* bt = smem + (size_t)s * Cfg::kStageBytes + kTcWBytes;
            const uint8_t* xsm = bt + Cfg::kBBytes + Cfg::kSBytes;
            float xs[2];
#pragma unroll
            for (int blk = 0; blk < 2; blk++) {
                const int r = 32 * blk + lane;  // row within the item
                uint8_t* tile = bt + (r >> 3) * Cfg::kBTile;
                const int kk = 2 * (r & 7);
                float xv;
                if constexpr (XF32) {
                    xv = reinterpret_cast<const float*>(xsm)[r];
                    const __half hi = __float2half_rn(xv);
                    const __half lo = __float2half_rn(xv - __half2float(hi));
                    *reinterpret_cast<__half*>(tile + btile_off(4 * blk + 0, kk)) = hi;
                    *reinterpret_cast<__half*>(tile + btile_off(4 * blk + 1, kk + 1)) = hi;
                    *reinterpret_cast<__half*>(tile + btile_off(4 * blk + 2, kk)) = lo;
                    *reinterpret_cast<__half*>(tile + btile_off(4 * blk + 3, kk + 1)) = lo;
                } else {
                    const __half h = reinterpret_cast<const __half*>(xsm)[r];
                    xv = __half2float(h);
                    *reinterpret_cast<__half*>(tile + btile_off(2 * blk + 0, kk)) = h;
                    *reinterpret_cast<__half*>(tile + btile_off(2 * blk + 1, kk + 1)) = h;
                }
                xs[blk] = xv;
            }
#pragma unroll
            for (int m = 16; m >= 1; m >>= 1) {
                xs[0] += __shfl_xor_sync(0xffffffffu, xs[0], m);
                xs[1] += __shfl_xor_sync(0xffffffffu, xs[1], m);
            }
            if (lane == 0) {
                s_xb[s][0] = xs[0];
                s_xb[s][1] = xs[1];
            }
            tc::fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(bfull_bar(s));
                mbar_arrive(wempty_bar(s));  // x slice consumed
            }
        }
    } else if (warp >= kTcDq0) {
        // ------------------------------------------------------- dequant + epilogue
        pdl_wait();
        const int qd = warp & 3;
        const int lam = 32 * qd + lane;                 // TMEM lane
        const int g = lam >> 2, p = lam & 3;
        const int c0 = 8 * g + p, c1 = c0 + 4;          // this lane's two columns of the tile
        const uint32_t sh = (uint32_t)(p >> 1) * 8u;
        const uint32_t mask = (p & 1) ? 0x00F000F0u : 0x000F000Fu;
        const float E = (p & 1) ? 1048576.0f : 16777216.0f;  // 2^20 / 2^24
        const uint32_t lane_addr = (uint32_t)(32 * qd) << 16;
        const long long t_first = ibeg / a.noct;
        const long long t_last = n_items > 0 ? (iend - 1) / a.noct : t_first - 1;
        const int dq = tid - kTcDq0 * 32;               // 0..127 among the dequant threads

        auto write_y = [&](long long t, int col, float v) {
            const TcSeg& sgm = tc_seg(a, tc_seg_of(a, t));
            const int n = ((int)t - sgm.tile0) * kTcTN + col;
            const float inv = SFMT == G4B_SCALE_E4M3 ? sgm.inv : 1.0f;
            if (n < sgm.N) {
                if (YF32) reinterpret_cast<float*>(sgm.y)[n] = v * inv;
                else reinterpret_cast<__half*>(sgm.y)[n] = __float2half_rn(v * inv);
            }
        };
        auto reduce_tile = [&](long long t) {
            const long long c_first = ((t * a.noct + 1) * a.G - 1) / a.total;
            const long long c_last = (((t + 1) * a.noct) * a.G - 1) / a.total;
#pragma unroll
            for (int h = 0; h < 2; h++) {
                const int col = h ? c1 : c0;
                float v = 0.f;
                for (long long cc = c_first; cc <= c_last; cc++) {
                    const long long sl = cc * a.maxseg + (t - s_ftile[cc]);
                    v += __ldcg(&a.partial[(size_t)sl * kTcTN + col]);
                }
                write_y(t, col, v);
            }
            if (dq == 0) a.counters[t] = 0u;  // ready for the next call
        };
        auto flush_tile = [&](long long t, float acc0, float acc1) {
            const long long c_first = ((t * a.noct + 1) * a.G - 1) / a.total;
            const long long c_last = (((t + 1) * a.noct) * a.G - 1) / a.total;
            const bool ok = !*abort_flag;
            if (c_first == c_last) {
                if (ok) {
                    write_y(t, c0, acc0);
                    write_y(t, c1, acc1);
                }
                return;
            }
            const long long slot = (long long)blockIdx.x * a.maxseg + (t - t_first);
            if (ok) {
                a.partial[(size_t)slot * kTcTN + c0] = acc0;
                a.partial[(size_t)slot * kTcTN + c1] = acc1;
            }
            named_bar_sync(1, 128);
            if (t < t_last) {
                if (dq == 0 && ok) {
                    __threadfence();
                    if (atomicAdd(&a.counters[t], 1u) == (unsigned)(c_last - c_first)) s_pending = t;
                }
            } else {
                if (dq == 0) {
                    unsigned last = 0;
                    if (ok) {
                        __threadfence();
                        last = atomicAdd(&a.counters[t], 1u) == (unsigned)(c_last - c_first) ? 1u : 0u;
                    }
                    s_last = last;
                }
                named_bar_sync(1, 128);
                if (s_last) {
                    __threadfence();
                    reduce_tile(t);
                }
            }
        };

        float acc0 = 0.f, acc1 = 0.f;
        // scales and block sums of the item whose epilogue is still pending
        float ps00 = 0.f, ps01 = 0.f, ps10 = 0.f, ps11 = 0.f, px0 = 0.f, px1 = 0.f;
        auto epilogue = [&](int i) -> bool {
            const int ab = i & 1;
            const bool good = mbar_wait(dfull_bar(ab), (uint32_t)(i >> 1) & 1u, abort_flag, &g_gemv_status);
            if (!__all_sync(0xffffffffu, good)) return false;
            tc::fence_after();
            uint32_t d[8];
            tc::ld_32x32b_x8(tmem + lane_addr + kTcDCol + 16u * ab, d);
            tc::wait_ld();
            float d00, d01, d10, d11;  // d<block><column>
            if constexpr (XF32) {
                d00 = __uint_as_float(d[0]) + __uint_as_float(d[2]);
                d01 = __uint_as_float(d[1]) + __uint_as_float(d[3]);
                d10 = __uint_as_float(d[4]) + __uint_as_float(d[6]);
                d11 = __uint_as_float(d[5]) + __uint_as_float(d[7]);
            } else {
                d00 = __uint_as_float(d[0]);
                d01 = __uint_as_float(d[1]);
                d10 = __uint_as_float(d[2]);
                d11 = __uint_as_float(d[3]);
            }
            acc0 = fmaf(ps00, fmaf(d00, E, -8.0f * px0), acc0);
            acc1 = fmaf(ps01, fmaf(d01, E, -8.0f * px0), acc1);
            acc0 = fmaf(ps10, fmaf(d10, E, -8.0f * px1), acc0);
            acc1 = fmaf(ps11, fmaf(d11, E, -8.0f * px1), acc1);
            tc::fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(dempty_bar(ab));
            return true;
        };

        // Every dequant warp runs the same sequence of items, epilogues and tile
        // flushes (with their named barriers) even after a wait has given up:
        // `ok` only turns the work off, never the control flow.
        bool ok = true;
        ItemCursor cur(ibeg, a.noct);
        int t_prev = cur.t;
        for (int i = 0; i < n_items; i++, t_prev = cur.t, cur.next()) {
            const int s = i % S, ab = i & 1;
            const uint32_t ps = (uint32_t)(i / S) & 1u;
            bool good = ok && mbar_wait(full_bar(s), ps, abort_flag, &g_gemv_status) &&
                        mbar_wait(bfull_bar(s), ps, abort_flag, &g_gemv_status) &&
                        (i < 2 || mbar_wait(aempty_bar(ab), ((uint32_t)(i >> 1) & 1u) ^ 1u, abort_flag, &g_gemv_status));
            ok = __all_sync(0xffffffffu, good);
            float s00 = 0.f, s01 = 0.f, s10 = 0.f, s11 = 0.f, x0 = 0.f, x1 = 0.f;
            if (ok) {
                tc::fence_after();
                const uint8_t* st = smem + (size_t)s * Cfg::kStageBytes;
                const uint8_t* sc = st + kTcWBytes + Cfg::kBBytes;
                if constexpr (SFMT == G4B_SCALE_F16) {
                    const __half* sh16 = reinterpret_cast<const __half*>(sc);
                    s00 = __half2float(sh16[c0]);
                    s01 = __half2float(sh16[c1]);
                    s10 = __half2float(sh16[kTcTN + c0]);
                    s11 = __half2float(sh16[kTcTN + c1]);
                } else {
                    s00 = e4m3_decode_ref(sc[c0]);
                    s01 = e4m3_decode_ref(sc[c1]);
                    s10 = e4m3_decode_ref(sc[kTcTN + c0]);
                    s11 = e4m3_decode_ref(sc[kTcTN + c1]);
                }
                x0 = s_xb[s][0];
                x1 = s_xb[s][1];
                const uint32_t* wr = reinterpret_cast<const uint32_t*>(st) + g;
#pragma unroll
                for (int hh = 0; hh < 2; hh++) {
                    uint32_t v[32];
#pragma unroll
                    for (int r = 0; r < 32; r++) v[r] = (wr[(32 * hh + r) * (kTcTN / 8)] >> sh) & mask;
                    tc::st_32x32b_x32(tmem + lane_addr + kTcACol + 64u * ab + 32u * hh, v);
                }
                tc::wait_st();
                tc::fence_before();
                __syncwarp();
                if (lane == 0) {
                    mbar_arrive(afull_bar(ab));
                    mbar_arrive(wempty_bar(s));
                }
            }
            // epilogue of the previous item (its MMAs ran while this item was dequantised)
            if (i > 0) {
                if (ok) ok = epilogue(i - 1);
                if (t_prev != cur.t) {  // item i - 1 was the last of its tile in this CTA
                    flush_tile(t_prev, acc0, acc1);
                    acc0 = acc1 = 0.f;
                }
            }
            ps00 = s00; ps01 = s01; ps10 = s10; ps11 = s11; px0 = x0; px1 = x1;
        }
        if (n_items > 0) {
            if (ok) ok = epilogue(n_items - 1);
            flush_tile(t_last, acc0, acc1);
        }
        // the deferred reduction of an earlier tile this CTA was the last to finish
        named_bar_sync(1, 128);
        if (s_pending >= 0 && !*abort_flag) {
            __threadfence();
            reduce_tile(s_pending);
        }
    }

    __syncwarp();
    tc::fence_before();
    __syncthreads();
    tc::fence_after();
    if (tid == 0 && *abort_flag) {
        const int issued = s_issued, xissued = s_xissued;
        for (int i = max(0, issued - S); i < issued; i++) mbar_wait_drain(full_bar(i % S), (i / S) & 1, &g_gemv_status);
        for (int i = max(0, xissued - S); i < xissued; i++)
            mbar_wait_drain(xfull_bar(i % S), (i / S) & 1, &g_gemv_status);
    }
    __syncthreads();
    if (warp == 1) tc::tmem_dealloc(tmem, 256);
}

struct TcPlan {
    int ntiles, noct, G, maxseg;
    long long total;
    size_t smem, ws_bytes;
};

static bool tc_ok(int M, int N, int K, int split) { return M == 1 && split == 0 && N % 32 == 0 && K % kTcRows == 0; }

static TcPlan tc_plan(int nseg, const int* Ns, int K, int sms, bool xf32, int sfmt) {
    TcPlan p{};
    p.noct = K / kTcRows;
    p.ntiles = 0;
    for (int i = 0; i < nseg; i++) p.ntiles += (Ns[i] + kTcTN - 1) / kTcTN;
    p.total = (long long)p.ntiles * p.noct;
    p.G = (int)std::max<long long>(1, std::min<long long>(std::min(std::max(sms, 1), kMaxCtas), p.total));
    const long long lmax = (p.total + p.G - 1) / p.G;
    p.maxseg = (int)((lmax + p.noct - 1) / p.noct + 1);
    p.smem = xf32 ? (sfmt == G4B_SCALE_F16 ? TcCfg<true, G4B_SCALE_F16>::kSmem : TcCfg<true, G4B_SCALE_E4M3>::kSmem)
                  : (sfmt == G4B_SCALE_F16 ? TcCfg<false, G4B_SCALE_F16>::kSmem : TcCfg<false, G4B_SCALE_E4M3>::kSmem);
    bool multi = false;
    for (int c = 1; c < p.G && !multi; c++)
        if (((long long)c * p.total / p.G) % p.noct) multi = true;
    if (multi) p.ws_bytes = kGemvCounterBytes + (((size_t)p.G * p.maxseg * kTcTN * sizeof(float) + 255) & ~(size_t)255);
    return p;
}

template <bool XF32, int SFMT, bool YF32>
static int launch_tc(const TcArgs& a, const TcPlan& p, const uint32_t* const* wps, const void* const* scales,
                     cudaStream_t s) {
    TcMaps maps;
    constexpr int ssz = SFMT == G4B_SCALE_F16 ? 2 : 1;
    for (int i = 0; i < kTcMaxSeg; i++) {
        const int k = i < a.nseg ? i : 0;  // unused slots repeat segment 0's maps
        const int N = k == 0 ? a.seg0.N : (k == 1 ? a.seg1.N : a.seg2.N);
        int st = tensor_map_2d(&maps.w[i], CU_TENSOR_MAP_DATA_TYPE_UINT32, wps[k], (uint64_t)N / 8, (uint64_t)a.K,
                               (uint64_t)N / 2, kTcTN / 8, kTcRows, CU_TENSOR_MAP_SWIZZLE_NONE,
                               CU_TENSOR_MAP_L2_PROMOTION_L2_128B);
        if (st != G4B_OK) return st;
        st = tensor_map_2d(&maps.s[i], CU_TENSOR_MAP_DATA_TYPE_UINT64, scales[k], (uint64_t)N * ssz / 8,
                           (uint64_t)a.K / 32, (uint64_t)N * ssz, kTcTN * ssz / 8, 2, CU_TENSOR_MAP_SWIZZLE_NONE);
        if (st != G4B_OK) return st;
    }
    auto kern = gemv_tc_kernel<XF32, SFMT, YF32>;
    static int attr_set_mask = 0;
    int dev = 0;
    cudaGetDevice(&dev);
    if (!(attr_set_mask & (1 << (dev & 31)))) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)TcCfg<XF32, SFMT>::kSmem);
        if (e != cudaSuccess) return fail(G4B_E_CUDA, "gemv_i4: cudaFuncSetAttribute: %s", cudaGetErrorString(e));
        attr_set_mask |= 1 << (dev & 31);
    }
    cudaError_t e = launch_k(kern, dim3(p.G), dim3(kTcThreads), TcCfg<XF32, SFMT>::kSmem, s, a, maps);
    if (e != cudaSuccess) return fail(G4B_E_CUDA, "gemv_i4: launch: %s", cudaGetErrorString(e));
    return G4B_OK;
}

static int dispatch_tc(const TcArgs& a, const TcPlan& p, const uint32_t* const* wp, const void* const* sc, bool xf32,
                       int sfmt, bool yf32, cudaStream_t s) {
    if (xf32) {
        if (sfmt == G4B_SCALE_F16)
            return yf32 ? launch_tc<true, G4B_SCALE_F16, true>(a, p, wp, sc, s)
                        : launch_tc<true, G4B_SCALE_F16, false>(a, p, wp, sc, s);
        return yf32 ? launch_tc<true, G4B_SCALE_E4M3, true>(a, p, wp, sc, s)
                    : launch_tc<true, G4B_SCALE_E4M3, false>(a, p, wp, sc, s);
    }
    if (sfmt == G4B_SCALE_F16)
        return yf32 ? launch_tc<false, G4B_SCALE_F16, true>(a, p, wp, sc, s)
                    : launch_tc<false, G4B_SCALE_F16, false>(a, p, wp, sc, s);
    return yf32 ? launch_tc<false, G4B_SCALE_E4M3, true>(a, p, wp, sc, s)
                : launch_tc<false, G4B_SCALE_E4M3, false>(a, p, wp, sc, s);
}

// Plan, check the workspace, and launch the tensor-core GEMV over `nseg`
// segments that share x (shapes already validated by the caller).
static int run_tc(const void* x, int x_dtype, int nseg, const g4b_gemv_segment* segs, int scale_fmt, int y_dtype,
                  int K, void* workspace, size_t ws_bytes, int sms, cudaStream_t s, const char* op) {
    int Ns[kTcMaxSeg];
    for (int i = 0; i < nseg; i++) Ns[i] = segs[i].N;
    const TcPlan p = tc_plan(nseg, Ns, K, sms, x_dtype == G4B_DT_F32, scale_fmt);
    G4B_REQUIRE(p.ntiles <= kGemvMaxTiles || p.ws_bytes == 0, G4B_E_SHAPE, "%s: too many columns for a split-K call",
                op);
    if (p.ws_bytes) {
        G4B_REQUIRE(workspace != nullptr && ws_bytes >= p.ws_bytes, G4B_E_WORKSPACE,
                    "%s: needs %zu bytes of workspace, got %zu", op, p.ws_bytes, workspace ? ws_bytes : 0);
        G4B_REQUIRE(aligned16(workspace), G4B_E_ALIGN, "%s: workspace must be 16-byte aligned", op);
    }
    TcArgs a{};
    a.x = x;
    TcSeg* dst[kTcMaxSeg] = {&a.seg0, &a.seg1, &a.seg2};
    const uint32_t* wps[kTcMaxSeg];
    const void* scs[kTcMaxSeg];
    int tile0 = 0;
    for (int i = 0; i < kTcMaxSeg; i++) {
        if (i < nseg) {
            dst[i]->y = segs[i].y;
            dst[i]->inv = segs[i].inv;
            dst[i]->N = segs[i].N;
            dst[i]->tile0 = tile0;
            tile0 += (segs[i].N + kTcTN - 1) / kTcTN;
            wps[i] = segs[i].wp;
            scs[i] = segs[i].scales;
        } else {
            *dst[i] = *dst[0];
            dst[i]->tile0 = 1 << 30;  // never reached
            wps[i] = segs[0].wp;
            scs[i] = segs[0].scales;
        }
    }
    a.nseg = nseg;
    a.K = K;
    a.noct = p.noct;
    a.ntiles = p.ntiles;
    a.G = p.G;
    a.maxseg = p.maxseg;
    a.total = p.total;
    if (p.ws_bytes) {
        a.counters = (unsigned*)workspace;
        a.partial = (float*)((char*)workspace + kGemvCounterBytes);
    }
    const int st = dispatch_tc(a, p, wps, scs, x_dtype == G4B_DT_F32, scale_fmt, y_dtype == G4B_DT_F32, s);
    if (st != G4B_OK) return st;
    count_launch();
    return launch_status(op);
}

// Plan, check the workspace, and launch the M = 1 kernel over `nseg` segments
// that share x (shapes already validated by the caller; K % 256 == 0).
static int run_m1(const void* x, int x_dtype, int nseg, const g4b_gemv_segment* segs, int scale_fmt, int y_dtype,
                  int K, void* workspace, size_t ws_bytes, int sms, cudaStream_t s, const char* op) {
    int Ns[kTcMaxSeg];
    for (int i = 0; i < nseg; i++) Ns[i] = segs[i].N;
    const M1Plan p = m1_plan(nseg, Ns, K, sms, x_dtype == G4B_DT_F32, scale_fmt);
    G4B_REQUIRE(p.ntiles <= kGemvMaxTiles || p.ws_bytes == 0, G4B_E_SHAPE, "%s: too many columns for a split-K call",
                op);
    if (p.ws_bytes) {
        G4B_REQUIRE(workspace != nullptr && ws_bytes >= p.ws_bytes, G4B_E_WORKSPACE,
                    "%s: needs %zu bytes of workspace, got %zu", op, p.ws_bytes, workspace ? ws_bytes : 0);
        G4B_REQUIRE(aligned16(workspace), G4B_E_ALIGN, "%s: workspace must be 16-byte aligned", op);
    }
    M1Args a{};
    a.x = x;
    TcSeg* dst[kTcMaxSeg] = {&a.seg0, &a.seg1, &a.seg2};
    const uint32_t* wps[kTcMaxSeg];
    const void* scs[kTcMaxSeg];
    int tile0 = 0;
    for (int i = 0; i < kTcMaxSeg; i++) {
        if (i < nseg) {
            dst[i]->y = segs[i].y;
            dst[i]->inv = segs[i].inv;
            dst[i]->N = segs[i].N;
            dst[i]->tile0 = tile0;
            tile0 += (segs[i].N + kStTN - 1) / kStTN;
            wps[i] = segs[i].wp;
            scs[i] = segs[i].scales;
        } else {
            *dst[i] = *dst[0];
            dst[i]->tile0 = 1 << 30;  // never reached
            wps[i] = segs[0].wp;
            scs[i] = segs[0].scales;
        }
    }
    a.nseg = nseg;
    a.K = K;
    a.noct = p.noct;
    a.ntiles = p.ntiles;
    a.G = p.G;
    a.maxseg = p.maxseg;
    a.mode = p.mode;
    a.total = p.total;
    a.stage_bytes = p.stage_bytes;
    a.s_bytes = p.s_bytes;
    if (p.ws_bytes) {
        a.counters = (unsigned*)workspace;
        a.partial = (float*)((char*)workspace + kGemvCounterBytes);
    }
    const int st = dispatch_m1(a, p, wps, scs, x_dtype == G4B_DT_F32, scale_fmt, y_dtype == G4B_DT_F32, s);
    if (st != G4B_OK) return st;
    count_launch();
    return launch_status(op);
}

unsigned read_status_gemv() {
    unsigned v = 0, z = 0;
    if (cudaMemcpyFromSymbol(&v, g_gemv_status, sizeof(v)) != cudaSuccess) return 0xffffffffu;
    if (v) cudaMemcpyToSymbol(g_gemv_status, &z, sizeof(z));
    return v;
}

struct StreamPlan {
    int ntiles, nquad, G, L, maxseg, stages, stage_bytes, s_bytes;
    long long total;
    size_t smem, part_bytes, ws_bytes;
};

static StreamPlan stream_plan(int M, int N, int K, int split, int sms, bool xf32, int sfmt) {
    StreamPlan p{};
    const int nblk = K / 32, mg = std::min(M, kGemvMaxTok);
    p.nquad = nblk / 4;
    p.ntiles = (N + kStTN - 1) / kStTN;
    p.total = (long long)p.ntiles * p.nquad;
    if (split > 0) {
        p.L = p.nquad / split;  // split divides nblk/4 here (checked by the caller)
        p.G = p.ntiles * split;
    } else {
        const int min_items = 2;  // at least 32 KB of weights per CTA
        long long G = std::min<long long>(2LL * std::max(sms, 1), (p.total + min_items - 1) / min_items);
        G = std::max<long long>(G, 1);
        p.L = (int)((p.total + G - 1) / G);
        p.G = (int)((p.total + p.L - 1) / p.L);
    }
    p.maxseg = (p.L + p.nquad - 1) / p.nquad + 1;
    p.s_bytes = 4 * kStTN * (sfmt == G4B_SCALE_F16 ? 2 : 1);
    const int nt = mg <= 4 ? 1 : 2;
    p.stage_bytes = (kStWBytes + p.s_bytes + mg * kStRows * (xf32 ? 4 : 2) + 127) & ~127;
    const size_t red_bytes = (size_t)4 * nt * 4 * 8 * 33 * sizeof(float);
    const size_t budget = 110 * 1024;  // two CTAs per SM
    p.stages = (int)std::max<size_t>(2, std::min<size_t>(kStMaxStages, (budget - red_bytes) / p.stage_bytes));
    p.smem = (size_t)p.stages * p.stage_bytes + red_bytes;
    const bool multi = (p.L % p.nquad) != 0;  // some tile is shared by several CTAs
    if (multi) {
        p.part_bytes = (size_t)p.G * p.maxseg * mg * kStTN * sizeof(float);
        p.ws_bytes = kGemvCounterBytes + ((p.part_bytes + 255) & ~(size_t)255);
    }
    return p;
}

template <bool XF32, int SFMT, int NT, bool YF32>
static int launch_stream(const StreamArgs& a, const StreamPlan& p, const uint32_t* wp, const void* scales,
                         cudaStream_t s) {
    CUtensorMap wmap, smap;
    int st = tensor_map_2d(&wmap, CU_TENSOR_MAP_DATA_TYPE_UINT32, wp, (uint64_t)a.N / 8, (uint64_t)a.K,
                           (uint64_t)a.N / 2, kStTN / 8, kStRows, CU_TENSOR_MAP_SWIZZLE_NONE,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_128B);
    if (st != G4B_OK) return st;
    constexpr int ssz = SFMT == G4B_SCALE_F16 ? 2 : 1;
    st = tensor_map_2d(&smap, CU_TENSOR_MAP_DATA_TYPE_UINT64, scales, (uint64_t)a.N * ssz / 8, (uint64_t)a.K / 32,
                       (uint64_t)a.N * ssz, kStTN * ssz / 8, 4, CU_TENSOR_MAP_SWIZZLE_NONE);
    if (st != G4B_OK) return st;
    auto kern = gemv_i4_stream_kernel<XF32, SFMT, NT, YF32>;
    static int attr_set_mask = 0;  // per device bit
    int dev = 0;
    cudaGetDevice(&dev);
    if (!(attr_set_mask & (1 << (dev & 31)))) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 112 * 1024);
        if (e != cudaSuccess) return fail(G4B_E_CUDA, "gemv_i4: cudaFuncSetAttribute: %s", cudaGetErrorString(e));
        attr_set_mask |= 1 << (dev & 31);
    }
    cudaError_t e = launch_k(kern, dim3(p.G), dim3(kStThreads), p.smem, s, a, wmap, smap);
    if (e != cudaSuccess) return fail(G4B_E_CUDA, "gemv_i4: launch: %s", cudaGetErrorString(e));
    return G4B_OK;
}

template <bool XF32, int SFMT>
static int dispatch_stream2(const StreamArgs& a, const StreamPlan& p, const uint32_t* wp, const void* sc, int nt,
                            bool yf32, cudaStream_t s) {
    if (nt == 1)
        return yf32 ? launch_stream<XF32, SFMT, 1, true>(a, p, wp, sc, s) : launch_stream<XF32, SFMT, 1, false>(a, p, wp, sc, s);
    return yf32 ? launch_stream<XF32, SFMT, 2, true>(a, p, wp, sc, s) : launch_stream<XF32, SFMT, 2, false>(a, p, wp, sc, s);
}

static int dispatch_stream(const StreamArgs& a, const StreamPlan& p, const uint32_t* wp, const void* sc, bool xf32,
                           int sfmt, int nt, bool yf32, cudaStream_t s) {
    if (xf32)
        return sfmt == G4B_SCALE_F16 ? dispatch_stream2<true, G4B_SCALE_F16>(a, p, wp, sc, nt, yf32, s)
                                     : dispatch_stream2<true, G4B_SCALE_E4M3>(a, p, wp, sc, nt, yf32, s);
    return sfmt == G4B_SCALE_F16 ? dispatch_stream2<false, G4B_SCALE_F16>(a, p, wp, sc, nt, yf32, s)
                                 : dispatch_stream2<false, G4B_SCALE_E4M3>(a, p, wp, sc, nt, yf32, s);
}

// The streaming kernel needs 16-byte rows (N % 32), whole block quads
// (K % 128) and, with a caller-given split, K-slices of whole quads.
static bool stream_ok(int N, int K, int split) {
    const int nblk = K / 32;
    return N % 32 == 0 && nblk % 4 == 0 && (split == 0 || (nblk / split) % 4 == 0);
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
        if (p.ntiles > kGemvMaxTiles) { p.slices = 1; p.bps = nblk; }
    }
    if (p.slices > 1) {
        p.part_bytes = align256((size_t)p.slices * p.mg * N * sizeof(float));
        p.ws_bytes = kGemvCounterBytes + p.part_bytes;
    }
    return p;
}

template <bool XF32, int SFMT, int NT, bool WIDE, bool YF32>
static void launch_gemv(const GemvArgs& a, const GemvPlan& p, cudaStream_t s) {
    dim3 grid(p.ntiles, p.slices);
    launch_k(gemv_i4_kernel<XF32, SFMT, NT, WIDE, YF32>, grid, dim3(kGemvThreads), 0, s, a);
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

// ------------------------------------------------- allocation-free variant
// Scratch for g4b_gemv_i4_noalloc: a fixed array in the library's own device
// memory, present on every GPU that loads the library until the process ends.
// Host code may only use its name through cudaGetSymbolAddress: on the host the
// symbol is a stand-in, not a device address.
constexpr size_t kNoAllocScratchBytes = 4u << 20;  // 4 MiB
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

static std::mutex g_noalloc_mu;
static void* g_noalloc_ptr[128];  // device address of the array, per device ordinal

// Resolve (once per device, with that device current) the array's device address.
static int noalloc_scratch(void** out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return fail(G4B_E_CUDA, "gemv_i4_noalloc: cudaGetDevice: %s", cudaGetErrorString(e));
    if (dev < 0 || dev >= 128) return fail(G4B_E_ARCH, "gemv_i4_noalloc: device index %d out of range", dev);
    std::lock_guard<std::mutex> lk(g_noalloc_mu);
    if (!g_noalloc_ptr[dev]) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess || !p)
            return fail(G4B_E_CUDA, "gemv_i4_noalloc: cudaGetSymbolAddress: %s", cudaGetErrorString(e));
        g_noalloc_ptr[dev] = p;
    }
    *out = g_noalloc_ptr[dev];
    return G4B_OK;
}

}  // namespace g4b

using namespace g4b;

extern "C" {

size_t g4b_gemv_workspace_bytes(int M, int N, int K, int split) {
    if (M <= 0 || N <= 0 || K <= 0 || K % 32 || N % 16) return 0;
    if (split > 0 && (K / 32) % split) return 0;
    int sms = 148;
    if (check_device(&sms) != G4B_OK) sms = 148;
    clear_error();
    // the activation and scale formats only change the shared-memory layout, not the workspace
    if (m1_ok(M, N, K, split)) return m1_plan(1, &N, K, sms, true, G4B_SCALE_F16).ws_bytes;
    if (tc_ok(M, N, K, split)) return tc_plan(1, &N, K, sms, true, G4B_SCALE_F16).ws_bytes;
    if (stream_ok(N, K, split)) return stream_plan(M, N, K, split, sms, true, G4B_SCALE_F16).ws_bytes;
    return gemv_plan(M, N, K, split, sms).ws_bytes;
}

static int gemv_i4_impl(const void* x, int x_dtype, int M, const uint32_t* wp, const void* scales, int scale_fmt,
                        float inv, void* y, int y_dtype, int N, int K, int split, void* workspace, size_t ws_bytes,
                        g4b_stream_t stream);

int g4b_gemv_i4(const void* x, int x_dtype, int M, const uint32_t* wp, const void* scales, int scale_fmt,
                float inv, void* y, int y_dtype, int N, int K, int split, void* workspace, size_t ws_bytes,
                g4b_stream_t stream) {
    G4B_ENTRY("gemv_i4");
    t_pdl = false;
    return gemv_i4_impl(x, x_dtype, M, wp, scales, scale_fmt, inv, y, y_dtype, N, K, split, workspace, ws_bytes, stream);
}

int g4b_gemv_i4_ex(const void* x, int x_dtype, int M, const uint32_t* wp, const void* scales, int scale_fmt,
                   float inv, void* y, int y_dtype, int N, int K, int split, void* workspace, size_t ws_bytes,
                   unsigned flags, g4b_stream_t stream) {
    G4B_ENTRY("gemv_i4");
    G4B_REQUIRE((flags & ~(unsigned)G4B_GEMV_PDL) == 0, G4B_E_ARG, "gemv_i4_ex: unknown flags 0x%x", flags);
    t_pdl = (flags & G4B_GEMV_PDL) != 0;
    const int st = gemv_i4_impl(x, x_dtype, M, wp, scales, scale_fmt, inv, y, y_dtype, N, K, split, workspace, ws_bytes,
                                stream);
    t_pdl = false;
    return st;
}

// Every argument check of g4b_gemv_i4 that needs no workspace: pointers, enums,
// sizes and alignment.  Shared with g4b_gemv_i4_noalloc, which runs it before it
// queues anything.
static int gemv_i4_check(const void* x, int x_dtype, int M, const uint32_t* wp, const void* scales, int scale_fmt,
                         void* y, int y_dtype, int N, int K, int split) {
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
    return G4B_OK;
}

static int gemv_i4_impl(const void* x, int x_dtype, int M, const uint32_t* wp, const void* scales, int scale_fmt,
                        float inv, void* y, int y_dtype, int N, int K, int split, void* workspace, size_t ws_bytes,
                        g4b_stream_t stream) {
    int st = gemv_i4_check(x, x_dtype, M, wp, scales, scale_fmt, y, y_dtype, N, K, split);
    if (st != G4B_OK) return st;
    const int nblk = K / 32;
    int sms = 0;
    st = check_device(&sms);
    if (st != G4B_OK) return st;
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    const size_t xe = x_dtype == G4B_DT_F32 ? 4 : 2, ye = y_dtype == G4B_DT_F32 ? 4 : 2;
    if (m1_ok(M, N, K, split)) {
        g4b_gemv_segment sg{wp, scales, inv, y, N};
        return run_m1(x, x_dtype, 1, &sg, scale_fmt, y_dtype, K, workspace, ws_bytes, sms, s, "gemv_i4");
    }
    if (tc_ok(M, N, K, split)) {
        g4b_gemv_segment sg{wp, scales, inv, y, N};
        return run_tc(x, x_dtype, 1, &sg, scale_fmt, y_dtype, K, workspace, ws_bytes, sms, s, "gemv_i4");
    }
    if (stream_ok(N, K, split)) {
        const StreamPlan p = stream_plan(M, N, K, split, sms, x_dtype == G4B_DT_F32, scale_fmt);
        if (p.ws_bytes) {
            G4B_REQUIRE(workspace != nullptr && ws_bytes >= p.ws_bytes, G4B_E_WORKSPACE,
                        "gemv_i4: needs %zu bytes of workspace, got %zu", p.ws_bytes, workspace ? ws_bytes : 0);
            G4B_REQUIRE(aligned16(workspace), G4B_E_ALIGN, "gemv_i4: workspace must be 16-byte aligned");
            G4B_REQUIRE(p.ntiles <= kGemvMaxTiles, G4B_E_SHAPE, "gemv_i4: N=%d too large for a split-K call", N);
        }
        for (int m0 = 0; m0 < M; m0 += kGemvMaxTok) {
            StreamArgs a{};
            a.M = std::min(kGemvMaxTok, M - m0);
            a.x = (const char*)x + (size_t)m0 * K * xe;
            a.y = (char*)y + (size_t)m0 * N * ye;
            a.inv = inv;
            a.N = N;
            a.K = K;
            a.nquad = p.nquad;
            a.ntiles = p.ntiles;
            a.L = p.L;
            a.maxseg = p.maxseg;
            a.total = p.total;
            a.stages = p.stages;
            a.stage_bytes = p.stage_bytes;
            a.s_bytes = p.s_bytes;
            if (p.ws_bytes) {
                a.counters = (unsigned*)workspace;
                a.partial = (float*)((char*)workspace + kGemvCounterBytes);
            }
            st = dispatch_stream(a, p, wp, scales, x_dtype == G4B_DT_F32, scale_fmt, a.M <= 4 ? 1 : 2,
                                 y_dtype == G4B_DT_F32, s);
            if (st != G4B_OK) return st;
            count_launch();
            st = launch_status("gemv_i4");
            if (st != G4B_OK) return st;
        }
        return G4B_OK;
    }
    // other shapes (N % 32 == 16, K % 128 != 0): the register-streaming kernel
    const GemvPlan p = gemv_plan(M, N, K, split, sms);
    if (p.slices > 1) {
        G4B_REQUIRE(workspace != nullptr && ws_bytes >= p.ws_bytes, G4B_E_WORKSPACE,
                    "gemv_i4: needs %zu bytes of workspace, got %zu", p.ws_bytes, workspace ? ws_bytes : 0);
        G4B_REQUIRE(aligned16(workspace), G4B_E_ALIGN, "gemv_i4: workspace must be 16-byte aligned");
        G4B_REQUIRE(p.ntiles <= kGemvMaxTiles, G4B_E_SHAPE, "gemv_i4: N=%d too large for a split-K call (split=1 only)",
                    N);
    }
    const bool wide = (N % 32) == 0;
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
            a.counters = (unsigned*)workspace;
            a.partial = (float*)((char*)workspace + kGemvCounterBytes);
        }
        const int nt = a.M <= 4 ? 1 : 2;
        dispatch_gemv(a, p, x_dtype == G4B_DT_F32, scale_fmt, nt, wide, y_dtype == G4B_DT_F32, s);
        count_launch();
        st = launch_status("gemv_i4");
        if (st != G4B_OK) return st;
    }
    return G4B_OK;
}

size_t g4b_gemv_fused_workspace_bytes(int nseg, const int* Ns, int K) {
    if (nseg < 1 || nseg > kTcMaxSeg || !Ns || K <= 0 || K % kTcRows) return 0;
    for (int i = 0; i < nseg; i++)
        if (Ns[i] <= 0 || Ns[i] % 32) return 0;
    int sms = 148;
    if (check_device(&sms) != G4B_OK) sms = 148;
    clear_error();
    if (K % 256 == 0) return m1_plan(nseg, Ns, K, sms, true, G4B_SCALE_F16).ws_bytes;
    return tc_plan(nseg, Ns, K, sms, true, G4B_SCALE_F16).ws_bytes;
}

int g4b_gemv_i4_fused(const void* x, int x_dtype, int nseg, const g4b_gemv_segment* segs, int scale_fmt, int y_dtype,
                      int K, void* workspace, size_t ws_bytes, unsigned flags, g4b_stream_t stream) {
    G4B_ENTRY("gemv_i4_fused");
    G4B_REQUIRE((flags & ~(unsigned)G4B_GEMV_PDL) == 0, G4B_E_ARG, "gemv_i4_fused: unknown flags 0x%x", flags);
    G4B_REQUIRE(x && segs, G4B_E_ARG, "gemv_i4_fused: NULL pointer argument");
    G4B_REQUIRE(nseg >= 1 && nseg <= kTcMaxSeg, G4B_E_ARG, "gemv_i4_fused: nseg=%d must be 1..%d", nseg, kTcMaxSeg);
    G4B_REQUIRE(x_dtype == G4B_DT_F32 || x_dtype == G4B_DT_F16, G4B_E_ARG, "gemv_i4_fused: bad x_dtype %d", x_dtype);
    G4B_REQUIRE(y_dtype == G4B_DT_F32 || y_dtype == G4B_DT_F16, G4B_E_ARG, "gemv_i4_fused: bad y_dtype %d", y_dtype);
    G4B_REQUIRE(scale_fmt == G4B_SCALE_F16 || scale_fmt == G4B_SCALE_E4M3, G4B_E_ARG,
                "gemv_i4_fused: bad scale_fmt %d", scale_fmt);
    G4B_REQUIRE(K > 0 && K % kTcRows == 0, G4B_E_SHAPE, "gemv_i4_fused: K=%d must be a multiple of %d", K, kTcRows);
    G4B_REQUIRE(aligned16(x), G4B_E_ALIGN, "gemv_i4_fused: x must be 16-byte aligned");
    for (int i = 0; i < nseg; i++) {
        const g4b_gemv_segment& g = segs[i];
        G4B_REQUIRE(g.wp && g.scales && g.y, G4B_E_ARG, "gemv_i4_fused: segment %d has a NULL pointer", i);
        G4B_REQUIRE(g.N > 0 && g.N % 32 == 0, G4B_E_SHAPE, "gemv_i4_fused: segment %d N=%d must be a multiple of 32",
                    i, g.N);
        G4B_REQUIRE(aligned16(g.wp) && aligned16(g.scales), G4B_E_ALIGN,
                    "gemv_i4_fused: segment %d wp and scales must be 16-byte aligned", i);
        G4B_REQUIRE(((uintptr_t)g.y & (y_dtype == G4B_DT_F32 ? 3u : 1u)) == 0, G4B_E_ALIGN,
                    "gemv_i4_fused: segment %d y misaligned", i);
    }
    int sms = 0;
    int st = check_device(&sms);
    if (st != G4B_OK) return st;
    t_pdl = (flags & G4B_GEMV_PDL) != 0;
    st = K % 256 == 0 ? run_m1(x, x_dtype, nseg, segs, scale_fmt, y_dtype, K, workspace, ws_bytes, sms,
                               reinterpret_cast<cudaStream_t>(stream), "gemv_i4_fused")
                      : run_tc(x, x_dtype, nseg, segs, scale_fmt, y_dtype, K, workspace, ws_bytes, sms,
                               reinterpret_cast<cudaStream_t>(stream), "gemv_i4_fused");
    t_pdl = false;
    return st;
}

}  // extern "C"

// ------------------------------------------------------------ GEMV chains
struct g4b_gemv_chain {
    int device = -1, nsteps = 0, x_dtype = 0, scale_fmt = 0, y_dtype = 0;
    int grid = 0, stage_bytes = 0, s_bytes = 0, maxtiles = 0, rank = 0, world = 1;
    int pf_items = 0;              // L2 prefetch distance in items (G4B_CHAIN_PREFETCH at create time)
    size_t smem = 0, sync_bytes = 0, ws_bytes = 0;
    size_t fwd_at = 0;             // workspace offset of the forward area (forwarded outputs' words)
    void* const* peers = nullptr;  // device array of the world exchange buffers (tensor parallel)
    // device: [nsteps][6] CUtensorMap, then [nsteps] ChainStep, then the steps' range / cspan tables
    void* plan = nullptr;
};

namespace g4b {

constexpr int kChainMaxSteps = 1 << 16;
// Default L2 prefetch distance of a chain: items (a 256 x 256 weight tile and its scales, 36 KB
// with f16 scales) each CTA keeps in flight to L2 ahead of its TMA producer; 8 items over 148
// SMs hold about 43 MB of the 126 MB L2.  G4B_CHAIN_PREFETCH=n at chain creation overrides it.
constexpr int kChainPrefetchItems = 8;

static size_t chain_maps_bytes(int nsteps) { return (size_t)nsteps * 2 * kTcMaxSeg * sizeof(CUtensorMap); }

// The partition of one step's items over the CTAs: range[c] .. range[c+1] for
// c < G (contiguous, item = tile * noct + k-chunk).  Two candidates:
//   balanced      CTA c owns [c*T/G, (c+1)*T/G): the fewest items per CTA,
//                 but a CTA may straddle two shared tiles, and then flushes
//                 twice and may run a deferred reduction;
//   tile-aligned  whole tiles per CTA when there are at least as many tiles
//                 as CTAs, otherwise each tile's k-chunks split evenly over
//                 G/ntiles CTAs: no CTA straddles a shared tile.
// The tile-aligned one is taken unless it costs more than one item over the
// balanced one's longest range plus a straddle.
static std::vector<int> chain_partition(int ntiles, int noct, int sms) {
    const long long total = (long long)ntiles * noct;
    const int G = (int)std::max<long long>(1, std::min<long long>(std::min(sms, kMaxCtas), total));
    std::vector<int> bal(G + 1), ta;
    for (int c = 0; c <= G; c++) bal[c] = (int)((long long)c * total / G);
    int max_bal = 0;
    bool straddle = false;
    for (int c = 0; c < G; c++) {
        max_bal = std::max(max_bal, bal[c + 1] - bal[c]);
        const int tf = bal[c] / noct, tl = (bal[c + 1] - 1) / noct;
        if (tl > tf && (bal[c] % noct != 0 || bal[c + 1] % noct != 0)) straddle = true;
    }
    if (ntiles >= G) {
        ta.resize(G + 1);
        for (int c = 0; c <= G; c++) ta[c] = (int)((long long)c * ntiles / G) * noct;
    } else {
        ta.push_back(0);
        const int q = G / ntiles, r = G % ntiles;
        for (int t = 0; t < ntiles; t++) {
            const int n = std::min(noct, q + (t < r ? 1 : 0));
            for (int k = 1; k <= n; k++) ta.push_back(t * noct + (int)((long long)k * noct / n));
        }
    }
    int max_ta = 0;
    for (size_t c = 0; c + 1 < ta.size(); c++) max_ta = std::max(max_ta, ta[c + 1] - ta[c]);
    return max_ta <= max_bal + (straddle ? 1 : 0) ? ta : bal;
}

template <bool XF32, int SFMT, bool YF32>
static int chain_prepare_kernel(size_t smem, int* resident) {
    auto kern = gemv_i4_chain_kernel<XF32, SFMT, YF32>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
    if (e != cudaSuccess) return fail(G4B_E_CUDA, "gemv_chain: cudaFuncSetAttribute: %s", cudaGetErrorString(e));
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(resident, kern, kChainThreads, smem);
    if (e != cudaSuccess) return fail(G4B_E_CUDA, "gemv_chain: occupancy query: %s", cudaGetErrorString(e));
    return G4B_OK;
}

static int chain_prepare(bool xf32, int sfmt, bool yf32, size_t smem, int* resident) {
    if (xf32) {
        if (sfmt == G4B_SCALE_F16) return yf32 ? chain_prepare_kernel<true, G4B_SCALE_F16, true>(smem, resident) : chain_prepare_kernel<true, G4B_SCALE_F16, false>(smem, resident);
        return yf32 ? chain_prepare_kernel<true, G4B_SCALE_E4M3, true>(smem, resident) : chain_prepare_kernel<true, G4B_SCALE_E4M3, false>(smem, resident);
    }
    if (sfmt == G4B_SCALE_F16) return yf32 ? chain_prepare_kernel<false, G4B_SCALE_F16, true>(smem, resident) : chain_prepare_kernel<false, G4B_SCALE_F16, false>(smem, resident);
    return yf32 ? chain_prepare_kernel<false, G4B_SCALE_E4M3, true>(smem, resident) : chain_prepare_kernel<false, G4B_SCALE_E4M3, false>(smem, resident);
}

template <bool XF32, int SFMT, bool YF32>
static cudaError_t chain_launch_kernel(const g4b_gemv_chain* c, const ChainArgs& ch, bool pdl, cudaStream_t s) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(c->grid);
    cfg.blockDim = dim3(kChainThreads);
    cfg.dynamicSmemBytes = c->smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeCooperative;  // every CTA resident: the steps wait on one another
    attr[0].val.cooperative = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 2 : 1;
    return cudaLaunchKernelEx(&cfg, gemv_i4_chain_kernel<XF32, SFMT, YF32>, ch);
}

static cudaError_t chain_launch(const g4b_gemv_chain* c, const ChainArgs& ch, bool pdl, cudaStream_t s) {
    const bool xf32 = c->x_dtype == G4B_DT_F32, yf32 = c->y_dtype == G4B_DT_F32;
    if (xf32) {
        if (c->scale_fmt == G4B_SCALE_F16) return yf32 ? chain_launch_kernel<true, G4B_SCALE_F16, true>(c, ch, pdl, s) : chain_launch_kernel<true, G4B_SCALE_F16, false>(c, ch, pdl, s);
        return yf32 ? chain_launch_kernel<true, G4B_SCALE_E4M3, true>(c, ch, pdl, s) : chain_launch_kernel<true, G4B_SCALE_E4M3, false>(c, ch, pdl, s);
    }
    if (c->scale_fmt == G4B_SCALE_F16) return yf32 ? chain_launch_kernel<false, G4B_SCALE_F16, true>(c, ch, pdl, s) : chain_launch_kernel<false, G4B_SCALE_F16, false>(c, ch, pdl, s);
    return yf32 ? chain_launch_kernel<false, G4B_SCALE_E4M3, true>(c, ch, pdl, s) : chain_launch_kernel<false, G4B_SCALE_E4M3, false>(c, ch, pdl, s);
}

}  // namespace g4b

// Exchange-buffer words (u64) the steps' all-reduces need: world slots of N
// words per flagged step; -1 if the flags are inconsistent.
static long long chain_exchange_words(const g4b_gemv_chain_step* steps, int nsteps, int world) {
    long long words = 0;
    for (int j = 0; j < nsteps; j++) {
        if (!(steps[j].flags & G4B_CHAIN_ALLREDUCE)) continue;
        if (j + 1 >= nsteps || steps[j].nseg != 1 || steps[j + 1].K != steps[j].seg[0].N) return -1;
        words += (long long)world * steps[j].seg[0].N;
    }
    return words;
}

extern "C" {

size_t g4b_gemv_chain_exchange_bytes(const g4b_gemv_chain_step* steps, int nsteps, int world) {
    if (!steps || nsteps < 1 || world < 1 || world > 8) return 0;
    const long long w = chain_exchange_words(steps, nsteps, world);
    return w < 0 ? 0 : (size_t)w * sizeof(unsigned long long);
}

int g4b_gemv_chain_create(const g4b_gemv_chain_step* steps, int nsteps, int x_dtype, int scale_fmt, int y_dtype,
                          g4b_gemv_chain** chain) {
    return g4b_gemv_chain_create_tp(steps, nsteps, x_dtype, scale_fmt, y_dtype, nullptr, 0, 1, 0, chain);
}

static int chain_create_impl(const g4b_gemv_chain_step* steps, const g4b_chain_xform* xf, int nsteps, int x_dtype,
                             int scale_fmt, int y_dtype, void* const* peers_dev, int rank, int world,
                             size_t exchange_bytes, g4b_gemv_chain** chain);

int g4b_gemv_chain_create_tp(const g4b_gemv_chain_step* steps, int nsteps, int x_dtype, int scale_fmt, int y_dtype,
                             void* const* peers_dev, int rank, int world, size_t exchange_bytes,
                             g4b_gemv_chain** chain) {
    G4B_ENTRY("gemv_chain_create");
    return chain_create_impl(steps, nullptr, nsteps, x_dtype, scale_fmt, y_dtype, peers_dev, rank, world,
                             exchange_bytes, chain);
}

int g4b_gemv_chain_create_fused(const g4b_gemv_chain_step* steps, const g4b_chain_xform* xforms, int nsteps,
                                int x_dtype, int scale_fmt, int y_dtype, g4b_gemv_chain** chain) {
    G4B_ENTRY("gemv_chain_create_fused");
    G4B_REQUIRE(xforms, G4B_E_ARG, "gemv_chain_create_fused: NULL xforms");
    return chain_create_impl(steps, xforms, nsteps, x_dtype, scale_fmt, y_dtype, nullptr, 0, 1, 0, chain);
}

// Check step j's element-wise work (g4b_chain_xform) against the steps.
static int chain_check_xform(const g4b_gemv_chain_step* steps, const g4b_chain_xform* xf, int j) {
    const g4b_chain_xform& f = xf[j];
    const int K = steps[j].K;
    G4B_REQUIRE(f.kind >= G4B_XF_NONE && f.kind <= G4B_XF_GELU_MUL, G4B_E_ARG,
                "gemv_chain_create_fused: step %d has unknown xform kind %d", j, f.kind);
    if (f.kind == G4B_XF_NONE) return G4B_OK;
    G4B_REQUIRE(!(steps[j].flags & G4B_CHAIN_ALLREDUCE) && (j == 0 || !(steps[j - 1].flags & G4B_CHAIN_ALLREDUCE)),
                G4B_E_ARG, "gemv_chain_create_fused: step %d: element-wise work next to an all-reduced step", j);
    G4B_REQUIRE(f.a && aligned16(f.a), G4B_E_ARG, "gemv_chain_create_fused: step %d xform needs a 16-byte aligned a",
                j);
    const bool produced = j > 0 && f.a == steps[j - 1].seg[0].y;
    G4B_REQUIRE(!produced || steps[j - 1].seg[0].N == K, G4B_E_SHAPE,
                "gemv_chain_create_fused: step %d reads step %d's output of %d values as its %d inputs", j, j - 1,
                steps[j - 1].seg[0].N, K);
    if (f.kind == G4B_XF_GELU_MUL) {
        G4B_REQUIRE(j > 0 && f.b && aligned16(f.b), G4B_E_ARG,
                    "gemv_chain_create_fused: step %d GELU_MUL needs 16-byte aligned a and b written by earlier steps",
                    j);
        return G4B_OK;
    }
    G4B_REQUIRE(f.w && aligned16(f.w), G4B_E_ARG, "gemv_chain_create_fused: step %d needs a 16-byte aligned w", j);
    G4B_REQUIRE(f.eps >= 0.f, G4B_E_ARG, "gemv_chain_create_fused: step %d eps must be >= 0", j);
    if (f.kind == G4B_XF_NORMADD) {
        G4B_REQUIRE(produced, G4B_E_ARG,
                    "gemv_chain_create_fused: step %d NORMADD: a must be step %d's first output", j, j - 1);
        G4B_REQUIRE(f.b && f.w_post && f.h_out && aligned16(f.b) && aligned16(f.w_post) && aligned16(f.h_out),
                    G4B_E_ARG, "gemv_chain_create_fused: step %d NORMADD needs 16-byte aligned b, w_post and h_out", j);
        const char* hb = reinterpret_cast<const char*>(f.h_out);
        const char* bb = reinterpret_cast<const char*>(f.b);
        G4B_REQUIRE(hb + (size_t)K * 4 <= bb || bb + (size_t)K * 4 <= hb, G4B_E_ARG,
                    "gemv_chain_create_fused: step %d NORMADD h_out overlaps b", j);
    }
    return G4B_OK;
}

// Step j's outputs (every segment's y) against what step j-1 reads from memory (its x, its
// element-wise inputs) or writes (its outputs, its h_out).  A step that reads forwarded x does not wait
// for step j-1 to finish, so an overlap there must keep the whole-step wait.
static bool ranges_overlap(const void* a, size_t na, const void* b, size_t nb) {
    if (!a || !b || !na || !nb) return false;
    const uintptr_t a0 = reinterpret_cast<uintptr_t>(a), b0 = reinterpret_cast<uintptr_t>(b);
    return a0 < b0 + nb && b0 < a0 + na;
}
static bool chain_outputs_touch_prev(const g4b_gemv_chain_step* steps, const g4b_chain_xform* xf, int j, int x_dtype,
                                     int y_dtype, bool prev_x_in_memory) {
    const size_t ysz = y_dtype == G4B_DT_F32 ? 4 : 2, xsz = x_dtype == G4B_DT_F32 ? 4 : 2;
    const g4b_gemv_chain_step& p = steps[j - 1];
    for (int i = 0; i < steps[j].nseg; i++) {
        const void* y = steps[j].seg[i].y;
        const size_t ny = (size_t)steps[j].seg[i].N * ysz;
        // (step j-1's own x only when it loads it from memory, not as forwarded or all-reduced words)
        if (prev_x_in_memory && ranges_overlap(y, ny, p.x, (size_t)p.K * xsz)) return true;
        for (int q = 0; q < p.nseg; q++)
            if (ranges_overlap(y, ny, p.seg[q].y, (size_t)p.seg[q].N * ysz)) return true;
        if (xf && xf[j - 1].kind != G4B_XF_NONE) {
            const g4b_chain_xform& f = xf[j - 1];
            const size_t nk = (size_t)p.K;
            if (ranges_overlap(y, ny, f.a, nk * 4) || ranges_overlap(y, ny, f.b, nk * 4) ||
                ranges_overlap(y, ny, f.h_out, nk * 4))
                return true;
        }
    }
    return false;
}

// Where each step's x comes from -- the decisions chain creation makes, on the host only:
//   fwd[j]    x is step j-1's first output (same dtype, no element-wise work, no all-reduce between them,
//             no overlap that the whole-step wait would have to order), read as forwarded words;
//   wlo[j]    the first step whose completion count step j's activation load waits for (it waits for
//             wlo .. j-1 unless its x is forwarded or all-reduced): back over the forwarded steps, which
//             waited on no count themselves;
//   early[j]  x written by no step (no output or h_out range overlaps it): its first slice is loaded
//             before that wait.
// G4B_CHAIN_FORWARD=0 in the environment turns forwarding and the early load off.
struct ChainXPlan {
    std::vector<int> fwd, wlo, early;
};
static ChainXPlan chain_plan_x(const g4b_gemv_chain_step* steps, const g4b_chain_xform* xf, int nsteps, int x_dtype,
                               int y_dtype) {
    const char* env = getenv("G4B_CHAIN_FORWARD");
    const bool off = env && atoi(env) == 0;
    const bool fwd_on = x_dtype == y_dtype && !off;
    const size_t ysz = y_dtype == G4B_DT_F32 ? 4 : 2, xsz = x_dtype == G4B_DT_F32 ? 4 : 2;
    ChainXPlan p;
    p.fwd.assign(nsteps, 0);
    p.wlo.assign(nsteps, 0);
    p.early.assign(nsteps, 0);
    auto xreg = [&](int j) { return j > 0 && (steps[j - 1].flags & G4B_CHAIN_ALLREDUCE) != 0; };
    auto xform = [&](int j) { return xf && xf[j].kind != G4B_XF_NONE; };
    for (int j = 1; j < nsteps; j++) {
        const g4b_gemv_chain_step& cs = steps[j];
        p.fwd[j] = fwd_on && cs.x && cs.x == steps[j - 1].seg[0].y && !xform(j) &&
                   !(steps[j - 1].flags & G4B_CHAIN_ALLREDUCE) && cs.K <= steps[j - 1].seg[0].N &&
                   !chain_outputs_touch_prev(steps, xf, j, x_dtype, y_dtype, !p.fwd[j - 1] && !xreg(j - 1));
    }
    for (int j = 1; j < nsteps; j++) {
        int lo = j - 1;
        while (lo > 0 && p.fwd[lo]) lo--;
        p.wlo[j] = lo;
        if (off || !steps[j].x || xreg(j) || p.fwd[j] || xform(j)) continue;
        bool written = false;
        for (int k = 0; k < nsteps && !written; k++) {
            for (int i = 0; i < steps[k].nseg && !written; i++)
                written = ranges_overlap(steps[j].x, (size_t)steps[j].K * xsz, steps[k].seg[i].y,
                                         (size_t)steps[k].seg[i].N * ysz);
            if (!written && xf && xf[k].kind == G4B_XF_NORMADD)
                written = ranges_overlap(steps[j].x, (size_t)steps[j].K * xsz, xf[k].h_out, (size_t)steps[k].K * 4);
        }
        p.early[j] = written ? 0 : 1;
    }
    return p;
}

static int chain_create_impl(const g4b_gemv_chain_step* steps, const g4b_chain_xform* xf, int nsteps, int x_dtype,
                             int scale_fmt, int y_dtype, void* const* peers_dev, int rank, int world,
                             size_t exchange_bytes, g4b_gemv_chain** chain) {
    G4B_REQUIRE(steps && chain, G4B_E_ARG, "gemv_chain_create: NULL pointer argument");
    *chain = nullptr;
    G4B_REQUIRE(world >= 1 && world <= 8 && rank >= 0 && rank < world, G4B_E_ARG,
                "gemv_chain_create: rank %d / world %d (1..8 ranks)", rank, world);
    G4B_REQUIRE(nsteps >= 1 && nsteps <= kChainMaxSteps, G4B_E_ARG, "gemv_chain_create: nsteps=%d (1..%d)", nsteps,
                kChainMaxSteps);
    G4B_REQUIRE(x_dtype == G4B_DT_F32 || x_dtype == G4B_DT_F16, G4B_E_ARG, "gemv_chain_create: bad x_dtype %d",
                x_dtype);
    G4B_REQUIRE(y_dtype == G4B_DT_F32 || y_dtype == G4B_DT_F16, G4B_E_ARG, "gemv_chain_create: bad y_dtype %d",
                y_dtype);
    G4B_REQUIRE(scale_fmt == G4B_SCALE_F16 || scale_fmt == G4B_SCALE_E4M3, G4B_E_ARG,
                "gemv_chain_create: bad scale_fmt %d", scale_fmt);
    const long long xwords = chain_exchange_words(steps, nsteps, world);
    G4B_REQUIRE(xwords >= 0, G4B_E_ARG,
                "gemv_chain_create: an all-reduced step needs one segment and a next step with K = its N");
    G4B_REQUIRE(xwords == 0 || (peers_dev && world > 1), G4B_E_ARG,
                "gemv_chain_create: all-reduced steps need the exchange buffers of 2 or more ranks");
    G4B_REQUIRE((size_t)xwords * sizeof(unsigned long long) <= exchange_bytes || xwords == 0, G4B_E_WORKSPACE,
                "gemv_chain_create: the all-reduces need %lld exchange bytes, got %zu",
                xwords * (long long)sizeof(unsigned long long), exchange_bytes);
    for (int j = 0; j < nsteps; j++) {
        const g4b_gemv_chain_step& st = steps[j];
        G4B_REQUIRE((st.flags & ~(unsigned)G4B_CHAIN_ALLREDUCE) == 0, G4B_E_ARG,
                    "gemv_chain_create: step %d has unknown flags 0x%x", j, st.flags);
        const bool x_from_peers = j > 0 && (steps[j - 1].flags & G4B_CHAIN_ALLREDUCE);
        const bool x_fused = xf && xf[j].kind != G4B_XF_NONE;
        G4B_REQUIRE(st.x || x_from_peers || x_fused, G4B_E_ARG, "gemv_chain_create: step %d has a NULL x", j);
        G4B_REQUIRE(x_from_peers || x_fused || aligned16(st.x), G4B_E_ALIGN,
                    "gemv_chain_create: step %d x must be 16-byte aligned", j);
        if (xf) {
            const int xs = chain_check_xform(steps, xf, j);
            if (xs != G4B_OK) return xs;
        }
        G4B_REQUIRE(st.nseg >= 1 && st.nseg <= kTcMaxSeg, G4B_E_ARG, "gemv_chain_create: step %d nseg=%d (1..%d)", j,
                    st.nseg, kTcMaxSeg);
        G4B_REQUIRE(st.K > 0 && st.K % 256 == 0, G4B_E_SHAPE, "gemv_chain_create: step %d K=%d must be a multiple of 256",
                    j, st.K);
        int ntiles = 0;
        for (int i = 0; i < st.nseg; i++) {
            const g4b_gemv_segment& g = st.seg[i];
            G4B_REQUIRE(g.wp && g.scales && g.y, G4B_E_ARG, "gemv_chain_create: step %d segment %d has a NULL pointer",
                        j, i);
            G4B_REQUIRE(g.N > 0 && g.N % 32 == 0, G4B_E_SHAPE,
                        "gemv_chain_create: step %d segment %d N=%d must be a multiple of 32", j, i, g.N);
            G4B_REQUIRE(aligned16(g.wp) && aligned16(g.scales), G4B_E_ALIGN,
                        "gemv_chain_create: step %d segment %d wp and scales must be 16-byte aligned", j, i);
            G4B_REQUIRE(((uintptr_t)g.y & (y_dtype == G4B_DT_F32 ? 3u : 1u)) == 0, G4B_E_ALIGN,
                        "gemv_chain_create: step %d segment %d y misaligned", j, i);
            ntiles += (g.N + kStTN - 1) / kStTN;
        }
        G4B_REQUIRE(ntiles <= kGemvMaxTiles, G4B_E_SHAPE, "gemv_chain_create: step %d has %d column tiles (max %d)", j,
                    ntiles, kGemvMaxTiles);
        G4B_REQUIRE((long long)ntiles * (st.K / 256) < (1LL << 30), G4B_E_SHAPE,
                    "gemv_chain_create: step %d has too many weight tiles", j);
    }
    int sms = 0;
    int st = check_device(&sms);
    if (st != G4B_OK) return st;
    int attr = 0;
    int dev = 0;
    cudaGetDevice(&dev);
    if (cudaDeviceGetAttribute(&attr, cudaDevAttrCooperativeLaunch, dev) != cudaSuccess || !attr)
        return fail(G4B_E_CUDA, "gemv_chain_create: device %d has no cooperative launch", dev);

    const bool xf32 = x_dtype == G4B_DT_F32;
    const int ssz = scale_fmt == G4B_SCALE_F16 ? 2 : 1;
    std::vector<ChainStep> hsteps((size_t)nsteps);
    std::vector<CUtensorMap> hmaps((size_t)nsteps * 2 * kTcMaxSeg);
    std::vector<int> tables;           // every step's range[G + 1] and cspan[ntiles][2]
    std::vector<size_t> range_at(nsteps), cspan_at(nsteps);
    std::vector<size_t> sums_at(nsteps, (size_t)-1);  // float offset of a producer step's tile sums
    size_t sums_words = 0;
    int grid = 1, maxtiles = 0;
    long long region = 0;  // next free exchange word
    // Forwarded x (chain_plan_x): a step whose x is the step before's first output reads it as
    // epoch-tagged words in the workspace, each 256-row slice as soon as its own words are stored.
    const ChainXPlan xp = chain_plan_x(steps, xf, nsteps, x_dtype, y_dtype);
    long long fwd_words = 0;
    for (int j = 0; j < nsteps; j++) {
        const g4b_gemv_chain_step& cs = steps[j];
        ChainStep& d = hsteps[j];
        d = ChainStep{};
        d.x = cs.x;
        d.xreg = -1;
        d.yreg = -1;
        d.xfw = -1;
        d.yfw = -1;
        if (j > 0 && (steps[j - 1].flags & G4B_CHAIN_ALLREDUCE)) d.xreg = hsteps[j - 1].yreg;
        if (cs.flags & G4B_CHAIN_ALLREDUCE) {
            d.yreg = (int)region;
            region += (long long)world * cs.seg[0].N;
        }
        if (xp.fwd[j]) {
            ChainStep& pd = hsteps[j - 1];
            if (pd.yfw < 0) {
                pd.yfw = (int)fwd_words;
                fwd_words += (steps[j - 1].seg[0].N + 31) & ~31;  // 256-byte aligned regions
            }
            d.xfw = pd.yfw;
        }
        TcSeg* dst[kTcMaxSeg] = {&d.seg0, &d.seg1, &d.seg2};
        const uint32_t* wps[kTcMaxSeg];
        const void* scs[kTcMaxSeg];
        int tile0 = 0;
        for (int i = 0; i < kTcMaxSeg; i++) {
            if (i < cs.nseg) {
                dst[i]->y = cs.seg[i].y;
                dst[i]->inv = cs.seg[i].inv;
                dst[i]->N = cs.seg[i].N;
                dst[i]->tile0 = tile0;
                tile0 += (cs.seg[i].N + kStTN - 1) / kStTN;
                wps[i] = cs.seg[i].wp;
                scs[i] = cs.seg[i].scales;
            } else {
                *dst[i] = *dst[0];
                dst[i]->tile0 = 1 << 30;  // never reached
                wps[i] = cs.seg[0].wp;
                scs[i] = cs.seg[0].scales;
            }
        }
        d.nseg = cs.nseg;
        d.K = cs.K;
        d.noct = cs.K / 256;
        d.ntiles = tile0;
        d.done = tile0;
        if (xf && xf[j].kind != G4B_XF_NONE) {
            const g4b_chain_xform& f = xf[j];
            d.xf_kind = f.kind;
            d.xf_a = f.a;
            d.xf_b = f.b;
            d.xf_w = f.w;
            d.xf_wpost = f.w_post;
            d.xf_hout = f.h_out;
            d.xf_scale = f.kind == G4B_XF_NORMADD ? f.scale : 1.0f;
            d.xf_eps = f.eps;
            const bool produced = j > 0 && f.a == steps[j - 1].seg[0].y;
            d.xf_self = f.kind == G4B_XF_RMSNORM && !produced;
            if (f.kind != G4B_XF_GELU_MUL && produced) {
                // the step before hands its first output's tile sums to this step's norm
                ChainStep& pd = hsteps[j - 1];
                d.xf_ptiles = (steps[j - 1].seg[0].N + kStTN - 1) / kStTN;
                sums_at[j - 1] = sums_words;
                sums_words += (size_t)4 * d.xf_ptiles;
                if (f.kind == G4B_XF_NORMADD) {
                    pd.sum_res = reinterpret_cast<const float*>(f.b);
                    pd.sum_wpost = f.w_post;
                }
            }
            if (f.kind == G4B_XF_NORMADD) d.done = tile0 + d.noct;  // + the h_out slices its loads write
        }
        const std::vector<int> range = chain_partition(d.ntiles, d.noct, sms);
        d.G = (int)range.size() - 1;
        range_at[j] = tables.size();
        tables.insert(tables.end(), range.begin(), range.end());
        cspan_at[j] = tables.size();
        std::vector<int> cspan((size_t)2 * d.ntiles);
        for (int cc = 0; cc < d.G; cc++) {
            if (range[cc + 1] <= range[cc]) continue;
            const int tf = range[cc] / d.noct, tl = (range[cc + 1] - 1) / d.noct;
            // CTAs come in item order: the last CTA to touch a tile is the latest; the first is the one
            // whose range holds the tile's first k-chunk
            for (int t = tf; t <= tl; t++) {
                cspan[2 * t + 1] = cc;
                if (t != tf) cspan[2 * t] = cc | (int)0x80000000u;  // cc's share of t sits in its last slot
                else if (range[cc] % d.noct == 0) cspan[2 * t] = cc;
            }
        }
        tables.insert(tables.end(), cspan.begin(), cspan.end());
        grid = std::max(grid, d.G);
        maxtiles = std::max(maxtiles, d.ntiles);
        CUtensorMap* wm = &hmaps[(size_t)j * 2 * kTcMaxSeg];
        for (int i = 0; i < kTcMaxSeg; i++) {
            const int k = i < cs.nseg ? i : 0;
            const int N = cs.seg[k].N;
            st = tensor_map_2d(&wm[i], CU_TENSOR_MAP_DATA_TYPE_UINT32, wps[k], (uint64_t)N / 8, (uint64_t)cs.K,
                               (uint64_t)N / 2, kStTN / 8, kM1Rows, CU_TENSOR_MAP_SWIZZLE_128B,
                               CU_TENSOR_MAP_L2_PROMOTION_L2_128B);
            if (st != G4B_OK) return st;
            st = tensor_map_2d(&wm[kTcMaxSeg + i], CU_TENSOR_MAP_DATA_TYPE_UINT64, scs[k], (uint64_t)N * ssz / 8,
                               (uint64_t)cs.K / 32, (uint64_t)N * ssz, kStTN * ssz / 8, 8, CU_TENSOR_MAP_SWIZZLE_NONE);
            if (st != G4B_OK) return st;
        }
    }
    G4B_REQUIRE(fwd_words < (1LL << 31), G4B_E_SHAPE, "gemv_chain_create: the forwarded outputs are too long");
    for (int j = 0; j < nsteps; j++) {
        hsteps[j].wlo = xp.wlo[j];
        hsteps[j].xind = xp.early[j];
    }
    // x slice: f32 as f16 hi | lo words, or f16 stored twice over (see chain_xoff16): 1 KB either way,
    // then (f32 x) its 8 block sums
    const int stage_bytes = (kM1WBytes + 8 * kStTN * ssz + kChainXBytes + (xf32 ? kChainXSumBytes : 0) + 1023) & ~1023;
    const size_t smem = (size_t)kM1Stages * stage_bytes + 1024;
    int resident = 0;
    st = chain_prepare(xf32, scale_fmt, y_dtype == G4B_DT_F32, smem, &resident);
    if (st != G4B_OK) return st;
    G4B_REQUIRE(resident >= 1 && grid <= sms * resident, G4B_E_CUDA,
                "gemv_chain_create: %d CTAs cannot all be resident (%d per SM, %d SMs)", grid, resident, sms);

    const size_t maps_bytes = chain_maps_bytes(nsteps);
    const size_t steps_bytes = (size_t)nsteps * sizeof(ChainStep);
    const size_t tables_bytes = (tables.size() * sizeof(int) + 15) & ~(size_t)15;
    // the tile sums (written by every run) follow the read-only plan in the same allocation
    const size_t plan_bytes = maps_bytes + steps_bytes + tables_bytes + sums_words * sizeof(float);
    void* plan = nullptr;
    cudaError_t e = cudaMalloc(&plan, plan_bytes);
    if (e != cudaSuccess) return fail(G4B_E_CUDA, "gemv_chain_create: cudaMalloc: %s", cudaGetErrorString(e));
    const int* tables_dev = reinterpret_cast<const int*>(reinterpret_cast<uint8_t*>(plan) + maps_bytes + steps_bytes);
    float* sums_dev = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(plan) + maps_bytes + steps_bytes +
                                               tables_bytes);
    for (int j = 0; j < nsteps; j++) {
        hsteps[j].range = tables_dev + range_at[j];
        hsteps[j].cspan = tables_dev + cspan_at[j];
        if (sums_at[j] != (size_t)-1) {
            hsteps[j].sums_out = sums_dev + sums_at[j];
            hsteps[j + 1].xf_sums = sums_dev + sums_at[j];
        }
    }
    std::vector<uint8_t> host(plan_bytes, 0);
    memcpy(host.data(), hmaps.data(), maps_bytes);
    memcpy(host.data() + maps_bytes, hsteps.data(), steps_bytes);
    memcpy(host.data() + maps_bytes + steps_bytes, tables.data(), tables.size() * sizeof(int));
    e = cudaMemcpy(plan, host.data(), plan_bytes, cudaMemcpyHostToDevice);
    if (e != cudaSuccess) {
        cudaFree(plan);
        return fail(G4B_E_CUDA, "gemv_chain_create: cudaMemcpy: %s", cudaGetErrorString(e));
    }
    g4b_gemv_chain* c = new g4b_gemv_chain();
    c->device = dev;
    c->nsteps = nsteps;
    c->x_dtype = x_dtype;
    c->scale_fmt = scale_fmt;
    c->y_dtype = y_dtype;
    c->grid = grid;
    c->stage_bytes = stage_bytes;
    c->s_bytes = 8 * kStTN * ssz;
    c->maxtiles = maxtiles;
    c->smem = smem;
    c->sync_bytes = ((size_t)(nsteps + 3) * sizeof(unsigned) + 255) & ~(size_t)255;
    c->fwd_at = c->sync_bytes + (size_t)2 * 2 * grid * kStTN * sizeof(unsigned long long);
    c->ws_bytes = c->fwd_at + (size_t)fwd_words * sizeof(unsigned long long);
    c->plan = plan;
    c->peers = peers_dev;
    c->rank = rank;
    c->world = world;
    c->pf_items = kChainPrefetchItems;
    if (const char* pf = getenv("G4B_CHAIN_PREFETCH")) c->pf_items = std::max(0, std::min(64, atoi(pf)));
    *chain = c;
    return G4B_OK;
}

int g4b_gemv_chain_plan(const g4b_gemv_chain_step* steps, const g4b_chain_xform* xforms, int nsteps, int x_dtype,
                        int y_dtype, g4b_chain_step_plan* out) {
    G4B_ENTRY("gemv_chain_plan");
    G4B_REQUIRE(steps && out, G4B_E_ARG, "gemv_chain_plan: NULL pointer argument");
    G4B_REQUIRE(nsteps >= 1 && nsteps <= kChainMaxSteps, G4B_E_ARG, "gemv_chain_plan: nsteps=%d (1..%d)", nsteps,
                kChainMaxSteps);
    G4B_REQUIRE((x_dtype == G4B_DT_F32 || x_dtype == G4B_DT_F16) && (y_dtype == G4B_DT_F32 || y_dtype == G4B_DT_F16),
                G4B_E_ARG, "gemv_chain_plan: bad dtype %d / %d", x_dtype, y_dtype);
    for (int j = 0; j < nsteps; j++)
        G4B_REQUIRE(steps[j].nseg >= 1 && steps[j].nseg <= kTcMaxSeg && steps[j].K > 0, G4B_E_ARG,
                    "gemv_chain_plan: step %d nseg=%d K=%d", j, steps[j].nseg, steps[j].K);
    const ChainXPlan xp = chain_plan_x(steps, xforms, nsteps, x_dtype, y_dtype);
    for (int j = 0; j < nsteps; j++) {
        out[j].x_forwarded = xp.fwd[j];
        out[j].wait_from = xp.wlo[j];
        out[j].x_early = xp.early[j];
        out[j].reserved = 0;
    }
    return G4B_OK;
}

size_t g4b_gemv_chain_workspace_bytes(const g4b_gemv_chain* chain) { return chain ? chain->ws_bytes : 0; }

int g4b_gemv_chain_run(const g4b_gemv_chain* chain, void* workspace, size_t ws_bytes, g4b_stream_t stream) {
    return g4b_gemv_chain_run_ex(chain, workspace, ws_bytes, 0u, stream);
}

int g4b_gemv_chain_run_ex(const g4b_gemv_chain* chain, void* workspace, size_t ws_bytes, unsigned flags,
                          g4b_stream_t stream) {
    G4B_ENTRY("gemv_chain_run");
    G4B_REQUIRE((flags & ~G4B_CHAIN_RUN_PDL) == 0u, G4B_E_ARG, "gemv_chain_run: unknown flags 0x%x", flags);
    G4B_REQUIRE(chain && chain->plan, G4B_E_ARG, "gemv_chain_run: NULL chain");
    G4B_REQUIRE(workspace && ws_bytes >= chain->ws_bytes, G4B_E_WORKSPACE,
                "gemv_chain_run: needs %zu bytes of workspace, got %zu", chain->ws_bytes, workspace ? ws_bytes : 0);
    G4B_REQUIRE(aligned16(workspace), G4B_E_ALIGN, "gemv_chain_run: workspace must be 16-byte aligned");
    int st = check_device(nullptr);
    if (st != G4B_OK) return st;
    int dev = -1;
    cudaGetDevice(&dev);
    G4B_REQUIRE(dev == chain->device, G4B_E_ARG, "gemv_chain_run: chain built on device %d, current device %d",
                chain->device, dev);
    ChainArgs ch{};
    ch.maps = reinterpret_cast<const CUtensorMap*>(chain->plan);
    ch.steps = reinterpret_cast<const ChainStep*>(reinterpret_cast<const uint8_t*>(chain->plan) +
                                                  chain_maps_bytes(chain->nsteps));
    uint8_t* ws = reinterpret_cast<uint8_t*>(workspace);
    ch.sync = reinterpret_cast<unsigned*>(ws);
    ch.partial = reinterpret_cast<unsigned long long*>(ws + chain->sync_bytes);
    ch.fwd = reinterpret_cast<unsigned long long*>(ws + chain->fwd_at);
    ch.peers = reinterpret_cast<unsigned long long* const*>(chain->peers);
    ch.nsteps = chain->nsteps;
    ch.stage_bytes = chain->stage_bytes;
    ch.s_bytes = chain->s_bytes;
    ch.maxtiles = chain->maxtiles;
    ch.G = chain->grid;
    ch.rank = chain->rank;
    ch.world = chain->world;
    ch.pf_items = chain->pf_items;
    cudaError_t e = chain_launch(chain, ch, (flags & G4B_CHAIN_RUN_PDL) != 0u, reinterpret_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return fail(G4B_E_CUDA, "gemv_chain_run: launch: %s", cudaGetErrorString(e));
    count_launch();
    return launch_status("gemv_chain_run");
}

void g4b_gemv_chain_destroy(g4b_gemv_chain* chain) {
    if (!chain) return;
    if (chain->plan) cudaFree(chain->plan);
    delete chain;
}

int g4b_gemv_i4_noalloc(const void* x, int x_dtype, int M, const uint32_t* wp, const void* scales, int scale_fmt,
                        float inv, void* y, int y_dtype, int N, int K, int split, g4b_stream_t stream) {
    G4B_ENTRY("gemv_i4_noalloc");
    // every argument check first: a rejected call must not have queued the counter clear below
    int st = gemv_i4_check(x, x_dtype, M, wp, scales, scale_fmt, y, y_dtype, N, K, split);
    if (st != G4B_OK) return st;
    st = check_device(nullptr);
    if (st != G4B_OK) return st;
    const size_t need = g4b_gemv_workspace_bytes(M, N, K, split);
    clear_error();
    G4B_REQUIRE(need <= kNoAllocScratchBytes, G4B_E_WORKSPACE,
                "gemv_i4_noalloc: these sizes need %zu bytes of scratch; the built-in scratch holds %zu "
                "(use g4b_gemv_i4 with a caller-provided workspace)",
                need, kNoAllocScratchBytes);
    void* ws = nullptr;
    if (need) {
        st = noalloc_scratch(&ws);
        if (st != G4B_OK) return st;
        // the arrival counters at the front of the scratch must start at zero; a previous call
        // leaves them zero, but one that gave up (kernel status) may not.  The clear is queued by
        // the kernel launch itself, after gemv_i4_impl's remaining checks have all passed.
        t_clear_ptr = ws;
        t_clear_bytes = kGemvCounterBytes;
    }
    t_pdl = false;
    st = gemv_i4_impl(x, x_dtype, M, wp, scales, scale_fmt, inv, y, y_dtype, N, K, split, ws, need, stream);
    t_clear_ptr = nullptr;  // unused if the call failed before its launch
    return st;
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
