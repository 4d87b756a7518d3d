// g4b_gemm.cu -- prefill GEMMs on the packed int4 weights (tcgen05 / TMEM / TMA).
//
// W4A16 (vk/coopgemm_i4h.comp:13-35, vk/coopgemm_i4.comp:14-36,
// vk/coopgemm_i4f.comp:12-35; dispatched by gmm(), src/vk_engine.py:391-400):
//     Y[m, n] = sum_k f16(X[m, k]) * f16((q[k, n] - 8) * f32(scale[k/32, n]))
//
// B200 design.  The product is computed transposed, D[n, m] = W^T[n, :] . X[m, :],
// so that the dequantised weights are the MMA's A operand and can live in
// tensor memory: dequant warps turn packed nibbles into f16 pairs in registers
// and write them straight to TMEM with tcgen05.st, and the tensor core reads
// them from there.  Dequantised weights never touch shared memory, which keeps
// the shared-memory port for the TMA-fed activation tiles (the B operand).
//
//   CTA tile: 128 weight columns (n, TMEM lanes = MMA M) x 256 tokens (m, MMA N),
//   K staged 64 at a time.  Persistent CTAs walk the tiles with a static stride.
//   warp 0      TMA producer: X tile [256 x 64] f16 (128-byte swizzle), packed
//               words [64 x 16] u32 and f16 scales [2 x 128] per stage.
//   warp 1      allocates TMEM; one lane issues tcgen05.mma (4 x K=16 per stage).
//   warps 2-17  dequant: warp w owns TMEM lanes 32*(w%4).., one 32-row scale
//               block of a stage, and every other stage (two warps share each
//               (lanes, block) pair, so one's loads overlap the other's math);
//               per element 2.5 ALU ops, exact f16((q-8)*s) (HSUB2 of the
//               1024+q exponent trick, then HMUL2).
//   warps 18-21 epilogue: tcgen05.ld of the f32 accumulator, convert, store.
// TMEM: accumulator columns [0, 256), A stages at [256, 256 + 32*stages) (448 of 512); the 64-token
// instance (batched decode): two accumulators [0, 128), 4 stages of 3 K blocks (96 A columns each).
// Shared-memory stage s and TMEM A stage s are recycled together: the MMA's
// commit on empty[s] frees both.
#include <algorithm>
#include <cstdlib>

#include "g4b_tcgen05.cuh"

namespace g4b {

static __device__ unsigned g_gemm_status;

unsigned read_status_gemm() {
    unsigned v = 0, z = 0;
    if (cudaMemcpyFromSymbol(&v, g_gemm_status, sizeof(v)) != cudaSuccess) return 0xffffffffu;
    if (v) cudaMemcpyToSymbol(g_gemm_status, &z, sizeof(z));
    return v;
}

// ------------------------------------------------------------------ W4A16
constexpr int kW4BN = 128;      // weight columns per tile (TMEM lanes)
constexpr int kW4BT = 256;      // tokens per tile (MMA N) for prefill
constexpr int kW4BTSmall = 64;  // tokens per tile for M <= 64 (batched decode): no MMA work on padding rows
constexpr int kW4BK = 64;       // K rows per stage
constexpr int kW4DqWarps = 16;
constexpr int kW4Threads = (2 + kW4DqWarps + 4) * 32;
constexpr int kW4WBytes = kW4BK * (kW4BN / 8) * 4;    // 4 KB
constexpr int kW4SBytes = (kW4BK / 32) * kW4BN * 2;   // 512 B
constexpr int kW4TmemCols = 512;
constexpr int kW4MaxSplit = 16;
// Per instance: stages in flight (even: dequant warps alternate stages) and accumulator buffers.  The
// 64-token instance (batched decode) is latency-bound on its small stages, so it keeps 12 in flight and
// two 64-column accumulators (the epilogue of one tile overlaps the next tile's MMAs); TMEM holds the
// accumulators, then 32 A columns per stage.
// A stage carries w4_sub(bt) consecutive 64-row K blocks: the small-M instance's stages are otherwise too
// small for their fixed hand-off (TMA landing, TMEM stores, MMA issue and commit) to hide behind.  Measured at
// M = 8 on the lm_head shape: 1 block x 6 stages 350 us, 1 x 12 327-340 us, 2 x 6 274 us, 3 x 4 246-264 us.
__host__ __device__ constexpr int w4_stages(int bt) { return bt == kW4BTSmall ? 4 : 6; }
__host__ __device__ constexpr int w4_sub(int bt) { return bt == kW4BTSmall ? 3 : 1; }
__host__ __device__ constexpr int w4_nacc(int bt) { return bt == kW4BTSmall ? 2 : 1; }
constexpr int kW4MaxStages = 6;
static_assert(w4_stages(kW4BT) % 2 == 0 && w4_stages(kW4BTSmall) % 2 == 0, "dequant warps alternate stages");
static_assert(w4_nacc(kW4BT) * kW4BT + 32 * w4_sub(kW4BT) * w4_stages(kW4BT) <= kW4TmemCols, "TMEM budget (prefill)");
static_assert(w4_nacc(kW4BTSmall) * kW4BTSmall + 32 * w4_sub(kW4BTSmall) * w4_stages(kW4BTSmall) <= kW4TmemCols,
              "TMEM budget (small M)");
__host__ __device__ constexpr int w4_xbytes(int bt) { return bt * kW4BK * 2; }  // 32 KB / 8 KB per K block
__host__ __device__ constexpr size_t w4_smem(int bt) {
    return 1024 + (size_t)w4_stages(bt) * w4_sub(bt) * (w4_xbytes(bt) + kW4WBytes + kW4SBytes);
}

// Split-K: tile t of the launch is (column tile, token tile) t / S with the K range of split t % S;
// with S > 1 each split writes its f32 partial to part[split][M][N] and a second kernel sums the
// splits in order into y.
// Fused weights (the small-M instance only): up to 3 weights that share X run as one launch, segment g
// owning column tiles [tile0[g], tile0[g + 1]) and writing ys[g] [M, Ns[g]]; N is then their total and the
// split partials are laid out over it.
constexpr int kW4MaxSeg = 3;
struct W4Segs {
    int nseg;
    int tile0[kW4MaxSeg + 1];
    void* ys[kW4MaxSeg];
    int Ns[kW4MaxSeg];
};

struct W4Args {
    void* y;
    float* part;
    int M, N, K, nkb, ntm, ntiles, S;
    W4Segs seg;
};

// the segment of global column tile nt
__device__ __forceinline__ int w4_seg_of(const W4Segs& g, int nt) {
    return nt >= g.tile0[1] ? (nt >= g.tile0[2] ? 2 : 1) : 0;
}
// segment sg's output, width and first column tile (constant indices: no local-memory copy of the params)
__device__ __forceinline__ void w4_seg_out(const W4Segs& g, int sg, void*& y, int& N, int& tile0) {
    y = sg == 0 ? g.ys[0] : (sg == 1 ? g.ys[1] : g.ys[2]);
    N = sg == 0 ? g.Ns[0] : (sg == 1 ? g.Ns[1] : g.Ns[2]);
    tile0 = sg == 0 ? g.tile0[0] : (sg == 1 ? g.tile0[1] : g.tile0[2]);
}

template <bool YF32, int BT, bool SPLIT>
__global__ void __launch_bounds__(kW4Threads, 1) gemm_w4a16_kernel(const W4Args a,
                                                                   const __grid_constant__ CUtensorMap xmap,
                                                                   const __grid_constant__ CUtensorMap wmap,
                                                                   const __grid_constant__ CUtensorMap smap,
                                                                   const __grid_constant__ CUtensorMap wmap1,
                                                                   const __grid_constant__ CUtensorMap smap1,
                                                                   const __grid_constant__ CUtensorMap wmap2,
                                                                   const __grid_constant__ CUtensorMap smap2) {
    // the weight / scale maps and local column tile of global column tile nt (segments: SPLIT instance only)
    auto seg_maps = [&](int nt, const CUtensorMap*& wm, const CUtensorMap*& smp, int& ntl) {
        wm = &wmap;
        smp = &smap;
        ntl = nt;
        if constexpr (SPLIT) {
            const int sg = w4_seg_of(a.seg, nt);
            if (sg == 1) {
                wm = &wmap1;
                smp = &smap1;
            } else if (sg == 2) {
                wm = &wmap2;
                smp = &smap2;
            }
            ntl = nt - (sg == 0 ? a.seg.tile0[0] : (sg == 1 ? a.seg.tile0[1] : a.seg.tile0[2]));
        }
    };
    constexpr int kW4XBytes = w4_xbytes(BT);
    constexpr int kW4Stages = w4_stages(BT), kNAcc = w4_nacc(BT), kSub = w4_sub(BT);
    // dequant warps per stage: each of 8 warps takes one (lane quarter, 32-row scale block) of every
    // other stage (giving the small-M instance's 4 warps a quarter's 64 rows of every fourth stage
    // measured no faster)
    constexpr int kPar = 2, kDqPerStage = kW4DqWarps / kPar;
    static_assert(kW4Stages % kPar == 0, "stages a multiple of the dequant rotation");
    constexpr int kW4ACol = kNAcc * BT;   // first A column (after the accumulators)
    constexpr int kACols = kSub * (kW4BK / 2);   // A columns per stage
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    __shared__ uint64_t bars[3 * kW4MaxStages + 2 * 2 + 1];
    __shared__ uint32_t s_tmem;
    __shared__ int s_abort;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    volatile int* abort_flag = &s_abort;
    const uint32_t raw0 = smem_u32(smem_raw);
    const uint32_t sm0 = (raw0 + 1023u) & ~1023u;          // X stages (1024-aligned for the swizzle)
    // stage s, K block j of the stage: X at sm0 + (s kSub + j) kW4XBytes, words and scales likewise
    const uint32_t smw = sm0 + kW4Stages * kSub * kW4XBytes;   // packed words
    const uint32_t sms = smw + kW4Stages * kSub * kW4WBytes;   // scales
    const uint8_t* gsm = smem_raw + (sm0 - raw0);
    const uint32_t* wsm = reinterpret_cast<const uint32_t*>(gsm + kW4Stages * kSub * kW4XBytes);
    const uint16_t* ssm = reinterpret_cast<const uint16_t*>(gsm + kW4Stages * kSub * (kW4XBytes + kW4WBytes));
    const uint32_t bar0 = smem_u32(bars);
    auto full_bar = [&](int s) { return bar0 + 8u * s; };
    auto empty_bar = [&](int s) { return bar0 + 8u * (kW4Stages + s); };
    auto afull_bar = [&](int s) { return bar0 + 8u * (2 * kW4Stages + s); };
    // accumulator buffer b: dfull(b) (MMA commit -> epilogue), dempty(b) (epilogue -> MMA)
    auto dfull_bar = [&](int b) { return bar0 + 8u * (3 * kW4Stages + 2 * b); };
    auto dempty_bar = [&](int b) { return bar0 + 8u * (3 * kW4Stages + 2 * b + 1); };
    const uint32_t drain_bar = bar0 + 8u * (3 * kW4Stages + 2 * kNAcc);

    if (tid == 0) {
        for (int s = 0; s < kW4Stages; s++) {
            mbar_init(full_bar(s), 1);
            mbar_init(empty_bar(s), kDqPerStage + 1);  // the stage's dequant warps + the MMA commit
            mbar_init(afull_bar(s), kDqPerStage);
        }
        for (int b = 0; b < kNAcc; b++) {
            mbar_init(dfull_bar(b), 1);
            mbar_init(dempty_bar(b), 4);
        }
        mbar_init(drain_bar, 1);
        s_abort = 0;
        fence_mbar_init();
    }
    if (warp == 1) {
        tc::tmem_alloc(smem_u32(&s_tmem), kW4TmemCols);
        tc::tmem_relinquish();
    }
    tc::fence_before();
    __syncthreads();
    tc::fence_after();
    const uint32_t tmem = s_tmem;
    pdl_launch_dependents();   // a programmatic dependent may be scheduled now; it waits for this grid
    const int nks = a.nkb;  // K stages per tile
    // K splits: only the SPLIT instance (small M) reads a.S; the prefill instance keeps every tile whole
    const int S = SPLIT ? a.S : 1;

    if (warp == 0) {
        // ------------------------------------------------------- TMA producer
        if (lane == 0) {
            prefetch_tensor_map(&xmap);
            prefetch_tensor_map(&wmap);
            prefetch_tensor_map(&smap);
            const uint64_t pol_w = l2_evict_first_policy();
            uint64_t pol_x;
            asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(pol_x));
            // launched as a programmatic dependent (G4B_GEMM_PDL): warm L2 with the first tile's first weight
            // blocks while the kernel before finishes, then wait for it before the first X load
            if (blockIdx.x < a.ntiles) {
                const int t = blockIdx.x, tb = SPLIT ? t / S : t, ks = SPLIT ? t % S : 0;
                const int kb0 = SPLIT ? ks * nks / S : 0, kb1 = SPLIT ? (ks + 1) * nks / S : nks;
                const CUtensorMap *wm, *smp;
                int ntl;
                seg_maps(tb / a.ntm, wm, smp, ntl);
                for (int kb = kb0; kb < std::min(kb1, kb0 + kW4Stages * kSub); kb++) {
                    tma_prefetch_l2_2d(wm, ntl * (kW4BN / 8), kb * kW4BK);
                    tma_prefetch_l2_2d(smp, ntl * kW4BN, kb * (kW4BK / 32));
                }
            }
            pdl_wait();
            int it = 0;
            bool ok = true;
            for (int t = blockIdx.x; ok && t < a.ntiles; t += gridDim.x) {
                const int tb = SPLIT ? t / S : t, ks = SPLIT ? t % S : 0;
                const int nt = tb / a.ntm, mt = tb % a.ntm;
                const int kb0 = SPLIT ? ks * nks / S : 0, kb1 = SPLIT ? (ks + 1) * nks / S : nks;
                const CUtensorMap *wm, *smp;
                int ntl;
                seg_maps(nt, wm, smp, ntl);
                for (int kb = kb0; kb < kb1; kb += kSub, it++) {
                    const int s = it % kW4Stages, sub = min(kSub, kb1 - kb);
                    if (it >= kW4Stages &&
                        !mbar_wait(empty_bar(s), ((it / kW4Stages) & 1) ^ 1, abort_flag, &g_gemm_status)) {
                        ok = false;
                        break;
                    }
                    mbar_arrive_expect_tx(full_bar(s), (uint32_t)sub * (kW4XBytes + kW4WBytes + kW4SBytes));
                    for (int j = 0; j < sub; j++) {
                        const int sj = s * kSub + j;
                        tma_load_2d(sm0 + sj * kW4XBytes, &xmap, (kb + j) * kW4BK, mt * BT, full_bar(s), pol_x);
                        tma_load_2d(smw + sj * kW4WBytes, wm, ntl * (kW4BN / 8), (kb + j) * kW4BK, full_bar(s),
                                    pol_w);
                        tma_load_2d(sms + sj * kW4SBytes, smp, ntl * kW4BN, (kb + j) * (kW4BK / 32), full_bar(s),
                                    pol_w);
                    }
                }
            }
            // drain: the copies already issued must land before the CTA exits
            for (int i = std::max(0, it - kW4Stages); i < it; i++)
                mbar_wait_drain(full_bar(i % kW4Stages), (i / kW4Stages) & 1, &g_gemm_status);
        }
    } else if (warp == 1) {
        // ------------------------------------------------------- MMA issuer
        if (lane == 0) {
            constexpr uint32_t idesc = tc::idesc(1, 0, 0, 0, 0, BT, kW4BN);
            int it = 0, tc_i = 0;
            bool ok = true;
            for (int t = blockIdx.x; ok && t < a.ntiles; t += gridDim.x, tc_i++) {
                const int ab = tc_i % kNAcc;
                if (!mbar_wait(dempty_bar(ab), ((tc_i / kNAcc) & 1) ^ 1, abort_flag, &g_gemm_status)) break;
                tc::fence_after();
                const int ks = SPLIT ? t % S : 0;
                const int kb0 = SPLIT ? ks * nks / S : 0, kb1 = SPLIT ? (ks + 1) * nks / S : nks;
                for (int kb = kb0; kb < kb1; kb += kSub, it++) {
                    const int s = it % kW4Stages, sub = min(kSub, kb1 - kb);
                    const uint32_t ph = (it / kW4Stages) & 1;
                    if (!mbar_wait(full_bar(s), ph, abort_flag, &g_gemm_status) ||
                        !mbar_wait(afull_bar(s), ph, abort_flag, &g_gemm_status)) {
                        ok = false;
                        break;
                    }
                    tc::fence_after();
                    for (int j = 0; j < sub; j++) {
                        const uint64_t bdesc = tc::sdesc_sw128(sm0 + (s * kSub + j) * kW4XBytes, 16, 1024);
#pragma unroll
                        for (int kk = 0; kk < kW4BK / 16; kk++)
                            tc::mma_f16_ts(tmem + ab * BT, tmem + kW4ACol + s * kACols + j * (kW4BK / 2) + kk * 8,
                                           bdesc + (uint64_t)(kk * 2), idesc,
                                           (kb + j != kb0 || kk != 0) ? 1u : 0u);
                    }
                    tc::commit(empty_bar(s));
                }
                if (ok) tc::commit(dfull_bar(ab));
            }
            // drain: every MMA issued must be complete before TMEM is released
            tc::commit(drain_bar);
            mbar_wait_drain(drain_bar, 0, &g_gemm_status);
        }
    } else if (warp < 2 + kW4DqWarps) {
        // ------------------------------------------------------- dequant
        const int q = warp & 3;             // TMEM lane quarter this warp may access
        // the 32-row scale blocks of a stage this warp dequantises, and which stages: it % kPar == par
        const int kh0 = kPar == 2 ? ((warp - 2) >> 2) & 1 : 0, nkh = kPar == 2 ? 1 : 2;
        const int par = kPar == 2 ? (warp - 2) >> 3 : (warp - 2) >> 2;
        const int nl = q * 32 + lane;       // weight column within the tile
        const int g = nl >> 3, j = nl & 7;
        const uint32_t sel = (uint32_t)(j >> 1) | ((uint32_t)(4 + (j >> 1)) << 8);
        const uint32_t sh = (uint32_t)(j & 1) * 4u;
        const uint32_t lane_addr = (uint32_t)(q * 32) << 16;
        int it = 0;
        bool ok = true;
        for (int t = blockIdx.x; ok && t < a.ntiles; t += gridDim.x) {
            const int ks = SPLIT ? t % S : 0;
            const int kb0 = SPLIT ? ks * nks / S : 0, kb1 = SPLIT ? (ks + 1) * nks / S : nks;
            for (int kb = kb0; kb < kb1; kb += kSub, it++) {
                if ((it % kPar) != par) continue;
                const int s = it % kW4Stages, sub = min(kSub, kb1 - kb);
                if (!mbar_wait(full_bar(s), (it / kW4Stages) & 1, abort_flag, &g_gemm_status)) {
                    ok = false;
                    break;
                }
                tc::fence_after();
                for (int jk = 0; jk < sub * nkh; jk++) {
                    const int j = jk / nkh, kh = kh0 + jk % nkh, sj = s * kSub + j;
                    const uint32_t* wr = wsm + sj * (kW4WBytes / 4) + kh * 32 * (kW4BN / 8) + g;
                    const uint32_t sc = ssm[sj * (kW4SBytes / 2) + kh * kW4BN + nl];
                    const uint32_t s2 = sc | (sc << 16);
                    uint32_t v[16];
#pragma unroll
                    for (int p = 0; p < 16; p++) {
                        const uint32_t w0 = wr[(2 * p) * (kW4BN / 8)], w1 = wr[(2 * p + 1) * (kW4BN / 8)];
                        uint32_t u = prmt(w0, w1, sel) >> sh;
                        u = and_or(u, 0x000F000Fu, 0x64006400u);  // f16 pair (1024 + q_k, 1024 + q_k+1)
                        u = hsub2_u(u, 0x64086408u);               // exact (q - 8)
                        v[p] = hmul2_u(u, s2);                     // f16((q - 8) * s), one rounding
                    }
                    tc::st_32x32b_x16(tmem + lane_addr + kW4ACol + s * kACols + j * (kW4BK / 2) + kh * 16, v);
                }
                tc::wait_st();
                tc::fence_before();
                __syncwarp();
                if (lane == 0) {
                    mbar_arrive(afull_bar(s));
                    mbar_arrive(empty_bar(s));
                }
            }
        }
    } else {
        // ------------------------------------------------------- epilogue
        const int q = warp & 3;
        const int nl = q * 32 + lane;
        const uint32_t lane_addr = (uint32_t)(q * 32) << 16;
        int tc_i = 0;
        for (int t = blockIdx.x; t < a.ntiles; t += gridDim.x, tc_i++) {
            const int ab = tc_i % kNAcc;
            if (!mbar_wait(dfull_bar(ab), (tc_i / kNAcc) & 1, abort_flag, &g_gemm_status)) break;
            tc::fence_after();
            const int tb = SPLIT ? t / S : t, ks = SPLIT ? t % S : 0;
            const int nt = tb / a.ntm, mt = tb % a.ntm;
            const int n = nt * kW4BN + nl;   // over all segments: the partials' column
            const int m0 = mt * BT;
            float* const part = SPLIT && S > 1 ? a.part + (size_t)ks * a.M * a.N : nullptr;
            // y of this tile's segment
            void* yseg = a.y;
            int nseg_col = n, Nseg = a.N;
            if constexpr (SPLIT) {
                int t0;
                w4_seg_out(a.seg, w4_seg_of(a.seg, nt), yseg, Nseg, t0);
                nseg_col = n - t0 * kW4BN;
            }
#pragma unroll 1
            for (int c = 0; c < BT / 32; c++) {
                uint32_t r[32];
                tc::ld_32x32b_x32(tmem + lane_addr + ab * BT + c * 32, r);
                tc::wait_ld();
                const int mb = m0 + c * 32;
                // the f32 partials of a K split, or y; the row index is checked per element (M may end mid-tile)
                if (SPLIT && part) {
                    float* pp = part + (size_t)mb * a.N + n;  // one running address: no extra registers
#pragma unroll
                    for (int i = 0; i < 32; i++, pp += a.N)
                        if (mb + i < a.M) *pp = __uint_as_float(r[i]);
                } else {
#pragma unroll
                    for (int i = 0; i < 32; i++) {
                        const int m = mb + i;
                        if (m < a.M) {
                            const float f = __uint_as_float(r[i]);
                            if (YF32)
                                reinterpret_cast<float*>(yseg)[(size_t)m * Nseg + nseg_col] = f;
                            else
                                reinterpret_cast<__half*>(yseg)[(size_t)m * Nseg + nseg_col] = __float2half_rn(f);
                        }
                    }
                }
            }
            tc::fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(dempty_bar(ab));
        }
    }

    __syncwarp();
    tc::fence_before();
    __syncthreads();
    tc::fence_after();
    if (warp == 1) tc::tmem_dealloc(tmem, kW4TmemCols);
}

// ------------------------------------------------------------ W8A8 / W4A8
// vk/coopgemm_w8a8.comp:18-37 and vk/coopgemm_w4a8.comp:21-50:
//     C[m, n] = sum_k A8[m, k] * W8[k, n]            (exact int32)
//     Y[m, n] = f16((float(C) * sa[m]) * f32(sw[n]))
// with W8 either the prepared int8 weights [K, N] (W8A8) or, for W4A8, the
// packed int4 words requantised in the kernel against a per-column scale:
//     W8[k, n] = clamp(round_half_even((q - 8) * f32(ratio[k/32, n])), -127, 127)
//
// Same transposed product as W4A16: D[n, m] in tensor memory, weight columns
// on the 128 lanes, 256 tokens per tile.  tcgen05.mma kind::i8.
//   W8A8: both operands come from shared memory.  The weight tile is TMA'd
//         straight from the reference's [K, N] row-major int8 array, which is
//         an MN-major operand (128-byte swizzle, one 128-column group per
//         tile), so no repacking of the weights is needed.  Two accumulator
//         buffers (2 x 256 TMEM columns) let the epilogue of one tile overlap
//         the MMAs of the next.
//   W4A8: 16 requant warps write the int8 weights to tensor memory as the
//         MMA's A operand (four K values per 32-bit column), like the W4A16
//         dequant.  Exact round-half-even without any conversion
//         instruction: fma.rn.f16x2((q - 8), r, 1536) rounds the exact
//         product once at a spacing of 1.0, and the low byte of the f16
//         result is the int8 two's-complement value.
constexpr int kS8BN = 128;                              // weight columns per tile
constexpr int kS8BT = 256;                              // tokens per tile
constexpr int kS8BK = 128;                              // K per stage (one 128-byte swizzle row)
constexpr int kS8Stages = 4;
constexpr int kS8ABytes = kS8BT * kS8BK;                // activations [256 x 128] s8: 32 KB
constexpr int kS8W8Bytes = kS8BK * kS8BN;               // W8 [128 K x 128 n] s8: 16 KB
constexpr int kS8WpBytes = kS8BK * (kS8BN / 8) * 4;     // packed words [128 K x 16]: 8 KB
constexpr int kS8RBytes = (kS8BK / 32) * kS8BN * 2;     // ratio [4 x 128] f16: 1 KB
constexpr int kS8DqWarps = 16;

template <bool W4>
struct S8Cfg {
    static constexpr int kDq = W4 ? kS8DqWarps : 0;
    static constexpr int kThreads = (2 + kDq + 4) * 32;
    static constexpr int kWBytes = W4 ? kS8WpBytes + kS8RBytes : kS8W8Bytes;
    static constexpr int kStageBytes = kS8ABytes + kWBytes;
    static constexpr int kAccBufs = W4 ? 1 : 2;
    static constexpr int kACol = 256;                   // W4A8: first tensor-memory A column
    static constexpr size_t kSmem = 1024 + (size_t)kS8Stages * kStageBytes;
};
static_assert(256 + 32 * kS8Stages <= 512, "TMEM budget");

// Tile t is (token tile t / ntn, column tile t % ntn): the CTAs resident at once share a few
// activation panels and sweep every column tile, so the whole int8 weight (59 MB at config 4)
// stays in L2 across waves and each activation panel is read from DRAM about once.
//
// Work units: the first nfull units are whole tiles; when the tiles leave a last wave that fills at most a
// quarter of the CTAs (W8A8), each tile of that wave runs as four units of 64 tokens instead (unit
// nfull + 4 i + sub: token rows sub * 64 .. +64 of tile nfull + i), so the last wave ends in about a
// quarter of a tile's time instead of a whole one.  Every unit still owns its outputs: no partial sums.
constexpr int kS8Sub = 4;
constexpr int kS8SubT = kS8BT / kS8Sub;                 // tokens per quarter unit
struct S8Args {
    void* y;
    int32_t* c;           // nullable raw accumulators
    const float* sa;      // [M]
    const uint16_t* sw;   // [N] f16
    int M, N, K, nkb, ntm, ntiles, nfull, nunits;
};

// unit u -> token tile, column tile and quarter (-1: the whole tile)
__device__ __forceinline__ void s8_unit(const S8Args& a, int u, int& mt, int& nt, int& sub) {
    int t = u;
    sub = -1;
    if (u >= a.nfull) {
        t = a.nfull + (u - a.nfull) / kS8Sub;
        sub = (u - a.nfull) % kS8Sub;
    }
    const int ntn = a.ntiles / a.ntm;
    mt = t / ntn;
    nt = t % ntn;
}

template <bool W4, bool YF32>
__global__ void __launch_bounds__(S8Cfg<W4>::kThreads, 1)
    gemm_s8_kernel(const S8Args a, const __grid_constant__ CUtensorMap amap, const __grid_constant__ CUtensorMap wmap,
                   const __grid_constant__ CUtensorMap rmap, const __grid_constant__ CUtensorMap amap_q) {
    using Cfg = S8Cfg<W4>;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    __shared__ uint64_t bars[3 * kS8Stages + 5];
    __shared__ uint32_t s_tmem;
    __shared__ int s_abort;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    volatile int* abort_flag = &s_abort;
    const uint32_t raw0 = smem_u32(smem_raw);
    const uint32_t sm0 = (raw0 + 1023u) & ~1023u;            // activation stages (1024-aligned)
    const uint32_t smw = sm0 + kS8Stages * kS8ABytes;         // weight stages (W8, or words + ratio)
    const uint8_t* gsm = smem_raw + (sm0 - raw0);
    const uint8_t* wsm_b = gsm + kS8Stages * kS8ABytes;
    const uint32_t bar0 = smem_u32(bars);
    auto full_bar = [&](int s) { return bar0 + 8u * s; };
    auto empty_bar = [&](int s) { return bar0 + 8u * (kS8Stages + s); };
    auto afull_bar = [&](int s) { return bar0 + 8u * (2 * kS8Stages + s); };
    auto dfull_bar = [&](int b) { return bar0 + 8u * (3 * kS8Stages + b); };
    auto dempty_bar = [&](int b) { return bar0 + 8u * (3 * kS8Stages + 2 + b); };
    const uint32_t drain_bar = bar0 + 8u * (3 * kS8Stages + 4);

    if (tid == 0) {
        for (int s = 0; s < kS8Stages; s++) {
            mbar_init(full_bar(s), 1);
            mbar_init(empty_bar(s), Cfg::kDq + 1);  // requant warps + the MMA commit
            mbar_init(afull_bar(s), Cfg::kDq > 0 ? Cfg::kDq : 1);
        }
        for (int b = 0; b < 2; b++) {
            mbar_init(dfull_bar(b), 1);
            mbar_init(dempty_bar(b), 4);
        }
        mbar_init(drain_bar, 1);
        s_abort = 0;
        fence_mbar_init();
    }
    if (warp == 1) {
        tc::tmem_alloc(smem_u32(&s_tmem), 512);
        tc::tmem_relinquish();
    }
    tc::fence_before();
    __syncthreads();
    tc::fence_after();
    const uint32_t tmem = s_tmem;
    const int nks = a.nkb;

    if (warp == 0) {
        // ------------------------------------------------------- TMA producer
        if (lane == 0) {
            prefetch_tensor_map(&amap);
            prefetch_tensor_map(&wmap);
            if (W4) prefetch_tensor_map(&rmap);
            if (a.nunits > a.nfull) prefetch_tensor_map(&amap_q);
            // the weights are swept again by every wave of tiles: keep them in L2; an activation panel
            // is read by the CTAs of one wave only (token-tile-major order), so it may go first
            uint64_t pol_keep;
            asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(pol_keep));
            const uint64_t pol_once = l2_evict_first_policy();
            int it = 0;
            bool ok = true;
            for (int u = blockIdx.x; ok && u < a.nunits; u += gridDim.x) {
                int mt, nt, sub;
                s8_unit(a, u, mt, nt, sub);  // token-tile major: see S8Args
                for (int kb = 0; kb < nks; kb++, it++) {
                    const int s = it % kS8Stages;
                    if (it >= kS8Stages &&
                        !mbar_wait(empty_bar(s), ((it / kS8Stages) & 1) ^ 1, abort_flag, &g_gemm_status)) {
                        ok = false;
                        break;
                    }
                    if (sub < 0) {
                        mbar_arrive_expect_tx(full_bar(s), Cfg::kStageBytes);
                        tma_load_2d(sm0 + s * kS8ABytes, &amap, kb * kS8BK, mt * kS8BT, full_bar(s), pol_once);
                    } else {
                        mbar_arrive_expect_tx(full_bar(s), Cfg::kStageBytes - kS8ABytes + kS8ABytes / kS8Sub);
                        tma_load_2d(sm0 + s * kS8ABytes, &amap_q, kb * kS8BK, mt * kS8BT + sub * kS8SubT, full_bar(s),
                                    pol_once);
                    }
                    if (W4) {
                        const uint32_t dst = smw + s * Cfg::kWBytes;
                        tma_load_2d(dst, &wmap, nt * (kS8BN / 8), kb * kS8BK, full_bar(s), pol_keep);
                        tma_load_2d(dst + kS8WpBytes, &rmap, nt * kS8BN, kb * (kS8BK / 32), full_bar(s), pol_keep);
                    } else {
                        tma_load_2d(smw + s * Cfg::kWBytes, &wmap, nt * kS8BN, kb * kS8BK, full_bar(s), pol_keep);
                    }
                }
            }
            for (int i = std::max(0, it - kS8Stages); i < it; i++)
                mbar_wait_drain(full_bar(i % kS8Stages), (i / kS8Stages) & 1, &g_gemm_status);
        }
    } else if (warp == 1) {
        // ------------------------------------------------------- MMA issuer
        if (lane == 0) {
            // D s32, A/B s8; A MN-major from shared memory (W8A8) or K-major from TMEM (W4A8)
            constexpr uint32_t idesc_full = tc::idesc(2, 1, 1, W4 ? 0 : 1, 0, kS8BT, kS8BN);
            constexpr uint32_t idesc_q = tc::idesc(2, 1, 1, W4 ? 0 : 1, 0, kS8SubT, kS8BN);
            int it = 0, tc_i = 0;
            bool ok = true;
            for (int u = blockIdx.x; ok && u < a.nunits; u += gridDim.x, tc_i++) {
                const uint32_t idesc = u < a.nfull ? idesc_full : idesc_q;
                const int buf = tc_i % Cfg::kAccBufs;
                const uint32_t use = (uint32_t)(tc_i / Cfg::kAccBufs);
                if (!mbar_wait(dempty_bar(buf), (use & 1) ^ 1, abort_flag, &g_gemm_status)) break;
                tc::fence_after();
                const uint32_t dt = tmem + (uint32_t)(buf * kS8BT);
                for (int kb = 0; kb < nks; kb++, it++) {
                    const int s = it % kS8Stages;
                    const uint32_t ph = (it / kS8Stages) & 1;
                    if (!mbar_wait(full_bar(s), ph, abort_flag, &g_gemm_status) ||
                        (W4 && !mbar_wait(afull_bar(s), ph, abort_flag, &g_gemm_status))) {
                        ok = false;
                        break;
                    }
                    tc::fence_after();
                    const uint64_t bdesc = tc::sdesc_sw128(sm0 + s * kS8ABytes, 16, 1024);
#pragma unroll
                    for (int kk = 0; kk < kS8BK / 32; kk++) {
                        if (W4) {
                            tc::mma_i8_ts(dt, tmem + Cfg::kACol + s * (kS8BK / 4) + kk * 8, bdesc + (uint64_t)(kk * 2),
                                          idesc, (kb | kk) != 0);
                        } else {
                            // MN-major A: 32 K rows of 128 bytes per MMA step
                            const uint64_t adesc =
                                tc::sdesc_sw128(smw + s * Cfg::kWBytes + kk * 32 * 128, kS8W8Bytes, 1024);
                            tc::mma_i8_ss(dt, adesc, bdesc + (uint64_t)(kk * 2), idesc, (kb | kk) != 0);
                        }
                    }
                    tc::commit(empty_bar(s));
                }
                if (ok) tc::commit(dfull_bar(buf));
            }
            tc::commit(drain_bar);
            mbar_wait_drain(drain_bar, 0, &g_gemm_status);
        }
    } else if (W4 && warp < 2 + Cfg::kDq) {
        // ------------------------------------------------------- W4A8 requant
        const int q = warp & 3;                 // TMEM lane quarter this warp may access
        const int kq = (warp - 2) >> 2;         // which 32-row block of the stage
        const int nl = q * 32 + lane;
        const int g = nl >> 3, j = nl & 7;
        const uint32_t sel = (uint32_t)(j >> 1) | ((uint32_t)(4 + (j >> 1)) << 8);
        const uint32_t sh = (uint32_t)(j & 1) * 4u;
        const uint32_t lane_addr = (uint32_t)(q * 32) << 16;
        int it = 0;
        bool ok = true;
        for (int u = blockIdx.x; ok && u < a.nunits; u += gridDim.x) {
            for (int kb = 0; kb < nks; kb++, it++) {
                const int s = it % kS8Stages;
                if (!mbar_wait(full_bar(s), (it / kS8Stages) & 1, abort_flag, &g_gemm_status)) {
                    ok = false;
                    break;
                }
                const uint32_t* wr =
                    reinterpret_cast<const uint32_t*>(wsm_b + s * Cfg::kWBytes) + kq * 32 * (kS8BN / 8) + g;
                const uint32_t r = reinterpret_cast<const uint16_t*>(wsm_b + s * Cfg::kWBytes + kS8WpBytes)[kq * kS8BN + nl];
                const uint32_t r2 = r | (r << 16);
                // |(q - 8) * r| < 127.5 whenever |r| < 15.9375: no clamp needed
                const bool big = (r & 0x7fffu) >= 0x4bf8u;
                uint32_t v[8];
                if (!__any_sync(0xffffffffu, big)) {
#pragma unroll
                    for (int p = 0; p < 8; p++) {
                        uint32_t t2[2];
#pragma unroll
                        for (int h = 0; h < 2; h++) {
                            const int k = 4 * p + 2 * h;
                            uint32_t u = prmt(wr[k * (kS8BN / 8)], wr[(k + 1) * (kS8BN / 8)], sel) >> sh;
                            u = and_or(u, 0x000F000Fu, 0x64006400u);      // f16 (1024 + q) pair
                            u = hsub2_u(u, 0x64086408u);                   // exact q - 8
                            t2[h] = hfma2_u(u, r2, 0x66006600u);           // 1536 + rne((q - 8) * r)
                        }
                        v[p] = prmt(t2[0], t2[1], 0x6420u);                // low bytes: the int8 values
                    }
                } else {
#pragma unroll
                    for (int p = 0; p < 8; p++) {
                        uint32_t t2[2];
#pragma unroll
                        for (int h = 0; h < 2; h++) {
                            const int k = 4 * p + 2 * h;
                            uint32_t u = prmt(wr[k * (kS8BN / 8)], wr[(k + 1) * (kS8BN / 8)], sel) >> sh;
                            u = and_or(u, 0x000F000Fu, 0x64006400u);
                            u = hsub2_u(u, 0x64086408u);
                            u = hfma2_u(u, r2, 0x66006600u);
                            t2[h] = hmin2_u(hmax2_u(u, 0x65816581u), 0x667F667Fu);  // clamp to 1536 -+ 127
                        }
                        v[p] = prmt(t2[0], t2[1], 0x6420u);
                    }
                }
                tc::st_32x32b_x8(tmem + lane_addr + Cfg::kACol + s * (kS8BK / 4) + kq * 8, v);
                tc::wait_st();
                tc::fence_before();
                __syncwarp();
                if (lane == 0) {
                    mbar_arrive(afull_bar(s));
                    mbar_arrive(empty_bar(s));
                }
            }
        }
    } else if (warp >= 2 + Cfg::kDq) {
        // ------------------------------------------------------- epilogue
        const int q = warp & 3;
        const int nl = q * 32 + lane;
        const uint32_t lane_addr = (uint32_t)(q * 32) << 16;
        int tc_i = 0;
        for (int u = blockIdx.x; u < a.nunits; u += gridDim.x, tc_i++) {
            const int buf = tc_i % Cfg::kAccBufs;
            const uint32_t use = (uint32_t)(tc_i / Cfg::kAccBufs);
            if (!mbar_wait(dfull_bar(buf), use & 1, abort_flag, &g_gemm_status)) break;
            tc::fence_after();
            int mt, nt, sub;
            s8_unit(a, u, mt, nt, sub);  // token-tile major: see S8Args
            const int n = nt * kS8BN + nl;
            const bool nok = n < a.N;
            const float swf = nok ? __half2float(__ushort_as_half(a.sw[n])) : 0.0f;
            const int m0 = mt * kS8BT + (sub < 0 ? 0 : sub * kS8SubT);
            const int nchunk = (sub < 0 ? kS8BT : kS8SubT) / 32;
#pragma unroll 1
            for (int c = 0; c < nchunk; c++) {
                const int mb = m0 + c * 32;
                if (mb >= a.M) break;
                uint32_t r[32];
                tc::ld_32x32b_x32(tmem + lane_addr + (uint32_t)(buf * kS8BT + c * 32), r);
                tc::wait_ld();
                const float sav = mb + lane < a.M ? a.sa[mb + lane] : 0.0f;
#pragma unroll
                for (int i = 0; i < 32; i++) {
                    const float sam = __shfl_sync(0xffffffffu, sav, i);
                    const int m = mb + i;
                    if (m < a.M && nok) {
                        const int32_t cv = (int32_t)r[i];
                        if (a.c) a.c[(size_t)m * a.N + n] = cv;
                        const float f = __fmul_rn(__fmul_rn((float)cv, sam), swf);
                        if (YF32)
                            reinterpret_cast<float*>(a.y)[(size_t)m * a.N + n] = f;
                        else
                            reinterpret_cast<__half*>(a.y)[(size_t)m * a.N + n] = __float2half_rn(f);
                    }
                }
            }
            tc::fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(dempty_bar(buf));
        }
    }

    __syncwarp();
    tc::fence_before();
    __syncthreads();
    tc::fence_after();
    if (warp == 1) tc::tmem_dealloc(tmem, 512);
}

// y[i] = sum over the splits s = 0 .. S-1 of part[s][i], in split order (deterministic)
template <bool YF32>
__global__ void w4a16_splitk_reduce(const float* __restrict__ part, const W4Segs g, size_t n4, size_t stride,
                                    int S, int N) {
    pdl_launch_dependents();
    pdl_wait();   // launched as a programmatic dependent of its GEMM: the partials are complete after this
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n4; i += (size_t)gridDim.x * blockDim.x) {
        // element 4i of the [M, N] partials: row m, column ncol, in the segment holding it (segments start on
        // 128-column tiles, so a group of 4 never straddles two)
        const size_t m = 4 * i / N;
        const int ncol = (int)(4 * i - m * N);
        void* y;
        int Ns, t0;
        w4_seg_out(g, w4_seg_of(g, ncol / kW4BN), y, Ns, t0);
        const size_t yo = (m * Ns + (ncol - t0 * kW4BN)) / 4;
        float4 v = __ldg(reinterpret_cast<const float4*>(part) + i);
        for (int s = 1; s < S; s++) {
            const float4 u = __ldg(reinterpret_cast<const float4*>(part + (size_t)s * stride) + i);
            v.x += u.x;
            v.y += u.y;
            v.z += u.z;
            v.w += u.w;
        }
        if (YF32) {
            reinterpret_cast<float4*>(y)[yo] = v;
        } else {
            uint2 h;
            h.x = pack_half2(__float2half_rn(v.x), __float2half_rn(v.y));
            h.y = pack_half2(__float2half_rn(v.z), __float2half_rn(v.w));
            reinterpret_cast<uint2*>(y)[yo] = h;
        }
    }
}

// How a W4A16 GEMM is tiled: the token-tile width and the number of K splits.  Small-M GEMMs
// (batched decode) use 64-token tiles, and when their column tiles cannot fill the SMs they split
// K so that about one tile per SM runs, keeping at least 4 K stages (256 rows) per split.
struct W4Plan {
    int bt, ntm, base, S;
    size_t xconv_bytes, part_bytes;
};

static W4Plan w4a16_plan(int M, int N, int K, int x_dtype, int sms) {
    W4Plan p{};
    p.bt = M <= kW4BTSmall ? kW4BTSmall : kW4BT;
    p.ntm = (M + p.bt - 1) / p.bt;
    p.base = (N / kW4BN) * p.ntm;
    const int nkb = K / kW4BK;
    p.S = 1;
    if (p.bt == kW4BTSmall && p.base * 2 <= sms && nkb >= 8)
        p.S = std::max(1, std::min({sms / std::max(p.base, 1), nkb / 4, kW4MaxSplit}));
    p.xconv_bytes = x_dtype == G4B_DT_F32 ? (((size_t)M * K * 2 + 255) & ~(size_t)255) : 0;
    p.part_bytes = p.S > 1 ? (size_t)p.S * M * N * sizeof(float) : 0;
    return p;
}

static size_t w4a16_ws(const W4Plan& p) { return p.xconv_bytes + p.part_bytes; }

}  // namespace g4b

using namespace g4b;

extern "C" {

size_t g4b_gemm_i4_workspace_bytes(int M, int N, int K, int x_dtype) {
    if (M <= 0 || K <= 0 || N <= 0 || N % kW4BN || K % kW4BK) return 0;
    int sms = 148;
    if (check_device(&sms) != G4B_OK) sms = 148;
    clear_error();
    return w4a16_ws(w4a16_plan(M, N, K, x_dtype, sms));
}

int g4b_gemm_i4(const void* X, int x_dtype, const uint32_t* wp, const uint16_t* scales_f16, void* Y, int y_dtype,
                int M, int N, int K, void* workspace, size_t ws_bytes, g4b_stream_t stream) {
    return g4b_gemm_i4_ex(X, x_dtype, wp, scales_f16, Y, y_dtype, M, N, K, workspace, ws_bytes, 0u, stream);
}

}  // extern "C"

// g4b_gemm_i4_ex (one weight) and g4b_gemm_i4_fused (2-3 weights sharing X, M <= 64): every check, then the
// launches
static int gemm_i4_impl(const char* op, const void* X, int x_dtype, int M, int K, int nseg, const g4b_gemm_seg* segs,
                        int y_dtype, void* workspace, size_t ws_bytes, unsigned flags, g4b_stream_t stream) {
    G4B_REQUIRE((flags & ~G4B_GEMM_PDL) == 0u, G4B_E_ARG, "%s: unknown flags 0x%x", op, flags);
    G4B_REQUIRE(X && segs, G4B_E_ARG, "%s: NULL pointer", op);
    G4B_REQUIRE(x_dtype == G4B_DT_F32 || x_dtype == G4B_DT_F16, G4B_E_ARG, "%s: bad x_dtype %d", op, x_dtype);
    G4B_REQUIRE(y_dtype == G4B_DT_F32 || y_dtype == G4B_DT_F16, G4B_E_ARG, "%s: bad y_dtype %d", op, y_dtype);
    G4B_REQUIRE(nseg >= 1 && nseg <= kW4MaxSeg, G4B_E_ARG, "%s: 1 to %d weights, got %d", op, kW4MaxSeg, nseg);
    G4B_REQUIRE(nseg == 1 || M <= kW4BTSmall, G4B_E_SHAPE, "%s: several weights in one launch need M <= %d (got %d)",
                op, kW4BTSmall, M);
    G4B_REQUIRE(M >= 1 && K >= kW4BK && K % kW4BK == 0, G4B_E_SHAPE, "%s: need M >= 1, K %% %d == 0 (got M=%d K=%d)",
                op, kW4BK, M, K);
    long long Ntot = 0;
    for (int g = 0; g < nseg; g++) {
        const g4b_gemm_seg& sg = segs[g];
        G4B_REQUIRE(sg.wp && sg.scales_f16 && sg.y, G4B_E_ARG, "%s: NULL pointer in weight %d", op, g);
        G4B_REQUIRE(sg.N >= kW4BN && sg.N % kW4BN == 0, G4B_E_SHAPE, "%s: weight %d: N %% %d == 0 (got N=%d)", op, g,
                    kW4BN, sg.N);
        G4B_REQUIRE(aligned16(sg.wp) && aligned16(sg.scales_f16) && aligned16(sg.y), G4B_E_ALIGN,
                    "%s: weight %d: wp, scales and Y must be 16-byte aligned", op, g);
        Ntot += sg.N;
    }
    G4B_REQUIRE(Ntot <= 0x7fffffffLL && (long long)M * K < (1ll << 40) && (long long)M * Ntot < (1ll << 40),
                G4B_E_SHAPE, "%s: too large", op);
    G4B_REQUIRE(aligned16(X), G4B_E_ALIGN, "%s: X must be 16-byte aligned", op);
    const int N = (int)Ntot;
    int sms = 0;
    int st = check_device(&sms);
    if (st != G4B_OK) return st;
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    W4Plan p = w4a16_plan(M, N, K, x_dtype, sms);
    if (p.S > 1 && (!workspace || ws_bytes < w4a16_ws(p))) {
        // the split-K partials do not fit the caller's workspace: one split (always correct)
        p.S = 1;
        p.part_bytes = 0;
    }
    const size_t need = w4a16_ws(p);
    G4B_REQUIRE(ws_bytes >= need && (need == 0 || workspace), G4B_E_WORKSPACE,
                "%s: f32 X needs a %zu-byte workspace (got %zu)", op, need, ws_bytes);
    G4B_REQUIRE(need == 0 || aligned16(workspace), G4B_E_ALIGN, "%s: workspace must be 16-byte aligned", op);
    // encode the tensor maps first: nothing is queued until every check has passed
    const void* X16 = x_dtype == G4B_DT_F32 ? workspace : X;
    CUtensorMap xmap, wmap[kW4MaxSeg], smap[kW4MaxSeg];
    st = tensor_map_2d(&xmap, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, X16, (uint64_t)K, (uint64_t)M, (uint64_t)K * 2, kW4BK,
                       p.bt, CU_TENSOR_MAP_SWIZZLE_128B);
    for (int g = 0; g < kW4MaxSeg && st == G4B_OK; g++) {
        const g4b_gemm_seg& sg = segs[g < nseg ? g : 0];   // unused maps repeat weight 0's
        st = tensor_map_2d(&wmap[g], CU_TENSOR_MAP_DATA_TYPE_UINT32, sg.wp, (uint64_t)sg.N / 8, (uint64_t)K,
                           (uint64_t)sg.N / 2, kW4BN / 8, kW4BK, CU_TENSOR_MAP_SWIZZLE_NONE);
        if (st == G4B_OK)
            st = tensor_map_2d(&smap[g], CU_TENSOR_MAP_DATA_TYPE_FLOAT16, sg.scales_f16, (uint64_t)sg.N,
                               (uint64_t)K / 32, (uint64_t)sg.N * 2, kW4BN, kW4BK / 32, CU_TENSOR_MAP_SWIZZLE_NONE);
    }
    if (st != G4B_OK) return st;
    W4Args a{};
    a.y = segs[0].y;
    a.part = p.part_bytes ? reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(workspace) + p.xconv_bytes) : nullptr;
    a.M = M;
    a.N = N;
    a.K = K;
    a.nkb = K / kW4BK;
    a.ntm = p.ntm;
    a.S = p.S;
    a.ntiles = p.base * p.S;
    a.seg.nseg = nseg;
    for (int g = 0, t0 = 0; g <= kW4MaxSeg; g++) {
        a.seg.tile0[g] = g < nseg ? t0 : (g == nseg ? t0 : 0x3fffffff);
        if (g < nseg) {
            a.seg.ys[g] = segs[g].y;
            a.seg.Ns[g] = segs[g].N;
            t0 += segs[g].N / kW4BN;
        }
    }
    for (int g = nseg; g < kW4MaxSeg; g++) {
        a.seg.ys[g] = segs[0].y;
        a.seg.Ns[g] = segs[0].N;
    }
    const bool yf32 = y_dtype == G4B_DT_F32;
    auto kern = p.bt == kW4BT ? (yf32 ? gemm_w4a16_kernel<true, kW4BT, false> : gemm_w4a16_kernel<false, kW4BT, false>)
                              : (yf32 ? gemm_w4a16_kernel<true, kW4BTSmall, true>
                                      : gemm_w4a16_kernel<false, kW4BTSmall, true>);
    const size_t smem = w4_smem(p.bt);
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return fail(G4B_E_CUDA, "%s: cudaFuncSetAttribute: %s", op, cudaGetErrorString(e));
    if (x_dtype == G4B_DT_F32) {
        st = cast_f32_to_f16_async(reinterpret_cast<const float*>(X), reinterpret_cast<__half*>(workspace),
                                   (size_t)M * K, s);
        if (st != G4B_OK) return st;
    }
    const int grid = std::min(a.ntiles, sms);
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kW4Threads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cfg.attrs = attr;
    // a GEMM after the f32 -> f16 cast (its own kernel) does not overlap it
    cfg.numAttrs = (flags & G4B_GEMM_PDL) && x_dtype != G4B_DT_F32 ? 1 : 0;
    e = cudaLaunchKernelEx(&cfg, kern, a, xmap, wmap[0], smap[0], wmap[1], smap[1], wmap[2], smap[2]);
    if (e != cudaSuccess) return fail(G4B_E_CUDA, "%s: launch: %s", op, cudaGetErrorString(e));
    count_launch();
    st = launch_status(op);
    if (st != G4B_OK || p.S == 1) return st;
    // the split sum, as a programmatic dependent of the GEMM (it waits for the partials)
    const size_t n4 = (size_t)M * N / 4;
    const int threads = 256, blocks = (int)std::min<size_t>((n4 + threads - 1) / threads, (size_t)sms * 8);
    cudaLaunchConfig_t rcfg{};
    rcfg.gridDim = dim3(blocks);
    rcfg.blockDim = dim3(threads);
    rcfg.stream = s;
    rcfg.attrs = attr;
    rcfg.numAttrs = 1;
    e = yf32 ? cudaLaunchKernelEx(&rcfg, w4a16_splitk_reduce<true>, (const float*)a.part, a.seg, n4, (size_t)M * N,
                                  p.S, N)
             : cudaLaunchKernelEx(&rcfg, w4a16_splitk_reduce<false>, (const float*)a.part, a.seg, n4, (size_t)M * N,
                                  p.S, N);
    if (e != cudaSuccess) return fail(G4B_E_CUDA, "%s: split-sum launch: %s", op, cudaGetErrorString(e));
    count_launch();
    return launch_status(op);
}

extern "C" {

int g4b_gemm_i4_ex(const void* X, int x_dtype, const uint32_t* wp, const uint16_t* scales_f16, void* Y, int y_dtype,
                   int M, int N, int K, void* workspace, size_t ws_bytes, unsigned flags, g4b_stream_t stream) {
    G4B_ENTRY("gemm_i4");
    const g4b_gemm_seg one{wp, scales_f16, Y, N};
    return gemm_i4_impl("gemm_i4", X, x_dtype, M, K, 1, &one, y_dtype, workspace, ws_bytes, flags, stream);
}

int g4b_gemm_i4_fused(const void* X, int x_dtype, int M, int K, const g4b_gemm_seg* segs, int nseg, int y_dtype,
                      void* workspace, size_t ws_bytes, unsigned flags, g4b_stream_t stream) {
    G4B_ENTRY("gemm_i4_fused");
    return gemm_i4_impl("gemm_i4_fused", X, x_dtype, M, K, nseg, segs, y_dtype, workspace, ws_bytes, flags, stream);
}

}  // extern "C"

namespace g4b {

template <bool W4>
static int launch_s8(const char* op, const int8_t* A8, const void* W, const uint16_t* ratio, const float* sa,
                     const uint16_t* sw, void* Y, int y_dtype, int32_t* C, int M, int N, int K, cudaStream_t s) {
    using Cfg = S8Cfg<W4>;
    int sms = 0;
    int st = check_device(&sms);
    if (st != G4B_OK) return st;
    CUtensorMap amap, wmap, rmap, amap_q;
    st = tensor_map_2d(&amap, CU_TENSOR_MAP_DATA_TYPE_UINT8, A8, (uint64_t)K, (uint64_t)M, (uint64_t)K, kS8BK, kS8BT,
                       CU_TENSOR_MAP_SWIZZLE_128B);
    if (st == G4B_OK)
        st = tensor_map_2d(&amap_q, CU_TENSOR_MAP_DATA_TYPE_UINT8, A8, (uint64_t)K, (uint64_t)M, (uint64_t)K, kS8BK,
                           kS8SubT, CU_TENSOR_MAP_SWIZZLE_128B);
    if (st == G4B_OK) {
        if (W4)
            st = tensor_map_2d(&wmap, CU_TENSOR_MAP_DATA_TYPE_UINT32, W, (uint64_t)N / 8, (uint64_t)K, (uint64_t)N / 2,
                               kS8BN / 8, kS8BK, CU_TENSOR_MAP_SWIZZLE_NONE);
        else
            st = tensor_map_2d(&wmap, CU_TENSOR_MAP_DATA_TYPE_UINT8, W, (uint64_t)N, (uint64_t)K, (uint64_t)N, kS8BN,
                               kS8BK, CU_TENSOR_MAP_SWIZZLE_128B);
    }
    if (st == G4B_OK && W4)
        st = tensor_map_2d(&rmap, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, ratio, (uint64_t)N, (uint64_t)K / 32,
                           (uint64_t)N * 2, kS8BN, kS8BK / 32, CU_TENSOR_MAP_SWIZZLE_NONE);
    if (st != G4B_OK) return st;
    if (!W4) rmap = wmap;  // unused
    S8Args a;
    a.y = Y;
    a.c = C;
    a.sa = sa;
    a.sw = sw;
    a.M = M;
    a.N = N;
    a.K = K;
    a.nkb = (K + kS8BK - 1) / kS8BK;
    a.ntm = (M + kS8BT - 1) / kS8BT;
    a.ntiles = ((N + kS8BN - 1) / kS8BN) * a.ntm;
    // the last wave's tiles as quarter units when that wave fills at most a quarter of the SMs (W8A8: the
    // W4A8 requant costs the same per stage whatever the token count, so a quarter unit would not be faster)
    const int tail = a.ntiles % sms;
    // G4B_S8_QUARTER_TAIL=0 in the environment keeps whole tiles throughout
    const char* qenv = std::getenv("G4B_S8_QUARTER_TAIL");
    const bool quarter = !W4 && !(qenv && std::atoi(qenv) == 0) && tail > 0 && kS8Sub * tail <= sms;
    a.nfull = quarter ? a.ntiles - tail : a.ntiles;
    a.nunits = quarter ? a.nfull + kS8Sub * tail : a.ntiles;
    auto kern = y_dtype == G4B_DT_F32 ? gemm_s8_kernel<W4, true> : gemm_s8_kernel<W4, false>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)Cfg::kSmem);
    if (e != cudaSuccess) return fail(G4B_E_CUDA, "%s: cudaFuncSetAttribute: %s", op, cudaGetErrorString(e));
    const int grid = std::min(a.nunits, sms);
    kern<<<grid, Cfg::kThreads, Cfg::kSmem, s>>>(a, amap, wmap, rmap, amap_q);
    count_launch();
    return launch_status(op);
}

}  // namespace g4b

extern "C" {

int g4b_gemm_w8a8(const int8_t* A8, const int8_t* W8, const float* sa, const uint16_t* sw_f16, void* Y, int y_dtype,
                  int32_t* C_debug, int M, int N, int K, g4b_stream_t stream) {
    G4B_ENTRY("gemm_w8a8");
    G4B_REQUIRE(A8 && W8 && sa && sw_f16 && Y, G4B_E_ARG, "gemm_w8a8: NULL pointer");
    G4B_REQUIRE(y_dtype == G4B_DT_F32 || y_dtype == G4B_DT_F16, G4B_E_ARG, "gemm_w8a8: bad y_dtype %d", y_dtype);
    G4B_REQUIRE(M >= 1 && N >= 16 && K >= 32 && N % 16 == 0 && K % 32 == 0, G4B_E_SHAPE,
                "gemm_w8a8: need M >= 1, N %% 16 == 0, K %% 32 == 0 (got M=%d N=%d K=%d)", M, N, K);
    G4B_REQUIRE((long long)M * K < (1ll << 40) && (long long)M * N < (1ll << 40) && (long long)K * N < (1ll << 40),
                G4B_E_SHAPE, "gemm_w8a8: too large");
    G4B_REQUIRE(aligned16(A8) && aligned16(W8) && aligned16(Y) && (!C_debug || aligned16(C_debug)), G4B_E_ALIGN,
                "gemm_w8a8: A8, W8, Y and C_debug must be 16-byte aligned");
    return launch_s8<false>("gemm_w8a8", A8, W8, nullptr, sa, sw_f16, Y, y_dtype, C_debug, M, N, K,
                            reinterpret_cast<cudaStream_t>(stream));
}

int g4b_gemm_w4a8(const int8_t* A8, const uint32_t* wp, const uint16_t* ratio_f16, const float* sa,
                  const uint16_t* sw_f16, void* Y, int y_dtype, int32_t* C_debug, int M, int N, int K,
                  g4b_stream_t stream) {
    G4B_ENTRY("gemm_w4a8");
    G4B_REQUIRE(A8 && wp && ratio_f16 && sa && sw_f16 && Y, G4B_E_ARG, "gemm_w4a8: NULL pointer");
    G4B_REQUIRE(y_dtype == G4B_DT_F32 || y_dtype == G4B_DT_F16, G4B_E_ARG, "gemm_w4a8: bad y_dtype %d", y_dtype);
    G4B_REQUIRE(M >= 1 && N >= 32 && K >= 32 && N % 32 == 0 && K % 32 == 0, G4B_E_SHAPE,
                "gemm_w4a8: need M >= 1, N %% 32 == 0, K %% 32 == 0 (got M=%d N=%d K=%d)", M, N, K);
    G4B_REQUIRE((long long)M * K < (1ll << 40) && (long long)M * N < (1ll << 40) && (long long)K * N < (1ll << 40),
                G4B_E_SHAPE, "gemm_w4a8: too large");
    G4B_REQUIRE(aligned16(A8) && aligned16(wp) && aligned16(ratio_f16) && aligned16(Y) &&
                    (!C_debug || aligned16(C_debug)),
                G4B_E_ALIGN, "gemm_w4a8: A8, wp, ratio, Y and C_debug must be 16-byte aligned");
    return launch_s8<true>("gemm_w4a8", A8, wp, ratio_f16, sa, sw_f16, Y, y_dtype, C_debug, M, N, K,
                           reinterpret_cast<cudaStream_t>(stream));
}

}  // extern "C"
