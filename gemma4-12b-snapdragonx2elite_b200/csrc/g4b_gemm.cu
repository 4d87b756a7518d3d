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
// TMEM: accumulator columns [0, 256), A stages at [256, 256 + 32*stages) (448 of 512).
// Shared-memory stage s and TMEM A stage s are recycled together: the MMA's
// commit on empty[s] frees both.
#include <algorithm>

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
constexpr int kW4BT = 256;      // tokens per tile (MMA N)
constexpr int kW4BK = 64;       // K rows per stage
constexpr int kW4Stages = 6;  // even: dequant warps alternate stages
constexpr int kW4DqWarps = 16;
constexpr int kW4Threads = (2 + kW4DqWarps + 4) * 32;
constexpr int kW4XBytes = kW4BT * kW4BK * 2;          // 32 KB
constexpr int kW4WBytes = kW4BK * (kW4BN / 8) * 4;    // 4 KB
constexpr int kW4SBytes = (kW4BK / 32) * kW4BN * 2;   // 512 B
constexpr int kW4TmemCols = 512;
static_assert(kW4Stages % 2 == 0 && 256 + 32 * kW4Stages <= kW4TmemCols, "TMEM budget");
constexpr int kW4ACol = kW4BT;                         // first A column
constexpr size_t kW4Smem = 1024 + (size_t)kW4Stages * (kW4XBytes + kW4WBytes + kW4SBytes);

struct W4Args {
    void* y;
    int M, N, K, nkb, ntm, ntiles;
};

template <bool YF32>
__global__ void __launch_bounds__(kW4Threads, 1) gemm_w4a16_kernel(const W4Args a,
                                                                   const __grid_constant__ CUtensorMap xmap,
                                                                   const __grid_constant__ CUtensorMap wmap,
                                                                   const __grid_constant__ CUtensorMap smap) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    __shared__ uint64_t bars[3 * kW4Stages + 3];
    __shared__ uint32_t s_tmem;
    __shared__ int s_abort;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    volatile int* abort_flag = &s_abort;
    const uint32_t raw0 = smem_u32(smem_raw);
    const uint32_t sm0 = (raw0 + 1023u) & ~1023u;          // X stages (1024-aligned for the swizzle)
    const uint32_t smw = sm0 + kW4Stages * kW4XBytes;        // packed words
    const uint32_t sms = smw + kW4Stages * kW4WBytes;        // scales
    const uint8_t* gsm = smem_raw + (sm0 - raw0);
    const uint32_t* wsm = reinterpret_cast<const uint32_t*>(gsm + kW4Stages * kW4XBytes);
    const uint16_t* ssm = reinterpret_cast<const uint16_t*>(gsm + kW4Stages * (kW4XBytes + kW4WBytes));
    const uint32_t bar0 = smem_u32(bars);
    auto full_bar = [&](int s) { return bar0 + 8u * s; };
    auto empty_bar = [&](int s) { return bar0 + 8u * (kW4Stages + s); };
    auto afull_bar = [&](int s) { return bar0 + 8u * (2 * kW4Stages + s); };
    const uint32_t dfull_bar = bar0 + 8u * (3 * kW4Stages);
    const uint32_t dempty_bar = dfull_bar + 8u;
    const uint32_t drain_bar = dfull_bar + 16u;

    if (tid == 0) {
        for (int s = 0; s < kW4Stages; s++) {
            mbar_init(full_bar(s), 1);
            mbar_init(empty_bar(s), 8 + 1);  // 8 dequant warps + the MMA commit
            mbar_init(afull_bar(s), 8);
        }
        mbar_init(dfull_bar, 1);
        mbar_init(dempty_bar, 4);
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
    const int nks = a.nkb;  // K stages per tile

    if (warp == 0) {
        // ------------------------------------------------------- TMA producer
        if (lane == 0) {
            prefetch_tensor_map(&xmap);
            prefetch_tensor_map(&wmap);
            prefetch_tensor_map(&smap);
            const uint64_t pol_w = l2_evict_first_policy();
            uint64_t pol_x;
            asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(pol_x));
            int it = 0;
            bool ok = true;
            for (int t = blockIdx.x; ok && t < a.ntiles; t += gridDim.x) {
                const int nt = t / a.ntm, mt = t % a.ntm;
                for (int kb = 0; kb < nks; kb++, it++) {
                    const int s = it % kW4Stages;
                    if (it >= kW4Stages &&
                        !mbar_wait(empty_bar(s), ((it / kW4Stages) & 1) ^ 1, abort_flag, &g_gemm_status)) {
                        ok = false;
                        break;
                    }
                    mbar_arrive_expect_tx(full_bar(s), kW4XBytes + kW4WBytes + kW4SBytes);
                    tma_load_2d(sm0 + s * kW4XBytes, &xmap, kb * kW4BK, mt * kW4BT, full_bar(s), pol_x);
                    tma_load_2d(smw + s * kW4WBytes, &wmap, nt * (kW4BN / 8), kb * kW4BK, full_bar(s), pol_w);
                    tma_load_2d(sms + s * kW4SBytes, &smap, nt * kW4BN, kb * (kW4BK / 32), full_bar(s), pol_w);
                }
            }
            // drain: the copies already issued must land before the CTA exits
            for (int i = std::max(0, it - kW4Stages); i < it; i++)
                mbar_wait_drain(full_bar(i % kW4Stages), (i / kW4Stages) & 1, &g_gemm_status);
        }
    } else if (warp == 1) {
        // ------------------------------------------------------- MMA issuer
        if (lane == 0) {
            constexpr uint32_t idesc = tc::idesc(1, 0, 0, 0, 0, kW4BT, kW4BN);
            int it = 0, tc_i = 0;
            bool ok = true;
            for (int t = blockIdx.x; ok && t < a.ntiles; t += gridDim.x, tc_i++) {
                if (!mbar_wait(dempty_bar, (tc_i & 1) ^ 1, abort_flag, &g_gemm_status)) break;
                tc::fence_after();
                for (int kb = 0; kb < nks; kb++, it++) {
                    const int s = it % kW4Stages;
                    const uint32_t ph = (it / kW4Stages) & 1;
                    if (!mbar_wait(full_bar(s), ph, abort_flag, &g_gemm_status) ||
                        !mbar_wait(afull_bar(s), ph, abort_flag, &g_gemm_status)) {
                        ok = false;
                        break;
                    }
                    tc::fence_after();
                    const uint64_t bdesc = tc::sdesc_sw128(sm0 + s * kW4XBytes, 16, 1024);
#pragma unroll
                    for (int kk = 0; kk < kW4BK / 16; kk++)
                        tc::mma_f16_ts(tmem, tmem + kW4ACol + s * (kW4BK / 2) + kk * 8, bdesc + (uint64_t)(kk * 2),
                                       idesc, (kb | kk) != 0);
                    tc::commit(empty_bar(s));
                }
                if (ok) tc::commit(dfull_bar);
            }
            // drain: every MMA issued must be complete before TMEM is released
            tc::commit(drain_bar);
            mbar_wait_drain(drain_bar, 0, &g_gemm_status);
        }
    } else if (warp < 2 + kW4DqWarps) {
        // ------------------------------------------------------- dequant
        const int q = warp & 3;             // TMEM lane quarter this warp may access
        const int kh = ((warp - 2) >> 2) & 1;  // which 32-row scale block of the stage
        const int par = (warp - 2) >> 3;       // which stages: it % 2 == par
        const int nl = q * 32 + lane;       // weight column within the tile
        const int g = nl >> 3, j = nl & 7;
        const uint32_t sel = (uint32_t)(j >> 1) | ((uint32_t)(4 + (j >> 1)) << 8);
        const uint32_t sh = (uint32_t)(j & 1) * 4u;
        const uint32_t lane_addr = (uint32_t)(q * 32) << 16;
        int it = 0;
        bool ok = true;
        for (int t = blockIdx.x; ok && t < a.ntiles; t += gridDim.x) {
            for (int kb = 0; kb < nks; kb++, it++) {
                if ((it & 1) != par) continue;
                const int s = it % kW4Stages;
                if (!mbar_wait(full_bar(s), (it / kW4Stages) & 1, abort_flag, &g_gemm_status)) {
                    ok = false;
                    break;
                }
                tc::fence_after();
                const uint32_t* wr = wsm + s * (kW4WBytes / 4) + kh * 32 * (kW4BN / 8) + g;
                const uint32_t sc = ssm[s * (kW4SBytes / 2) + kh * kW4BN + nl];
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
                tc::st_32x32b_x16(tmem + lane_addr + kW4ACol + s * (kW4BK / 2) + kh * 16, v);
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
            if (!mbar_wait(dfull_bar, tc_i & 1, abort_flag, &g_gemm_status)) break;
            tc::fence_after();
            const int nt = t / a.ntm, mt = t % a.ntm;
            const int n = nt * kW4BN + nl;
            const int m0 = mt * kW4BT;
#pragma unroll 1
            for (int c = 0; c < kW4BT / 32; c++) {
                uint32_t r[32];
                tc::ld_32x32b_x32(tmem + lane_addr + c * 32, r);
                tc::wait_ld();
                const int mb = m0 + c * 32;
#pragma unroll
                for (int i = 0; i < 32; i++) {
                    const int m = mb + i;
                    if (m < a.M) {
                        const float f = __uint_as_float(r[i]);
                        if (YF32)
                            reinterpret_cast<float*>(a.y)[(size_t)m * a.N + n] = f;
                        else
                            reinterpret_cast<__half*>(a.y)[(size_t)m * a.N + n] = __float2half_rn(f);
                    }
                }
            }
            tc::fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(dempty_bar);
        }
    }

    __syncwarp();
    tc::fence_before();
    __syncthreads();
    tc::fence_after();
    if (warp == 1) tc::tmem_dealloc(tmem, kW4TmemCols);
}

static size_t w4a16_ws(int M, int K, int x_dtype) {
    return x_dtype == G4B_DT_F32 ? (((size_t)M * K * 2 + 255) & ~(size_t)255) : 0;
}

}  // namespace g4b

using namespace g4b;

extern "C" {

size_t g4b_gemm_i4_workspace_bytes(int M, int N, int K, int x_dtype) {
    (void)N;
    if (M <= 0 || K <= 0) return 0;
    return w4a16_ws(M, K, x_dtype);
}

int g4b_gemm_i4(const void* X, int x_dtype, const uint32_t* wp, const uint16_t* scales_f16, void* Y, int y_dtype,
                int M, int N, int K, void* workspace, size_t ws_bytes, g4b_stream_t stream) {
    G4B_ENTRY("gemm_i4");
    G4B_REQUIRE(X && wp && scales_f16 && Y, G4B_E_ARG, "gemm_i4: NULL pointer");
    G4B_REQUIRE(x_dtype == G4B_DT_F32 || x_dtype == G4B_DT_F16, G4B_E_ARG, "gemm_i4: bad x_dtype %d", x_dtype);
    G4B_REQUIRE(y_dtype == G4B_DT_F32 || y_dtype == G4B_DT_F16, G4B_E_ARG, "gemm_i4: bad y_dtype %d", y_dtype);
    G4B_REQUIRE(M >= 1 && N >= kW4BN && K >= kW4BK && N % kW4BN == 0 && K % kW4BK == 0, G4B_E_SHAPE,
                "gemm_i4: need M >= 1, N %% %d == 0, K %% %d == 0 (got M=%d N=%d K=%d)", kW4BN, kW4BK, M, N, K);
    G4B_REQUIRE((long long)M * K < (1ll << 40) && (long long)M * N < (1ll << 40), G4B_E_SHAPE, "gemm_i4: too large");
    G4B_REQUIRE(aligned16(X) && aligned16(wp) && aligned16(scales_f16) && aligned16(Y), G4B_E_ALIGN,
                "gemm_i4: X, wp, scales and Y must be 16-byte aligned");
    int sms = 0;
    int st = check_device(&sms);
    if (st != G4B_OK) return st;
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    const size_t need = w4a16_ws(M, K, x_dtype);
    G4B_REQUIRE(ws_bytes >= need && (need == 0 || workspace), G4B_E_WORKSPACE,
                "gemm_i4: f32 X needs a %zu-byte workspace (got %zu)", need, ws_bytes);
    const void* X16 = X;
    if (x_dtype == G4B_DT_F32) {
        G4B_REQUIRE(aligned16(workspace), G4B_E_ALIGN, "gemm_i4: workspace must be 16-byte aligned");
        st = cast_f32_to_f16_async(reinterpret_cast<const float*>(X), reinterpret_cast<__half*>(workspace),
                                   (size_t)M * K, s);
        if (st != G4B_OK) return st;
        X16 = workspace;
    }
    CUtensorMap xmap, wmap, smap;
    st = tensor_map_2d(&xmap, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, X16, (uint64_t)K, (uint64_t)M, (uint64_t)K * 2, kW4BK,
                       kW4BT, CU_TENSOR_MAP_SWIZZLE_128B);
    if (st == G4B_OK)
        st = tensor_map_2d(&wmap, CU_TENSOR_MAP_DATA_TYPE_UINT32, wp, (uint64_t)N / 8, (uint64_t)K, (uint64_t)N / 2,
                           kW4BN / 8, kW4BK, CU_TENSOR_MAP_SWIZZLE_NONE);
    if (st == G4B_OK)
        st = tensor_map_2d(&smap, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, scales_f16, (uint64_t)N, (uint64_t)K / 32,
                           (uint64_t)N * 2, kW4BN, kW4BK / 32, CU_TENSOR_MAP_SWIZZLE_NONE);
    if (st != G4B_OK) return st;
    W4Args a;
    a.y = Y;
    a.M = M;
    a.N = N;
    a.K = K;
    a.nkb = K / kW4BK;
    a.ntm = (M + kW4BT - 1) / kW4BT;
    a.ntiles = (N / kW4BN) * a.ntm;
    auto kern = y_dtype == G4B_DT_F32 ? gemm_w4a16_kernel<true> : gemm_w4a16_kernel<false>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kW4Smem);
    if (e != cudaSuccess) return fail(G4B_E_CUDA, "gemm_i4: cudaFuncSetAttribute: %s", cudaGetErrorString(e));
    const int grid = std::min(a.ntiles, sms);
    kern<<<grid, kW4Threads, kW4Smem, s>>>(a, xmap, wmap, smap);
    count_launch();
    return launch_status("gemm_i4");
}

}  // extern "C"
