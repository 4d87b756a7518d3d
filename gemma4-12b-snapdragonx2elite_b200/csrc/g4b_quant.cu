// g4b_quant.cu -- the engine's weight packing, quant() (src/vk_engine.py:125-159),
// on the GPU.  Bit-for-bit the same buffers as the host packer:
//
//   g4b_quant_i4     scales = max(absmax/7, 1e-8) (f32), nibbles
//                    clip(rint(W/scale) + 8, 0, 15) packed into [K, N/8] words,
//                    f16 scales [K/32, N]                        (:126-131)
//   g4b_quant_e4m3   e4m3 bytes of clip(scale * 2^shift, 0, 448)   (:133-137)
//   g4b_quant_w8a8   s_w = max(rowmax|deq|/127, 1e-12), int8
//                    clip(rint(deq/s_w), -127, 127) as [K, N], f16 s_w  (:152-157)
//                    and the W4A8 ratio f16(scale / s_w)  (benchmarks/coopgemm_w4a8.py:84)
//
// The reference quantises on the host at every start-up (about four minutes
// for the 12B model); these kernels do it at HBM speed.  All divisions are
// correctly rounded and all roundings half-to-even, as numpy's are.
#include <algorithm>

#include "g4b_common.cuh"

namespace g4b {

// One thread per (8-column group g, scale block b).
__global__ void __launch_bounds__(128) quant_i4_kernel(const float* __restrict__ W, int N, int K,
                                                       uint32_t* __restrict__ wp, __half* __restrict__ sc16,
                                                       float* __restrict__ sc32, unsigned* __restrict__ amax_bits) {
    const int nb8 = N >> 3, nblk = K >> 5;
    const int g = blockIdx.x * blockDim.x + threadIdx.x;
    const int b = blockIdx.y;
    if (g >= nb8) return;
    float s[8];
    float smax = 0.f;
    #pragma unroll
    for (int j = 0; j < 8; j++) {
        const int n = 8 * g + j;
        const float4* row = (const float4*)(W + (size_t)n * K + 32 * b);
        float a = 0.f;
        #pragma unroll
        for (int i = 0; i < 8; i++) {
            const float4 v = __ldg(row + i);
            a = fmaxf(a, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
        }
        s[j] = fmaxf(__fdiv_rn(a, 7.0f), 1e-8f);
        smax = fmaxf(smax, s[j]);
        sc16[(size_t)b * N + n] = __float2half_rn(s[j]);
        if (sc32) sc32[(size_t)n * nblk + b] = s[j];
    }
    if (amax_bits) atomicMax(amax_bits, __float_as_uint(smax));
    for (int kk = 0; kk < 32; kk++) {
        uint32_t word = 0;
        #pragma unroll
        for (int j = 0; j < 8; j++) {
            const float v = __ldg(W + (size_t)(8 * g + j) * K + 32 * b + kk);
            float r = rintf(__fdiv_rn(v, s[j])) + 8.0f;
            r = fminf(fmaxf(r, 0.0f), 15.0f);
            word |= ((uint32_t)r & 15u) << (4 * j);
        }
        wp[(size_t)(32 * b + kk) * nb8 + g] = word;
    }
}

__device__ __forceinline__ uint8_t e4m3_rn(float v) {
    uint16_t d;
    asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(d) : "f"(0.0f), "f"(v));
    return (uint8_t)(d & 0xffu);  // the second source lands in the low byte
}

__global__ void quant_e4m3_kernel(const float* __restrict__ sc32, int N, int nblk, float mul, uint8_t* __restrict__ e8) {
    const size_t total = (size_t)N * nblk;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
        const int b = (int)(i / N), n = (int)(i % N);
        float v = __fmul_rn(sc32[(size_t)n * nblk + b], mul);
        v = fminf(fmaxf(v, 0.0f), 448.0f);
        e8[i] = e4m3_rn(v);
    }
}

// One thread per 8-column group: two passes down K.
__global__ void quant_w8a8_kernel(const uint32_t* __restrict__ wp, const float* __restrict__ sc32, int N, int K,
                                  int8_t* __restrict__ w8, __half* __restrict__ sw16, float* __restrict__ sw32,
                                  __half* __restrict__ ratio16) {
    const int nb8 = N >> 3, nblk = K >> 5;
    const int g = blockIdx.x * blockDim.x + threadIdx.x;
    if (g >= nb8) return;
    float m[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (int k = 0; k < K; k++) {
        const uint32_t w = __ldg(wp + (size_t)k * nb8 + g);
        #pragma unroll
        for (int j = 0; j < 8; j++) {
            const float d = __fmul_rn((float)((w >> (4 * j)) & 15u) - 8.0f, sc32[(size_t)(8 * g + j) * nblk + (k >> 5)]);
            m[j] = fmaxf(m[j], fabsf(d));
        }
    }
    float sw[8];
    #pragma unroll
    for (int j = 0; j < 8; j++) {
        sw[j] = fmaxf(__fdiv_rn(m[j], 127.0f), 1e-12f);
        sw16[8 * g + j] = __float2half_rn(sw[j]);
        if (sw32) sw32[8 * g + j] = sw[j];
        if (ratio16)
            for (int b = 0; b < nblk; b++)
                ratio16[(size_t)b * N + 8 * g + j] =
                    __float2half_rn(__fdiv_rn(sc32[(size_t)(8 * g + j) * nblk + b], sw[j]));
    }
    for (int k = 0; k < K; k++) {
        const uint32_t w = __ldg(wp + (size_t)k * nb8 + g);
        uint32_t lo = 0, hi = 0;
        #pragma unroll
        for (int j = 0; j < 8; j++) {
            const float d = __fmul_rn((float)((w >> (4 * j)) & 15u) - 8.0f, sc32[(size_t)(8 * g + j) * nblk + (k >> 5)]);
            float r = rintf(__fdiv_rn(d, sw[j]));
            r = fminf(fmaxf(r, -127.0f), 127.0f);
            const uint32_t byte = (uint32_t)((int)r) & 0xffu;
            if (j < 4) lo |= byte << (8 * j); else hi |= byte << (8 * (j - 4));
        }
        *(uint2*)(w8 + (size_t)k * N + 8 * g) = make_uint2(lo, hi);
    }
}

}  // namespace g4b

using namespace g4b;

extern "C" {

int g4b_quant_i4(const float* W, int N, int K, uint32_t* wp, uint16_t* scales_f16, float* scales_f32,
                 uint32_t* amax_bits, g4b_stream_t stream) {
    G4B_ENTRY("quant_i4");
    G4B_REQUIRE(W && wp && scales_f16, G4B_E_ARG, "quant_i4: NULL pointer argument");
    G4B_REQUIRE(N > 0 && N % 8 == 0 && K > 0 && K % 32 == 0, G4B_E_SHAPE,
                "quant_i4: N=%d (multiple of 8), K=%d (multiple of 32)", N, K);
    G4B_REQUIRE(aligned16(W) && ((uintptr_t)wp & 3u) == 0 && ((uintptr_t)scales_f16 & 1u) == 0, G4B_E_ALIGN,
                "quant_i4: W must be 16-byte aligned");
    int st = check_device(nullptr);
    if (st != G4B_OK) return st;
    dim3 grid((N / 8 + 127) / 128, K / 32);
    quant_i4_kernel<<<grid, 128, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
        W, N, K, wp, (__half*)scales_f16, scales_f32, amax_bits);
    count_launch();
    return launch_status("quant_i4");
}

int g4b_quant_e4m3(const float* scales_f32, int N, int K, int shift, uint8_t* scales_e4m3, g4b_stream_t stream) {
    G4B_ENTRY("quant_e4m3");
    G4B_REQUIRE(scales_f32 && scales_e4m3, G4B_E_ARG, "quant_e4m3: NULL pointer argument");
    G4B_REQUIRE(N > 0 && K > 0 && K % 32 == 0, G4B_E_SHAPE, "quant_e4m3: N=%d, K=%d (multiple of 32)", N, K);
    G4B_REQUIRE(shift > -126 && shift < 127, G4B_E_ARG, "quant_e4m3: shift %d out of range", shift);
    int sms = 148;
    int st = check_device(&sms);
    if (st != G4B_OK) return st;
    const size_t total = (size_t)N * (K / 32);
    const int blocks = (int)std::min<size_t>((total + 255) / 256, (size_t)sms * 8);
    quant_e4m3_kernel<<<blocks, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
        scales_f32, N, K / 32, ldexpf(1.0f, shift), scales_e4m3);
    count_launch();
    return launch_status("quant_e4m3");
}

int g4b_quant_w8a8(const uint32_t* wp, const float* scales_f32, int N, int K, int8_t* w8, uint16_t* sw_f16,
                   float* sw_f32, uint16_t* ratio_f16, g4b_stream_t stream) {
    G4B_ENTRY("quant_w8a8");
    G4B_REQUIRE(wp && scales_f32 && w8 && sw_f16, G4B_E_ARG, "quant_w8a8: NULL pointer argument");
    G4B_REQUIRE(N > 0 && N % 8 == 0 && K > 0 && K % 32 == 0, G4B_E_SHAPE,
                "quant_w8a8: N=%d (multiple of 8), K=%d (multiple of 32)", N, K);
    G4B_REQUIRE(((uintptr_t)w8 & 7u) == 0, G4B_E_ALIGN, "quant_w8a8: w8 must be 8-byte aligned");
    int st = check_device(nullptr);
    if (st != G4B_OK) return st;
    quant_w8a8_kernel<<<(N / 8 + 63) / 64, 64, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
        wp, scales_f32, N, K, w8, (__half*)sw_f16, sw_f32, (__half*)ratio_f16);
    count_launch();
    return launch_status("quant_w8a8");
}

}  // extern "C"
