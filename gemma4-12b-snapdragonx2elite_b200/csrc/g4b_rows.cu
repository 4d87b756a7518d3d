// g4b_rows.cu -- the prefill layer's element-wise dispatches over [M, D] rows of tokens:
//   rows_rmsnorm   vk/pre_norm.comp:8-13    y[m] = x[m] * rsqrt(mean(x[m]^2) + 1e-6) * w
//   rows_normadd   vk/pre_na.comp:9-15      h[m] = (h[m] + x[m] * rsqrt(mean(x[m]^2) + 1e-6) * w) * scl
//   gelumul        vk/gelumul.comp:7-8      out = gelu_tanh(gate) * up, element-wise
// recorded around each layer's prefill GEMMs (src/vk_engine.py:413-424).
//
// All three are HBM-bound streams.  The two norms run one CTA per row: a vectorised sum-of-squares
// pass, a block reduction, then a second pass over the same row (L1/L2-resident by then), so HBM sees
// each byte once.  x and y / out may be f32 or f16 (the GEMMs' operands); the residual h is f32, as in
// the engine.
#include <algorithm>

#include "g4b_common.cuh"

namespace g4b {

constexpr int kRowThreads = 256;
constexpr float kRowEps = 1e-6f;   // vk/pre_norm.comp:12, vk/pre_na.comp:13

// 4 consecutive values as f32 / stored from f32
template <bool F32>
__device__ __forceinline__ float4 ld4(const void* p, size_t i4) {
    if constexpr (F32) return __ldg(reinterpret_cast<const float4*>(p) + i4);
    const uint2 u = __ldg(reinterpret_cast<const uint2*>(p) + i4);
    return make_float4(h_lo(u.x), h_hi(u.x), h_lo(u.y), h_hi(u.y));
}
template <bool F32>
__device__ __forceinline__ void st4(void* p, size_t i4, float4 v) {
    if constexpr (F32) {
        reinterpret_cast<float4*>(p)[i4] = v;
    } else {
        uint2 u;
        u.x = pack_half2(__float2half_rn(v.x), __float2half_rn(v.y));
        u.y = pack_half2(__float2half_rn(v.z), __float2half_rn(v.w));
        reinterpret_cast<uint2*>(p)[i4] = u;
    }
}

// rsqrt(mean(x^2) + eps) of the CTA's row (x as f32 or f16, D % 4 == 0)
template <bool XF32>
__device__ __forceinline__ float row_inv_rms(const void* x, size_t row4, int D4, float* red) {
    float s = 0.f;
    for (int i = threadIdx.x; i < D4; i += kRowThreads) {
        const float4 v = ld4<XF32>(x, row4 + i);
        s = fmaf(v.x, v.x, s);
        s = fmaf(v.y, v.y, s);
        s = fmaf(v.z, v.z, s);
        s = fmaf(v.w, v.w, s);
    }
    #pragma unroll
    for (int m = 16; m >= 1; m >>= 1) s += __shfl_xor_sync(0xffffffffu, s, m);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
    __syncthreads();
    float tot = 0.f;
    #pragma unroll
    for (int w = 0; w < kRowThreads / 32; w++) tot += red[w];
    return rsqrtf(tot / (float)(4 * D4) + kRowEps);
}

template <bool XF32, bool YF32>
__global__ void __launch_bounds__(kRowThreads) rows_rmsnorm_kernel(const void* __restrict__ x,
                                                                  const float* __restrict__ w, void* __restrict__ y,
                                                                  int D) {
    __shared__ float red[kRowThreads / 32];
    const int D4 = D / 4;
    const size_t row4 = (size_t)blockIdx.x * D4;
    const float inv = row_inv_rms<XF32>(x, row4, D4, red);
    for (int i = threadIdx.x; i < D4; i += kRowThreads) {
        const float4 v = ld4<XF32>(x, row4 + i), g = __ldg(reinterpret_cast<const float4*>(w) + i);
        st4<YF32>(y, row4 + i, make_float4(v.x * inv * g.x, v.y * inv * g.y, v.z * inv * g.z, v.w * inv * g.w));
    }
}

template <bool XF32>
__global__ void __launch_bounds__(kRowThreads) rows_normadd_kernel(const void* __restrict__ x,
                                                                  const float* __restrict__ w, float* __restrict__ h,
                                                                  int D, float scl) {
    __shared__ float red[kRowThreads / 32];
    const int D4 = D / 4;
    const size_t row4 = (size_t)blockIdx.x * D4;
    const float inv = row_inv_rms<XF32>(x, row4, D4, red);
    float4* h4 = reinterpret_cast<float4*>(h);
    for (int i = threadIdx.x; i < D4; i += kRowThreads) {
        const float4 v = ld4<XF32>(x, row4 + i), g = __ldg(reinterpret_cast<const float4*>(w) + i);
        float4 o = h4[row4 + i];
        o.x = (o.x + v.x * inv * g.x) * scl;
        o.y = (o.y + v.y * inv * g.y) * scl;
        o.z = (o.z + v.z * inv * g.z) * scl;
        o.w = (o.w + v.w * inv * g.w) * scl;
        h4[row4 + i] = o;
    }
}

__device__ __forceinline__ float gelu_tanh(float x) {
    // vk/gelumul.comp:8, the tanh approximation with the shader's constants
    return 0.5f * x * (1.0f + tanhf(0.7978845608028654f * (x + 0.044715f * x * x * x)));
}

template <bool XF32, bool YF32>
__global__ void __launch_bounds__(kRowThreads) gelumul_kernel(const void* __restrict__ gate, const void* __restrict__ up,
                                                             void* __restrict__ out, size_t n4) {
    const size_t stride = (size_t)gridDim.x * blockDim.x;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n4; i += stride) {
        const float4 g = ld4<XF32>(gate, i), u = ld4<XF32>(up, i);
        st4<YF32>(out, i, make_float4(gelu_tanh(g.x) * u.x, gelu_tanh(g.y) * u.y, gelu_tanh(g.z) * u.z,
                                      gelu_tanh(g.w) * u.w));
    }
}

static bool dt_ok(int dt) { return dt == G4B_DT_F32 || dt == G4B_DT_F16; }

}  // namespace g4b

using namespace g4b;

extern "C" {

int g4b_rows_rmsnorm(const void* x, int x_dtype, const float* w, void* y, int y_dtype, int M, int D,
                     g4b_stream_t stream) {
    G4B_ENTRY("rows_rmsnorm");
    G4B_REQUIRE(x && w && y, G4B_E_ARG, "rows_rmsnorm: NULL pointer");
    G4B_REQUIRE(dt_ok(x_dtype) && dt_ok(y_dtype), G4B_E_ARG, "rows_rmsnorm: bad dtype %d / %d", x_dtype, y_dtype);
    G4B_REQUIRE(M >= 1 && M <= 0x7fffffff && D >= 4 && D % 4 == 0, G4B_E_SHAPE,
                "rows_rmsnorm: M=%d D=%d (D a multiple of 4)", M, D);
    G4B_REQUIRE(aligned16(x) && aligned16(w) && aligned16(y), G4B_E_ALIGN,
                "rows_rmsnorm: x, w and y must be 16-byte aligned");
    int st = check_device(nullptr);
    if (st != G4B_OK) return st;
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    const bool xf = x_dtype == G4B_DT_F32, yf = y_dtype == G4B_DT_F32;
    if (xf && yf) rows_rmsnorm_kernel<true, true><<<M, kRowThreads, 0, s>>>(x, w, y, D);
    else if (xf) rows_rmsnorm_kernel<true, false><<<M, kRowThreads, 0, s>>>(x, w, y, D);
    else if (yf) rows_rmsnorm_kernel<false, true><<<M, kRowThreads, 0, s>>>(x, w, y, D);
    else rows_rmsnorm_kernel<false, false><<<M, kRowThreads, 0, s>>>(x, w, y, D);
    count_launch();
    return launch_status("rows_rmsnorm");
}

int g4b_rows_normadd(const void* x, int x_dtype, const float* w, float* h, int M, int D, float scl,
                     g4b_stream_t stream) {
    G4B_ENTRY("rows_normadd");
    G4B_REQUIRE(x && w && h, G4B_E_ARG, "rows_normadd: NULL pointer");
    G4B_REQUIRE(dt_ok(x_dtype), G4B_E_ARG, "rows_normadd: bad dtype %d", x_dtype);
    G4B_REQUIRE(M >= 1 && D >= 4 && D % 4 == 0, G4B_E_SHAPE, "rows_normadd: M=%d D=%d (D a multiple of 4)", M, D);
    G4B_REQUIRE(aligned16(x) && aligned16(w) && aligned16(h), G4B_E_ALIGN,
                "rows_normadd: x, w and h must be 16-byte aligned");
    int st = check_device(nullptr);
    if (st != G4B_OK) return st;
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    if (x_dtype == G4B_DT_F32) rows_normadd_kernel<true><<<M, kRowThreads, 0, s>>>(x, w, h, D, scl);
    else rows_normadd_kernel<false><<<M, kRowThreads, 0, s>>>(x, w, h, D, scl);
    count_launch();
    return launch_status("rows_normadd");
}

int g4b_gelumul(const void* gate, const void* up, int dtype, void* out, int out_dtype, size_t n,
                g4b_stream_t stream) {
    G4B_ENTRY("gelumul");
    G4B_REQUIRE(gate && up && out, G4B_E_ARG, "gelumul: NULL pointer");
    G4B_REQUIRE(dt_ok(dtype) && dt_ok(out_dtype), G4B_E_ARG, "gelumul: bad dtype %d / %d", dtype, out_dtype);
    G4B_REQUIRE(n >= 4 && n % 4 == 0, G4B_E_SHAPE, "gelumul: n=%zu (a multiple of 4)", n);
    G4B_REQUIRE(aligned16(gate) && aligned16(up) && aligned16(out), G4B_E_ALIGN,
                "gelumul: gate, up and out must be 16-byte aligned");
    int sms = 148;
    int st = check_device(&sms);
    if (st != G4B_OK) return st;
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    const size_t n4 = n / 4;
    const int grid = (int)std::min<size_t>((n4 + kRowThreads - 1) / kRowThreads, (size_t)sms * 8);
    const bool xf = dtype == G4B_DT_F32, yf = out_dtype == G4B_DT_F32;
    if (xf && yf) gelumul_kernel<true, true><<<grid, kRowThreads, 0, s>>>(gate, up, out, n4);
    else if (xf) gelumul_kernel<true, false><<<grid, kRowThreads, 0, s>>>(gate, up, out, n4);
    else if (yf) gelumul_kernel<false, true><<<grid, kRowThreads, 0, s>>>(gate, up, out, n4);
    else gelumul_kernel<false, false><<<grid, kRowThreads, 0, s>>>(gate, up, out, n4);
    count_launch();
    return launch_status("gelumul");
}

}  // extern "C"
