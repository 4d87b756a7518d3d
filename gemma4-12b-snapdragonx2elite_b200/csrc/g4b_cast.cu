// g4b_cast.cu -- element-wise f32 <-> f16 casts (vk/cast_dn.comp, vk/cast_up.comp)
// and the per-token int8 activation quantiser (vk/cast_i8.comp).
//
// All three are HBM-bound streams.  cast_i8 runs one CTA per row (token): a
// vectorised max-abs pass, a block reduction, then a second pass over the same
// row, which the first pass has just brought into L1/L2, so HBM sees each
// activation byte once.
#include <algorithm>

#include "g4b_common.cuh"

namespace g4b {

__global__ void cast_f32_to_f16_kernel(const float* __restrict__ src, __half* __restrict__ dst, size_t n) {
    const size_t n8 = n / 8;
    const size_t stride = (size_t)gridDim.x * blockDim.x;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n8; i += stride) {
        const float4 a = __ldcs((const float4*)src + 2 * i);
        const float4 b = __ldcs((const float4*)src + 2 * i + 1);
        uint4 o;
        o.x = pack_half2(__float2half_rn(a.x), __float2half_rn(a.y));
        o.y = pack_half2(__float2half_rn(a.z), __float2half_rn(a.w));
        o.z = pack_half2(__float2half_rn(b.x), __float2half_rn(b.y));
        o.w = pack_half2(__float2half_rn(b.z), __float2half_rn(b.w));
        __stcs((uint4*)dst + i, o);
    }
    for (size_t i = n8 * 8 + blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += stride)
        dst[i] = __float2half_rn(src[i]);
}

__global__ void cast_f16_to_f32_kernel(const __half* __restrict__ src, float* __restrict__ dst, size_t n) {
    const size_t n8 = n / 8;
    const size_t stride = (size_t)gridDim.x * blockDim.x;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n8; i += stride) {
        const uint4 v = __ldcs((const uint4*)src + i);
        __stcs((float4*)dst + 2 * i, make_float4(h_lo(v.x), h_hi(v.x), h_lo(v.y), h_hi(v.y)));
        __stcs((float4*)dst + 2 * i + 1, make_float4(h_lo(v.z), h_hi(v.z), h_lo(v.w), h_hi(v.w)));
    }
    for (size_t i = n8 * 8 + blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += stride)
        dst[i] = __half2float(src[i]);
}

// 8 consecutive activations of a row as f32
template <bool XF16>
__device__ __forceinline__ void load8(const void* row, int i8, float (&v)[8]) {
    if (XF16) {
        const uint4 u = __ldg((const uint4*)row + i8);
        v[0] = h_lo(u.x); v[1] = h_hi(u.x); v[2] = h_lo(u.y); v[3] = h_hi(u.y);
        v[4] = h_lo(u.z); v[5] = h_hi(u.z); v[6] = h_lo(u.w); v[7] = h_hi(u.w);
    } else {
        const float4 a = __ldg((const float4*)row + 2 * i8), b = __ldg((const float4*)row + 2 * i8 + 1);
        v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
    }
}

__device__ __forceinline__ uint32_t q4(float a, float b, float c, float d, float inv) {
    // round-half-even of x * inv (cvt.rni), clamped to [-127, 127], vk/cast_i8.comp:18
    int qa = max(-127, min(127, __float2int_rn(__fmul_rn(a, inv))));
    int qb = max(-127, min(127, __float2int_rn(__fmul_rn(b, inv))));
    int qc = max(-127, min(127, __float2int_rn(__fmul_rn(c, inv))));
    int qd = max(-127, min(127, __float2int_rn(__fmul_rn(d, inv))));
    return (uint32_t)(qa & 0xff) | ((uint32_t)(qb & 0xff) << 8) | ((uint32_t)(qc & 0xff) << 16) |
           ((uint32_t)(qd & 0xff) << 24);
}

template <bool XF16>
__global__ void __launch_bounds__(256) cast_i8_kernel(const void* __restrict__ X, int8_t* __restrict__ A8,
                                                      float* __restrict__ sa, int K) {
    const int m = blockIdx.x;
    const void* row = (const char*)X + (size_t)m * K * (XF16 ? 2 : 4);
    const int k8 = K / 8;
    float mx = 0.f;
    for (int i = threadIdx.x; i < k8; i += blockDim.x) {
        float v[8];
        load8<XF16>(row, i, v);
        #pragma unroll
        for (int j = 0; j < 8; j++) mx = fmaxf(mx, fabsf(v[j]));
    }
    #pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    __shared__ float wmax[8];
    __shared__ float s_inv;
    if ((threadIdx.x & 31) == 0) wmax[threadIdx.x >> 5] = mx;
    __syncthreads();
    if (threadIdx.x == 0) {
        float a = 0.f;
        for (int w = 0; w < (int)(blockDim.x >> 5); w++) a = fmaxf(a, wmax[w]);
        // s = max(amax / 127, 1e-12); inv = 1 / s -- correctly rounded, vk/cast_i8.comp:16
        const float s = fmaxf(__fdiv_rn(a, 127.0f), 1e-12f);
        sa[m] = s;
        s_inv = __fdiv_rn(1.0f, s);
    }
    __syncthreads();
    const float inv = s_inv;
    int8_t* out = A8 + (size_t)m * K;
    for (int i = threadIdx.x; i < k8; i += blockDim.x) {
        float v[8];
        load8<XF16>(row, i, v);
        uint2 o;
        o.x = q4(v[0], v[1], v[2], v[3], inv);
        o.y = q4(v[4], v[5], v[6], v[7], inv);
        *((uint2*)out + i) = o;
    }
}

// f32 -> f16 (RNE) on `s` for the library's own use (the GEMMs' cast_dn step).
int cast_f32_to_f16_async(const float* src, __half* dst, size_t n, cudaStream_t s) {
    int sms = 148;
    int st = check_device(&sms);
    if (st != G4B_OK) return st;
    const int threads = 256;
    const int blocks = (int)std::max<size_t>(1, std::min<size_t>((n / 8 + threads - 1) / threads, (size_t)sms * 8));
    cast_f32_to_f16_kernel<<<blocks, threads, 0, s>>>(src, dst, n);
    count_launch();
    return launch_status("cast f32->f16");
}

}  // namespace g4b

using namespace g4b;

extern "C" {

int g4b_cast(const void* src, int src_dtype, void* dst, int dst_dtype, size_t n, g4b_stream_t stream) {
    G4B_ENTRY("cast");
    G4B_REQUIRE(src && dst, G4B_E_ARG, "cast: NULL pointer argument");
    G4B_REQUIRE((src_dtype == G4B_DT_F32 && dst_dtype == G4B_DT_F16) ||
                    (src_dtype == G4B_DT_F16 && dst_dtype == G4B_DT_F32),
                G4B_E_ARG, "cast: only f32->f16 and f16->f32 are supported");
    G4B_REQUIRE(aligned16(src) && aligned16(dst), G4B_E_ALIGN, "cast: pointers must be 16-byte aligned");
    if (n == 0) return G4B_OK;
    int sms = 148;
    int st = check_device(&sms);
    if (st != G4B_OK) return st;
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    const int threads = 256;
    const int blocks = (int)std::max<size_t>(1, std::min<size_t>((n / 8 + threads - 1) / threads, (size_t)sms * 8));
    if (src_dtype == G4B_DT_F32)
        cast_f32_to_f16_kernel<<<blocks, threads, 0, s>>>((const float*)src, (__half*)dst, n);
    else
        cast_f16_to_f32_kernel<<<blocks, threads, 0, s>>>((const __half*)src, (float*)dst, n);
    count_launch();
    return launch_status("cast");
}

int g4b_cast_i8(const void* X, int x_dtype, int8_t* A8, float* sa, int M, int K, g4b_stream_t stream) {
    G4B_ENTRY("cast_i8");
    G4B_REQUIRE(X && A8 && sa, G4B_E_ARG, "cast_i8: NULL pointer argument");
    G4B_REQUIRE(x_dtype == G4B_DT_F32 || x_dtype == G4B_DT_F16, G4B_E_ARG, "cast_i8: bad x_dtype %d", x_dtype);
    G4B_REQUIRE(M > 0 && K > 0 && K % 16 == 0, G4B_E_SHAPE, "cast_i8: M=%d, K=%d (multiple of 16)", M, K);
    G4B_REQUIRE(M <= 0x7fffffff && aligned16(X) && aligned16(A8), G4B_E_ALIGN,
                "cast_i8: X and A8 must be 16-byte aligned");
    G4B_REQUIRE(((uintptr_t)sa & 3u) == 0, G4B_E_ALIGN, "cast_i8: sa misaligned");
    int st = check_device(nullptr);
    if (st != G4B_OK) return st;
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    if (x_dtype == G4B_DT_F16) cast_i8_kernel<true><<<M, 256, 0, s>>>(X, A8, sa, K);
    else cast_i8_kernel<false><<<M, 256, 0, s>>>(X, A8, sa, K);
    count_launch();
    return launch_status("cast_i8");
}

}  // extern "C"
