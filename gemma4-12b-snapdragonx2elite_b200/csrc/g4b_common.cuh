// g4b_common.cuh -- shared host plumbing and device helpers of the g4b library.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <stdio.h>

#include "g4b.h"

namespace g4b {

// ------------------------------------------------------------------ host side
// Record `msg` as this host thread's last error and return `code`.
int fail(int code, const char* fmt, ...);
// Clear the last error (called at the start of every entry point).
void clear_error();
// Fault injector: G4B_FAULT="op:n[,op:n...]" makes the n-th call (1-based) of
// entry point `op` fail with G4B_E_FAULT_INJECTED before anything is launched.
bool fault_hit(const char* op);
// Current device is an sm_100 part (the kernels are built for sm_100a only).
int check_device(int* sm_count);
// Count one kernel launch (reported by g4b_query(G4B_Q_LAUNCHES)).
void count_launch(int n = 1);
// Turn the last CUDA error after a launch into a status.
int launch_status(const char* op);

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

#define G4B_ENTRY(opname)                                  \
    g4b::clear_error();                                    \
    if (g4b::fault_hit(opname))                            \
        return g4b::fail(G4B_E_FAULT_INJECTED, "%s: fault injected by G4B_FAULT", opname);

#define G4B_REQUIRE(cond, code, ...) \
    do { if (!(cond)) return g4b::fail((code), __VA_ARGS__); } while (0)

// ---------------------------------------------------------------- device side
__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
    uint32_t d;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
    return d;
}

// d = (a & b) | c  -- one LOP3 (immLut 0xEA)
__device__ __forceinline__ uint32_t and_or(uint32_t a, uint32_t b, uint32_t c) {
    uint32_t d;
    asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

__device__ __forceinline__ uint32_t hsub2_u(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
}

__device__ __forceinline__ uint32_t hfma2_u(uint32_t a, uint32_t b, uint32_t c) {
    uint32_t d;
    asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

__device__ __forceinline__ uint32_t hmul2_u(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
}

// Two packed e4m3 bytes (low 16 bits of `v`) -> f16x2, exact.
__device__ __forceinline__ uint32_t e4m3x2_to_f16x2(uint16_t v) {
    uint32_t d;
    asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(d) : "h"(v));
    return d;
}

__device__ __forceinline__ float h_lo(uint32_t v) { return __half2float(__ushort_as_half((uint16_t)(v & 0xffffu))); }
__device__ __forceinline__ float h_hi(uint32_t v) { return __half2float(__ushort_as_half((uint16_t)(v >> 16))); }

__device__ __forceinline__ uint32_t pack_half2(__half lo, __half hi) {
    return (uint32_t)__half_as_ushort(lo) | ((uint32_t)__half_as_ushort(hi) << 16);
}

// The reference shader's e4m3 decode (vk/gemv_fp8.comp:14-18), exact for all
// 256 codes: exponent 0 -> m * 2^-9, else (1 + m/8) * 2^(e-7); no NaN codes.
__device__ __forceinline__ float e4m3_decode_ref(uint32_t b) {
    uint32_t ex = (b >> 3) & 15u, m = b & 7u;
    float v = ex == 0u ? (float)m * (1.0f / 512.0f) : __uint_as_float(((ex + 120u) << 23) | (m << 20));
    return (b & 0x80u) ? -v : v;
}

// D = A(16x16 f16, row) * B(16x8 f16, col) + C, f32 accumulate.
__device__ __forceinline__ void mma_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                          uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
        "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Programmatic dependent launch controls (no-ops when launched without the attribute).
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

}  // namespace g4b
