// g4b_common.cuh -- shared host plumbing and device helpers of the g4b library.
#pragma once

#include <cuda.h>  // CUtensorMap and its enums (types only; the driver entry point is fetched at run time)
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
// Read-and-clear the device status words the kernels raise (bounded waits that
// gave up); 0 = clean.
unsigned read_status_gemv();
unsigned read_status_gemm();
unsigned read_status_comm();
// f32 -> f16 (RNE) launched on `s` (the GEMMs' cast_dn step).
int cast_f32_to_f16_async(const float* src, __half* dst, size_t n, cudaStream_t s);

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// A 2-D tiled TMA descriptor for a row-major [dim1, dim0] array (dim0
// innermost, rows stride1_bytes apart) with a box of [box1, box0] elements.
// `promo` is the L2 fill size of the box's row segments: the GEMV weight
// boxes are 128 bytes wide and read once, so they use 128-byte fills (a
// 256-byte fill would also fetch the neighbouring column strip, which another
// CTA reads much later, after L2 has evicted it: 1.36x the bytes from DRAM on
// the lm_head GEMV).  Encoded once per distinct argument set and cached (the
// encoding is a pure function of its inputs); returns G4B_OK or an error status.
int tensor_map_2d(CUtensorMap* out, CUtensorMapDataType dtype, const void* base, uint64_t dim0, uint64_t dim1,
                  uint64_t stride1_bytes, uint32_t box0, uint32_t box1, CUtensorMapSwizzle swizzle,
                  CUtensorMapL2promotion promo = CU_TENSOR_MAP_L2_PROMOTION_L2_256B);

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

__device__ __forceinline__ uint32_t hmin2_u(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("min.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
}

__device__ __forceinline__ uint32_t hmax2_u(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("max.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
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

// Four transposed 8x8 b16 matrices from shared memory: lane L supplies the
// address of row L%8 of matrix L/8; lane (g = L/4, q = L%4) receives, per
// matrix, rows 2q (low half) and 2q+1 (high half) of 16-bit column g.
__device__ __forceinline__ void ldsm_x4_trans(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}

// ------------------------------------------------------ mbarrier / bulk copy
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
    asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(bar),
                 "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.b32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}

// try_wait that lets the hardware suspend the thread until the phase completes
// (or `hint_ns` elapses), so a waiting warp does not take issue slots from the
// warps on its SM sub-partition that are doing the work.
__device__ __forceinline__ bool mbar_try_wait_suspend(uint32_t bar, uint32_t parity, uint32_t hint_ns) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\tselp.b32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity), "r"(hint_ns)
        : "memory");
    return ok != 0;
}
constexpr uint32_t kSuspendHintNs = 1000000u;  // 1 ms per suspension, then the bound and abort are checked

__device__ __forceinline__ uint64_t global_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}

// Every wait in the library's kernels is bounded: after kWaitLimitNs without
// progress (never reached by a correct launch) the waiting thread records
// kStatusTimeout in the kernel's status word and the kernel winds down.
constexpr uint64_t kWaitLimitNs = 2000000000ull;  // 2 s
constexpr unsigned kStatusTimeout = 1u;

// Bounded parity wait; returns false (and raises *abort) on timeout or if
// another thread of the CTA already aborted.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, volatile int* abort, unsigned* status) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = global_ns();
    for (;;) {
        if (mbar_try_wait_suspend(bar, parity, kSuspendHintNs)) return true;
        if (*abort) return false;
        if (global_ns() - t0 > kWaitLimitNs) {
            *abort = 1;
            atomicOr(status, kStatusTimeout);
            return false;
        }
    }
}

__device__ __forceinline__ uint64_t l2_evict_first_policy() {
    uint64_t pol;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
    return pol;
}

// 1-D bulk copy global -> this CTA's shared memory, completing on `bar`.
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar, uint64_t pol) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(dst),
        "l"(src), "r"(bytes), "r"(bar), "l"(pol)
        : "memory");
}

__device__ __forceinline__ void bulk_g2s_nohint(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
                 "l"(src), "r"(bytes), "r"(bar)
                 : "memory");
}

// 2-D tiled TMA load into this CTA's shared memory, completing on `bar`.
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int x, int y, uint32_t bar,
                                            uint64_t pol) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
        " [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar), "l"(pol)
        : "memory");
}

// Bring a 2-D tile of `map` into L2 without staging it anywhere: no shared
// memory, no barrier, nothing to wait for (a later TMA load of the same tile
// then reads L2 instead of HBM).
__device__ __forceinline__ void tma_prefetch_l2_2d(const CUtensorMap* map, int x, int y) {
    asm volatile("cp.async.bulk.prefetch.tensor.2d.L2.global.tile [%0, {%1, %2}];" ::"l"(reinterpret_cast<uint64_t>(map)),
                 "r"(x), "r"(y)
                 : "memory");
}

// Bring `bytes` (a multiple of 16, 16-byte aligned address) of global memory into L2.
__device__ __forceinline__ void bulk_prefetch_l2(const void* p, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(reinterpret_cast<uint64_t>(p)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void prefetch_tensor_map(const CUtensorMap* map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

__device__ __forceinline__ void named_bar_sync(int id, int nthreads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// Split-K arrival: one atomic add that releases this CTA's partials (stored by
// its threads before a CTA barrier) and, for the last arriver, acquires the
// other CTAs'.  Returns the old count.
__device__ __forceinline__ unsigned atom_add_acq_rel_gpu(unsigned* p, unsigned v) {
    unsigned old;
    asm volatile("atom.add.acq_rel.gpu.global.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
    return old;
}
// Count published with release semantics, without waiting for the old value.
__device__ __forceinline__ void red_add_release_gpu(unsigned* p, unsigned v) {
    asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Programmatic dependent launch controls (no-ops when launched without the attribute).
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

}  // namespace g4b
