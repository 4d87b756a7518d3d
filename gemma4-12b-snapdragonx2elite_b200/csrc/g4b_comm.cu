// g4b_comm.cu -- the per-layer all-reduce of a tensor-parallel decode, over
// NVLink peer memory.
//
// After the row-parallel o and down GEMVs every rank holds a partial hidden
// state (3840 f32 = 15 KB) that the ranks must sum: the cross-GPU counterpart
// of vk/reduce.comp:8-12.  At this size a collective is pure latency, so one
// small kernel does it in one shot, with no fence and no separate flag:
//   1. every rank stores each element of its partial, paired with the call's
//      epoch in one 64-bit word {f32 bits, epoch}, into slot [rank] of every
//      rank's exchange buffer (plain P2P stores over NVLink into CUDA-IPC
//      mapped buffers).  A 64-bit aligned store is single-copy atomic, so a
//      reader that sees the epoch also sees the value that came with it;
//   2. each thread polls its own elements of all `world` slots in its own
//      buffer until every word carries the epoch (bounded), and
//   3. adds the slots in rank order -- every rank gets the same bits.
// Two buffer halves alternate by epoch parity.  A rank can be at most one call
// ahead of any other: it cannot finish call e before every rank has started
// call e, and a rank starts call e only after its call e-1 kernel finished
// (the kernel waits for its predecessor in the stream before it stores
// anything), so no rank overwrites a half that a peer is still reading.
// With programmatic dependent launch the next kernel in the stream may start
// (and e.g. prefetch weights) while this one waits for the peers.
// No multicast object, no TMA: only ordinary loads and stores to peer memory.
#include <cstring>

#include "g4b_common.cuh"

namespace g4b {

static __device__ unsigned g_comm_status;

unsigned read_status_comm() {
    unsigned v = 0, z = 0;
    if (cudaMemcpyFromSymbol(&v, g_comm_status, sizeof(v)) != cudaSuccess) return 0xffffffffu;
    if (v) cudaMemcpyToSymbol(g_comm_status, &z, sizeof(z));
    return v;
}

constexpr int kArThreads = 256;  // small enough to share an SM with a GEMV CTA
constexpr int kArMaxWorld = 8;

// Exchange buffer of one rank: [2 halves][world][n] 64-bit words {f32, epoch}.
__host__ __device__ inline size_t ar_buffer_bytes(int world, int n) {
    return (size_t)2 * world * n * sizeof(unsigned long long);
}

__device__ __forceinline__ void st_relaxed_sys_u64(unsigned long long* p, unsigned long long v) {
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_relaxed_sys_u64(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

__global__ void __launch_bounds__(kArThreads) allreduce_f32_kernel(const float* x, float* y, int n, int rank,
                                                                  int world, void* const* bufs, unsigned* counter) {
    const int tid = threadIdx.x;
    pdl_wait();  // x is the previous kernel's output; nothing is stored before it completed
    const unsigned epoch = *counter + 1u;
    const int half = (int)(epoch & 1u);
    const unsigned long long tag = (unsigned long long)epoch << 32;
    // 1. this rank's partial, tagged, into slot [rank] of every rank's buffer
    for (int i = tid; i < n; i += kArThreads) {
        const unsigned long long w = tag | __float_as_uint(x[i]);
        for (int p = 0; p < world; p++) {
            unsigned long long* dst = reinterpret_cast<unsigned long long*>(bufs[p]) + ((size_t)half * world + rank) * n;
            st_relaxed_sys_u64(dst + i, w);
        }
    }
    pdl_launch_dependents();
    __syncthreads();
    // 2-3. poll this rank's own buffer until every slot of this thread's elements
    // carries the epoch (bounded), and sum in rank order.  A chunk's words are
    // all loaded at once (one round trip); only words still without the epoch
    // are loaded again.
    const unsigned long long* mine = reinterpret_cast<const unsigned long long*>(bufs[rank]) + (size_t)half * world * n;
    constexpr int kChunk = 8;  // elements per thread per round trip
    uint64_t t0 = 0;
    bool ok = true;
    for (int i0 = tid; i0 < n && ok; i0 += kChunk * kArThreads) {
        float v[kChunk];
        #pragma unroll
        for (int e = 0; e < kChunk; e++) v[e] = 0.f;
        for (int r = 0; r < world && ok; r++) {
            const unsigned long long* src = mine + (size_t)r * n;
            unsigned long long w[kChunk];
            #pragma unroll
            for (int e = 0; e < kChunk; e++) {
                const int i = i0 + e * kArThreads;
                w[e] = i < n ? ld_relaxed_sys_u64(src + i) : tag;
            }
            for (;;) {
                bool all = true;
                #pragma unroll
                for (int e = 0; e < kChunk; e++) all = all && (unsigned)(w[e] >> 32) == epoch;
                if (all) break;
                if (t0 == 0) t0 = global_ns();
                if (global_ns() - t0 > kWaitLimitNs) {
                    atomicOr(&g_comm_status, kStatusTimeout);
                    ok = false;
                    break;
                }
                __nanosleep(32);
                #pragma unroll
                for (int e = 0; e < kChunk; e++) {
                    const int i = i0 + e * kArThreads;
                    if ((unsigned)(w[e] >> 32) != epoch && i < n) w[e] = ld_relaxed_sys_u64(src + i);
                }
            }
            #pragma unroll
            for (int e = 0; e < kChunk; e++) v[e] += __uint_as_float((unsigned)w[e]);
        }
        if (ok) {
            #pragma unroll
            for (int e = 0; e < kChunk; e++) {
                const int i = i0 + e * kArThreads;
                if (i < n) y[i] = v[e];
            }
        }
    }
    __syncthreads();
    if (tid == 0) *counter = epoch;  // the next call's epoch, also after a timeout
}

}  // namespace g4b

using namespace g4b;

extern "C" {

size_t g4b_allreduce_buffer_bytes(int world, int n) {
    if (world < 1 || world > kArMaxWorld || n < 1 || n > (1 << 24)) return 0;
    return ar_buffer_bytes(world, n);
}

int g4b_allreduce_f32(const float* x, float* y, int n, int rank, int world, void* const* bufs_dev, unsigned* counter,
                      unsigned flags, g4b_stream_t stream) {
    G4B_ENTRY("allreduce_f32");
    G4B_REQUIRE((flags & ~(unsigned)G4B_GEMV_PDL) == 0, G4B_E_ARG, "allreduce_f32: unknown flags 0x%x", flags);
    G4B_REQUIRE(x && y && bufs_dev && counter, G4B_E_ARG, "allreduce_f32: NULL pointer");
    G4B_REQUIRE(world >= 1 && world <= kArMaxWorld && rank >= 0 && rank < world, G4B_E_ARG,
                "allreduce_f32: rank %d / world %d (1..%d ranks)", rank, world, kArMaxWorld);
    G4B_REQUIRE(n >= 1 && n <= (1 << 24), G4B_E_SHAPE, "allreduce_f32: n=%d", n);
    G4B_REQUIRE(((uintptr_t)x & 3u) == 0 && ((uintptr_t)y & 3u) == 0, G4B_E_ALIGN,
                "allreduce_f32: x and y must be 4-byte aligned");
    int st = check_device(nullptr);
    if (st != G4B_OK) return st;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(1);
    cfg.blockDim = dim3(kArThreads);
    cfg.stream = reinterpret_cast<cudaStream_t>(stream);
    cudaLaunchAttribute attr[1];
    if (flags & G4B_GEMV_PDL) {
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
    }
    cudaError_t e = cudaLaunchKernelEx(&cfg, allreduce_f32_kernel, x, y, n, rank, world, bufs_dev, counter);
    if (e != cudaSuccess) return fail(G4B_E_CUDA, "allreduce_f32: launch: %s", cudaGetErrorString(e));
    count_launch();
    return launch_status("allreduce_f32");
}

int g4b_comm_alloc(size_t bytes, void** dptr) {
    G4B_ENTRY("comm_alloc");
    G4B_REQUIRE(dptr && bytes > 0, G4B_E_ARG, "comm_alloc: bad arguments");
    void* p = nullptr;
    cudaError_t e = cudaMalloc(&p, bytes);
    if (e != cudaSuccess) return fail(G4B_E_CUDA, "comm_alloc: cudaMalloc: %s", cudaGetErrorString(e));
    e = cudaMemset(p, 0, bytes);
    if (e != cudaSuccess) {
        cudaFree(p);
        return fail(G4B_E_CUDA, "comm_alloc: cudaMemset: %s", cudaGetErrorString(e));
    }
    *dptr = p;
    return G4B_OK;
}

int g4b_comm_free(void* dptr) {
    G4B_ENTRY("comm_free");
    cudaError_t e = cudaFree(dptr);
    return e == cudaSuccess ? G4B_OK : fail(G4B_E_CUDA, "comm_free: %s", cudaGetErrorString(e));
}

int g4b_ipc_handle(const void* dptr, void* handle_out) {
    G4B_ENTRY("ipc_handle");
    G4B_REQUIRE(dptr && handle_out, G4B_E_ARG, "ipc_handle: NULL pointer");
    cudaIpcMemHandle_t h;
    cudaError_t e = cudaIpcGetMemHandle(&h, const_cast<void*>(dptr));
    if (e != cudaSuccess) return fail(G4B_E_CUDA, "ipc_handle: %s", cudaGetErrorString(e));
    memcpy(handle_out, &h, sizeof(h));
    return G4B_OK;
}

int g4b_ipc_open(const void* handle, void** dptr) {
    G4B_ENTRY("ipc_open");
    G4B_REQUIRE(handle && dptr, G4B_E_ARG, "ipc_open: NULL pointer");
    cudaIpcMemHandle_t h;
    memcpy(&h, handle, sizeof(h));
    cudaError_t e = cudaIpcOpenMemHandle(dptr, h, cudaIpcMemLazyEnablePeerAccess);
    return e == cudaSuccess ? G4B_OK : fail(G4B_E_CUDA, "ipc_open: %s", cudaGetErrorString(e));
}

int g4b_ipc_close(void* dptr) {
    G4B_ENTRY("ipc_close");
    cudaError_t e = cudaIpcCloseMemHandle(dptr);
    return e == cudaSuccess ? G4B_OK : fail(G4B_E_CUDA, "ipc_close: %s", cudaGetErrorString(e));
}

}  // extern "C"
