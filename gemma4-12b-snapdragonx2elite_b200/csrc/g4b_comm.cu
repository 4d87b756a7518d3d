// g4b_comm.cu -- the per-layer all-reduce of a tensor-parallel decode, over
// NVLink peer memory.
//
// After the row-parallel o and down GEMVs every rank holds a partial hidden
// state (3840 f32 = 15 KB) that the ranks must sum: the cross-GPU counterpart
// of vk/reduce.comp:8-12.  At this size a collective is pure latency, so one
// kernel does it in one shot:
//   1. every rank stores its partial into slot [rank] of every rank's exchange
//      buffer (plain P2P stores over NVLink; the buffers are CUDA-IPC mapped);
//   2. a system-scope fence, then a release store of the call's epoch into
//      flag [rank] of every rank's buffer;
//   3. each rank waits (bounded) until all `world` flags of its own buffer
//      carry the epoch, and
//   4. adds the `world` slots in rank order -- every rank gets the same bits.
// Two buffer halves alternate by epoch parity: a rank can be at most one call
// ahead of any other (it cannot pass call e+1 before every rank has finished
// call e), so it never overwrites a half that a peer is still reading.
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

constexpr int kArThreads = 512;
constexpr int kArMaxWorld = 8;

// Exchange buffer of one rank: [2 halves][world][n] f32 slots, then [2][world]
// u32 flags (16-byte aligned).
__host__ __device__ inline size_t ar_slots_bytes(int world, int n) {
    return (((size_t)2 * world * n * sizeof(float)) + 15) & ~(size_t)15;
}

__device__ __forceinline__ void st_release_sys(unsigned* p, unsigned v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__global__ void __launch_bounds__(kArThreads) allreduce_f32_kernel(const float* x, float* y, int n,
                                                                  int rank, int world, void* const* bufs,
                                                                  unsigned* counter) {
    __shared__ unsigned s_epoch;
    __shared__ int s_ok;
    const int tid = threadIdx.x;
    if (tid == 0) {
        s_epoch = *counter + 1u;
        s_ok = 1;
    }
    __syncthreads();
    const unsigned epoch = s_epoch;
    const int half = (int)(epoch & 1u);
    const size_t sb = ar_slots_bytes(world, n);
    // 1. this rank's partial into slot [rank] of every rank's buffer (vectorised when n % 4 == 0)
    for (int p = 0; p < world; p++) {
        float* dst = reinterpret_cast<float*>(bufs[p]) + ((size_t)half * world + rank) * n;
        if ((n & 3) == 0) {
            const float4* s4 = reinterpret_cast<const float4*>(x);
            float4* d4 = reinterpret_cast<float4*>(dst);
            for (int i = tid; i < n / 4; i += kArThreads) d4[i] = s4[i];
        } else {
            for (int i = tid; i < n; i += kArThreads) dst[i] = x[i];
        }
    }
    __threadfence_system();  // each thread's stores, at system scope
    __syncthreads();
    // 2. publish: raise this rank's flag in every rank's buffer (release, system scope)
    if (tid == 0) {
        for (int p = 0; p < world; p++) {
            unsigned* flags = reinterpret_cast<unsigned*>(reinterpret_cast<uint8_t*>(bufs[p]) + sb);
            st_release_sys(flags + half * world + rank, epoch);
        }
    }
    // 3. wait for every rank's flag in this rank's own buffer (bounded)
    if (tid < world) {
        const unsigned* flags = reinterpret_cast<const unsigned*>(reinterpret_cast<const uint8_t*>(bufs[rank]) + sb);
        const unsigned* f = flags + half * world + tid;
        if (ld_acquire_sys(f) != epoch) {
            const uint64_t t0 = global_ns();
            while (ld_acquire_sys(f) != epoch) {
                if (global_ns() - t0 > kWaitLimitNs) {
                    atomicOr(&g_comm_status, kStatusTimeout);
                    s_ok = 0;
                    break;
                }
                __nanosleep(64);
            }
        }
    }
    __syncthreads();
    // 4. sum the slots in rank order (identical on every rank)
    if (s_ok) {
        const float* mine = reinterpret_cast<const float*>(bufs[rank]) + (size_t)half * world * n;
        for (int i = tid; i < n; i += kArThreads) {
            float v = 0.f;
            for (int r = 0; r < world; r++) v += __ldcv(mine + (size_t)r * n + i);
            y[i] = v;
        }
    }
    __syncthreads();
    if (tid == 0) *counter = epoch;
}

}  // namespace g4b

using namespace g4b;

extern "C" {

size_t g4b_allreduce_buffer_bytes(int world, int n) {
    if (world < 1 || world > kArMaxWorld || n < 1) return 0;
    return ar_slots_bytes(world, n) + (size_t)2 * world * sizeof(unsigned);
}

int g4b_allreduce_f32(const float* x, float* y, int n, int rank, int world, void* const* bufs_dev, unsigned* counter,
                      g4b_stream_t stream) {
    G4B_ENTRY("allreduce_f32");
    G4B_REQUIRE(x && y && bufs_dev && counter, G4B_E_ARG, "allreduce_f32: NULL pointer");
    G4B_REQUIRE(world >= 1 && world <= kArMaxWorld && rank >= 0 && rank < world, G4B_E_ARG,
                "allreduce_f32: rank %d / world %d (1..%d ranks)", rank, world, kArMaxWorld);
    G4B_REQUIRE(n >= 1 && n <= (1 << 24), G4B_E_SHAPE, "allreduce_f32: n=%d", n);
    G4B_REQUIRE(aligned16(x) && aligned16(y), G4B_E_ALIGN, "allreduce_f32: x and y must be 16-byte aligned");
    int st = check_device(nullptr);
    if (st != G4B_OK) return st;
    allreduce_f32_kernel<<<1, kArThreads, 0, reinterpret_cast<cudaStream_t>(stream)>>>(x, y, n, rank, world, bufs_dev,
                                                                                       counter);
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
