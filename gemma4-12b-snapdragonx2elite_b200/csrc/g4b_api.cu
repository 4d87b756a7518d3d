// g4b_api.cu -- library-wide entry points and host plumbing: last-error
// reporting, the host-side fault injector, device checks and the bounded
// stream wait.
#include <atomic>
#include <chrono>
#include <cstdarg>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>
#include <thread>
#include <unordered_map>
#include <vector>

#include <cudaTypedefs.h>

#include "g4b_common.cuh"

#define G4B_VERSION_CODE 100  // 0.1.0

namespace g4b {

static thread_local char t_last_error[512] = {0};
static std::atomic<long long> g_launches{0};

int fail(int code, const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(t_last_error, sizeof(t_last_error), fmt, ap);
    va_end(ap);
    return code;
}

void clear_error() { t_last_error[0] = 0; }

void count_launch(int n) { g_launches.fetch_add(n, std::memory_order_relaxed); }

int launch_status(const char* op) {
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return fail(G4B_E_CUDA, "%s: launch failed: %s", op, cudaGetErrorString(e));
    return G4B_OK;
}

// ------------------------------------------------------------- fault injector
struct FaultRule {
    std::string op;
    long long nth;
    std::atomic<long long> seen{0};
};
static std::once_flag g_fault_once;
static std::vector<FaultRule*> g_fault_rules;
static std::atomic<long long> g_fault_calls{0};

static void parse_faults() {
    const char* env = std::getenv("G4B_FAULT");
    if (!env || !*env) return;
    std::string s(env);
    size_t pos = 0;
    while (pos < s.size()) {
        size_t comma = s.find(',', pos);
        std::string item = s.substr(pos, comma == std::string::npos ? std::string::npos : comma - pos);
        size_t colon = item.find(':');
        if (colon != std::string::npos) {
            auto* r = new FaultRule();
            r->op = item.substr(0, colon);
            r->nth = std::atoll(item.c_str() + colon + 1);
            if (r->nth > 0) g_fault_rules.push_back(r); else delete r;
        }
        if (comma == std::string::npos) break;
        pos = comma + 1;
    }
}

bool fault_hit(const char* op) {
    std::call_once(g_fault_once, parse_faults);
    if (g_fault_rules.empty()) return false;
    g_fault_calls.fetch_add(1, std::memory_order_relaxed);
    for (FaultRule* r : g_fault_rules) {
        if (r->op == op || r->op == "*") {
            long long n = r->seen.fetch_add(1) + 1;
            if (n == r->nth) return true;
        }
    }
    return false;
}

// --------------------------------------------------------------- device check
static int g_dev_ok[128];     // 0 unknown, 1 ok, -1 not ok
static int g_dev_sms[128];

int check_device(int* sm_count) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return fail(G4B_E_CUDA, "cudaGetDevice: %s", cudaGetErrorString(e));
    if (dev < 0 || dev >= 128) return fail(G4B_E_ARCH, "device index %d out of range", dev);
    if (g_dev_ok[dev] == 0) {
        int major = 0, minor = 0, sms = 0;
        if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess ||
            cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev) != cudaSuccess ||
            cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) {
            return fail(G4B_E_CUDA, "cudaDeviceGetAttribute failed: %s", cudaGetErrorString(cudaGetLastError()));
        }
        g_dev_sms[dev] = sms;
        g_dev_ok[dev] = (major == 10 && minor == 0) ? 1 : -1;
        if (g_dev_ok[dev] < 0)
            return fail(G4B_E_ARCH, "device %d is sm_%d%d; this library is built for sm_100a only", dev, major, minor);
    }
    if (g_dev_ok[dev] < 0) return fail(G4B_E_ARCH, "device %d is not an sm_100 GPU", dev);
    if (sm_count) *sm_count = g_dev_sms[dev];
    return G4B_OK;
}

// ------------------------------------------------------------- tensor maps
struct TmapKey {
    uintptr_t base;
    uint64_t dim0, dim1, stride1;
    uint32_t box0, box1, dtype, swizzle, promo;
    bool operator==(const TmapKey& o) const {
        return base == o.base && dim0 == o.dim0 && dim1 == o.dim1 && stride1 == o.stride1 && box0 == o.box0 &&
               box1 == o.box1 && dtype == o.dtype && swizzle == o.swizzle && promo == o.promo;
    }
};
struct TmapKeyHash {
    size_t operator()(const TmapKey& k) const {
        size_t h = std::hash<uint64_t>()(k.base);
        for (uint64_t v : {k.dim0, k.dim1, k.stride1, (uint64_t)k.box0 << 32 | k.box1, (uint64_t)k.dtype << 16 | k.swizzle << 8 | k.promo})
            h = h * 1000003u ^ std::hash<uint64_t>()(v);
        return h;
    }
};
static std::mutex g_tmap_mu;
static std::unordered_map<TmapKey, CUtensorMap, TmapKeyHash> g_tmaps;
static PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;

int tensor_map_2d(CUtensorMap* out, CUtensorMapDataType dtype, const void* base, uint64_t dim0, uint64_t dim1,
                  uint64_t stride1_bytes, uint32_t box0, uint32_t box1, CUtensorMapSwizzle swizzle,
                  CUtensorMapL2promotion promo) {
    TmapKey key{(uintptr_t)base, dim0, dim1, stride1_bytes, box0, box1, (uint32_t)dtype, (uint32_t)swizzle,
                (uint32_t)promo};
    std::lock_guard<std::mutex> lk(g_tmap_mu);
    auto it = g_tmaps.find(key);
    if (it != g_tmaps.end()) {
        *out = it->second;
        return G4B_OK;
    }
    if (!g_encode) {
        void* fn = nullptr;
        cudaDriverEntryPointQueryResult q{};
        cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q);
        if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || !fn)
            return fail(G4B_E_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
        g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    }
    const cuuint64_t dims[2] = {dim0, dim1};
    const cuuint64_t strides[1] = {stride1_bytes};
    const cuuint32_t box[2] = {box0, box1};
    const cuuint32_t estr[2] = {1, 1};
    CUtensorMap m;
    CUresult r = g_encode(&m, dtype, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                          swizzle, promo, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(G4B_E_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
    if (g_tmaps.size() > 8192) g_tmaps.clear();
    g_tmaps.emplace(key, m);
    *out = m;
    return G4B_OK;
}

}  // namespace g4b

extern "C" {

const char* g4b_last_error(void) { return g4b::t_last_error; }

int g4b_version(void) { return G4B_VERSION_CODE; }

long long g4b_query(int what) {
    switch (what) {
        case G4B_Q_VERSION: return G4B_VERSION_CODE;
        case G4B_Q_DEVICE_OK: return g4b::check_device(nullptr) == G4B_OK ? 1 : 0;
        case G4B_Q_SM_COUNT: {
            int sms = 0;
            return g4b::check_device(&sms) == G4B_OK ? sms : -1;
        }
        case G4B_Q_LAUNCHES: return g4b::g_launches.load();
        case G4B_Q_FAULT_COUNTER: return g4b::g_fault_calls.load();
        case G4B_Q_KERNEL_STATUS: {
            if (g4b::check_device(nullptr) != G4B_OK) return -1;
            return (long long)(g4b::read_status_gemv() | g4b::read_status_gemm() | g4b::read_status_comm());
        }
        default: return -1;
    }
}

int g4b_stream_wait(g4b_stream_t stream, int timeout_ms) {
    G4B_ENTRY("stream_wait");
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    auto t0 = std::chrono::steady_clock::now();
    for (;;) {
        cudaError_t e = cudaStreamQuery(s);
        if (e == cudaSuccess) return G4B_OK;
        if (e != cudaErrorNotReady)
            return g4b::fail(G4B_E_CUDA, "stream_wait: %s", cudaGetErrorString(e));
        if (timeout_ms > 0) {
            auto ms = std::chrono::duration_cast<std::chrono::milliseconds>(
                          std::chrono::steady_clock::now() - t0).count();
            if (ms >= timeout_ms)
                return g4b::fail(G4B_E_TIMEOUT, "stream_wait: GPU work still running after %d ms", timeout_ms);
        }
        std::this_thread::sleep_for(std::chrono::microseconds(50));
    }
}

}  // extern "C"
