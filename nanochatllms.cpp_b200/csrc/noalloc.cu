// gtn_matmul_2d_noalloc: the matmul_2d operator for callers that must not allocate device memory.
//
// Who needs it: code that runs where cudaMalloc / cudaMallocAsync are off limits — a host that
// owns a fixed device-memory budget and hands every byte out itself (an embedding runtime, an
// inference server with a preallocated pool), code running inside a memory-pool or allocator
// callback where allocating again would re-enter the allocator, and latency-critical paths that
// cannot afford an allocation's possible implicit synchronization. gtn_matmul_2d stages its fp32
// dot products in stream-ordered device scratch (cudaMallocAsync); this variant stages them in a
// fixed array that lives in the library itself instead.
//
// The scratch is a file-scope __device__ array of NOALLOC_MAX_FLOATS floats (8 MiB): every GPU
// that loads this library holds it until the process exits. Host code cannot use the array's
// name as a device address (on the host it only names a host-side shadow), so the device
// address is looked up with cudaGetSymbolAddress, with that device current, on the first call
// made on each device; make that first call before any stream capture. The address is kept per
// CUDA context: if the device's primary context is destroyed and created again (cudaDeviceReset),
// the module is loaded anew and the next call looks the address up again.
// All calls share the one array and it keeps the last call's contents: each call writes every
// scratch element it reads, so nothing needs clearing, but calls that overlap on the GPU (on
// different streams, or from different host threads without ordering) race on it.
#include <cstdarg>
#include <mutex>

#include "launch.cuh"

namespace gtn {

constexpr long NOALLOC_MAX_FLOATS = 1L << 21;  // 8 MiB of fp32 staging: M * n_out <= 2,097,152

static __device__ __align__(256) float g_noalloc_scratch[NOALLOC_MAX_FLOATS];

static int noalloc_fail(int code, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    return fail(code, "%s", buf);
}

// The driver's current context, reached through the runtime's driver entry point (no link to
// libcuda needed); nullptr if the entry point is unavailable.
typedef int (*CtxGetCurrentFn)(void**);
static void* current_context() {
    static CtxGetCurrentFn fn = [] {
        void* f = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &f, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            f = nullptr;
        return reinterpret_cast<CtxGetCurrentFn>(f);
    }();
    void* ctx = nullptr;
    if (fn && fn(&ctx) != 0) ctx = nullptr;
    return ctx;
}

// Device address of g_noalloc_scratch on the current device, looked up with that device current
// the first time a call runs on it (and again if the device's context has changed since).
static float* noalloc_scratch(int* rc) {
    static std::mutex mu;
    static float* addr[128] = {};
    static void* ctx_of[128] = {};
    int dev = -1;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess || dev < 0 || dev >= 128) {
        *rc = noalloc_fail(GTN_ERR_CUDA, "matmul_2d_noalloc: no usable current device (%s)", cudaGetErrorString(e));
        return nullptr;
    }
    std::lock_guard<std::mutex> lk(mu);
    void* ctx = current_context();
    if (!addr[dev] || ctx != ctx_of[dev]) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess || !p) {
            *rc = noalloc_fail(GTN_ERR_CUDA, "matmul_2d_noalloc: cudaGetSymbolAddress failed on device %d: %s", dev,
                               cudaGetErrorString(e));
            return nullptr;
        }
        addr[dev] = static_cast<float*>(p);
        ctx_of[dev] = current_context();  // the lookup makes the primary context current if none was
    }
    *rc = GTN_OK;
    return addr[dev];
}

}  // namespace gtn

using namespace gtn;

extern "C" int gtn_matmul_2d_noalloc(const gtn_tensor* x, const gtn_tensor* w, gtn_tensor* out, int start_pos,
                                     void* stream) {
    MatmulArgs a;
    const int arc = matmul_args(x, w, out, start_pos, "matmul_2d_noalloc", &a);
    if (arc != GTN_OK) return arc;
    const int M = a.M, N = a.N, K = a.K;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    cudaError_t e;
    if (a.odt == GTN_F32) {  // written directly, no staging needed
        float* Y = (float*)(a.out + (long)start_pos * a.os);
        e = matmul_f32(a.X, a.xs, a.xdt, M, a.W, a.ws, a.wdt, N, K, Y, a.one_d ? 0 : N, st, false);
    } else {
        if ((long)M * N > NOALLOC_MAX_FLOATS)
            return noalloc_fail(GTN_ERR_ARG,
                                "matmul_2d_noalloc: %d rows x %d outputs need %ld staging floats; the fixed scratch "
                                "holds %ld (use gtn_matmul_2d, or fewer rows per call)",
                                M, N, (long)M * N, NOALLOC_MAX_FLOATS);
        int rc = GTN_OK;
        float* Y = noalloc_scratch(&rc);
        if (!Y) return rc;
        e = matmul_f32(a.X, a.xs, a.xdt, M, a.W, a.ws, a.wdt, N, K, Y, N, st, false);
        if (e == cudaSuccess)
            e = launch_pdl(k_write_rows, dim3(((N + GTN_QBLK - 1) / GTN_QBLK + 3) / 4, M), dim3(128), 0, st,
                           (const float*)Y, (long)N, a.out, a.os, a.odt, N, start_pos);
    }
    if (e != cudaSuccess) return noalloc_fail(GTN_ERR_CUDA, "matmul_2d_noalloc: %s", cudaGetErrorString(e));
    return GTN_OK;
}
