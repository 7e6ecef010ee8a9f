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
// address is looked up once per device with cudaGetSymbolAddress, with that device current,
// on the first call made on that device; make that first call before any stream capture.
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

// Device address of g_noalloc_scratch on the current device (looked up once per device).
static float* noalloc_scratch(int* rc) {
    static std::mutex mu;
    static float* addr[128] = {};
    int dev = -1;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess || dev < 0 || dev >= 128) {
        *rc = noalloc_fail(GTN_ERR_CUDA, "matmul_2d_noalloc: no usable current device (%s)", cudaGetErrorString(e));
        return nullptr;
    }
    std::lock_guard<std::mutex> lk(mu);
    if (!addr[dev]) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess || !p) {
            *rc = noalloc_fail(GTN_ERR_CUDA, "matmul_2d_noalloc: cudaGetSymbolAddress failed on device %d: %s", dev,
                               cudaGetErrorString(e));
            return nullptr;
        }
        addr[dev] = static_cast<float*>(p);
    }
    *rc = GTN_OK;
    return addr[dev];
}

static long nb_stride(const gtn_tensor* t) {
    const long s = t->strides[0];
    switch (t->dtype) {
        case GTN_Q4: return s == 1 ? 1 : (s / GTN_QBLK) * GTN_Q4_BYTES;
        case GTN_Q8: return s == 1 ? 1 : (s / GTN_QBLK) * GTN_Q8_BYTES;
        case GTN_F16: return s * 2;
        default: return s * 4;
    }
}

}  // namespace gtn

using namespace gtn;

extern "C" int gtn_matmul_2d_noalloc(const gtn_tensor* x, const gtn_tensor* w, gtn_tensor* out, int start_pos,
                                     void* stream) {
    if (!x || !w || !out || !x->data || !w->data || !out->data)
        return noalloc_fail(GTN_ERR_ARG, "matmul_2d_noalloc: NULL tensor or data");
    if (x->ndim != 2 || w->ndim != 2 || w->shape[1] != x->shape[1])
        return noalloc_fail(GTN_ERR_ARG, "matmul_2d_noalloc: x [n_ctx, n_embd] and w [n_out, n_embd] expected");
    const int n_ctx = x->shape[0], K = x->shape[1], N = w->shape[0];
    if (n_ctx <= 0 || K <= 0 || N <= 0 || start_pos < 0 || start_pos >= n_ctx)
        return noalloc_fail(GTN_ERR_ARG, "matmul_2d_noalloc: start_pos %d out of [0, %d)", start_pos, n_ctx);
    if (out->ndim == 1) {
        if (n_ctx - start_pos != 1 || out->shape[0] != N)
            return noalloc_fail(GTN_ERR_ARG, "matmul_2d_noalloc: 1-D out needs one new row of %d", N);
    } else if (out->ndim != 2 || out->shape[0] != n_ctx || out->shape[1] != N) {
        return noalloc_fail(GTN_ERR_ARG, "matmul_2d_noalloc: out shape");
    }
    const bool q = x->dtype == GTN_Q8 && (w->dtype == GTN_Q8 || w->dtype == GTN_Q4);
    const bool h = x->dtype == GTN_F16 && w->dtype == GTN_F16;
    if (!(q || h)) return noalloc_fail(GTN_ERR_ARG, "matmul_2d_noalloc: unsupported dtypes x=%d w=%d", x->dtype, w->dtype);
    if (q && K % GTN_QBLK != 0) return noalloc_fail(GTN_ERR_ARG, "matmul_2d_noalloc: n_embd %d not a multiple of 32", K);
    if (out->dtype != GTN_F32 && out->dtype != x->dtype)
        return noalloc_fail(GTN_ERR_ARG, "matmul_2d_noalloc: out dtype");
    const int M = n_ctx - start_pos;
    if ((x->dtype == GTN_Q8 && M > 1 && K % GTN_QBLK) || (out->dtype == GTN_Q8 && n_ctx > 1 && N % GTN_QBLK))
        return noalloc_fail(GTN_ERR_ARG, "matmul_2d_noalloc: quantized rows not a multiple of 32 overlap");
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    const uint8_t* X = (const uint8_t*)x->data + (long)start_pos * nb_stride(x);
    const long os = out->ndim == 1 ? 0 : nb_stride(out);
    cudaError_t e;
    if (out->dtype == GTN_F32) {  // written directly, no staging needed
        float* Y = (float*)((uint8_t*)out->data + (long)start_pos * os);
        e = matmul_f32(X, nb_stride(x), x->dtype, M, (const uint8_t*)w->data, nb_stride(w), w->dtype, N, K, Y,
                       out->ndim == 1 ? 0 : N, st, false);
    } else {
        if ((long)M * N > NOALLOC_MAX_FLOATS)
            return noalloc_fail(GTN_ERR_ARG,
                                "matmul_2d_noalloc: %d rows x %d outputs need %ld staging floats; the fixed scratch "
                                "holds %ld (use gtn_matmul_2d, or fewer rows per call)",
                                M, N, (long)M * N, NOALLOC_MAX_FLOATS);
        int rc = GTN_OK;
        float* Y = noalloc_scratch(&rc);
        if (!Y) return rc;
        e = matmul_f32(X, nb_stride(x), x->dtype, M, (const uint8_t*)w->data, nb_stride(w), w->dtype, N, K, Y, N, st,
                       false);
        if (e == cudaSuccess)
            e = launch_pdl(k_write_rows, dim3(((N + GTN_QBLK - 1) / GTN_QBLK + 3) / 4, M), dim3(128), 0, st,
                           (const float*)Y, (long)N, (uint8_t*)out->data, os, (int)out->dtype, N, start_pos);
    }
    if (e != cudaSuccess) return noalloc_fail(GTN_ERR_CUDA, "matmul_2d_noalloc: %s", cudaGetErrorString(e));
    return GTN_OK;
}
