// Host-side launch helpers shared by the op-level ABI and the model engine.
#pragma once
#include <cuda_runtime.h>

#include <cstdio>
#include <string>
#include <vector>

#include "attention.cuh"
#include "gemm_tc.cuh"
#include "matmul.cuh"
#include "rowops.cuh"

// Seeded generator state of gtn_sample_topk (std::mt19937 restated on the device).
struct gtn_rng {
    uint32_t* state = nullptr;  // device: 624 words, then the index of the next output
    int device = 0;
};

namespace gtn {

void set_error(const std::string& msg);
int fail(int code, const char* fmt, ...);

// Number of kernels this library has launched in the process (gtn_kernel_launches).
void count_launch();

// Launches `kern` with programmatic dependent launch enabled (the kernel may start while the
// previous kernel in the stream finishes; it calls griddepcontrol.wait before reading its inputs).
template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                              Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    count_launch();
    return cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...);
}

// launch_pdl for a kernel launched as thread-block clusters of `cx` CTAs along x.
template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl_cluster(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                                      int cx, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = cx;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    count_launch();
    return cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...);
}

// True when `kern` on the current device has not yet been allowed `smem` bytes of dynamic shared
// memory (records the new maximum).
bool smem_attr_needed(const void* kern, size_t smem);

template <typename K>
inline cudaError_t ensure_smem(K kern, size_t smem) {
    if (smem <= 48 * 1024) return cudaSuccess;
    if (!smem_attr_needed(reinterpret_cast<const void*>(kern), smem)) return cudaSuccess;
    return cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
}

// Destination of one top-k draw (csrc/sample.cu): `out[0]` when out is set; when tok is set, the
// decode loop's bookkeeping of k_fargmax (the id becomes token pos[0] + 1 of tok and gen, pos[0]
// advances; at the end of the token rows bit 4 of *err is set instead).
struct SampleDst {
    int32_t* out = nullptr;
    int32_t* tok = nullptr;
    int32_t* gen = nullptr;
    int* pos = nullptr;
    int max_ctx = 0;
    unsigned int* err = nullptr;
};

// One top-k / temperature draw from n fp32 logits with the MT19937 state `mt` (k and temp already
// clamped and checked). Launched with programmatic dependent launch; counts one launch.
cudaError_t launch_topk_sample(cudaStream_t st, const float* logits, int n, float temp, int k, uint32_t* mt,
                               SampleDst dst);
// Sets the sampler's shared memory limit for n logits (outside stream capture; idempotent).
cudaError_t prepare_topk_sample(int n);

// Device error word written by kernels whose bounded waits expired (GTN_DEVERR_*).
unsigned int* device_error_word();
// Reads and clears the device error word (synchronous).
unsigned int take_device_error();

// fp32 matmul core used by both layers: Y[M, N] (row stride ldy floats) = X[M, K] . W[N, K]^T.
// xdt/wdt: (Q8, Q8), (Q8, Q4) or (F16, F16). Returns a cudaError_t.
// `padded`: W is 16-byte aligned and its allocation extends at least 16 bytes past the last row
// (the engine's arena guarantees it). Otherwise rows whose TMA tiles could leave the buffer are
// computed by the plain-load kernel, so no byte outside W is ever read.
// `tc`: device scratch for the tensor-core GEMM's expanded activation image (k_tc_expand); without
// it (or when it holds less than one 32-row tile) the CUDA-core kernels run. Larger M are done in
// passes of as many row tiles as the scratch holds.
struct TcScratch {
    uint8_t* p = nullptr;
    size_t bytes = 0;
};
cudaError_t matmul_f32(const uint8_t* X, long x_stride, int xdt, int M, const uint8_t* W, long w_stride, int wdt,
                       int N, int K, float* Y, long ldy, cudaStream_t st, bool padded = true,
                       const TcScratch& tc = TcScratch());

// Two-phase GEMV (k_gemv2) for M <= 4 activation rows of Q8 against Q8 or Q4 weights, with the
// same `padded` precondition on W as matmul_f32. `dry` only configures shared memory (so that a
// later launch can be captured into a CUDA graph). gemv_q_fits says whether a shape is supported.
constexpr size_t GV2_SMEM_LIMIT = 200 * 1024;
bool gemv_q_fits(int M, int wdt, int K);
cudaError_t gemv_q(const uint8_t* X, long xs, int M, const uint8_t* W, long ws, int wdt, int N, int K, float* Y,
                   long ldy, cudaStream_t st, bool dry);

// Exact fp16 x fp16 matmul (k_mm_f16, the reference's 8-lane order) for M activation rows; W 16-byte
// aligned with the `padded` precondition of matmul_f32. `dry` only configures shared memory.
cudaError_t gemm_f16(const uint8_t* X, long xs, int M, const uint8_t* W, long ws, int N, int K, float* Y, long ldy,
                     cudaStream_t st, bool dry);

// Exact GEMM for M >= 2 activation rows of Q8 against Q8 or Q4 weights (16-byte aligned weight
// rows, same `padded` precondition): the tensor-core kernel k_gemm_tc from TC_MIN_M rows on when
// `tc` scratch is given, else the persistent CUDA-core kernel k_gemm4 (k_gemm3 where its plan does
// not fit); `dry` only configures shared memory and prepares the weight tensor map (so that a later
// launch can be captured into a CUDA graph). From 16 rows the tensor-core kernel: in isolation
// k_gemm4 is faster on TinyLlama's shapes at 16 rows, but the graph-replayed decode steps of 16
// sequences are faster on the tensor cores (MiniCPM-2B Q8 7.3 ms vs 8.5 ms, TinyLlama Q8 and
// StableLM-2 Q4 by 1 % and 9 %).
constexpr int TC_MIN_M = 16;
bool gemm_q_fits(const uint8_t* W, long ws, int M, int wdt, int K, const TcScratch& tc = TcScratch());
cudaError_t gemm_q(const uint8_t* X, long xs, int M, const uint8_t* W, long ws, int wdt, int N, int K, float* Y,
                   long ldy, cudaStream_t st, bool dry, const TcScratch& tc = TcScratch());
// Whether matmul_f32 / gemm_q take the tensor-core path for this shape given scratch `tc`.
bool tc_fits(const uint8_t* W, long ws, int M, int wdt, int K, const TcScratch& tc);

// Checked arguments of matmul_2d (ops.cpp:617-636) in byte terms: rows [start_pos, n_ctx) of x
// (M rows from X, stride xs bytes), w [N, K] (stride ws), out (data, row stride os; 0 for a 1-D out).
struct MatmulArgs {
    bool quant, one_d;
    int M, N, K, xdt, wdt, odt;
    const uint8_t* X;
    const uint8_t* W;
    uint8_t* out;
    long xs, ws, os;
};
// The argument checks of gtn_matmul_2d (shapes, dtypes, start_pos, quantized row overlap); returns
// GTN_OK or GTN_ERR_ARG with the message prefixed by `who`.
int matmul_args(const gtn_tensor* x, const gtn_tensor* w, const gtn_tensor* out, int start_pos, const char* who,
                MatmulArgs* a);

// Host table of (cos, sin) for positions [0, npos) and j < rd/2, as rotary_emb_impl computes them
// (ops.cpp:791-812): theta = m * powf(10000, -((2j)/rd)), then cosf / sinf.
std::vector<float2> rope_table_host(int npos, int rd);

}  // namespace gtn
