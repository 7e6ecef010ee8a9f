// Op-level C ABI (include/gten_b200.h): gten::ops, the packer / quantizer and the argmax.
// Argument checks mirror the reference's GTEN_ASSERTs (src/gten/ops.cpp) but return GTN_ERR_ARG.
#include <atomic>
#include <cmath>
#include <cstdarg>
#include <map>
#include <mutex>
#include <tuple>

#include "launch.cuh"

namespace gtn {

static thread_local std::string g_last_error;

void set_error(const std::string& msg) { g_last_error = msg; }

int fail(int code, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    g_last_error = buf;
    return code;
}

static int cuda_status(cudaError_t e, const char* what) {
    if (e == cudaSuccess) return GTN_OK;
    return fail(e == cudaErrorMemoryAllocation ? GTN_ERR_OOM : GTN_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

static std::atomic<unsigned long long> g_launches{0};
void count_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }

bool smem_attr_needed(const void* kern, size_t smem) {
    static std::mutex mu;
    static std::map<std::pair<const void*, int>, size_t> done;
    int dev = 0;
    cudaGetDevice(&dev);
    std::lock_guard<std::mutex> lk(mu);
    size_t& cur = done[{kern, dev}];
    if (cur >= smem) return false;
    cur = smem;
    return true;
}

__device__ unsigned int g_dev_err;

unsigned int* device_error_word() {
    static thread_local int dev_cached = -1;
    static thread_local unsigned int* p = nullptr;
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev != dev_cached) {
        p = nullptr;
        if (cudaGetSymbolAddress((void**)&p, g_dev_err) != cudaSuccess) p = nullptr;
        dev_cached = dev;
    }
    return p;
}

unsigned int take_device_error() {
    unsigned int v = 0, zero = 0;
    unsigned int* p = device_error_word();
    if (!p) return 0;
    cudaMemcpy(&v, p, sizeof v, cudaMemcpyDeviceToHost);
    if (v) cudaMemcpy(p, &zero, sizeof zero, cudaMemcpyHostToDevice);
    return v;
}

std::vector<float2> rope_table_host(int npos, int rd) {
    const int half = rd / 2;
    const float d = (float)rd;
    std::vector<float2> t((size_t)npos * (half > 0 ? half : 1));
    for (int i = 0; i < npos; ++i) {
        const float m = (float)i;
        for (int j = 0; j < half; ++j) {
            const float e = -((2.0f * (float)j) / d);
            const float th = m * powf(10000.0f, e);
            t[(size_t)i * half + j] = make_float2(cosf(th), sinf(th));
        }
    }
    return t;
}

template <int WDT, int NW>
static cudaError_t launch_mm_q(const uint8_t* X, long xs, int M, const uint8_t* W, long ws, int N, int K, float* Y,
                               long ldy, cudaStream_t st, int mt) {
    const dim3 grid((N + NW * 8 - 1) / (NW * 8), (M + mt - 1) / mt);
    const size_t smem = mm_q_smem<WDT>(NW, mt, K);
    unsigned int* err = device_error_word();
    cudaError_t e;
#define GTN_MMQ(MTV)                                                                              \
    case MTV:                                                                                     \
        e = ensure_smem(k_mm_q<WDT, NW, MTV>, smem);                                              \
        if (e != cudaSuccess) return e;                                                           \
        return launch_pdl(k_mm_q<WDT, NW, MTV>, grid, dim3(NW * 32), smem, st, W, ws, N, K, X, xs, M, Y, ldy, err);
    switch (mt) {
        GTN_MMQ(1)
        GTN_MMQ(2)
        GTN_MMQ(4)
        default:
            GTN_MMQ(8)
    }
#undef GTN_MMQ
}

template <int NW>
static cudaError_t launch_mm_f16(const uint8_t* X, long xs, int M, const uint8_t* W, long ws, int N, int K, float* Y,
                                 long ldy, cudaStream_t st, int mt, bool dry = false) {
    const dim3 grid((N + NW * 4 - 1) / (NW * 4), (M + mt - 1) / mt);
    const size_t smem = mm_f16_smem(NW, mt, K);
    unsigned int* err = device_error_word();
    cudaError_t e;
#define GTN_MMF(MTV)                                                                              \
    case MTV:                                                                                     \
        e = ensure_smem(k_mm_f16<NW, MTV>, smem);                                                 \
        if (e != cudaSuccess || dry) return e;                                                    \
        return launch_pdl(k_mm_f16<NW, MTV>, grid, dim3(NW * 32), smem, st, W, ws, N, K, X, xs, M, Y, ldy, err);
    switch (mt) {
        GTN_MMF(1)
        GTN_MMF(2)
        GTN_MMF(4)
        default:
            GTN_MMF(8)
    }
#undef GTN_MMF
}

template <int WDT>
static cudaError_t launch_plain(const uint8_t* X, long xs, int M, const uint8_t* W, long ws, int row0, int nrows,
                                int K, float* Y, long ldy, cudaStream_t st) {
    return launch_pdl(k_mm_rows_plain<WDT>, dim3(nrows, M), dim3(32), 0, st, W, ws, row0, K, X, xs, Y, ldy);
}

static cudaError_t matmul_tma(const uint8_t* X, long xs, int M, const uint8_t* W, long ws, int wdt, int N, int K,
                              float* Y, long ldy, cudaStream_t st, const TcScratch& tc);

cudaError_t matmul_f32(const uint8_t* X, long xs, int xdt, int M, const uint8_t* W, long ws, int wdt, int N, int K,
                       float* Y, long ldy, cudaStream_t st, bool padded, const TcScratch& tc) {
    (void)xdt;
    auto plain = [&](int row0, int nrows) -> cudaError_t {
        if (wdt == GTN_Q8) return launch_plain<GTN_Q8>(X, xs, M, W, ws, row0, nrows, K, Y, ldy, st);
        if (wdt == GTN_Q4) return launch_plain<GTN_Q4>(X, xs, M, W, ws, row0, nrows, K, Y, ldy, st);
        return launch_plain<GTN_F16>(X, xs, M, W, ws, row0, nrows, K, Y, ldy, st);
    };
    if (!padded) {
        if (((uintptr_t)W & 15) != 0) return plain(0, N);
        // bytes the TMA tiles cover in the last row: whole blocks (Q) or the first K/8*8 halves (fp16)
        const long covered = wdt == GTN_F16 ? (long)(K / 8) * 16 : row_bytes(wdt, K);
        const uintptr_t end = (uintptr_t)W + (uintptr_t)(N - 1) * ws + covered;
        if ((end & 15) != 0 || (ws & 15) != 0) {
            // every row but the last reads at most into the following row; the last row goes plain
            if (N > 1) {
                const cudaError_t e = matmul_tma(X, xs, M, W, ws, wdt, N - 1, K, Y, ldy, st, tc);
                if (e != cudaSuccess) return e;
            }
            return plain(N - 1, 1);
        }
    }
    return matmul_tma(X, xs, M, W, ws, wdt, N, K, Y, ldy, st, tc);
}

static int sm_count() {
    static thread_local int dev_cached = -1, n = 148;
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev != dev_cached) {
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) n = 148;
        dev_cached = dev;
    }
    return n;
}

template <int WDT, int R, int MT>
static cudaError_t launch_gv2(const uint8_t* X, long xs, int M, const uint8_t* W, long ws, int N, int K, float* Y,
                              long ldy, cudaStream_t st, bool dry) {
    const size_t smem = gv2_smem<WDT>(R, MT, K);
    const cudaError_t e = ensure_smem(k_gemv2<WDT, R, MT>, smem);
    if (e != cudaSuccess || dry) return e;
    const int ngroups = (N + R - 1) / R;
    int occ = (int)((227 * 1024) / (smem + 2048));
    occ = occ < 1 ? 1 : (occ > 4 ? 4 : occ);
    const int gx = std::min(ngroups, sm_count() * occ);
    return launch_pdl(k_gemv2<WDT, R, MT>, dim3(gx, (M + MT - 1) / MT), dim3(GV2_THREADS), smem, st, W, ws, N, K, X,
                      xs, M, Y, ldy, device_error_word());
}

// Rows per group and batch tile for the two-phase GEMV, chosen by shared memory.
template <int WDT>
static cudaError_t gemv2(const uint8_t* X, long xs, int M, const uint8_t* W, long ws, int N, int K, float* Y, long ldy,
                         cudaStream_t st, bool dry) {
    const size_t lim = GV2_SMEM_LIMIT;
#define GV(R_, MT_) return launch_gv2<WDT, R_, MT_>(X, xs, M, W, ws, N, K, Y, ldy, st, dry)
    const int mt = M <= 1 ? 1 : (M <= 2 ? 2 : 4);
    if (mt == 1) {
        if (gv2_smem<WDT>(16, 1, K) <= lim) GV(16, 1);
        GV(8, 1);
    }
    if (mt == 2) {
        if (gv2_smem<WDT>(16, 2, K) <= lim) GV(16, 2);
        if (gv2_smem<WDT>(8, 2, K) <= lim) GV(8, 2);
        GV(8, 1);
    }
    if (gv2_smem<WDT>(16, 4, K) <= lim) GV(16, 4);
    if (gv2_smem<WDT>(8, 4, K) <= lim) GV(8, 4);
    if (gv2_smem<WDT>(8, 2, K) <= lim) GV(8, 2);
    GV(8, 1);
#undef GV
}

// k_gemv2 serves one activation row where k_gemv3 does not apply; two or more go to k_gemm4.
bool gemv_q_fits(int M, int wdt, int K) {
    return M == 1 && (wdt == GTN_Q8 || wdt == GTN_Q4) && gv2_smem<GTN_Q8>(8, 1, K) <= GV2_SMEM_LIMIT;
}

// k_gemv3 plan for one activation row: rows per stage R = RP * passes (RP = rows covered by one
// pass of 256 threads), as many passes (up to 16 rows) as keep two CTAs per SM.
template <int WDT>
static bool gv3_plan(const uint8_t* W, long ws, int N, int K, int* R, int* RP) {
    const int nb = K / GTN_QBLK;
    if (K % GTN_QBLK || nb % 4 || nb / 4 > GV3_THREADS || nb == 0) return false;
    if ((reinterpret_cast<uintptr_t>(W) & 15) || (ws & 15)) return false;
    const int rp = std::min(GV3_THREADS / (nb / 4), GV3_THREADS / 4);  // phase 2: 4 threads per row
    for (int passes = std::max(1, 16 / rp); passes >= 1; --passes)
        if (gv3_smem<WDT>(rp * passes, K) <= 110 * 1024) {
            *R = rp * passes;
            *RP = rp;
            // few rows (e.g. 2048-2560): halve the group so that every SM gets two groups
            if (passes == 1 && rp >= 16 && (N + rp - 1) / rp < 2 * sm_count()) *R = *RP = rp / 2;
            return true;
        }
    return false;
}

template <int WDT>
static cudaError_t launch_gv3(const uint8_t* X, const uint8_t* W, long ws, int N, int K, float* Y, int R, int RP,
                              cudaStream_t st, bool dry) {
    const size_t smem = gv3_smem<WDT>(R, K);
    const cudaError_t e = ensure_smem(k_gemv3<WDT>, smem);
    if (e != cudaSuccess || dry) return e;
    const int ngroups = (N + R - 1) / R;
    int occ = (int)((227 * 1024) / (smem + 2048));
    occ = occ < 1 ? 1 : (occ > 2 ? 2 : occ);
    const int gx = std::min(ngroups, sm_count() * occ);
    return launch_pdl(k_gemv3<WDT>, dim3(gx), dim3(GV3_THREADS), smem, st, W, ws, N, K, X, Y, R, RP,
                      device_error_word());
}

cudaError_t gemv_q(const uint8_t* X, long xs, int M, const uint8_t* W, long ws, int wdt, int N, int K, float* Y,
                   long ldy, cudaStream_t st, bool dry) {
    int R = 0, RP = 0;
    if (M == 1 && wdt == GTN_Q8 && gv3_plan<GTN_Q8>(W, ws, N, K, &R, &RP))
        return launch_gv3<GTN_Q8>(X, W, ws, N, K, Y, R, RP, st, dry);
    if (M == 1 && wdt == GTN_Q4 && gv3_plan<GTN_Q4>(W, ws, N, K, &R, &RP))
        return launch_gv3<GTN_Q4>(X, W, ws, N, K, Y, R, RP, st, dry);
    if (wdt == GTN_Q8) return gemv2<GTN_Q8>(X, xs, M, W, ws, N, K, Y, ldy, st, dry);
    return gemv2<GTN_Q4>(X, xs, M, W, ws, N, K, Y, ldy, st, dry);
}

// k_gemm3 plan: R rows per CTA (one pass of 256 threads over the 4-block groups), MT activation
// rows per CTA, MC rows per product chunk, within 200 KB of shared memory.
template <int WDT>
static bool gm3_plan(const uint8_t* W, long ws, int M, int K, GM3Plan* p) {
    const int nb = K / GTN_QBLK;
    if (K % GTN_QBLK || nb % 4 || nb == 0 || nb / 4 > GV3_THREADS) return false;
    if ((reinterpret_cast<uintptr_t>(W) & 15) || (ws & 15)) return false;
    const int R = std::min(GV3_THREADS / (nb / 4), 64);
    // two CTAs per SM if a plan fits in 110 KB (registers allow two), else one
    for (size_t lim : {(size_t)110 * 1024, (size_t)200 * 1024})
        for (int mt = std::min(M, 16); mt >= 1; mt = mt > 1 ? mt / 2 : 0) {
            for (int mc = std::min(mt, std::max(1, GV3_THREADS / (R * 4))); mc >= 1; --mc) {
                if (gm3_smem<WDT>(R, mt, mc, K) <= lim && (mt <= 4 || mc >= 2 || lim > 110 * 1024)) {
                    p->R = R;
                    p->MT = mt;
                    p->MC = mc;
                    return true;
                }
            }
        }
    return false;
}

template <int WDT>
static cudaError_t launch_gm3(const uint8_t* X, long xs, int M, const uint8_t* W, long ws, int N, int K, float* Y,
                              long ldy, const GM3Plan& p, cudaStream_t st, bool dry = false) {
    const size_t smem = gm3_smem<WDT>(p.R, p.MT, p.MC, K);
    const cudaError_t e = ensure_smem(k_gemm3<WDT>, smem);
    if (e != cudaSuccess || dry) return e;
    return launch_pdl(k_gemm3<WDT>, dim3((N + p.R - 1) / p.R, (M + p.MT - 1) / p.MT), dim3(GV3_THREADS), smem, st, W,
                      ws, N, K, X, xs, M, Y, ldy, p.R, p.MT, p.MC, device_error_word());
}

// k_gemm4 plan: R weight rows per group (one pass of 256 threads over the 4-block groups), the
// activation tile MT (all M rows, else halves) and MC rows per product chunk, preferring two CTAs
// per SM (within 110 KB of shared memory), then one (200 KB). Rows of 128 blocks or more (K >= 4096:
// 5 weight rows per group) take one CTA per SM at once: its larger chunks give phase 2 more chains
// at a time (MiniCPM-2B's batch-8 decode step 5.10 -> 4.72 ms).
template <int WDT>
static bool gm4_plan(const uint8_t* W, long ws, int M, int K, GM4Plan* p) {
    const int nb = K / GTN_QBLK;
    if (M < 2 || K % GTN_QBLK || nb % 4 || nb == 0 || nb / 4 > GV3_THREADS) return false;
    if ((reinterpret_cast<uintptr_t>(W) & 15) || (ws & 15)) return false;
    const int R = std::min(GV3_THREADS / (nb / 4), 64);
    for (int occ = nb >= 128 ? 1 : 2; occ >= 1; --occ) {
        const size_t lim = occ == 2 ? (size_t)110 * 1024 : (size_t)200 * 1024;
        for (int tiles = 1;; tiles *= 2) {
            const int mt = (M + tiles - 1) / tiles;
            for (int mc = std::min(mt, std::max(1, GV3_THREADS / (R * 4))); mc >= 1; --mc)
                if (gm4_smem<WDT>(R, mt, mc, K) <= lim) {
                    *p = GM4Plan{R, mt, mc, occ};
                    return true;
                }
            if (mt == 1) break;
        }
    }
    return false;
}

template <int WDT>
static cudaError_t launch_gm4(const uint8_t* X, long xs, int M, const uint8_t* W, long ws, int N, int K, float* Y,
                              long ldy, const GM4Plan& p, cudaStream_t st, bool dry = false) {
    // the model shapes' 4-block groups per row (K = 2048, 2304, 5632, 5760) at compile time
    const int nbg = K / (4 * GTN_QBLK);
    auto kern = nbg == 16 ? k_gemm4<WDT, 16> : nbg == 18 ? k_gemm4<WDT, 18> : nbg == 44 ? k_gemm4<WDT, 44>
              : nbg == 45 ? k_gemm4<WDT, 45> : k_gemm4<WDT, 0>;
    const size_t smem = gm4_smem<WDT>(p.R, p.MT, p.MC, K);
    const cudaError_t e = ensure_smem(kern, smem);
    if (e != cudaSuccess || dry) return e;
    const int ngroups = (N + p.R - 1) / p.R, mtiles = (M + p.MT - 1) / p.MT;
    const int gx = std::max(1, std::min(ngroups, sm_count() * p.occ / mtiles));
    return launch_pdl(kern, dim3(gx, mtiles), dim3(GV3_THREADS), smem, st, W, ws, N, K, X, xs, M, Y, ldy, p.R, p.MT,
                      p.MC, device_error_word());
}

// The CUDA-core GEMM for M >= 2 rows: k_gemm4 where its plan fits, else k_gemm3.
template <int WDT>
static bool cc_gemm_fits(const uint8_t* W, long ws, int M, int K) {
    GM4Plan p4{};
    GM3Plan p3{};
    return gm4_plan<WDT>(W, ws, M, K, &p4) || gm3_plan<WDT>(W, ws, M, K, &p3);
}
template <int WDT>
static cudaError_t cc_gemm(const uint8_t* X, long xs, int M, const uint8_t* W, long ws, int N, int K, float* Y,
                           long ldy, cudaStream_t st, bool dry) {
    GM4Plan p4{};
    if (gm4_plan<WDT>(W, ws, M, K, &p4)) return launch_gm4<WDT>(X, xs, M, W, ws, N, K, Y, ldy, p4, st, dry);
    GM3Plan p3{};
    if (gm3_plan<WDT>(W, ws, M, K, &p3)) return launch_gm3<WDT>(X, xs, M, W, ws, N, K, Y, ldy, p3, st, dry);
    return cudaErrorInvalidValue;
}

// ---- tensor-core GEMM (k_gemm_tc) -----------------------------------------------------------
// cuTensorMapEncodeTiled, reached through the runtime's driver entry point.
typedef CUresult (*TmapEncodeFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                 const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                 CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
static TmapEncodeFn tmap_encode_fn() {
    static TmapEncodeFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<TmapEncodeFn>(p);
    });
    return fn;
}

// A weight matrix (N rows, row stride ws bytes) as a 2-D uint16 tensor [N][ws / 2] whose box is
// nt rows x rstr bytes (8 blocks); rows past N and bytes past the row stride read as zeros. The
// map holds only the address and shape, so it is cached by them.
static bool weight_tmap(const uint8_t* W, long ws, int N, int rstr, int nt, CUtensorMap* out) {
    static std::mutex mu;
    static std::map<std::tuple<uintptr_t, long, int, int, int>, CUtensorMap> cache;
    std::lock_guard<std::mutex> lk(mu);
    const auto key = std::make_tuple(reinterpret_cast<uintptr_t>(W), ws, N, rstr, nt);
    const auto it = cache.find(key);
    if (it != cache.end()) {
        *out = it->second;
        return true;
    }
    const TmapEncodeFn fn = tmap_encode_fn();
    if (!fn) return false;
    const cuuint64_t dims[2] = {(cuuint64_t)(ws / 2), (cuuint64_t)N};
    const cuuint64_t strides[1] = {(cuuint64_t)ws};
    const cuuint32_t box[2] = {(cuuint32_t)(rstr / 2), (cuuint32_t)nt};
    const cuuint32_t es[2] = {1, 1};
    CUtensorMap m;
    if (fn(&m, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, const_cast<uint8_t*>(W), dims, strides, box, es,
           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
        return false;
    if (cache.size() >= 4096) cache.clear();
    cache.emplace(key, m);
    *out = m;
    return true;
}

// k_gemm_tc: at least TC_MIN_M rows, 16-byte aligned weight rows of at least one raw chunk (K >= 256),
// K a multiple of 32 * TC_G, and scratch for one 32-row activation image.
bool tc_fits(const uint8_t* W, long ws, int M, int wdt, int K, const TcScratch& tc) {
    if (M < TC_MIN_M || (wdt != GTN_Q8 && wdt != GTN_Q4) || K % GTN_QBLK || !tc.p) return false;
    const int nb = K / GTN_QBLK;
    const long rstr = wdt == GTN_Q8 ? tc_rstride<GTN_Q8>() : tc_rstride<GTN_Q4>();
    return nb % TC_G == 0 && ws >= rstr && tc.bytes >= tc_aimg_bytes(TC_MT, K) &&
           ((reinterpret_cast<uintptr_t>(W) & 15) | (uintptr_t)(ws & 15) | (reinterpret_cast<uintptr_t>(tc.p) & 15)) == 0;
}

template <int WDT, int NT>
static cudaError_t launch_tc_nt(const uint8_t* X, long xs, int M, const uint8_t* W, long ws, int N, int K, float* Y,
                                long ldy, const TcScratch& tc, cudaStream_t st, bool dry) {
    constexpr size_t smem = tc_smem<WDT, NT>();
    cudaError_t e = ensure_smem(k_gemm_tc<WDT, NT>, smem);
    if (e != cudaSuccess) return e;
    CUtensorMap map;
    if (!weight_tmap(W, ws, N, tc_rstride<WDT>(), NT, &map)) return cudaErrorInvalidValue;
    if (dry) return cudaSuccess;
    const int nb = K / GTN_QBLK;
    const int cap = (int)(tc.bytes / ((size_t)nb * TC_AIMG)) * TC_MT;  // rows per pass
    for (int r0 = 0; r0 < M; r0 += cap) {
        const int mm = std::min(cap, M - r0), tiles = (mm + TC_MT - 1) / TC_MT;
        e = launch_pdl(k_tc_expand, dim3(nb, tiles), dim3(128), 0, st, X + (long)r0 * xs, xs, mm, K, tc.p);
        if (e != cudaSuccess) return e;
        e = launch_pdl(k_gemm_tc<WDT, NT>, dim3((N + NT - 1) / NT, tiles), dim3(TcTile<NT>::THREADS), smem, st, map,
                       N, K, (const uint8_t*)tc.p, mm, Y + (long)r0 * ldy, ldy, device_error_word());
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}

// 64-row or 32-row weight tiles, by the waves of one-CTA-per-SM grids: a 32-row CTA takes about
// 0.71 of a 64-row CTA's time (measured on 2048 x 5632 at 64 rows: 43.9 vs 61.6 us), so the smaller
// tile wins when 1.4 x its waves stay below the 64-row waves (e.g. 64 CTAs -> 128, one wave each;
// not 80 -> 160, which needs a second wave).
template <int WDT>
static cudaError_t launch_tc(const uint8_t* X, long xs, int M, const uint8_t* W, long ws, int N, int K, float* Y,
                             long ldy, const TcScratch& tc, cudaStream_t st, bool dry) {
    const int nb = K / GTN_QBLK;
    const int cap = (int)(tc.bytes / ((size_t)nb * TC_AIMG)) * TC_MT;
    const long tiles = (std::min(M, cap) + TC_MT - 1) / TC_MT, sms = sm_count();
    const long waves64 = ((N + 63) / 64 * tiles + sms - 1) / sms, waves32 = ((N + 31) / 32 * tiles + sms - 1) / sms;
    if (10 * waves32 < 14 * waves64) return launch_tc_nt<WDT, 32>(X, xs, M, W, ws, N, K, Y, ldy, tc, st, dry);
    return launch_tc_nt<WDT, 64>(X, xs, M, W, ws, N, K, Y, ldy, tc, st, dry);
}

bool gemm_q_fits(const uint8_t* W, long ws, int M, int wdt, int K, const TcScratch& tc) {
    if (tc_fits(W, ws, M, wdt, K, tc)) return true;
    if (wdt == GTN_Q8) return cc_gemm_fits<GTN_Q8>(W, ws, M, K);
    if (wdt == GTN_Q4) return cc_gemm_fits<GTN_Q4>(W, ws, M, K);
    return false;
}

cudaError_t gemm_q(const uint8_t* X, long xs, int M, const uint8_t* W, long ws, int wdt, int N, int K, float* Y,
                   long ldy, cudaStream_t st, bool dry, const TcScratch& tc) {
    if (tc_fits(W, ws, M, wdt, K, tc))
        return wdt == GTN_Q8 ? launch_tc<GTN_Q8>(X, xs, M, W, ws, N, K, Y, ldy, tc, st, dry)
                             : launch_tc<GTN_Q4>(X, xs, M, W, ws, N, K, Y, ldy, tc, st, dry);
    if (wdt == GTN_Q8) return cc_gemm<GTN_Q8>(X, xs, M, W, ws, N, K, Y, ldy, st, dry);
    if (wdt == GTN_Q4) return cc_gemm<GTN_Q4>(X, xs, M, W, ws, N, K, Y, ldy, st, dry);
    return cudaErrorInvalidValue;
}

cudaError_t gemm_f16(const uint8_t* X, long xs, int M, const uint8_t* W, long ws, int N, int K, float* Y, long ldy,
                     cudaStream_t st, bool dry) {
    if (M >= 2) {
        // k_gemm_f16: 128 (or 32, for grids under two waves) weight rows x 16 activation rows per
        // CTA; 8 activation rows when the 32-row grid of 16-row tiles would still leave SMs with a
        // single CTA (two fit), or when M <= 8
        const long sms = sm_count();
        const int mt16 = (M + 15) / 16;
        const bool wide = (long)((N + mf_rows(4) - 1) / mf_rows(4)) * mt16 >= 2 * sms;
        const bool narrow = !wide && (M <= 8 || (long)((N + mf_rows(1) - 1) / mf_rows(1)) * mt16 < 2 * sms);
        const int mtile = narrow ? 8 : 16, rw = wide ? 4 : 1, mtiles = (M + mtile - 1) / mtile;
        const size_t smem = mf_smem(rw, mtile);
        auto kern = wide ? k_gemm_f16<4, 16> : (narrow ? k_gemm_f16<1, 8> : k_gemm_f16<1, 16>);
        const cudaError_t e = ensure_smem(kern, smem);
        if (e != cudaSuccess || dry) return e;
        return launch_pdl(kern, dim3((N + mf_rows(rw) - 1) / mf_rows(rw), mtiles), dim3(MF_THREADS), smem, st, W, ws,
                          N, K, X, xs, M, Y, ldy, device_error_word());
    }
    const int mt = M <= 1 ? 1 : (M <= 2 ? 2 : (M <= 4 ? 4 : 8));
    int nw = 4;
    while (nw > 1 && (N + nw * 4 - 1) / (nw * 4) < 296) nw >>= 1;
    int mtv = mt;
    while (mtv > 1 && mm_f16_smem(nw, mtv, K) > 200 * 1024) mtv >>= 1;
    if (nw == 4) return launch_mm_f16<4>(X, xs, M, W, ws, N, K, Y, ldy, st, mtv, dry);
    if (nw == 2) return launch_mm_f16<2>(X, xs, M, W, ws, N, K, Y, ldy, st, mtv, dry);
    return launch_mm_f16<1>(X, xs, M, W, ws, N, K, Y, ldy, st, mtv, dry);
}

static cudaError_t matmul_tma(const uint8_t* X, long xs, int M, const uint8_t* W, long ws, int wdt, int N, int K,
                              float* Y, long ldy, cudaStream_t st, const TcScratch& tc) {
    if (gemv_q_fits(M, wdt, K)) return gemv_q(X, xs, M, W, ws, wdt, N, K, Y, ldy, st, false);
    if (tc_fits(W, ws, M, wdt, K, tc)) return gemm_q(X, xs, M, W, ws, wdt, N, K, Y, ldy, st, false, tc);
    if (wdt == GTN_Q8 && cc_gemm_fits<GTN_Q8>(W, ws, M, K)) return cc_gemm<GTN_Q8>(X, xs, M, W, ws, N, K, Y, ldy, st, false);
    if (wdt == GTN_Q4 && cc_gemm_fits<GTN_Q4>(W, ws, M, K)) return cc_gemm<GTN_Q4>(X, xs, M, W, ws, N, K, Y, ldy, st, false);
    const int mt = M <= 1 ? 1 : (M <= 2 ? 2 : (M <= 4 ? 4 : 8));
    if (wdt == GTN_F16) return gemm_f16(X, xs, M, W, ws, N, K, Y, ldy, st, false);
    int nw = 4;
    while (nw > 1 && (N + nw * 8 - 1) / (nw * 8) < 296) nw >>= 1;
    int mtv = mt;
    if (wdt == GTN_Q8) {
        while (mtv > 1 && mm_q_smem<GTN_Q8>(nw, mtv, K) > 200 * 1024) mtv >>= 1;
        if (nw == 4) return launch_mm_q<GTN_Q8, 4>(X, xs, M, W, ws, N, K, Y, ldy, st, mtv);
        if (nw == 2) return launch_mm_q<GTN_Q8, 2>(X, xs, M, W, ws, N, K, Y, ldy, st, mtv);
        return launch_mm_q<GTN_Q8, 1>(X, xs, M, W, ws, N, K, Y, ldy, st, mtv);
    }
    while (mtv > 1 && mm_q_smem<GTN_Q4>(nw, mtv, K) > 200 * 1024) mtv >>= 1;
    if (nw == 4) return launch_mm_q<GTN_Q4, 4>(X, xs, M, W, ws, N, K, Y, ldy, st, mtv);
    if (nw == 2) return launch_mm_q<GTN_Q4, 2>(X, xs, M, W, ws, N, K, Y, ldy, st, mtv);
    return launch_mm_q<GTN_Q4, 1>(X, xs, M, W, ws, N, K, Y, ldy, st, mtv);
}

}  // namespace gtn

using namespace gtn;

// ---- tensor helpers (tensor.h:96-116 bstride) -------------------------------------------------
static bool valid_dtype(int dt) { return dt >= GTN_I32 && dt <= GTN_Q4; }

static long bstride(const gtn_tensor* t, int i) {
    const long s = t->strides[i];
    switch (t->dtype) {
        case GTN_Q4: return s == 1 ? 1 : (s / GTN_QBLK) * GTN_Q4_BYTES;
        case GTN_Q8: return s == 1 ? 1 : (s / GTN_QBLK) * GTN_Q8_BYTES;
        case GTN_F16: return s * 2;
        default: return s * 4;
    }
}

static int check_tensor(const gtn_tensor* t, const char* name) {
    if (!t) return fail(GTN_ERR_ARG, "%s is NULL", name);
    if (!t->data) return fail(GTN_ERR_ARG, "%s has no data", name);
    if (!valid_dtype(t->dtype)) return fail(GTN_ERR_ARG, "%s has invalid dtype %d", name, t->dtype);
    if (t->ndim < 1 || t->ndim > 3) return fail(GTN_ERR_ARG, "%s has %d dims", name, t->ndim);
    for (int i = 0; i < t->ndim; ++i)
        if (t->shape[i] <= 0) return fail(GTN_ERR_ARG, "%s dim %d is %d", name, i, t->shape[i]);
    // Quantized rows of a partial last block: the reference allocates ceil(n/32) blocks per row
    // (tensor.cpp:43-45) but steps rows by floor(n/32) blocks (tensor.h:196-200), so rows beyond
    // the first overlap. Only single-row use is well defined.
    if ((t->dtype == GTN_Q8 || t->dtype == GTN_Q4) && t->ndim >= 2 && t->shape[t->ndim - 1] % GTN_QBLK != 0) {
        long rows = 1;
        for (int i = 0; i < t->ndim - 1; ++i) rows *= t->shape[i];
        if (rows > 1)
            return fail(GTN_ERR_ARG, "%s: quantized rows of %d elements (not a multiple of 32) overlap", name,
                        t->shape[t->ndim - 1]);
    }
    return GTN_OK;
}

static bool shape_eq(const gtn_tensor* a, const gtn_tensor* b) {
    if (a->ndim != b->ndim) return false;
    for (int i = 0; i < a->ndim; ++i)
        if (a->shape[i] != b->shape[i]) return false;
    return true;
}

static cudaStream_t S(void* s) { return reinterpret_cast<cudaStream_t>(s); }

#define GTN_CHECK(expr)                 \
    do {                                \
        const int rc_ = (expr);         \
        if (rc_ != GTN_OK) return rc_;  \
    } while (0)
#define GTN_REQUIRE(cond, ...)                              \
    do {                                                    \
        if (!(cond)) return fail(GTN_ERR_ARG, __VA_ARGS__); \
    } while (0)

static int launched(const char* what) { return cuda_status(cudaGetLastError(), what); }

static int norm_common(const gtn_tensor* inp, const gtn_tensor* weight, const gtn_tensor* bias, gtn_tensor* out,
                       int start_pos, void* stream, bool layer) {
    GTN_CHECK(check_tensor(inp, "inp"));
    GTN_CHECK(check_tensor(weight, "weight"));
    GTN_CHECK(check_tensor(out, "out"));
    GTN_REQUIRE(inp->dtype == out->dtype, "norm: inp/out dtype");
    GTN_REQUIRE(inp->dtype == GTN_Q8 || inp->dtype == GTN_F16 || inp->dtype == GTN_F32, "norm: dtype");
    GTN_REQUIRE(weight->ndim == 1 && weight->dtype == GTN_F16, "norm: weight must be 1-D fp16");
    const int n_ctx = inp->shape[0];
    GTN_REQUIRE(start_pos >= 0 && start_pos < n_ctx, "norm: start_pos");
    int heads = 1, n = inp->ndim >= 2 ? inp->shape[1] : 0;
    long hs = 0;
    if (inp->ndim == 3) {
        GTN_REQUIRE(!layer, "layer_norm: 2-D input");
        heads = inp->shape[1];
        n = inp->shape[2];
        hs = bstride(inp, 1);
        GTN_REQUIRE(inp->dtype != GTN_Q8 || n % GTN_QBLK == 0, "rms_norm: 3-D Q8 head size %d", n);
    } else {
        GTN_REQUIRE(inp->ndim == 2, "norm: 2-D or 3-D input");
    }
    GTN_REQUIRE(weight->shape[0] == n, "norm: weight size %d != %d", weight->shape[0], n);
    if (layer) {
        GTN_CHECK(check_tensor(bias, "bias"));
        GTN_REQUIRE(bias->ndim == 1 && bias->dtype == GTN_F16 && bias->shape[0] == n, "layer_norm: bias");
    }
    const size_t smem = 2 * sizeof(float) * (size_t)n;  // values + the exact sum's scratch
    // the exact parallel sum (n > 256) keeps <= 8 terms per thread up to n = 4096; shorter rows sum
    // serially, with a block of at least one warp per 32-element block
    const int nthreads = n > 1024 ? 512 : (n > 256 ? 256 : ((n + 31) / 32 * 32 < 64 ? 64 : (n + 31) / 32 * 32));
    cudaError_t e;
    if (layer) {
        e = ensure_smem(k_norm<true>, smem);
        if (e == cudaSuccess)
            e = launch_pdl(k_norm<true>, dim3(heads, n_ctx - start_pos), dim3(nthreads), smem, S(stream),
                           (const uint8_t*)inp->data, bstride(inp, 0), hs, (uint8_t*)out->data, bstride(out, 0), hs,
                           (int)inp->dtype, n, start_pos, (const uint16_t*)weight->data,
                           (const uint16_t*)bias->data);
    } else {
        e = ensure_smem(k_norm<false>, smem);
        // The 3-D path writes out with the input's strides (ops.cpp:879).
        if (e == cudaSuccess)
            e = launch_pdl(k_norm<false>, dim3(heads, n_ctx - start_pos), dim3(nthreads), smem, S(stream),
                           (const uint8_t*)inp->data, bstride(inp, 0), hs, (uint8_t*)out->data,
                           inp->ndim == 3 ? bstride(inp, 0) : bstride(out, 0), hs, (int)inp->dtype, n, start_pos,
                           (const uint16_t*)weight->data, (const uint16_t*)nullptr);
    }
    return cuda_status(e, "norm");
}

template <int OP>
static int rowop(const gtn_tensor* a, const gtn_tensor* b, gtn_tensor* out, float s, const gtn_tensor* bias,
                 int start_pos, void* stream, const char* name) {
    GTN_CHECK(check_tensor(a, "inp0"));
    GTN_CHECK(check_tensor(out, "out"));
    GTN_REQUIRE(a->ndim == 2 && out->ndim == 2 && shape_eq(a, out), "%s: shapes", name);
    GTN_REQUIRE(a->dtype == out->dtype, "%s: dtypes", name);
    GTN_REQUIRE(a->dtype == GTN_Q8 || a->dtype == GTN_F16 || a->dtype == GTN_F32, "%s: dtype", name);
    if (b) {
        GTN_CHECK(check_tensor(b, "inp1"));
        GTN_REQUIRE(shape_eq(a, b) && a->dtype == b->dtype, "%s: inp1", name);
    }
    if (OP == ROP_BIAS) {
        GTN_CHECK(check_tensor(bias, "bias"));
        GTN_REQUIRE(bias->ndim == 1 && bias->dtype == GTN_F16 && bias->shape[0] == a->shape[1], "%s: bias", name);
    }
    const int n_ctx = a->shape[0], n = a->shape[1];
    GTN_REQUIRE(start_pos >= 0 && start_pos < n_ctx, "%s: start_pos", name);
    const int nb = (n + GTN_QBLK - 1) / GTN_QBLK;
    cudaError_t e = launch_pdl(k_rowop<OP>, dim3((nb + 3) / 4, n_ctx - start_pos), dim3(128), 0, S(stream),
                               (const uint8_t*)a->data, bstride(a, 0), (const uint8_t*)(b ? b->data : nullptr),
                               b ? bstride(b, 0) : 0L, (uint8_t*)out->data, bstride(out, 0), (int)a->dtype, n,
                               start_pos, s, (const uint16_t*)(bias ? bias->data : nullptr));
    return cuda_status(e, name);
}

namespace gtn {

// ops.cpp:617-636: the argument checks of matmul_2d, shared by gtn_matmul_2d and
// gtn_matmul_2d_noalloc (`who` prefixes the error text).
int matmul_args(const gtn_tensor* x, const gtn_tensor* w, const gtn_tensor* out, int start_pos, const char* who,
                MatmulArgs* a) {
    GTN_CHECK(check_tensor(x, "x"));
    GTN_CHECK(check_tensor(w, "w"));
    GTN_CHECK(check_tensor(out, "out"));
    GTN_REQUIRE(x->ndim == 2, "%s: x must be 2-D", who);
    GTN_REQUIRE(w->ndim == 2 && w->shape[1] == x->shape[1], "%s: w must be [n_out, n_embd]", who);
    const int n_ctx = x->shape[0], K = x->shape[1], N = w->shape[0];
    GTN_REQUIRE(start_pos >= 0 && start_pos < n_ctx, "%s: start_pos %d out of [0, %d)", who, start_pos, n_ctx);
    if (out->ndim == 1) {
        GTN_REQUIRE(n_ctx - start_pos == 1, "%s: 1-D out needs exactly one new row", who);
        GTN_REQUIRE(out->shape[0] == N, "%s: out shape", who);
    } else {
        GTN_REQUIRE(out->ndim == 2 && out->shape[0] == n_ctx && out->shape[1] == N, "%s: out shape", who);
    }
    const bool q = x->dtype == GTN_Q8 && (w->dtype == GTN_Q8 || w->dtype == GTN_Q4);
    const bool h = x->dtype == GTN_F16 && w->dtype == GTN_F16;
    GTN_REQUIRE(q || h, "%s: unsupported dtypes x=%d w=%d", who, x->dtype, w->dtype);
    GTN_REQUIRE(K % GTN_QBLK == 0 || h, "%s: n_embd %d not a multiple of 32", who, K);
    GTN_REQUIRE(out->dtype == GTN_F32 || out->dtype == x->dtype, "%s: out dtype", who);
    a->quant = q;
    a->M = n_ctx - start_pos;
    a->N = N;
    a->K = K;
    a->X = (const uint8_t*)x->data + (long)start_pos * bstride(x, 0);
    a->xs = bstride(x, 0);
    a->xdt = x->dtype;
    a->W = (const uint8_t*)w->data;
    a->ws = bstride(w, 0);
    a->wdt = w->dtype;
    a->os = out->ndim == 1 ? 0 : bstride(out, 0);
    a->odt = out->dtype;
    a->out = (uint8_t*)out->data;
    a->one_d = out->ndim == 1;
    return GTN_OK;
}

}  // namespace gtn

extern "C" {

const char* gtn_last_error(void) { return g_last_error.c_str(); }

unsigned long long gtn_kernel_launches(void) { return g_launches.load(); }

// ops.cpp:617-636
int gtn_matmul_2d(const gtn_tensor* x, const gtn_tensor* w, gtn_tensor* out, int start_pos, void* stream) {
    MatmulArgs a;
    GTN_CHECK(matmul_args(x, w, out, start_pos, "matmul_2d", &a));
    const int M = a.M, N = a.N, K = a.K;
    cudaStream_t st = S(stream);
    // the tensor-core path's expanded activation image (stream-ordered scratch, freed below)
    TcScratch tc;
    if (a.quant && M >= TC_MIN_M && K % GTN_QBLK == 0) {
        tc.bytes = tc_aimg_bytes(M, K);
        if (cudaMallocAsync((void**)&tc.p, tc.bytes, st) != cudaSuccess) {
            cudaGetLastError();
            tc = TcScratch();  // the CUDA-core kernels need no scratch
        }
    }
    cudaError_t e;
    if (a.odt == GTN_F32) {
        float* Y = (float*)(a.out + (long)start_pos * a.os);
        e = matmul_f32(a.X, a.xs, a.xdt, M, a.W, a.ws, a.wdt, N, K, Y, a.one_d ? 0 : N, st, false, tc);
    } else {
        float* Y = nullptr;
        e = cudaMallocAsync((void**)&Y, sizeof(float) * (size_t)M * N, st);
        if (e == cudaSuccess) {
            e = matmul_f32(a.X, a.xs, a.xdt, M, a.W, a.ws, a.wdt, N, K, Y, N, st, false, tc);
            if (e == cudaSuccess)
                e = launch_pdl(k_write_rows, dim3(((N + GTN_QBLK - 1) / GTN_QBLK + 3) / 4, M), dim3(128), 0, st,
                               (const float*)Y, (long)N, a.out, a.os, a.odt, N, start_pos);
            cudaFreeAsync(Y, st);
        }
    }
    if (tc.p) cudaFreeAsync(tc.p, st);
    return cuda_status(e, "matmul_2d");
}

// ops.cpp:1205-1220
int gtn_qkv_attn(const gtn_tensor* q, const gtn_tensor* k, const gtn_tensor* v, gtn_tensor* qk, gtn_tensor* qkv,
                 int max_ctx, int start_pos, void* stream) {
    (void)qk;
    GTN_CHECK(check_tensor(q, "q"));
    GTN_CHECK(check_tensor(k, "k"));
    GTN_CHECK(check_tensor(v, "v"));
    GTN_CHECK(check_tensor(qkv, "qkv"));
    GTN_REQUIRE(q->ndim == 2 && k->ndim == 2 && v->ndim == 2 && qkv->ndim == 2, "qkv_attn: 2-D tensors");
    const int n_ctx = q->shape[0], q_dim = q->shape[1], kv_dim = k->shape[1];
    GTN_REQUIRE(qkv->shape[0] == n_ctx && qkv->shape[1] == q_dim, "qkv_attn: qkv shape");
    GTN_REQUIRE(k->shape[0] >= n_ctx && v->shape[0] >= n_ctx && v->shape[1] == kv_dim, "qkv_attn: k/v shape");
    GTN_REQUIRE(q->dtype == k->dtype && k->dtype == v->dtype && v->dtype == qkv->dtype, "qkv_attn: dtypes differ");
    GTN_REQUIRE(q->dtype == GTN_Q8 || q->dtype == GTN_F16, "qkv_attn: dtype must be Q8 or F16");
    GTN_REQUIRE(max_ctx > 0 && max_ctx >= n_ctx, "qkv_attn: max_ctx");
    GTN_REQUIRE(start_pos >= 0 && start_pos < n_ctx, "qkv_attn: start_pos");
    const int d = 64;  // the reference's head size for every model
    GTN_REQUIRE(q_dim % d == 0 && kv_dim % d == 0, "qkv_attn: dims not multiples of 64");
    const int qh = q_dim / d, kvh = kv_dim / d;
    GTN_REQUIRE(qh % kvh == 0, "qkv_attn: heads %d not a multiple of kv heads %d", qh, kvh);
    const size_t smem = attn_smem(n_ctx, q->dtype, d);
    GTN_REQUIRE(smem <= 200 * 1024, "qkv_attn: n_ctx %d too large", n_ctx);
    cudaError_t e = ensure_smem(k_attn, smem);
    if (e == cudaSuccess)
        e = launch_pdl(k_attn, dim3(qh, n_ctx - start_pos), dim3(ATT_THREADS), smem, S(stream),
                       (const uint8_t*)q->data, bstride(q, 0), (const uint8_t*)k->data, bstride(k, 0),
                       row_bytes(k->dtype, d), (const uint8_t*)v->data, bstride(v, 0), row_bytes(v->dtype, d),
                       (uint8_t*)qkv->data, bstride(qkv, 0), (int)q->dtype, n_ctx, start_pos, qh, kvh, d,
                       device_error_word());
    return cuda_status(e, "qkv_attn");
}

int gtn_rms_norm(const gtn_tensor* inp, const gtn_tensor* weight, gtn_tensor* out, int start_pos, void* stream) {
    return norm_common(inp, weight, nullptr, out, start_pos, stream, false);
}

int gtn_layer_norm(const gtn_tensor* inp, const gtn_tensor* weight, const gtn_tensor* bias, gtn_tensor* out,
                   int start_pos, void* stream) {
    GTN_REQUIRE(inp && out && shape_eq(inp, out), "layer_norm: inp/out shapes differ");
    return norm_common(inp, weight, bias, out, start_pos, stream, true);
}

// ops.cpp:775-827. The (cos, sin) table for this call's positions is computed on the host with the
// reference's expression and uploaded once per (rd, device) and growth of the position count.
int gtn_rotary_emb(const gtn_tensor* inp, gtn_tensor* out, int d_head, float rope_pct, int start_pos, void* stream) {
    GTN_CHECK(check_tensor(inp, "inp"));
    GTN_CHECK(check_tensor(out, "out"));
    GTN_REQUIRE(inp->ndim == 2 && out->ndim == 2, "rotary_emb: 2-D tensors");
    GTN_REQUIRE(rope_pct >= 0.0f && rope_pct <= 1.0f, "rotary_emb: rope_pct");
    GTN_REQUIRE(d_head > 0 && d_head % 32 == 0 && d_head <= 256, "rotary_emb: d_head %d unsupported", d_head);
    const int n_ctx = inp->shape[0], n_embd = inp->shape[1];
    GTN_REQUIRE(n_embd % d_head == 0 && out->shape[0] >= n_ctx && out->shape[1] == n_embd, "rotary_emb: shapes");
    GTN_REQUIRE(inp->dtype == out->dtype, "rotary_emb: dtypes");
    GTN_REQUIRE(inp->dtype == GTN_Q8 || inp->dtype == GTN_F16 || inp->dtype == GTN_F32, "rotary_emb: dtype");
    GTN_REQUIRE(start_pos >= 0 && start_pos < n_ctx, "rotary_emb: start_pos");
    const int rd = (int)((float)d_head * rope_pct);
    const int half = rd / 2;
    static std::mutex mu;
    struct Entry { int rd, dev, npos; float2* tab; };
    static std::vector<Entry> cache;
    float2* tab = nullptr;
    {
        std::lock_guard<std::mutex> lk(mu);
        int dev = 0;
        cudaGetDevice(&dev);
        for (auto& c : cache)
            if (c.rd == rd && c.dev == dev && c.npos >= n_ctx) tab = c.tab;
        if (!tab) {
            const int npos = n_ctx < 4096 ? 4096 : n_ctx;
            auto hst = rope_table_host(npos, rd);
            GTN_CHECK(cuda_status(cudaMalloc((void**)&tab, hst.size() * sizeof(float2)), "rope table"));
            GTN_CHECK(cuda_status(cudaMemcpy(tab, hst.data(), hst.size() * sizeof(float2), cudaMemcpyHostToDevice),
                                  "rope table"));
            cache.push_back({rd, dev, npos, tab});
        }
    }
    cudaError_t e = launch_pdl(k_rope, dim3(n_embd / d_head, n_ctx - start_pos), dim3(32), 0, S(stream),
                               (const uint8_t*)inp->data, bstride(inp, 0), (uint8_t*)out->data, bstride(inp, 0),
                               (int)inp->dtype, n_embd, d_head, half, start_pos, (const float2*)tab,
                               half > 0 ? half : 1);
    return cuda_status(e, "rotary_emb");
}

int gtn_silu(const gtn_tensor* inp, gtn_tensor* out, int start_pos, void* stream) {
    return rowop<ROP_SILU>(inp, nullptr, out, 0.0f, nullptr, start_pos, stream, "silu");
}
int gtn_silu_inplace(gtn_tensor* inp, int start_pos, void* stream) {
    return rowop<ROP_SILU>(inp, nullptr, inp, 0.0f, nullptr, start_pos, stream, "silu_inplace");
}
int gtn_multiply(const gtn_tensor* inp0, const gtn_tensor* inp1, gtn_tensor* out, int start_pos, void* stream) {
    return rowop<ROP_MUL>(inp0, inp1, out, 0.0f, nullptr, start_pos, stream, "multiply");
}
int gtn_multiply_inplace(gtn_tensor* inp0, const gtn_tensor* inp1, int start_pos, void* stream) {
    return rowop<ROP_MUL>(inp0, inp1, inp0, 0.0f, nullptr, start_pos, stream, "multiply_inplace");
}
int gtn_add(const gtn_tensor* inp0, const gtn_tensor* inp1, gtn_tensor* out, int start_pos, void* stream) {
    return rowop<ROP_ADD>(inp0, inp1, out, 0.0f, nullptr, start_pos, stream, "add");
}
int gtn_scale(gtn_tensor* inp, float scaler, int start_pos, void* stream) {
    return rowop<ROP_SCALE>(inp, nullptr, inp, scaler, nullptr, start_pos, stream, "scale");
}
int gtn_bias_add_inplace(gtn_tensor* inp, const gtn_tensor* bias, int start_pos, void* stream) {
    return rowop<ROP_BIAS>(inp, nullptr, inp, 0.0f, bias, start_pos, stream, "bias_add_inplace");
}

// ops.cpp:566-576
int gtn_token_embed(const gtn_tensor* weight, const gtn_tensor* tokens, gtn_tensor* out, int start_pos,
                    void* stream) {
    GTN_CHECK(check_tensor(weight, "weight"));
    GTN_CHECK(check_tensor(tokens, "tokens"));
    GTN_CHECK(check_tensor(out, "out"));
    GTN_REQUIRE(weight->ndim == 2, "token_embed: weight 2-D");
    GTN_REQUIRE(tokens->ndim == 1 && tokens->dtype == GTN_I32, "token_embed: tokens 1-D int32");
    const int n_ctx = tokens->shape[0], n = weight->shape[1];
    GTN_REQUIRE(out->ndim == 2 && out->shape[0] == n_ctx && out->shape[1] == n, "token_embed: out shape");
    GTN_REQUIRE(weight->dtype == GTN_Q4 ? out->dtype == GTN_Q8 : out->dtype == weight->dtype, "token_embed: dtypes");
    GTN_REQUIRE(start_pos >= 0 && start_pos < n_ctx, "token_embed: start_pos");
    const int nb = (n + GTN_QBLK - 1) / GTN_QBLK;
    cudaError_t e = launch_pdl(k_embed, dim3((nb + 3) / 4, n_ctx - start_pos), dim3(128), 0, S(stream),
                               (const uint8_t*)weight->data, bstride(weight, 0), (int)weight->dtype,
                               (const int32_t*)tokens->data, (uint8_t*)out->data, bstride(out, 0), (int)out->dtype, n,
                               start_pos, weight->shape[0], device_error_word());
    return cuda_status(e, "token_embed");
}

int gtn_pack_q8(const float* w, int64_t rows, int64_t cols, void* out, void* stream) {
    GTN_REQUIRE(w && out && rows > 0 && cols > 0 && cols % GTN_QBLK == 0, "pack_q8: arguments");
    GTN_REQUIRE(((uintptr_t)w & 15) == 0, "pack_q8: w must be 16-byte aligned");
    const long nb = rows * (cols / GTN_QBLK);
    count_launch();
    k_pack<false><<<(unsigned)((nb + 255) / 256), 256, 0, S(stream)>>>(w, nb, (uint8_t*)out);
    return launched("pack_q8");
}

int gtn_pack_q4(const float* w, int64_t rows, int64_t cols, void* out, void* stream) {
    GTN_REQUIRE(w && out && rows > 0 && cols > 0 && cols % GTN_QBLK == 0, "pack_q4: arguments");
    GTN_REQUIRE(((uintptr_t)w & 15) == 0, "pack_q4: w must be 16-byte aligned");
    const long nb = rows * (cols / GTN_QBLK);
    count_launch();
    k_pack<true><<<(unsigned)((nb + 255) / 256), 256, 0, S(stream)>>>(w, nb, (uint8_t*)out);
    return launched("pack_q4");
}

int gtn_quantize_q8_rows(const float* x, int64_t rows, int64_t cols, void* out, void* stream) {
    GTN_REQUIRE(x && out && rows > 0 && cols > 0 && rows < 65536, "quantize_q8_rows: arguments");
    const int nb = (int)((cols + GTN_QBLK - 1) / GTN_QBLK);
    cudaError_t e = launch_pdl(k_quant_rows, dim3((nb + 3) / 4, (unsigned)rows), dim3(128), 0, S(stream), x,
                               (long)cols, (uint8_t*)out, (long)nb * GTN_Q8_BYTES, (int)cols);
    return cuda_status(e, "quantize_q8_rows");
}

int gtn_argmax(const float* logits, int n, int32_t* out_index, void* stream) {
    GTN_REQUIRE(logits && out_index && n > 0, "argmax: arguments");
    cudaError_t e = launch_pdl(k_argmax, dim3(1), dim3(1024), 0, S(stream), logits, n, out_index, 0L, 0L);
    return cuda_status(e, "argmax");
}

}  // extern "C"
