// Exact (reference-order) matmul kernels: Y[m, n] = dot(X[m, :], W[n, :]) in fp32.
//
// Reference: ops.cpp:579-636 matmul_2d_impl, with the dot products of ops.cpp:208-523.
// The reference's AVX build accumulates
//   * Q8 x Q8 and Q8 x Q4 (ops.cpp:292-490) in 4 fp32 lanes: lane l owns elements
//     {c+2l, c+2l+1 : c in {0,8,16,24}} of each 32-element block; per block the exact int32 lane
//     sum is converted to fp32, multiplied by fp16(da)*fp16(dw) and added to the lane, blocks in
//     order; the result is (L0+L1)+(L2+L3);
//   * fp16 x fp16 (ops.cpp:208-242) in 8 fp32 lanes over elements 8i+l (products are exact in
//     fp32), lanes summed left to right, then the scalar tail.
// Here one thread owns one (output row, lane) accumulator, so the per-lane chains keep exactly
// that order and the results are bit-identical. Integer lane sums use dp4a on the lane's 8
// bytes (2 words); Q4 nibbles are unpacked with shifts/masks and the +7 bias is removed with the
// activation lane sum (sum((q-7)*a) = sum(q*a) - 7*sum(a), exact in int32).
//
// Weight streaming: W rows are read with 1-D TMA bulk copies (cp.async.bulk) into a 4-stage
// shared-memory ring per CTA, one copy per row per K tile, completion on an mbarrier (waits are
// bounded). Activations are prepared once per CTA in shared memory in lane order.
#pragma once
#include "common.cuh"

namespace gtn {

constexpr int MM_STAGES = 4;

// After an aborted pipeline: wait (bounded again) for copies that may still be in flight into this
// CTA's shared memory before it exits. Stage s has an outstanding phase for the last tile issued to it.
__device__ __forceinline__ void drain_stages(uint64_t* bars, int nkt, int tid) {
    if (tid != 0) return;
    for (int s = 0; s < MM_STAGES && s < nkt; ++s) {
        const int last = s + ((nkt - 1 - s) / MM_STAGES) * MM_STAGES;
        for (uint32_t it = 0; it < GTN_WAIT_LIMIT; ++it)
            if (mbar_try_wait(&bars[s], (last / MM_STAGES) & 1)) break;
    }
}

// Per (activation row, block, lane): the lane's 8 activation int8 in two words ordered like the
// weight words below, their sum (for the Q4 bias), and fp16(da) as float.
struct __align__(16) LanePrep {
    int a0, a1, s;
    float da;
};

// Builds LanePrep for rows [m0, m0+mt) of a Q8 activation matrix; all threads of the CTA.
__device__ __forceinline__ void build_prep_q8(const uint8_t* X, long x_stride, int m0, int mt, int nb,
                                              LanePrep* prep) {
    const int total = mt * nb * 4;
    for (int i = threadIdx.x; i < total; i += blockDim.x) {
        const int l = i & 3, b = (i >> 2) % nb, m = (i >> 2) / nb;
        const uint8_t* blk = X + (long)(m0 + m) * x_stride + (long)b * GTN_Q8_BYTES;
        const int8_t* q = reinterpret_cast<const int8_t*>(blk + 2);
        const int e0 = q[2 * l], e1 = q[2 * l + 1], e2 = q[8 + 2 * l], e3 = q[9 + 2 * l];
        const int e4 = q[16 + 2 * l], e5 = q[17 + 2 * l], e6 = q[24 + 2 * l], e7 = q[25 + 2 * l];
        LanePrep p;
        p.a0 = (e0 & 255) | ((e1 & 255) << 8) | ((e2 & 255) << 16) | ((e3 & 255) << 24);
        p.a1 = (e4 & 255) | ((e5 & 255) << 8) | ((e6 & 255) << 16) | ((e7 & 255) << 24);
        p.s = e0 + e1 + e2 + e3 + e4 + e5 + e6 + e7;
        p.da = h2f(ld_u16(blk));
        prep[i] = p;
    }
}

// Weight lane words of one Q8 block (34 bytes at p): bytes {2l,2l+1,8+2l,9+2l} and
// {16+2l,17+2l,24+2l,25+2l} of the data. All 16-bit loads are aligned (block starts are even).
__device__ __forceinline__ int q8_block_lane_dot(const uint8_t* p, int l, const LanePrep& a) {
    const uint8_t* d = p + 2;
    const int w0 = (int)ld_u16(d + 2 * l) | ((int)ld_u16(d + 8 + 2 * l) << 16);
    const int w1 = (int)ld_u16(d + 16 + 2 * l) | ((int)ld_u16(d + 24 + 2 * l) << 16);
    return dp4a(w0, a.a0, dp4a(w1, a.a1, 0));
}
// Q4 block (18 bytes at p): byte j = (q[j] << 4) | q[j+16]; lane l's 8 weights are the high and low
// nibbles of bytes {2l, 2l+1, 8+2l, 9+2l}.
__device__ __forceinline__ int q4_block_lane_dot(const uint8_t* p, int l, const LanePrep& a) {
    const uint8_t* d = p + 2;
    const int wb = (int)ld_u16(d + 2 * l) | ((int)ld_u16(d + 8 + 2 * l) << 16);
    const int hi = (wb >> 4) & 0x0f0f0f0f, lo = wb & 0x0f0f0f0f;
    return dp4a(hi, a.a0, dp4a(lo, a.a1, 0)) - 7 * a.s;
}

template <int WDT>
struct MMCfg;
template <>
struct MMCfg<GTN_Q8> {
    static constexpr int LANES = 4, BLK_BYTES = GTN_Q8_BYTES, KT_BLOCKS = 16;
};
template <>
struct MMCfg<GTN_Q4> {
    static constexpr int LANES = 4, BLK_BYTES = GTN_Q4_BYTES, KT_BLOCKS = 32;
};

// Shared memory bytes of k_mm_q for (NW warps, MT activation rows, K).
template <int WDT>
__host__ __device__ inline int mm_q_tile_stride() {
    return ((MMCfg<WDT>::KT_BLOCKS * MMCfg<WDT>::BLK_BYTES + 15) / 16) * 16 + 16;
}
template <int WDT>
__host__ __device__ inline size_t mm_q_smem(int nw, int mt, int K) {
    const int rows = nw * 8;
    const int nb = K / GTN_QBLK;
    return 128 + (size_t)MM_STAGES * rows * mm_q_tile_stride<WDT>() + (size_t)mt * nb * 4 * sizeof(LanePrep);
}

// Q8/Q4 weights x Q8 activations. grid.x = ceil(N / (8*NW)), grid.y = ceil(M / MT).
// W: row stride w_stride bytes (any alignment: copies start at the 16-byte boundary below the
// row tile and the tile is read at the remainder; the allocation must extend 16 bytes past the
// last row unless rows and tiles are 16-byte multiples). X: Q8 rows, stride x_stride bytes.
// Y: fp32, row stride y_stride elements.
template <int WDT, int NW, int MT>
__global__ void __launch_bounds__(NW * 32) k_mm_q(const uint8_t* __restrict__ W, long w_stride, int N, int K,
                                                  const uint8_t* __restrict__ X, long x_stride, int M,
                                                  float* __restrict__ Y, long y_stride, unsigned int* err) {
    using C = MMCfg<WDT>;
    constexpr int ROWS = NW * 8;
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ int abort_flag;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem);
    const int tstride = mm_q_tile_stride<WDT>();
    uint8_t* stages = smem + 128;
    const int nb = K / GTN_QBLK;
    LanePrep* prep = reinterpret_cast<LanePrep*>(stages + (size_t)MM_STAGES * ROWS * tstride);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int r_local = warp * 8 + (lane >> 2), l = lane & 3;
    const int row0 = blockIdx.x * ROWS;
    const int nrows = min(ROWS, N - row0);
    const int m0 = blockIdx.y * MT;
    const int mt = min(MT, M - m0);
    const int nkt = (nb + C::KT_BLOCKS - 1) / C::KT_BLOCKS;

    auto issue = [&](int kt) {
        // warp 0: lane 0 arms the stage barrier, then lane r copies row r's tile.
        const int s = kt % MM_STAGES;
        const int b0 = kt * C::KT_BLOCKS;
        const int nbt = min(C::KT_BLOCKS, nb - b0);
        uint32_t total = 0;
        for (int r = 0; r < nrows; ++r) {
            const uintptr_t src = reinterpret_cast<uintptr_t>(W) + (uintptr_t)(row0 + r) * w_stride +
                                  (uintptr_t)b0 * C::BLK_BYTES;
            const uint32_t off = (uint32_t)(src & 15);
            total += (off + nbt * C::BLK_BYTES + 15) & ~15u;
        }
        if (lane == 0) mbar_arrive_expect_tx(&bars[s], total);
        __syncwarp();
        for (int r = lane; r < nrows; r += 32) {
            const uintptr_t src = reinterpret_cast<uintptr_t>(W) + (uintptr_t)(row0 + r) * w_stride +
                                  (uintptr_t)b0 * C::BLK_BYTES;
            const uint32_t off = (uint32_t)(src & 15);
            const uint32_t bytes = (off + nbt * C::BLK_BYTES + 15) & ~15u;
            bulk_g2s(stages + ((size_t)s * ROWS + r) * tstride, reinterpret_cast<const void*>(src - off), bytes,
                     &bars[s]);
        }
    };

    if (tid == 0) {
        for (int s = 0; s < MM_STAGES; ++s) mbar_init(&bars[s], 1);
        fence_mbar_init();
        abort_flag = 0;
    }
    __syncthreads();
    if (warp == 0)
        for (int kt = 0; kt < min(MM_STAGES, nkt); ++kt) issue(kt);

    // Weights do not depend on the previous kernel; activations do (programmatic dependent launch).
    asm volatile("griddepcontrol.wait;" ::: "memory");
    build_prep_q8(X, x_stride, m0, mt, nb, prep);
    __syncthreads();

    float acc[MT];
#pragma unroll
    for (int m = 0; m < MT; ++m) acc[m] = 0.0f;
    for (int kt = 0; kt < nkt; ++kt) {
        const int s = kt % MM_STAGES;
        // A timed-out wait marks the CTA aborted; every thread still reaches each barrier.
        if (!abort_flag && !mbar_wait_bounded(&bars[s], (kt / MM_STAGES) & 1, err)) abort_flag = 1;
        const int b0 = kt * C::KT_BLOCKS;
        const int nbt = min(C::KT_BLOCKS, nb - b0);
        if (!abort_flag && r_local < nrows) {
            const uintptr_t src = reinterpret_cast<uintptr_t>(W) + (uintptr_t)(row0 + r_local) * w_stride +
                                  (uintptr_t)b0 * C::BLK_BYTES;
            const uint8_t* t = stages + ((size_t)s * ROWS + r_local) * tstride + (src & 15);
            for (int b = 0; b < nbt; ++b) {
                const uint8_t* p = t + b * C::BLK_BYTES;
                const float dw = h2f(ld_u16(p));
#pragma unroll
                for (int m = 0; m < MT; ++m) {
                    if (m < mt) {
                        const LanePrep a = prep[((size_t)m * nb + b0 + b) * 4 + l];
                        const int L = WDT == GTN_Q8 ? q8_block_lane_dot(p, l, a) : q4_block_lane_dot(p, l, a);
                        const float sc = a.da * dw;
                        const float pr = lane_sum_f32(L) * sc;
                        acc[m] = acc[m] + pr;
                    }
                }
            }
        }
        __syncthreads();
        if (warp == 0 && !abort_flag && kt + MM_STAGES < nkt) issue(kt + MM_STAGES);
    }
    asm volatile("griddepcontrol.launch_dependents;");
    if (abort_flag) {
        drain_stages(bars, nkt, tid);
        return;
    }
#pragma unroll
    for (int m = 0; m < MT; ++m) {
        const float t01 = acc[m] + __shfl_xor_sync(0xffffffffu, acc[m], 1);
        const float t = t01 + __shfl_xor_sync(0xffffffffu, t01, 2);
        if (l == 0 && r_local < nrows && m < mt) Y[(long)(m0 + m) * y_stride + row0 + r_local] = t;
    }
}

// fp16 weights x fp16 activations, 8 lanes per row: CTA = NW warps x 4 rows.
constexpr int MM_F16_KT = 256;  // elements per K tile (512 bytes per row)
__host__ __device__ inline int mm_f16_tile_stride() { return MM_F16_KT * 2 + 16; }
__host__ __device__ inline size_t mm_f16_smem(int nw, int mt, int K) {
    return 128 + (size_t)MM_STAGES * nw * 4 * mm_f16_tile_stride() + (size_t)mt * K * 2 + 16;
}

template <int NW, int MT>
__global__ void __launch_bounds__(NW * 32) k_mm_f16(const uint8_t* __restrict__ W, long w_stride, int N, int K,
                                                    const uint8_t* __restrict__ X, long x_stride, int M,
                                                    float* __restrict__ Y, long y_stride, unsigned int* err) {
    constexpr int ROWS = NW * 4;
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ int abort_flag;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem);
    const int tstride = mm_f16_tile_stride();
    uint8_t* stages = smem + 128;
    uint16_t* xs = reinterpret_cast<uint16_t*>(stages + (size_t)MM_STAGES * ROWS * tstride);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int r_local = warp * 4 + (lane >> 3), l = lane & 7;
    const int row0 = blockIdx.x * ROWS;
    const int nrows = min(ROWS, N - row0);
    const int m0 = blockIdx.y * MT;
    const int mt = min(MT, M - m0);
    const int K8 = (K / 8) * 8;
    const int nkt = (K8 + MM_F16_KT - 1) / MM_F16_KT;

    auto issue = [&](int kt) {
        const int s = kt % MM_STAGES;
        const int e0 = kt * MM_F16_KT;
        const int ne = min(MM_F16_KT, K8 - e0);
        uint32_t total = 0;
        for (int r = 0; r < nrows; ++r) {
            const uintptr_t src = reinterpret_cast<uintptr_t>(W) + (uintptr_t)(row0 + r) * w_stride + (uintptr_t)e0 * 2;
            total += ((uint32_t)(src & 15) + ne * 2 + 15) & ~15u;
        }
        if (lane == 0) mbar_arrive_expect_tx(&bars[s], total);
        __syncwarp();
        for (int r = lane; r < nrows; r += 32) {
            const uintptr_t src = reinterpret_cast<uintptr_t>(W) + (uintptr_t)(row0 + r) * w_stride + (uintptr_t)e0 * 2;
            const uint32_t off = (uint32_t)(src & 15);
            bulk_g2s(stages + ((size_t)s * ROWS + r) * tstride, reinterpret_cast<const void*>(src - off),
                     (off + ne * 2 + 15) & ~15u, &bars[s]);
        }
    };

    if (tid == 0) {
        for (int s = 0; s < MM_STAGES; ++s) mbar_init(&bars[s], 1);
        fence_mbar_init();
        abort_flag = 0;
    }
    __syncthreads();
    if (warp == 0)
        for (int kt = 0; kt < min(MM_STAGES, nkt); ++kt) issue(kt);
    asm volatile("griddepcontrol.wait;" ::: "memory");
    for (int i = tid; i < mt * K; i += blockDim.x) {
        const int m = i / K, k = i % K;
        xs[i] = reinterpret_cast<const uint16_t*>(X + (long)(m0 + m) * x_stride)[k];
    }
    __syncthreads();

    float acc[MT];
#pragma unroll
    for (int m = 0; m < MT; ++m) acc[m] = 0.0f;
    for (int kt = 0; kt < nkt; ++kt) {
        const int s = kt % MM_STAGES;
        if (!abort_flag && !mbar_wait_bounded(&bars[s], (kt / MM_STAGES) & 1, err)) abort_flag = 1;
        const int e0 = kt * MM_F16_KT;
        const int ne = min(MM_F16_KT, K8 - e0);
        if (!abort_flag && r_local < nrows) {
            const uintptr_t src = reinterpret_cast<uintptr_t>(W) + (uintptr_t)(row0 + r_local) * w_stride + (uintptr_t)e0 * 2;
            const uint16_t* t = reinterpret_cast<const uint16_t*>(stages + ((size_t)s * ROWS + r_local) * tstride + (src & 15));
            for (int i = l; i < ne; i += 8) {
                const float w = h2f(t[i]);
#pragma unroll
                for (int m = 0; m < MT; ++m) {
                    if (m < mt) {
                        const float pr = h2f(xs[m * K + e0 + i]) * w;
                        acc[m] = pr + acc[m];
                    }
                }
            }
        }
        __syncthreads();
        if (warp == 0 && !abort_flag && kt + MM_STAGES < nkt) issue(kt + MM_STAGES);
    }
    asm volatile("griddepcontrol.launch_dependents;");
    if (abort_flag) {
        drain_stages(bars, nkt, tid);
        return;
    }
    // lanes summed left to right (simd_ops.h:75-78), then the scalar tail (ops.cpp:224-228).
    const int base = lane & ~7;
#pragma unroll
    for (int m = 0; m < MT; ++m) {
        float v[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) v[j] = __shfl_sync(0xffffffffu, acc[m], base + j);
        if (l == 0 && r_local < nrows && m < mt) {
            float d = v[0] + v[1];
            d = d + v[2];
            d = d + v[3];
            d = d + v[4];
            d = d + v[5];
            d = d + v[6];
            d = d + v[7];
            const uint16_t* wr = reinterpret_cast<const uint16_t*>(W + (long)(row0 + r_local) * w_stride);
            for (int k = K8; k < K; ++k) {
                const float pr = h2f(xs[m * K + k]) * h2f(wr[k]);
                d = d + pr;
            }
            Y[(long)(m0 + m) * y_stride + row0 + r_local] = d;
        }
    }
}

// ---- exact fp16 GEMM for several activation rows (prefill, batched decode) ----------------------
// The arithmetic of k_mm_f16 (8 fp32 lanes over elements 8i+l, lanes summed left to right, then the
// scalar tail) for a tile of 32 * RW weight rows x MF_MT activation rows per CTA of 256 threads:
// thread (row slot r, lane l) owns weight rows r + 32 i (i < RW) and keeps RW x MF_MT accumulators.
// The reference multiplies and adds with separate roundings (no FMA in its build); a product of
// two fp16 values is exact in fp32 (at most 22 significant bits, exponents within range), so
// fma(x, w, acc) rounds exactly once, like fl(fl(x * w) + acc): one instruction per product here.
// Per K tile (MF_KT(RW) elements) the weight rows and the activation rows arrive by TMA bulk copies
// (an MM_STAGES-deep ring; activations 16-byte aligned, else loaded directly), and the activation
// tile is converted once to fp32 in an [element][row] layout (row stride padded to 68 floats: the
// 8 lanes of a slot read 8 consecutive elements with conflict-free 16-byte loads), so every float4
// load feeds 4 * RW products. grid (ceil(N / (32 RW)), ceil(M / MF_MT)).
// MF_MT activation rows per CTA: 16, or 8 when the 16-row grid would leave SMs with one CTA
// (e.g. M = 32 against 2048 weight rows: 128 CTAs instead of 256) or M <= 8.
constexpr int MF_STAGES = MM_STAGES, MF_THREADS = 256;
// floats per element of the fp32 activation tile: the rows + 4 (bank spread of the 16-byte loads)
__host__ __device__ constexpr int mf_xstr(int mt) { return mt == 16 ? 68 : 36; }
__host__ __device__ constexpr int mf_rows(int rw) { return 32 * rw; }
__host__ __device__ constexpr int mf_kt(int rw) { return rw == 1 ? 128 : 64; }
__host__ __device__ constexpr int mf_wstride(int rw) { return mf_kt(rw) * 2 + 16; }
__host__ __device__ inline size_t mf_smem(int rw, int mt = 16) {
    return 128 + (size_t)MF_STAGES * (mf_rows(rw) * mf_wstride(rw) + mt * mf_kt(rw) * 2) +
           (size_t)mf_kt(rw) * mf_xstr(mt) * sizeof(float);
}

template <int RW, int MF_MT>
static __global__ void __launch_bounds__(MF_THREADS, 2) k_gemm_f16(const uint8_t* __restrict__ W, long w_stride,
                                                                   int N, int K, const uint8_t* __restrict__ X,
                                                                   long x_stride, int M, float* __restrict__ Y,
                                                                   long y_stride, unsigned int* err) {
    constexpr int ROWS = mf_rows(RW), KT = mf_kt(RW), MF_XSTR = mf_xstr(MF_MT);
    static_assert(MF_MT == 8 || MF_MT == 16, "8- or 16-row activation tiles");
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ int abort_flag;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem);
    constexpr int WST = mf_wstride(RW);
    uint8_t* stages = smem + 128;
    uint8_t* xst = stages + (size_t)MF_STAGES * ROWS * WST;  // [stage][MF_MT][KT] fp16 activation rows
    float* xt = reinterpret_cast<float*>(xst + (size_t)MF_STAGES * MF_MT * KT * 2);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int r = tid >> 3, l = tid & 7;
    const int row0 = blockIdx.x * ROWS, nrows = min(ROWS, N - row0);
    const int m0 = blockIdx.y * MF_MT, mt = min(MF_MT, M - m0);
    const int K8 = (K / 8) * 8;
    const int nkt = (K8 + KT - 1) / KT;
    // activation rows by bulk copy when every tile starts on a 16-byte boundary (tile sizes are
    // multiples of 8 elements)
    const bool xbulk = ((reinterpret_cast<uintptr_t>(X) | (uintptr_t)x_stride) & 15) == 0;

    // Copies of one K tile: every warp copies its own weight rows (slots 4w..4w+3: rows slot + 32 i;
    // lanes 0..4 RW-1) and two activation rows (lanes 16, 17); thread 0 arms the stage's mbarrier
    // with the tile's bytes before any of them is issued. The activation rows come from the
    // previous kernel: for the stages armed before griddepcontrol.wait they are copied after it.
    auto wrow_bytes = [&](int ne) {  // bytes of the tile's weight copies (16-byte rounded per row)
        if (((reinterpret_cast<uintptr_t>(W) | (uintptr_t)w_stride) & 15) == 0) return (uint32_t)(nrows * ne * 2);
        uint32_t t = 0;
        for (int i = 0; i < nrows; ++i)
            t += ((uint32_t)((reinterpret_cast<uintptr_t>(W) + (uintptr_t)(row0 + i) * w_stride) & 15) + ne * 2 + 15) &
                 ~15u;
        return t;
    };
    const int ne_last = K8 - (nkt - 1) * KT;
    const uint32_t wb_full = tid == 0 ? wrow_bytes(KT) : 0u, wb_last = tid == 0 ? wrow_bytes(ne_last) : 0u;
    auto arm = [&](int kt) {  // thread 0
        const int ne = min(KT, K8 - kt * KT);
        mbar_arrive_expect_tx(&bars[kt % MF_STAGES],
                              (ne == KT ? wb_full : wb_last) + (xbulk ? (uint32_t)(mt * ne * 2) : 0u));
    };
    auto copy_w = [&](int kt) {
        const int s = kt % MF_STAGES, e0 = kt * KT, ne = min(KT, K8 - e0);
        if (lane < 4 * RW) {
            const int i = 4 * warp + (lane & 3) + 32 * (lane >> 2);
            if (i < nrows) {
                const uintptr_t src =
                    reinterpret_cast<uintptr_t>(W) + (uintptr_t)(row0 + i) * w_stride + (uintptr_t)e0 * 2;
                const uint32_t off = (uint32_t)(src & 15);
                bulk_g2s(stages + ((size_t)s * ROWS + i) * WST, reinterpret_cast<const void*>(src - off),
                         (off + ne * 2 + 15) & ~15u, &bars[s]);
            }
        }
    };
    auto copy_x = [&](int kt) {
        const int s = kt % MF_STAGES, e0 = kt * KT, ne = min(KT, K8 - e0);
        const int m = 2 * warp + (lane - 16);
        if (xbulk && lane >= 16 && lane < 18 && m < mt)
            bulk_g2s(xst + ((size_t)s * MF_MT + m) * KT * 2, X + (long)(m0 + m) * x_stride + (long)e0 * 2,
                     (uint32_t)(ne * 2), &bars[s]);
    };

    if (tid == 0) {
        for (int s = 0; s < MF_STAGES; ++s) mbar_init(&bars[s], 1);
        fence_mbar_init();
        abort_flag = 0;
        for (int kt = 0; kt < min(MF_STAGES, nkt); ++kt) arm(kt);
    }
    __syncthreads();
    for (int kt = 0; kt < min(MF_STAGES, nkt); ++kt) copy_w(kt);  // weights: independent of it
    asm volatile("griddepcontrol.wait;" ::: "memory");
    for (int kt = 0; kt < min(MF_STAGES, nkt); ++kt) copy_x(kt);

    float acc[RW][MF_MT];
#pragma unroll
    for (int i = 0; i < RW; ++i)
#pragma unroll
        for (int m = 0; m < MF_MT; ++m) acc[i][m] = 0.0f;
    for (int kt = 0; kt < nkt; ++kt) {
        const int s = kt % MF_STAGES, e0 = kt * KT, ne = min(KT, K8 - e0);
        if (!abort_flag && !mbar_wait_bounded(&bars[s], (kt / MF_STAGES) & 1, err)) abort_flag = 1;
        // the activation tile as fp32, [element][row] (rows past M are 0); consecutive threads take
        // consecutive rows of one element pair (conflict-free stores)
        for (int i = tid; i < MF_MT * (KT / 2); i += MF_THREADS) {
            const int m = i % MF_MT, e = 2 * (i / MF_MT);
            float2 v = make_float2(0.0f, 0.0f);
            if (m < mt && e < ne) {  // ne and e are even: both elements lie in the row
                const uint16_t* xr = xbulk ? reinterpret_cast<const uint16_t*>(xst + ((size_t)s * MF_MT + m) * KT * 2) + e
                                           : reinterpret_cast<const uint16_t*>(X + (long)(m0 + m) * x_stride) + e0 + e;
                v.x = h2f(xr[0]);
                v.y = h2f(xr[1]);
            }
            xt[e * MF_XSTR + m] = v.x;
            xt[(e + 1) * MF_XSTR + m] = v.y;
        }
        __syncthreads();
        if (!abort_flag) {
            const uint8_t* st = stages + (size_t)s * ROWS * WST;
            const uint16_t* wt[RW];
#pragma unroll
            for (int i = 0; i < RW; ++i) {
                const int rr = min(r + 32 * i, nrows - 1);  // rows past N: computed, never stored
                const uintptr_t src =
                    reinterpret_cast<uintptr_t>(W) + (uintptr_t)(row0 + rr) * w_stride + (uintptr_t)e0 * 2;
                wt[i] = reinterpret_cast<const uint16_t*>(st + (size_t)(r + 32 * i) * WST + (src & 15));
            }
            for (int e = l; e < ne; e += 8) {
                float w[RW];
#pragma unroll
                for (int i = 0; i < RW; ++i) w[i] = h2f(wt[i][e]);
                const float4* xv = reinterpret_cast<const float4*>(xt + (size_t)e * MF_XSTR);
#pragma unroll
                for (int q = 0; q < MF_MT / 4; ++q) {
                    const float4 x4 = xv[q];
#pragma unroll
                    for (int i = 0; i < RW; ++i) {  // exact products: one rounding, as mul then add
                        acc[i][4 * q] = __fmaf_rn(x4.x, w[i], acc[i][4 * q]);
                        acc[i][4 * q + 1] = __fmaf_rn(x4.y, w[i], acc[i][4 * q + 1]);
                        acc[i][4 * q + 2] = __fmaf_rn(x4.z, w[i], acc[i][4 * q + 2]);
                        acc[i][4 * q + 3] = __fmaf_rn(x4.w, w[i], acc[i][4 * q + 3]);
                    }
                }
            }
        }
        if (tid == 0 && !abort_flag && kt + MF_STAGES < nkt) arm(kt + MF_STAGES);  // every thread passed the wait
        __syncthreads();  // the stage and the activation tile are rewritten next
        if (!abort_flag && kt + MF_STAGES < nkt) {
            copy_w(kt + MF_STAGES);
            copy_x(kt + MF_STAGES);
        }
    }
    asm volatile("griddepcontrol.launch_dependents;");
    if (abort_flag) {
        drain_stages(bars, nkt, tid);  // MF_STAGES == MM_STAGES: the same ring
        return;
    }
    // lanes summed left to right (simd_ops.h:75-78), then the scalar tail (ops.cpp:224-228)
    const int base = lane & ~7;
#pragma unroll
    for (int i = 0; i < RW; ++i) {
        const int rr = r + 32 * i;
#pragma unroll
        for (int m = 0; m < MF_MT; ++m) {
            float v[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) v[j] = __shfl_sync(0xffffffffu, acc[i][m], base + j);
            if (l == 0 && rr < nrows && m < mt) {
                float d = v[0] + v[1];
                d = d + v[2];
                d = d + v[3];
                d = d + v[4];
                d = d + v[5];
                d = d + v[6];
                d = d + v[7];
                const uint16_t* wr = reinterpret_cast<const uint16_t*>(W + (long)(row0 + rr) * w_stride);
                const uint16_t* xr = reinterpret_cast<const uint16_t*>(X + (long)(m0 + m) * x_stride);
                for (int k = K8; k < K; ++k) {
                    const float pr = h2f(xr[k]) * h2f(wr[k]);
                    d = d + pr;
                }
                Y[(long)(m0 + m) * y_stride + row0 + rr] = d;
            }
        }
    }
}

// ---- two-phase exact GEMV for small M --------------------------------------------------------
// At M = 1 there are only N*4 lane chains, too few threads to cover latency when each walks K/32
// dependent steps. Here a persistent CTA of 256 threads takes groups of R weight rows (whole rows,
// TMA double-buffered): phase 1 computes every per-block lane product fl(float(L) * (da*dw)) in
// parallel into shared memory, phase 2 runs the per-lane fp32 chains over the blocks in order
// (acc = acc + p, exactly the reference's order), phase 3 forms (L0+L1)+(L2+L3).
constexpr int GV2_THREADS = 256;

template <int WDT>
__host__ __device__ inline int gv2_rstride(int K) {
    const long rb = (long)(K / GTN_QBLK) * MMCfg<WDT>::BLK_BYTES;
    return (int)(((rb + 15) & ~15L) + 16);
}
template <int WDT>
__host__ __device__ inline size_t gv2_smem(int R, int mt, int K) {
    const int nb = K / GTN_QBLK;
    return 128 + (size_t)2 * R * gv2_rstride<WDT>(K) + (size_t)mt * nb * 4 * sizeof(LanePrep) +
           (size_t)mt * R * 4 * (nb + 1) * sizeof(float) + (size_t)mt * R * 4 * sizeof(float);
}

template <int WDT, int R, int MT>
__global__ void __launch_bounds__(GV2_THREADS) k_gemv2(const uint8_t* __restrict__ W, long w_stride, int N, int K,
                                                       const uint8_t* __restrict__ X, long x_stride, int M,
                                                       float* __restrict__ Y, long y_stride, unsigned int* err) {
    using C = MMCfg<WDT>;
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ int abort_flag;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem);
    const int nb = K / GTN_QBLK;
    const long rb = (long)nb * C::BLK_BYTES;
    const int rstride = gv2_rstride<WDT>(K);
    uint8_t* stage = smem + 128;
    LanePrep* prep = reinterpret_cast<LanePrep*>(stage + (size_t)2 * R * rstride);
    const int m0 = blockIdx.y * MT;
    const int mt = min(MT, M - m0);
    float* prod = reinterpret_cast<float*>(prep + (size_t)MT * nb * 4);
    const int pstr = nb + 1;
    float* res = prod + (size_t)MT * R * 4 * pstr;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int ngroups = (N + R - 1) / R;

    auto issue = [&](int g, int s) {  // warp 0
        const int r0 = g * R, nr = min(R, N - r0);
        uint32_t total = 0;
        for (int r = 0; r < nr; ++r) {
            const uintptr_t src = reinterpret_cast<uintptr_t>(W) + (uintptr_t)(r0 + r) * w_stride;
            total += ((uint32_t)(src & 15) + (uint32_t)rb + 15) & ~15u;
        }
        if (lane == 0) mbar_arrive_expect_tx(&bars[s], total);
        __syncwarp();
        for (int r = lane; r < nr; r += 32) {
            const uintptr_t src = reinterpret_cast<uintptr_t>(W) + (uintptr_t)(r0 + r) * w_stride;
            const uint32_t off = (uint32_t)(src & 15);
            bulk_g2s(stage + ((size_t)s * R + r) * rstride, reinterpret_cast<const void*>(src - off),
                     (off + (uint32_t)rb + 15) & ~15u, &bars[s]);
        }
    };

    if (tid == 0) {
        mbar_init(&bars[0], 1);
        mbar_init(&bars[1], 1);
        fence_mbar_init();
        abort_flag = 0;
    }
    __syncthreads();
    const int g0 = blockIdx.x;
    int nissued[2] = {0, 0};  // meaningful in warp 0, which issues every copy
    if (warp == 0) {
        if (g0 < ngroups) issue(g0, 0), ++nissued[0];
        if (g0 + (int)gridDim.x < ngroups) issue(g0 + gridDim.x, 1), ++nissued[1];
    }
    asm volatile("griddepcontrol.wait;" ::: "memory");
    build_prep_q8(X, x_stride, m0, mt, nb, prep);
    __syncthreads();
    int it = 0;
    for (int g = g0; g < ngroups; g += gridDim.x, ++it) {
        const int s = it & 1;
        const int r0 = g * R, nr = min(R, N - r0);
        if (!abort_flag && !mbar_wait_bounded(&bars[s], (it >> 1) & 1, err)) abort_flag = 1;
        __syncthreads();
        if (!abort_flag) {
            for (int item = tid; item < nr * nb; item += GV2_THREADS) {
                const int r = item / nb, b = item - r * nb;
                const uintptr_t src = reinterpret_cast<uintptr_t>(W) + (uintptr_t)(r0 + r) * w_stride;
                const uint8_t* p = stage + ((size_t)s * R + r) * rstride + (src & 15) + (size_t)b * C::BLK_BYTES;
                const float dw = h2f(ld_u16(p));
#pragma unroll
                for (int m = 0; m < MT; ++m) {
                    if (m < mt) {
#pragma unroll
                        for (int l = 0; l < 4; ++l) {
                            const LanePrep av = prep[((size_t)m * nb + b) * 4 + l];
                            const int L = WDT == GTN_Q8 ? q8_block_lane_dot(p, l, av) : q4_block_lane_dot(p, l, av);
                            const float sc = av.da * dw;
                            prod[((size_t)(m * R + r) * 4 + l) * pstr + b] = lane_sum_f32(L) * sc;
                        }
                    }
                }
            }
        }
        __syncthreads();
        if (warp == 0 && !abort_flag && g + 2 * (int)gridDim.x < ngroups) issue(g + 2 * gridDim.x, s), ++nissued[s];
        if (!abort_flag) {
            for (int c = tid; c < mt * nr * 4; c += GV2_THREADS) {
                const int m = c / (nr * 4), rl = c - m * nr * 4;  // rl = r*4 + l
                const float* pp = prod + ((size_t)(m * R) * 4 + rl) * pstr;
                float acc = 0.0f;
#pragma unroll 8
                for (int b = 0; b < nb; ++b) acc = acc + pp[b];
                res[c] = acc;
            }
        }
        __syncthreads();
        if (!abort_flag) {
            for (int t = tid; t < mt * nr; t += GV2_THREADS) {
                const int m = t / nr, r = t - m * nr;
                const float* q = res + (size_t)t * 4;
                const float y = (q[0] + q[1]) + (q[2] + q[3]);
                Y[(long)(m0 + m) * y_stride + r0 + r] = y;
            }
        }
        __syncthreads();
    }
    asm volatile("griddepcontrol.launch_dependents;");
    if (abort_flag && tid == 0) {
        // bounded wait for the last copy issued into each stage (phase nissued-1)
        for (int s = 0; s < 2; ++s) {
            if (nissued[s] == 0) continue;
            for (uint32_t i = 0; i < GTN_WAIT_LIMIT; ++i)
                if (mbar_try_wait(&bars[s], (uint32_t)(nissued[s] - 1) & 1)) break;
        }
    }
}

// ---- single-row GEMV with the activation in registers (M = 1, 16-byte aligned weight rows) ------
// Same arithmetic and order as k_gemv2. Thread (row slot rs, block group j) keeps the lane words of
// activation blocks 4j..4j+3 in registers for the whole launch; weight rows arrive by TMA into a
// double-buffered stage; phase 1 reads a thread's 4 weight blocks with 8-byte shared loads
// (conflict-free: a half-warp covers 16 consecutive groups of one row), extracts the lane words
// with byte permutes and writes the 16 products as four float4 (one per lane, blocks 4j..4j+3);
// phase 2 runs the lane chains (acc = acc + p in block order) and the final (L0+L1)+(L2+L3).
// Row stride of the products: a multiple of 4 floats, odd in float4 units (conflict-free float4
// reads across 8 consecutive chains). grid: persistent over groups of R rows; block 256.
constexpr int GV3_THREADS = 256;

template <int WDT>
__host__ __device__ inline int gv3_rstride(int K) {
    return ((K / GTN_QBLK) * MMCfg<WDT>::BLK_BYTES + 15) & ~15;
}
__host__ __device__ inline int gv3_pstr(int nb) { return ((nb + 7) & ~7) + 4; }
template <int WDT>
__host__ __device__ inline size_t gv3_smem(int R, int K) {
    return 128 + (size_t)2 * R * gv3_rstride<WDT>(K) + (size_t)R * 4 * gv3_pstr(K / GTN_QBLK) * sizeof(float) +
           (((size_t)(K / GTN_QBLK) * GTN_Q8_BYTES + 15) & ~(size_t)15);  // + the activation row
}

// Little-endian u16 at even byte offset o of a register-resident byte array (o folds at compile
// time once the loops are unrolled).
__device__ __forceinline__ uint32_t gv3_u16(const uint32_t* w, int o) { return (w[o >> 2] >> ((o & 2) * 8)) & 0xffffu; }
// (u16 at o1) | (u16 at o2) << 16
__device__ __forceinline__ int gv3_pair(const uint32_t* w, int o1, int o2) {
    const unsigned sel = (unsigned)(o1 & 2) | ((unsigned)((o1 & 2) + 1) << 4) | ((unsigned)(4 + (o2 & 2)) << 8) |
                         ((unsigned)(5 + (o2 & 2)) << 12);
    return (int)__byte_perm(w[o1 >> 2], w[o2 >> 2], sel);
}

// Shared memory of k_gemv3: [mbarriers 128][2 stages of R weight rows][products R*4 rows of pstr
// floats][the activation row]. gv3_bars / gv3_stage / gv3_prod / gv3_xs give the pieces.
template <int WDT>
__device__ __forceinline__ uint8_t* gv3_stage(uint8_t* smem) { return smem + 128; }
template <int WDT>
__device__ __forceinline__ float* gv3_prod(uint8_t* smem, int R, int K) {
    return reinterpret_cast<float*>(smem + 128 + (size_t)2 * R * gv3_rstride<WDT>(K));
}
template <int WDT>
__device__ __forceinline__ uint8_t* gv3_xs(uint8_t* smem, int R, int K) {
    return reinterpret_cast<uint8_t*>(gv3_prod<WDT>(smem, R, K) + (size_t)R * 4 * gv3_pstr(K / GTN_QBLK));
}

// Issues the TMA copies of group g (R rows, W and w_stride 16-byte aligned) into stage s; warp 0.
template <int WDT>
__device__ __forceinline__ void gv3_issue(uint8_t* smem, const uint8_t* W, long w_stride, int N, int K, int R, int g,
                                          int s) {
    const int lane = threadIdx.x & 31, rstride = gv3_rstride<WDT>(K);
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem);
    uint8_t* stage = gv3_stage<WDT>(smem);
    const int r0 = g * R, nr = min(R, N - r0);
    if (lane == 0) mbar_arrive_expect_tx(&bars[s], (uint32_t)rstride * (uint32_t)nr);
    __syncwarp();
    for (int r = lane; r < nr; r += 32)
        bulk_g2s(stage + ((size_t)s * R + r) * rstride, W + (size_t)(r0 + r) * w_stride, (uint32_t)rstride, &bars[s]);
}

// Before the kernel waits for its predecessor: barrier init and the copies of this CTA's first two
// groups. nissued[s]: copies issued into stage s (meaningful in warp 0).
template <int WDT>
__device__ __forceinline__ void gv3_prefetch(uint8_t* smem, const uint8_t* W, long w_stride, int N, int K, int R,
                                             int* abort_flag, int nissued[2]) {
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem);
    if (threadIdx.x == 0) {
        mbar_init(&bars[0], 1);
        mbar_init(&bars[1], 1);
        fence_mbar_init();
        *abort_flag = 0;
    }
    __syncthreads();
    const int ngroups = (N + R - 1) / R, g0 = blockIdx.x;
    nissued[0] = nissued[1] = 0;
    if ((threadIdx.x >> 5) == 0) {
        if (g0 < ngroups) gv3_issue<WDT>(smem, W, w_stride, N, K, R, g0, 0), ++nissued[0];
        if (g0 + (int)gridDim.x < ngroups) gv3_issue<WDT>(smem, W, w_stride, N, K, R, g0 + gridDim.x, 1), ++nissued[1];
    }
}

// The GEMV over this CTA's groups once the Q8 activation row is in shared memory (gv3_xs): phase 1
// products, phase 2 lane chains, Y[r] = (L0+L1)+(L2+L3). Ends with griddepcontrol.launch_dependents.
template <int WDT>
__device__ __forceinline__ void gv3_main(uint8_t* smem, const uint8_t* __restrict__ W, long w_stride, int N, int K,
                                         float* __restrict__ Y, int R, int RP, unsigned int* err, int* abort_flag,
                                         int nissued[2]) {
    using C = MMCfg<WDT>;
    constexpr int GB = 4 * C::BLK_BYTES, GW = GB / 4;  // bytes / words of 4 weight blocks
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem);
    const int nb = K / GTN_QBLK, nbg = nb / 4;
    const int rstride = gv3_rstride<WDT>(K);
    const int pstr = gv3_pstr(nb);
    uint8_t* stage = gv3_stage<WDT>(smem);
    float* prod = gv3_prod<WDT>(smem, R, K);
    const uint8_t* xs = gv3_xs<WDT>(smem, R, K);
    const int tid = threadIdx.x, warp = tid >> 5;
    const int j = tid % nbg, rs = tid / nbg;
    const bool p1 = rs < RP;
    const int ngroups = (N + R - 1) / R, g0 = blockIdx.x;
    // this thread's lane words of activation blocks 4j..4j+3 (same packing as build_prep_q8) from
    // four 34-byte blocks read as 8-byte words
    int a0[16], a1[16], asum[16];
    float da[4];
    {
        uint32_t xw[34];
        const uint2* xsrc = reinterpret_cast<const uint2*>(xs + (size_t)j * 4 * GTN_Q8_BYTES);  // 8-byte aligned
#pragma unroll
        for (int q = 0; q < 17; ++q) {
            const uint2 t = p1 ? xsrc[q] : make_uint2(0u, 0u);
            xw[2 * q] = t.x;
            xw[2 * q + 1] = t.y;
        }
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const int ob = k * GTN_Q8_BYTES;
            da[k] = h2f((uint16_t)gv3_u16(xw, ob));
#pragma unroll
            for (int l = 0; l < 4; ++l) {
                const int w0 = gv3_pair(xw, ob + 2 + 2 * l, ob + 10 + 2 * l);
                const int w1 = gv3_pair(xw, ob + 18 + 2 * l, ob + 26 + 2 * l);
                a0[k * 4 + l] = w0;
                a1[k * 4 + l] = w1;
                asum[k * 4 + l] = dp4a(w0, 0x01010101, dp4a(w1, 0x01010101, 0));
            }
        }
    }
    int it = 0;
    for (int g = g0; g < ngroups; g += gridDim.x, ++it) {
        const int s = it & 1;
        const int r0 = g * R, nr = min(R, N - r0);
        if (!*abort_flag && !mbar_wait_bounded(&bars[s], (it >> 1) & 1, err)) *abort_flag = 1;
        __syncthreads();
        if (*abort_flag) break;
        if (p1) {
            for (int r = rs; r < nr; r += RP) {
                const uint2* src = reinterpret_cast<const uint2*>(stage + ((size_t)s * R + r) * rstride + (size_t)j * GB);
                uint32_t w[GW];
#pragma unroll
                for (int q = 0; q < GW / 2; ++q) {
                    const uint2 t = src[q];
                    w[2 * q] = t.x;
                    w[2 * q + 1] = t.y;
                }
                float o[4][4];  // [lane][block]
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    const int ob = k * C::BLK_BYTES;
                    const float sc = da[k] * h2f((uint16_t)gv3_u16(w, ob));
#pragma unroll
                    for (int l = 0; l < 4; ++l) {
                        int L;
                        if (WDT == GTN_Q8) {
                            const int w0 = gv3_pair(w, ob + 2 + 2 * l, ob + 10 + 2 * l);
                            const int w1 = gv3_pair(w, ob + 18 + 2 * l, ob + 26 + 2 * l);
                            L = dp4a(w0, a0[k * 4 + l], dp4a(w1, a1[k * 4 + l], 0));
                        } else {
                            const int wb = gv3_pair(w, ob + 2 + 2 * l, ob + 10 + 2 * l);
                            const int hi = (wb >> 4) & 0x0f0f0f0f, lo = wb & 0x0f0f0f0f;
                            L = dp4a(hi, a0[k * 4 + l], dp4a(lo, a1[k * 4 + l], 0)) - 7 * asum[k * 4 + l];
                        }
                        o[l][k] = lane_sum_f32(L) * sc;
                    }
                }
#pragma unroll
                for (int l = 0; l < 4; ++l)
                    *reinterpret_cast<float4*>(prod + (size_t)(r * 4 + l) * pstr + 4 * j) =
                        make_float4(o[l][0], o[l][1], o[l][2], o[l][3]);
            }
        }
        __syncthreads();
        if (warp == 0 && g + 2 * (int)gridDim.x < ngroups) {
            gv3_issue<WDT>(smem, W, w_stride, N, K, R, g + 2 * gridDim.x, s);
            ++nissued[s];
        }
        if (tid < ((R * 4 + 31) & ~31)) {  // whole warps: the combine shuffles need every lane
            const int r = tid >> 2, l = tid & 3;
            float acc = 0.0f;
            if (r < nr) {
                const float4* pp = reinterpret_cast<const float4*>(prod + (size_t)(r * 4 + l) * pstr);
                for (int b4 = 0; b4 < nbg; ++b4) {
                    const float4 v = pp[b4];
                    acc = acc + v.x;
                    acc = acc + v.y;
                    acc = acc + v.z;
                    acc = acc + v.w;
                }
            }
            const float t01 = acc + __shfl_xor_sync(0xffffffffu, acc, 1);
            const float t = t01 + __shfl_xor_sync(0xffffffffu, t01, 2);
            if (l == 0 && r < nr) Y[r0 + r] = t;
        }
        __syncthreads();  // the products are rewritten by the next group
    }
    asm volatile("griddepcontrol.launch_dependents;");
    if (*abort_flag && tid == 0) {
        // bounded wait for the last copy issued into each stage (phase nissued-1)
        for (int s = 0; s < 2; ++s) {
            if (nissued[s] == 0) continue;
            for (uint32_t i = 0; i < GTN_WAIT_LIMIT; ++i)
                if (mbar_try_wait(&bars[s], (uint32_t)(nissued[s] - 1) & 1)) break;
        }
    }
}

template <int WDT>
__global__ void __launch_bounds__(GV3_THREADS, 2) k_gemv3(const uint8_t* __restrict__ W, long w_stride, int N, int K,
                                                         const uint8_t* __restrict__ X, float* __restrict__ Y, int R,
                                                         int RP, unsigned int* err) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ int abort_flag;
    int nissued[2];
    gv3_prefetch<WDT>(smem, W, w_stride, N, K, R, &abort_flag, nissued);
    asm volatile("griddepcontrol.wait;" ::: "memory");
    // the activation row into shared memory (coalesced)
    uint8_t* xs = gv3_xs<WDT>(smem, R, K);
    const int xbytes = (K / GTN_QBLK) * GTN_Q8_BYTES, tid = threadIdx.x;
    if ((reinterpret_cast<uintptr_t>(X) & 3) == 0) {
        for (int i = tid; i < xbytes / 4; i += GV3_THREADS)
            reinterpret_cast<uint32_t*>(xs)[i] = reinterpret_cast<const uint32_t*>(X)[i];
        if (tid < (xbytes & 3)) xs[(xbytes & ~3) + tid] = X[(xbytes & ~3) + tid];
    } else {
        for (int i = tid; i < xbytes; i += GV3_THREADS) xs[i] = X[i];
    }
    __syncthreads();
    gv3_main<WDT>(smem, W, w_stride, N, K, Y, R, RP, err, &abort_flag, nissued);
}

// ---- exact GEMM for M >= 2 activation rows (prefill, batched decode) ----------------------------
// The arithmetic and order of k_gemv3, for a tile of R weight rows x MT activation rows per CTA:
// thread (row slot rs < R, block group j) keeps the weight bytes of blocks 4j..4j+3 of its row in
// registers; the activation lane words of the MT rows are built once in shared memory; the rows
// are processed MC at a time: phase 1 writes the 16 products per (activation row, thread) as four
// float4, phase 2 runs the MC*R*4 lane chains in block order and the (L0+L1)+(L2+L3) combine.
// The R weight rows arrive with one TMA bulk copy each (16-byte aligned rows). grid (ceil(N/R),
// ceil(M/MT)); block 256.
struct GM3Plan {
    int R, MT, MC;
};
template <int WDT>
__host__ __device__ inline size_t gm3_smem(int R, int MT, int MC, int K) {
    const int nb = K / GTN_QBLK;
    const size_t prep = (size_t)MT * nb * (4 * 8 + 4 + (WDT == GTN_Q4 ? 16 : 0));  // lane words, da, [sums]
    return 128 + (size_t)R * gv3_rstride<WDT>(K) + ((prep + 15) & ~(size_t)15) +
           (size_t)MC * R * 4 * gv3_pstr(nb) * sizeof(float);
}

template <int WDT>
__global__ void __launch_bounds__(GV3_THREADS, 2) k_gemm3(const uint8_t* __restrict__ W, long w_stride, int N, int K,
                                                         const uint8_t* __restrict__ X, long x_stride, int M,
                                                         float* __restrict__ Y, long y_stride, int R, int MT, int MC,
                                                         unsigned int* err) {
    using C = MMCfg<WDT>;
    constexpr int GB = 4 * C::BLK_BYTES, GW = GB / 4;
    extern __shared__ __align__(128) uint8_t smem[];
    uint64_t* bar = reinterpret_cast<uint64_t*>(smem);
    const int nb = K / GTN_QBLK, nbg = nb / 4;
    const int rstride = gv3_rstride<WDT>(K), pstr = gv3_pstr(nb);
    uint8_t* stage = smem + 128;
    // activation lane words [MT][4 blocks k][4 lanes][nbg groups j] (block 4j+k): a warp's threads
    // (consecutive j) read consecutive words; da [MT][4][nbg]; lane sums (Q4) like the words
    int2* pa = reinterpret_cast<int2*>(stage + (size_t)R * rstride);
    float* pda = reinterpret_cast<float*>(pa + (size_t)MT * nb * 4);
    int* ps = reinterpret_cast<int*>(pda + (size_t)MT * nb);
    const size_t prep = (size_t)MT * nb * (4 * 8 + 4 + (WDT == GTN_Q4 ? 16 : 0));
    float* prod = reinterpret_cast<float*>(stage + (size_t)R * rstride + ((prep + 15) & ~(size_t)15));
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int j = tid % nbg, rs = tid / nbg;
    const int r0 = blockIdx.x * R, nr = min(R, N - r0);
    const int m0 = blockIdx.y * MT, mt = min(MT, M - m0);
    const bool p1 = rs < nr;
    if (tid == 0) {
        mbar_init(bar, 1);
        fence_mbar_init();
        mbar_arrive_expect_tx(bar, (uint32_t)rstride * (uint32_t)nr);
    }
    __syncwarp();
    if (warp == 0)
        for (int r = lane; r < nr; r += 32)
            bulk_g2s(stage + (size_t)r * rstride, W + (size_t)(r0 + r) * w_stride, (uint32_t)rstride, bar);
    asm volatile("griddepcontrol.wait;" ::: "memory");
    // activation lane words of the MT rows; the raw rows are first copied with coalesced 4-byte
    // loads into the (not yet used) product buffer when they fit there and are word aligned
    const int xrow = nb * GTN_Q8_BYTES;
    const bool stage_x = (size_t)mt * xrow <= (size_t)MC * R * 4 * pstr * sizeof(float) &&
                         ((reinterpret_cast<uintptr_t>(X) | (uintptr_t)x_stride | (uintptr_t)xrow) & 3) == 0;
    const uint8_t* xsrc = X + (long)m0 * x_stride;
    long xss = x_stride;
    if (stage_x) {
        const int wpr = xrow / 4;
        uint32_t* xd = reinterpret_cast<uint32_t*>(prod);
        for (int i = tid; i < mt * wpr; i += GV3_THREADS) {
            const int m = i / wpr, w = i - m * wpr;
            xd[i] = reinterpret_cast<const uint32_t*>(xsrc + (long)m * x_stride)[w];
        }
        __syncthreads();
        xsrc = reinterpret_cast<const uint8_t*>(prod);
        xss = xrow;
    }
    for (int i = tid; i < mt * nb * 4; i += GV3_THREADS) {
        const int l = i & 3, b = (i >> 2) % nb, m = (i >> 2) / nb;
        const uint8_t* blk = xsrc + (long)m * xss + (long)b * GTN_Q8_BYTES;
        const uint8_t* q = blk + 2;
        const int w0 = (int)ld_u16(q + 2 * l) | ((int)ld_u16(q + 8 + 2 * l) << 16);
        const int w1 = (int)ld_u16(q + 16 + 2 * l) | ((int)ld_u16(q + 24 + 2 * l) << 16);
        const int jj = b >> 2, k = b & 3;
        const size_t o = ((size_t)(m * 4 + k) * 4 + l) * nbg + jj;
        pa[o] = make_int2(w0, w1);
        if (WDT == GTN_Q4) ps[o] = dp4a(w0, 0x01010101, dp4a(w1, 0x01010101, 0));
        if (l == 0) pda[(size_t)(m * 4 + k) * nbg + jj] = h2f(ld_u16(blk));
    }
    const bool ok = __syncthreads_and(mbar_wait_bounded(bar, 0, err));
    if (!ok) {  // the copy did not land in time: wait (bounded) for it before leaving
        if (tid == 0)
            for (uint32_t it = 0; it < GTN_WAIT_LIMIT; ++it)
                if (mbar_try_wait(bar, 0)) break;
        return;
    }
    uint32_t w[GW];
    if (p1) {
        const uint2* src = reinterpret_cast<const uint2*>(stage + (size_t)rs * rstride + (size_t)j * GB);
#pragma unroll
        for (int q = 0; q < GW / 2; ++q) {
            const uint2 t = src[q];
            w[2 * q] = t.x;
            w[2 * q + 1] = t.y;
        }
    }
    float dw[4];
    int wl0[16], wl1[16];  // weight lane words per (block, lane)
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const int ob = k * C::BLK_BYTES;
        dw[k] = p1 ? h2f((uint16_t)gv3_u16(w, ob)) : 0.0f;
#pragma unroll
        for (int l = 0; l < 4; ++l) {
            if (WDT == GTN_Q8) {
                wl0[k * 4 + l] = p1 ? gv3_pair(w, ob + 2 + 2 * l, ob + 10 + 2 * l) : 0;
                wl1[k * 4 + l] = p1 ? gv3_pair(w, ob + 18 + 2 * l, ob + 26 + 2 * l) : 0;
            } else {
                const int wb = p1 ? gv3_pair(w, ob + 2 + 2 * l, ob + 10 + 2 * l) : 0;
                wl0[k * 4 + l] = (wb >> 4) & 0x0f0f0f0f;
                wl1[k * 4 + l] = wb & 0x0f0f0f0f;
            }
        }
    }
    const int nch = R * 4;  // chains per activation row
    for (int c0 = 0; c0 < mt; c0 += MC) {
        const int mc = min(MC, mt - c0);
        if (p1) {
            for (int mm = 0; mm < mc; ++mm) {
                const int m = c0 + mm;
                float o[4][4];
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    const float sc = pda[(size_t)(m * 4 + k) * nbg + j] * dw[k];
#pragma unroll
                    for (int l = 0; l < 4; ++l) {
                        const size_t o2 = ((size_t)(m * 4 + k) * 4 + l) * nbg + j;
                        const int2 av = pa[o2];
                        int L = dp4a(wl0[k * 4 + l], av.x, dp4a(wl1[k * 4 + l], av.y, 0));
                        if (WDT == GTN_Q4) L -= 7 * ps[o2];
                        o[l][k] = lane_sum_f32(L) * sc;
                    }
                }
#pragma unroll
                for (int l = 0; l < 4; ++l)
                    *reinterpret_cast<float4*>(prod + ((size_t)(mm * R + rs) * 4 + l) * pstr + 4 * j) =
                        make_float4(o[l][0], o[l][1], o[l][2], o[l][3]);
            }
        }
        __syncthreads();
        for (int cb = 0; cb < mc * nch; cb += GV3_THREADS) {  // whole warps: the combine shuffles
            const int c = cb + tid;
            const int mm = c / nch, rl = c - mm * nch, r = rl >> 2;
            const bool valid = c < mc * nch && r < nr;
            float acc = 0.0f;
            if (valid) {
                const float4* pp = reinterpret_cast<const float4*>(prod + (size_t)c * pstr);
                for (int b4 = 0; b4 < nbg; ++b4) {
                    const float4 v = pp[b4];
                    acc = acc + v.x;
                    acc = acc + v.y;
                    acc = acc + v.z;
                    acc = acc + v.w;
                }
            }
            const float t01 = acc + __shfl_xor_sync(0xffffffffu, acc, 1);
            const float t = t01 + __shfl_xor_sync(0xffffffffu, t01, 2);
            if (valid && (c & 3) == 0) Y[(long)(m0 + c0 + mm) * y_stride + r0 + r] = t;
        }
        __syncthreads();
    }
    asm volatile("griddepcontrol.launch_dependents;");
}

// ---- persistent exact GEMM for a few activation rows (batched decode steps) -----------------------
// The arithmetic and order of k_gemm3 (and k_gemv3) for M >= 2 rows, arranged so that the weight
// stream overlaps the arithmetic: a CTA prepares the lane words of its MT-row activation tile once
// (k_gemm3's conflict-free layout) and then walks groups of R weight rows (one thread per (row,
// 4-block group)) persistently. Per group it waits for the group's TMA bulk copies, moves its
// weight lane words into registers, releases the single stage and at once issues the copies of
// its next group, which land while this group computes: per chunk of MC activation rows, phase 1
// writes the 16 products of each (activation row, thread) as four float4 and phase 2 runs the
// MC * R * 4 lane chains in block order and the (L0 + L1) + (L2 + L3) combine.
// Per product: two dp4a accumulating onto the bias 0x4B400000 (so the int32 lane sum L arrives as
// the fp32 bit pattern of 1.5 * 2^23 + L, exact for |L| < 2^22), one subtraction of 1.5 * 2^23 (the
// exact fp32 value of L) and the multiply by fp32(da) * fp32(dw); the activation lane words of
// two lanes come in one 16-byte shared load ([row][block k][lane pair][group j] layout, threads of
// consecutive groups read consecutive 16 bytes). NBG > 0 fixes K / 128 (the 4-block groups per
// row) at compile time, so that every shared-memory offset is an immediate; NBG = 0 reads it from K.
// grid (persistent over the groups, ceil(M / MT)); block 256; two CTAs per SM when shared memory
// allows. W rows 16-byte aligned (rstride-byte copies).
struct GM4Plan {
    int R, MT, MC, occ;
};
template <int WDT>
__host__ __device__ inline size_t gm4_prep_bytes(int MT, int nb) {
    return ((size_t)MT * nb * (4 * 8 + 4 + (WDT == GTN_Q4 ? 16 : 0)) + 15) & ~(size_t)15;
}
template <int WDT>
__host__ __device__ inline size_t gm4_smem(int R, int MT, int MC, int K) {
    const int nb = K / GTN_QBLK;
    return 128 + (size_t)R * gv3_rstride<WDT>(K) + gm4_prep_bytes<WDT>(MT, nb) +
           (size_t)MC * R * 4 * gv3_pstr(nb) * sizeof(float);
}

template <int WDT, int NBG>
__global__ void __launch_bounds__(GV3_THREADS, 2) k_gemm4(const uint8_t* __restrict__ W, long w_stride, int N, int K,
                                                         const uint8_t* __restrict__ X, long x_stride, int M,
                                                         float* __restrict__ Y, long y_stride, int R, int MT, int MC,
                                                         unsigned int* err) {
    using C = MMCfg<WDT>;
    constexpr int GB = 4 * C::BLK_BYTES, GW = GB / 4;
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ int abort_flag;
    uint64_t* bar = reinterpret_cast<uint64_t*>(smem);
    const int nbg = NBG > 0 ? NBG : K / (4 * GTN_QBLK), nb = 4 * nbg;
    const int rstride = gv3_rstride<WDT>(K), pstr = gv3_pstr(nb);
    uint8_t* stage = smem + 128;
    int4* pa = reinterpret_cast<int4*>(stage + (size_t)R * rstride);  // [MT][4 k][2 lane pairs][nbg]
    float* pda = reinterpret_cast<float*>(pa + (size_t)MT * nb * 2);  // [MT][4 k][nbg]
    int* ps = reinterpret_cast<int*>(pda + (size_t)MT * nb);          // Q4: lane sums [MT][4 k][4 l][nbg]
    float* prod = reinterpret_cast<float*>(stage + (size_t)R * rstride + gm4_prep_bytes<WDT>(MT, nb));
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int j = tid % nbg, rs = tid / nbg;
    const int m0 = blockIdx.y * MT, mt = min(MT, M - m0);
    const int ngroups = (N + R - 1) / R;
    int nissued = 0;  // copies issued into the stage (warp 0)
    auto issue = [&](int g) {  // warp 0: the rows of group g into the stage
        const int r0 = g * R, nr = min(R, N - r0);
        if (lane == 0) mbar_arrive_expect_tx(bar, (uint32_t)rstride * (uint32_t)nr);
        __syncwarp();
        for (int r = lane; r < nr; r += 32)
            bulk_g2s(stage + (size_t)r * rstride, W + (size_t)(r0 + r) * w_stride, (uint32_t)rstride, bar);
    };
    if (tid == 0) {
        mbar_init(bar, 1);
        fence_mbar_init();
        abort_flag = 0;
    }
    __syncthreads();
    if (warp == 0 && (int)blockIdx.x < ngroups) {  // weights do not depend on the previous kernel
        issue(blockIdx.x);
        ++nissued;
    }
    asm volatile("griddepcontrol.wait;" ::: "memory");
    // the tile's activation lane words. Word-aligned rows are first copied with coalesced 4-byte
    // loads into the (not yet used) product buffer, as many rows per pass as fit there (long rows
    // take several passes); converting straight from global memory with 2-byte loads is one chain
    // of L2 round trips per thread
    const int xrow = nb * GTN_Q8_BYTES;
    const size_t pbytes = (size_t)MC * R * 4 * pstr * sizeof(float);
    const bool aligned = ((reinterpret_cast<uintptr_t>(X) | (uintptr_t)x_stride | (uintptr_t)xrow) & 3) == 0;
    const int per_pass = aligned ? (int)min((size_t)mt, pbytes / (size_t)xrow) : 0;
    const int step = per_pass > 0 ? per_pass : mt;
    for (int p0 = 0; p0 < mt; p0 += step) {
        const int pr = min(step, mt - p0);
        const uint8_t* xsrc = X + (long)(m0 + p0) * x_stride;
        long xss = x_stride;
        if (per_pass > 0) {
            const int wpr = xrow / 4;
            uint32_t* xd = reinterpret_cast<uint32_t*>(prod);
            for (int i = tid; i < pr * wpr; i += GV3_THREADS) {
                const int m = i / wpr, w = i - m * wpr;
                xd[i] = reinterpret_cast<const uint32_t*>(xsrc + (long)m * x_stride)[w];
            }
            __syncthreads();
            xsrc = reinterpret_cast<const uint8_t*>(prod);
            xss = xrow;
        }
        for (int i = tid; i < pr * nb * 4; i += GV3_THREADS) {
            const int l = i & 3, b = (i >> 2) % nb, mp = (i >> 2) / nb, m = p0 + mp;
            const uint8_t* blk = xsrc + (long)mp * xss + (long)b * GTN_Q8_BYTES;
            const uint8_t* q = blk + 2;
            const int w0 = (int)ld_u16(q + 2 * l) | ((int)ld_u16(q + 8 + 2 * l) << 16);
            const int w1 = (int)ld_u16(q + 16 + 2 * l) | ((int)ld_u16(q + 24 + 2 * l) << 16);
            const int jj = b >> 2, k = b & 3;
            int* pw = reinterpret_cast<int*>(pa + ((size_t)(m * 4 + k) * 2 + (l >> 1)) * nbg + jj) + 2 * (l & 1);
            pw[0] = w0;
            pw[1] = w1;
            if (WDT == GTN_Q4)
                ps[((size_t)(m * 4 + k) * 4 + l) * nbg + jj] = dp4a(w0, 0x01010101, dp4a(w1, 0x01010101, 0));
            if (l == 0) pda[(size_t)(m * 4 + k) * nbg + jj] = h2f(ld_u16(blk));
        }
        __syncthreads();  // this pass's lane words in place; the staged rows may be overwritten
    }
    const int nch = R * 4;  // chains per activation row
    int it = 0;
    for (int g = blockIdx.x; g < ngroups; g += gridDim.x, ++it) {
        const int r0 = g * R, nr = min(R, N - r0);
        const bool p1 = rs < nr;  // rs < R for every thread below R * nbg
        if (!abort_flag && !mbar_wait_bounded(bar, (uint32_t)it & 1u, err)) abort_flag = 1;
        __syncthreads();
        if (abort_flag) break;
        float dw[4];
        int wl0[16], wl1[16];  // weight lane words per (block, lane)
        {
            uint32_t w[GW];
            if (p1) {
                const uint2* src = reinterpret_cast<const uint2*>(stage + (size_t)rs * rstride + (size_t)j * GB);
#pragma unroll
                for (int q = 0; q < GW / 2; ++q) {
                    const uint2 t = src[q];
                    w[2 * q] = t.x;
                    w[2 * q + 1] = t.y;
                }
            }
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const int ob = k * C::BLK_BYTES;
                dw[k] = p1 ? h2f((uint16_t)gv3_u16(w, ob)) : 0.0f;
#pragma unroll
                for (int l = 0; l < 4; ++l) {
                    if (WDT == GTN_Q8) {
                        wl0[k * 4 + l] = p1 ? gv3_pair(w, ob + 2 + 2 * l, ob + 10 + 2 * l) : 0;
                        wl1[k * 4 + l] = p1 ? gv3_pair(w, ob + 18 + 2 * l, ob + 26 + 2 * l) : 0;
                    } else {
                        const int wb = p1 ? gv3_pair(w, ob + 2 + 2 * l, ob + 10 + 2 * l) : 0;
                        wl0[k * 4 + l] = (wb >> 4) & 0x0f0f0f0f;
                        wl1[k * 4 + l] = wb & 0x0f0f0f0f;
                    }
                }
            }
        }
        __syncthreads();  // the stage is free: the next group's copies land while this one computes
        if (warp == 0 && g + (int)gridDim.x < ngroups) {
            issue(g + gridDim.x);
            ++nissued;
        }
        for (int c0 = 0; c0 < mt; c0 += MC) {
            const int mc = min(MC, mt - c0);
            if (p1) {
                for (int mm = 0; mm < mc; ++mm) {
                    const int m = c0 + mm;
                    const int4* pam = pa + (size_t)m * 8 * nbg + j;
                    const float* pdm = pda + (size_t)m * 4 * nbg + j;
                    float o[4][4];
#pragma unroll
                    for (int k = 0; k < 4; ++k) {
                        const float sc = pdm[k * nbg] * dw[k];
#pragma unroll
                        for (int lp = 0; lp < 2; ++lp) {
                            const int4 av = pam[(k * 2 + lp) * nbg];  // lanes 2 lp and 2 lp + 1
#pragma unroll
                            for (int h = 0; h < 2; ++h) {
                                const int l = 2 * lp + h;
                                int Lb = dp4a(wl0[k * 4 + l], h ? av.z : av.x,
                                              dp4a(wl1[k * 4 + l], h ? av.w : av.y, 0x4B400000));
                                if (WDT == GTN_Q4) Lb -= 7 * ps[((size_t)(m * 4 + k) * 4 + l) * nbg + j];
                                o[l][k] = (__int_as_float(Lb) - 12582912.0f) * sc;
                            }
                        }
                    }
#pragma unroll
                    for (int l = 0; l < 4; ++l)
                        *reinterpret_cast<float4*>(prod + ((size_t)(mm * R + rs) * 4 + l) * pstr + 4 * j) =
                            make_float4(o[l][0], o[l][1], o[l][2], o[l][3]);
                }
            }
            __syncthreads();
            for (int cb = 0; cb < mc * nch; cb += GV3_THREADS) {  // whole warps: the combine shuffles
                const int c = cb + tid;
                const int mm = c / nch, rl = c - mm * nch, r = rl >> 2;
                const bool valid = c < mc * nch && r < nr;
                float acc = 0.0f;
                if (valid) {
                    const float4* pp = reinterpret_cast<const float4*>(prod + (size_t)c * pstr);
                    for (int b4 = 0; b4 < nbg; ++b4) {
                        const float4 v = pp[b4];
                        acc = acc + v.x;
                        acc = acc + v.y;
                        acc = acc + v.z;
                        acc = acc + v.w;
                    }
                }
                const float t01 = acc + __shfl_xor_sync(0xffffffffu, acc, 1);
                const float t = t01 + __shfl_xor_sync(0xffffffffu, t01, 2);
                if (valid && (c & 3) == 0) Y[(long)(m0 + c0 + mm) * y_stride + r0 + r] = t;
            }
            __syncthreads();  // the products are rewritten by the next chunk
        }
    }
    asm volatile("griddepcontrol.launch_dependents;");
    if (abort_flag && tid == 0 && nissued > 0) {
        // bounded wait for the last copy issued into the stage (phase nissued - 1)
        for (uint32_t i = 0; i < GTN_WAIT_LIMIT; ++i)
            if (mbar_try_wait(bar, (uint32_t)(nissued - 1) & 1u)) break;
    }
}

// Plain-load variant for rows whose TMA tiles could reach outside the caller's weight buffer (an
// unaligned base, or a last row that does not end on a 16-byte boundary). One warp per
// (row, activation row): lanes 0..3 (Q8/Q4) or 0..7 (fp16) run the reference's lane chains with
// the same arithmetic as k_mm_q / k_mm_f16. grid (rows, M); block 32.
template <int WDT>
__global__ void k_mm_rows_plain(const uint8_t* __restrict__ W, long w_stride, int row0, int K,
                                const uint8_t* __restrict__ X, long x_stride, float* __restrict__ Y, long y_stride) {
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const int row = row0 + blockIdx.x, m = blockIdx.y, l = threadIdx.x;
    const uint8_t* wr = W + (long)row * w_stride;
    const uint8_t* xr = X + (long)m * x_stride;
    float acc = 0.0f;
    if (WDT == GTN_F16) {
        const int K8 = (K / 8) * 8;
        if (l < 8) {
            for (int i = l; i < K8; i += 8) {
                const uint16_t wv = (uint16_t)(wr[2 * i] | (wr[2 * i + 1] << 8));
                const uint16_t xv = (uint16_t)(xr[2 * i] | (xr[2 * i + 1] << 8));
                const float pr = h2f(xv) * h2f(wv);
                acc = pr + acc;
            }
        }
        float v[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) v[j] = __shfl_sync(0xffffffffu, acc, j);
        if (l == 0) {
            float d = v[0] + v[1];
            for (int j = 2; j < 8; ++j) d = d + v[j];
            for (int k = K8; k < K; ++k) {
                const uint16_t wv = (uint16_t)(wr[2 * k] | (wr[2 * k + 1] << 8));
                const uint16_t xv = (uint16_t)(xr[2 * k] | (xr[2 * k + 1] << 8));
                const float pr = h2f(xv) * h2f(wv);
                d = d + pr;
            }
            Y[(long)m * y_stride + row] = d;
        }
        return;
    }
    constexpr int BB = WDT == GTN_Q8 ? GTN_Q8_BYTES : GTN_Q4_BYTES;
    if (l < 4) {
        for (int b = 0; b < K / GTN_QBLK; ++b) {
            const uint8_t* xb = xr + (long)b * GTN_Q8_BYTES;
            const uint8_t* wb = wr + (long)b * BB;
            const int8_t* xq = reinterpret_cast<const int8_t*>(xb + 2);
            int L = 0;
            for (int c = 0; c < GTN_QBLK; c += 8) {
                for (int e = c + 2 * l; e < c + 2 * l + 2; ++e) {
                    int wv;
                    if (WDT == GTN_Q8) {
                        wv = (int)(int8_t)wb[2 + e];
                    } else {
                        const uint8_t p = wb[2 + (e & 15)];
                        wv = (e < 16 ? (p >> 4) : (p & 15)) - 7;
                    }
                    L += (int)xq[e] * wv;
                }
            }
            const float da = h2f((uint16_t)(xb[0] | (xb[1] << 8)));
            const float dw = h2f((uint16_t)(wb[0] | (wb[1] << 8)));
            const float sc = da * dw;
            const float pr = lane_sum_f32(L) * sc;
            acc = acc + pr;
        }
    }
    const float t01 = acc + __shfl_xor_sync(0xffffffffu, acc, 1);
    const float t = t01 + __shfl_xor_sync(0xffffffffu, t01, 2);
    if (l == 0) Y[(long)m * y_stride + row] = t;
}

}  // namespace gtn
