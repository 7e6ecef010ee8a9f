// Exact Q8/Q4 GEMM on the 5th-generation tensor cores (tcgen05) for M >= 16 activation rows:
// prefill and batched decode steps.
//
// Reference: ops.cpp:292-490 (vec_dot_product_q8, vec_dot_product_q8_q4) inside matmul_2d_impl
// (ops.cpp:579-636). The reference keeps 4 fp32 lanes per dot product; lane l owns the elements
// k of every 32-element block with (k % 8) / 2 == l, its int32 sum L over those 8 products is
// converted to fp32, multiplied by fp32(da) * fp32(dw) and added to the lane, blocks in order;
// the result is (L0 + L1) + (L2 + L3).
//
// Split of the work:
//   * tensor cores: the exact integer lane sums. Q8 values (-128..127) and Q4 values (nibble - 7)
//     are exact in fp16, every product is an integer below 2^15 and a lane sum of 8 of them stays
//     below 2^18, so kind::f16 with fp32 accumulation returns L exactly. To get one lane per
//     accumulator row, the activation tile is expanded 4x: row r = l * 32 + m of A' holds row m
//     of the activations masked to lane l's elements (zeros elsewhere). One block (K = 32) is two
//     MMAs (K = 16 each) into its own TMEM region of 128 lanes x NT columns; D[l*32+m][n] = L.
//   * CUDA cores: the reference's fp32 epilogue. Thread (warp w, lane m) reads TMEM lane quarter
//     l = w % 4 (its own accumulator rows) and owns the chains (m, l, n) of NT/2 weight rows n; per
//     block it computes s = da * dw, p = L * s and acc = acc + p, blocks in order, so every
//     chain is the reference's. The four lane chains of an output meet in shared memory at the
//     end for (L0 + L1) + (L2 + L3).
//
// Data movement:
//   * activations: a pre-pass (k_tc_expand) writes, per 32-row tile and block, the expanded A'
//     tile in the MMA's canonical K-major fp16 layout (8-row x 16-byte core matrices, no swizzle)
//     followed by the 32 activation scales: 8320 bytes that the GEMM fetches with one bulk copy
//     (the image is small and stays in L2; every CTA of a row tile reads the same image);
//   * weights: raw rows (34/18-byte blocks, 16-byte aligned row stride) through a 2-D TMA tensor
//     map, one copy per NT rows x 8 blocks into a 3-stage ring; each converter thread turns one
//     (row, block) into the four 16-byte K-chunk rows of the canonical fp16 tile (aligned word
//     loads, byte permutes and one exact fp16 subtraction per pair).
// 512 / (4 NT) groups of 4 blocks are in flight (tile, TMEM and scale slots; all of TMEM).
// Roles: a producer warp (copies), converter warps (weight tiles), an MMA warp, epilogue warps.
// Every wait is bounded (about 2 s of device time); on expiry the kernel flags the device error
// word, waits (bounded) for its own copies and MMAs, frees its TMEM and returns.
#pragma once
#include <cuda.h>

#include "common.cuh"

namespace gtn {

constexpr int TC_EPI_WARPS = 8;                  // epilogue warps: warp w reads TMEM lane quarter w % 4
constexpr int TC_MT = 32;                        // activation rows per CTA (x 4 lanes = 128 MMA rows)
constexpr int TC_G = 4;                          // blocks per group (one commit)
constexpr int TC_KB = 8;                         // blocks per raw weight chunk (one TMA copy)
constexpr int TC_RS = 3;                         // raw chunk stages
constexpr int TC_TMEM_COLS = 512;                // the whole TMEM (one CTA per SM)
constexpr int TC_ATILE = 128 * 64;               // expanded activation tile of one block: 128 rows x 32 fp16
constexpr int TC_AIMG = TC_ATILE + TC_MT * 4;    // + the 32 activation scales (fp32): one bulk copy
constexpr int TC_COMB_STRIDE = 65;               // floats per (lane, row) in the final combine (bank spread)

// Tile of one CTA: NT weight rows (the MMA's N) — 64, or 32 when a grid of 64-row tiles would leave
// SMs idle. The slots in flight fill TMEM; converter threads cover one (block, weight row) each.
template <int NT>
struct TcTile {
    static constexpr int S = TC_TMEM_COLS / (TC_G * NT);  // groups in flight (tile / TMEM / scale slots)
    static constexpr int CONV_WARPS = TC_G * NT / 32;
    static constexpr int CONV_THREADS = 32 * CONV_WARPS;
    static constexpr int PROD_WARP = TC_EPI_WARPS + CONV_WARPS;  // producer warp (copies)
    static constexpr int MMA_WARP = PROD_WARP + 1;               // MMA issue warp
    static constexpr int THREADS = 32 * (MMA_WARP + 1);
    static constexpr int BTILE = NT * 64;  // weight tile of one block: NT rows x 32 fp16
    static constexpr int COLS = NT / 2;    // epilogue columns per thread (two threads per row and lane)
    // instruction descriptor: kind::f16, A = B = fp16, D = fp32, both K-major, M = 128, N = NT
    static constexpr uint32_t IDESC = (1u << 4) | ((uint32_t)(NT >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
    static_assert(NT == 32 || NT == 64, "32- or 64-row tiles");
};

// Bytes of the expanded activation image of M rows and K columns (k_tc_expand's output).
__host__ __device__ inline size_t tc_aimg_bytes(int M, int K) {
    return (size_t)((M + TC_MT - 1) / TC_MT) * (size_t)(K / GTN_QBLK) * TC_AIMG;
}
template <int WDT>
__host__ __device__ constexpr int tc_rstride() {  // raw chunk row: 8 blocks (272 / 144 bytes)
    return TC_KB * (WDT == GTN_Q8 ? GTN_Q8_BYTES : GTN_Q4_BYTES);
}
template <int WDT, int NT>
__host__ __device__ constexpr size_t tc_smem() {
    return 1024 + (size_t)TcTile<NT>::S * TC_G * (TC_AIMG + TcTile<NT>::BTILE) +
           (size_t)TC_RS * NT * tc_rstride<WDT>() + (size_t)TcTile<NT>::S * TC_G * NT * sizeof(float) + 64;
}
static_assert(tc_rstride<GTN_Q8>() % 16 == 0 && tc_rstride<GTN_Q4>() % 16 == 0, "TMA boxes are 16-byte rows");
static_assert((size_t)4 * TC_MT * TC_COMB_STRIDE * sizeof(float) <= (size_t)2 * TC_G * TC_AIMG,
              "the combine buffer reuses the activation tiles");
static_assert(tc_smem<GTN_Q8, 32>() <= 227 * 1024 && tc_smem<GTN_Q8, 64>() <= 227 * 1024, "shared memory");
static_assert(TC_KB % TC_G == 0, "groups never straddle raw chunks");

// Shared-memory matrix descriptor (tcgen05): K-major, no swizzle; LBO = bytes between the two
// 16-byte K chunks of a core-matrix row group, SBO = bytes between 8-row groups; version 1.
__device__ __forceinline__ uint64_t tc_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
    return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)((lbo >> 4) & 0x3FFFu) << 16) |
           ((uint64_t)((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46);
}
__device__ __forceinline__ void tc_mma(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(d),
        "l"(a), "l"(b), "r"(idesc), "r"(accumulate)
        : "memory");
}
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
// Bounded mbarrier wait: at most about TC_WAIT_NS of device time (%globaltimer), then the device
// error word is flagged and false returned.
constexpr uint64_t TC_WAIT_NS = 2000000000ull;
__device__ __forceinline__ uint64_t globaltimer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
__device__ __forceinline__ bool tc_wait(uint64_t* bar, uint32_t phase, unsigned int* err) {
    if (mbar_try_wait(bar, phase)) return true;
    const uint64_t t0 = globaltimer_ns();
    for (uint32_t it = 0; it < GTN_WAIT_LIMIT; ++it) {
        if (mbar_try_wait(bar, phase)) return true;
        if ((it & 255u) == 255u && globaltimer_ns() - t0 > TC_WAIT_NS) break;
    }
    if (err) atomicOr(err, GTN_DEVERR_TIMEOUT);
    return false;
}

// 16 consecutive TMEM columns of this warp's lane quarter (one lane per thread), not waited for:
// the registers are valid after tc_wait_ld, which names them as in-out operands so that no use
// is scheduled before the wait.
#define TC_R16(a) "=r"(a[0]), "=r"(a[1]), "=r"(a[2]), "=r"(a[3]), "=r"(a[4]), "=r"(a[5]), "=r"(a[6]), "=r"(a[7]), \
    "=r"(a[8]), "=r"(a[9]), "=r"(a[10]), "=r"(a[11]), "=r"(a[12]), "=r"(a[13]), "=r"(a[14]), "=r"(a[15])
#define TC_RW16(a) "+r"(a[0]), "+r"(a[1]), "+r"(a[2]), "+r"(a[3]), "+r"(a[4]), "+r"(a[5]), "+r"(a[6]), "+r"(a[7]), \
    "+r"(a[8]), "+r"(a[9]), "+r"(a[10]), "+r"(a[11]), "+r"(a[12]), "+r"(a[13]), "+r"(a[14]), "+r"(a[15])
__device__ __forceinline__ void tc_ld16(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15}, [%16];\n"
        : TC_R16(r)
        : "r"(taddr)
        : "memory");
}
__device__ __forceinline__ void tc_wait_ld(uint32_t (&r)[16]) {
    asm volatile("tcgen05.wait::ld.sync.aligned;\n" : TC_RW16(r) : : "memory");
}

// Four int8 (as bytes b0..b3 of x, each biased by `bias` so that it is 0..255) -> two fp16 pairs
// of (byte - sub): 1024 + byte has the fp16 bits 0x6400 | byte, and subtracting 1024 + bias in fp16
// is exact (both operands lie in [1024, 1280)).
__device__ __forceinline__ uint2 tc_bytes_to_f16x4(uint32_t x, uint32_t sub2) {
    const uint32_t lo = __byte_perm(x, 0x64646464u, 0x4140), hi = __byte_perm(x, 0x64646464u, 0x4342);
    const __half2 s = *reinterpret_cast<const __half2*>(&sub2);
    const __half2 a = __hsub2(*reinterpret_cast<const __half2*>(&lo), s);
    const __half2 b = __hsub2(*reinterpret_cast<const __half2*>(&hi), s);
    return make_uint2(*reinterpret_cast<const uint32_t*>(&a), *reinterpret_cast<const uint32_t*>(&b));
}

__device__ __forceinline__ bool mbar_test(uint64_t* bar, uint32_t phase) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(phase)
        : "memory");
    return ok != 0;
}
// 2-D TMA tile load (no multicast) of box (x, y) of `map` into shared memory, counted on `bar`.
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}

// Expanded activation image for k_gemm_tc: for each 32-row tile t and block b, at
// img + (t * nb + b) * TC_AIMG, the A' tile (row r = l * 32 + m holds the lane-l elements of
// activation row m as fp16, zeros elsewhere; canonical K-major layout) and the 32 row scales as
// fp32 (0 for rows past M). X: Q8 rows, stride x_stride. grid (nb, ceil(M / 32)), block 128.
static __global__ void __launch_bounds__(128) k_tc_expand(const uint8_t* __restrict__ X, long x_stride, int M, int K,
                                                         uint8_t* __restrict__ img) {
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const int b = blockIdx.x, t = blockIdx.y, nb = K / GTN_QBLK;
    const int m0 = t * TC_MT, mr = min(TC_MT, M - m0);
    uint8_t* tile = img + ((size_t)t * nb + b) * TC_AIMG;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int u = threadIdx.x + 128 * i;  // 16-byte core row: chunk c, A' row r
        const int c = u & 3, r = u >> 2, l = r >> 5, m = r & 31;
        uint32_t w = 0u;
        if (m < mr) {
            const uint32_t v = ld_u16(X + (long)(m0 + m) * x_stride + (long)b * GTN_Q8_BYTES + 2 + 8 * c + 2 * l);
            w = tc_bytes_to_f16x4(v ^ 0x8080u, 0x64806480u).x;  // (q + 128) - 1152
        }
        uint4 o = make_uint4(0u, 0u, 0u, 0u);
        if (l == 0) o.x = w;
        if (l == 1) o.y = w;
        if (l == 2) o.z = w;
        if (l == 3) o.w = w;
        *reinterpret_cast<uint4*>(tile + (r >> 3) * 512 + c * 128 + (r & 7) * 16) = o;
    }
    if (threadIdx.x < TC_MT) {
        const int m = threadIdx.x;
        reinterpret_cast<float*>(tile + TC_ATILE)[m] =
            m < mr ? h2f(ld_u16(X + (long)(m0 + m) * x_stride + (long)b * GTN_Q8_BYTES)) : 0.0f;
    }
    asm volatile("griddepcontrol.launch_dependents;");
}

// Y[m, n] (fp32, row stride y_stride) = dot(X[m, :], W[n, :]) for Q8 activations and Q8/Q4
// weights, bit-identical to the reference. `img`: k_tc_expand's image of X (M rows). `wmap`: the
// weight matrix as a 2-D uint16 tensor (inner extent w_stride / 2, N rows, row stride w_stride),
// box (tc_rstride / 2, NT); rows past N read as zeros. K / 32 a multiple of TC_G.
// grid (ceil(N / NT), ceil(M / 32)), block TcTile<NT>::THREADS, dynamic shared memory tc_smem<WDT, NT>();
// one CTA per SM (it holds all of TMEM).
//
// Roles, synchronised only by mbarriers (no block-wide barrier inside the main loop):
//   producer warp: weight chunks (raw_full / raw_empty ring) and the A' images of group g into
//     slot s = g % T::S once the epilogue released the slot (tmem_empty of group g - T::S);
//   converter warps: wait for the slot and the raw chunk, write the weight tile and scales, arrive
//     on b_full[s] (and on raw_empty once a chunk's last group is converted);
//   MMA warp: waits for b_full[s] and a_full[s], issues the group's MMAs into TMEM slot s and
//     commits them to mma_done[s];
//   epilogue warps: wait mma_done[s], read the lane sums from TMEM, run the fp32 chains, release
//     slot s (tmem_empty[s], 256 arrivals).
template <int WDT, int NT>
__global__ void __launch_bounds__(TcTile<NT>::THREADS, 1) k_gemm_tc(const __grid_constant__ CUtensorMap wmap, int N, int K,
                                                           const uint8_t* __restrict__ img, int M,
                                                           float* __restrict__ Y, long y_stride, unsigned int* err) {
    using T = TcTile<NT>;
    constexpr int BB = WDT == GTN_Q8 ? GTN_Q8_BYTES : GTN_Q4_BYTES;
    constexpr int RSTR = tc_rstride<WDT>();
    constexpr uint32_t CHUNK_BYTES = (uint32_t)RSTR * NT;
    extern __shared__ __align__(128) uint8_t smem[];  // every TMA destination and MMA tile sits at a 128-byte multiple
    uint64_t* raw_full = reinterpret_cast<uint64_t*>(smem);  // [TC_RS]
    uint64_t* raw_empty = raw_full + TC_RS;                   // [TC_RS]
    uint64_t* a_full = raw_empty + TC_RS;                     // [T::S]
    uint64_t* b_full = a_full + T::S;                         // [T::S]
    uint64_t* mma_done = b_full + T::S;                       // [T::S]
    uint64_t* tmem_empty = mma_done + T::S;                   // [T::S]
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tmem_empty + T::S);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
    uint8_t* atile = smem + 1024;                             // [T::S * TC_G][TC_AIMG]
    uint8_t* btile = atile + T::S * TC_G * TC_AIMG;           // [T::S * TC_G][T::BTILE]
    uint8_t* raw = btile + T::S * TC_G * T::BTILE;            // [TC_RS][NT][RSTR]
    float* dw_s = reinterpret_cast<float*>(raw + (size_t)TC_RS * NT * RSTR);  // [T::S][TC_G][NT]
    float* comb = reinterpret_cast<float*>(atile);  // [4][TC_MT][TC_COMB_STRIDE], after the last MMA

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int n0 = blockIdx.x * NT, nr = min(NT, N - n0);
    const int m0 = blockIdx.y * TC_MT, mr = min(TC_MT, M - m0);
    const int nb = K / GTN_QBLK, ngroups = nb / TC_G, nchunks = (nb + TC_KB - 1) / TC_KB;
    constexpr int CW0 = TC_EPI_WARPS;  // first converter warp

    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(TC_TMEM_COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    if (tid == 32) {
        for (int s = 0; s < TC_RS; ++s) {
            mbar_init(&raw_full[s], 1);
            mbar_init(&raw_empty[s], T::CONV_THREADS);
        }
        for (int s = 0; s < T::S; ++s) {
            mbar_init(&a_full[s], 1);
            mbar_init(&b_full[s], T::CONV_THREADS);
            mbar_init(&mma_done[s], 1);
            mbar_init(&tmem_empty[s], 32 * TC_EPI_WARPS);
        }
        *abort_flag = 0;
        fence_mbar_init();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    float acc[T::COLS];
#pragma unroll
    for (int j = 0; j < T::COLS; ++j) acc[j] = 0.0f;
    int g_issued = 0;                // MMA warp: groups whose MMAs were issued
    int a_issued = 0, w_issued = 0;  // producer: groups of A' images and weight chunks issued

    if (warp == T::PROD_WARP) {
        // ---- producer (one thread) ----
        if (lane == 0) {
            for (int c = 0; c < min(TC_RS, nchunks); ++c) {  // weights: independent of the previous kernel
                mbar_arrive_expect_tx(&raw_full[c], CHUNK_BYTES);
                tma_load_2d(raw + (size_t)c * NT * RSTR, &wmap, c * (RSTR / 2), n0, &raw_full[c]);
            }
            w_issued = min(TC_RS, nchunks);
            asm volatile("griddepcontrol.wait;" ::: "memory");  // the A' image comes from the pre-pass
            const uint8_t* aimg = img + (size_t)blockIdx.y * nb * TC_AIMG;
            uint64_t t0 = globaltimer_ns();
            while (a_issued < ngroups || w_issued < nchunks) {
                bool progressed = false;
                if (a_issued < ngroups) {
                    const int g = a_issued, s = g % T::S;
                    if (g < T::S || mbar_test(&tmem_empty[s], (uint32_t)(g / T::S - 1) & 1u)) {
                        mbar_arrive_expect_tx(&a_full[s], (uint32_t)(TC_G * TC_AIMG));
                        for (int blk = 0; blk < TC_G; ++blk)
                            bulk_g2s(atile + (size_t)(s * TC_G + blk) * TC_AIMG,
                                     aimg + (size_t)(g * TC_G + blk) * TC_AIMG, (uint32_t)TC_AIMG, &a_full[s]);
                        ++a_issued;
                        progressed = true;
                    }
                }
                if (w_issued < nchunks) {
                    const int c = w_issued, st = c % TC_RS;
                    if (mbar_test(&raw_empty[st], (uint32_t)(c / TC_RS - 1) & 1u)) {
                        mbar_arrive_expect_tx(&raw_full[st], CHUNK_BYTES);
                        tma_load_2d(raw + (size_t)st * NT * RSTR, &wmap, c * (RSTR / 2), n0, &raw_full[st]);
                        ++w_issued;
                        progressed = true;
                    }
                }
                if (progressed) {
                    t0 = globaltimer_ns();
                } else if (*abort_flag != 0 || globaltimer_ns() - t0 > TC_WAIT_NS) {
                    *abort_flag = 1;
                    if (err) atomicOr(err, GTN_DEVERR_TIMEOUT);
                    break;
                } else {
                    __nanosleep(64);
                }
            }
        }
        __syncwarp();
    } else if (warp >= CW0 && warp < CW0 + T::CONV_WARPS) {
        // ---- converters: thread -> (block blk of the group, weight row n); the whole 32-element
        // block is read as aligned words (the block data starts 2 bytes past a word boundary in even
        // blocks) and written as the four 16-byte K-chunk rows of the fp16 tile ----
        const int ct = tid - 32 * CW0;
        const int blk = ct / NT, n = ct % NT;
        for (int g = 0; g < ngroups; ++g) {
            const int s = g % T::S, chunk = (g * TC_G) / TC_KB, stage = chunk % TC_RS;
            bool ok = *abort_flag == 0;
            if (ok && g >= T::S) ok = tc_wait(&tmem_empty[s], (uint32_t)(g / T::S - 1) & 1u, err);
            if (ok) ok = tc_wait(&raw_full[stage], (uint32_t)(chunk / TC_RS) & 1u, err);
            if (ok) {
                const int boff = ((g * TC_G + blk) % TC_KB) * BB;  // block offset in the raw row
                const uint8_t* row = raw + (size_t)stage * NT * RSTR + (size_t)n * RSTR;
                const int sh = ((boff + 2) & 3) * 8;                // 16 (even blocks) or 0 bits
                const uint32_t* wp = reinterpret_cast<const uint32_t*>(row + ((boff + 2) & ~3));
                uint8_t* dst = btile + (size_t)(s * TC_G + blk) * T::BTILE + (n >> 3) * 512 + (n & 7) * 16;
                if (WDT == GTN_Q8) {
                    uint32_t w[9], d[8];
#pragma unroll
                    for (int i = 0; i < 9; ++i) w[i] = wp[i];
#pragma unroll
                    for (int i = 0; i < 8; ++i) d[i] = __funnelshift_r(w[i], w[i + 1], sh) ^ 0x80808080u;
#pragma unroll
                    for (int c = 0; c < 4; ++c) {  // K chunk c: elements 8c .. 8c+7
                        const uint2 lo = tc_bytes_to_f16x4(d[2 * c], 0x64806480u);  // (q + 128) - 1152
                        const uint2 hi = tc_bytes_to_f16x4(d[2 * c + 1], 0x64806480u);
                        *reinterpret_cast<uint4*>(dst + c * 128) = make_uint4(lo.x, lo.y, hi.x, hi.y);
                    }
                } else {
                    uint32_t w[5], d[4];
#pragma unroll
                    for (int i = 0; i < 5; ++i) w[i] = wp[i];
#pragma unroll
                    for (int i = 0; i < 4; ++i) d[i] = __funnelshift_r(w[i], w[i + 1], sh);
#pragma unroll
                    for (int c = 0; c < 4; ++c) {  // elements 8c..8c+7: high nibbles (c < 2) or low nibbles
                        const uint32_t b0 = d[2 * (c & 1)], b1 = d[2 * (c & 1) + 1];
                        const uint32_t q0 = c < 2 ? (b0 >> 4) & 0x0F0F0F0Fu : b0 & 0x0F0F0F0Fu;
                        const uint32_t q1 = c < 2 ? (b1 >> 4) & 0x0F0F0F0Fu : b1 & 0x0F0F0F0Fu;
                        const uint2 lo = tc_bytes_to_f16x4(q0, 0x64076407u);  // nibble - 7
                        const uint2 hi = tc_bytes_to_f16x4(q1, 0x64076407u);
                        *reinterpret_cast<uint4*>(dst + c * 128) = make_uint4(lo.x, lo.y, hi.x, hi.y);
                    }
                }
                dw_s[s * TC_G * NT + ct] = h2f(ld_u16(row + boff));  // rows past N are zeros (scale 0)
                fence_async_smem();  // generic-proxy tile writes -> visible to the tensor cores
            }
            if (!ok) {
                *abort_flag = 1;
                break;
            }
            mbar_arrive(&b_full[s]);
            if ((g + 1) * TC_G % TC_KB == 0 || g + 1 == ngroups) mbar_arrive(&raw_empty[stage]);  // chunk done
        }
    } else if (warp == T::MMA_WARP) {
        // ---- MMA issue (one thread) ----
        if (lane == 0) {
            for (int g = 0; g < ngroups; ++g) {
                const int s = g % T::S;
                const uint32_t ph = (uint32_t)(g / T::S) & 1u;
                if (*abort_flag != 0 || !tc_wait(&b_full[s], ph, err) || !tc_wait(&a_full[s], ph, err)) {
                    *abort_flag = 1;
                    break;
                }
                tc_fence_after();
#pragma unroll
                for (int b2 = 0; b2 < TC_G; ++b2) {
                    const int t = s * TC_G + b2;
                    const uint32_t a = smem_u32(atile + (size_t)t * TC_AIMG);
                    const uint32_t b = smem_u32(btile + (size_t)t * T::BTILE);
                    const uint32_t d = tmem + (uint32_t)(t * NT);
                    tc_mma(d, tc_desc(a, 128, 512), tc_desc(b, 128, 512), T::IDESC, 0u);
                    tc_mma(d, tc_desc(a + 256, 128, 512), tc_desc(b + 256, 128, 512), T::IDESC, 1u);
                }
                tc_commit(&mma_done[s]);
                g_issued = g + 1;
            }
        }
        __syncwarp();
    } else {
        // ---- epilogue: thread (quarter q = reference lane l, column half, row m = lane) ----
        const int q = warp & 3, half = warp >> 2;
        for (int g = 0; g < ngroups; ++g) {
            const int s = g % T::S;
            if (*abort_flag != 0 || !tc_wait(&mma_done[s], (uint32_t)(g / T::S) & 1u, err)) {
                *abort_flag = 1;
                break;
            }
            tc_fence_after();
            // 16-column chunks i = CPB * block + sub: the TMEM load of chunk i + 1 is in flight while
            // chunk i is accumulated
            constexpr int CPB = T::COLS / 16, NCH = TC_G * CPB;
            const uint32_t tq = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(s * TC_G * NT + half * T::COLS);
            uint32_t va[16], vb[16];
            tc_ld16(tq, va);
            tc_wait_ld(va);
#pragma unroll
            for (int i = 0; i < NCH; ++i) {
                uint32_t(&cur)[16] = (i & 1) ? vb : va;
                uint32_t(&nxt)[16] = (i & 1) ? va : vb;
                if (i + 1 < NCH) tc_ld16(tq + (uint32_t)(((i + 1) / CPB) * NT + ((i + 1) % CPB) * 16), nxt);
                const int t = s * TC_G + i / CPB, sub = i % CPB;
                const float da = reinterpret_cast<const float*>(atile + (size_t)t * TC_AIMG + TC_ATILE)[lane];
                const float4* dw4 = reinterpret_cast<const float4*>(dw_s + t * NT + half * T::COLS + sub * 16);
#pragma unroll
                for (int j4 = 0; j4 < 4; ++j4) {
                    const float4 w = dw4[j4];
                    const int j = sub * 16 + 4 * j4;
                    const float s0 = da * w.x, s1 = da * w.y, s2 = da * w.z, s3 = da * w.w;
                    const float p0 = __uint_as_float(cur[4 * j4]) * s0, p1 = __uint_as_float(cur[4 * j4 + 1]) * s1;
                    const float p2 = __uint_as_float(cur[4 * j4 + 2]) * s2, p3 = __uint_as_float(cur[4 * j4 + 3]) * s3;
                    acc[j] = acc[j] + p0;
                    acc[j + 1] = acc[j + 1] + p1;
                    acc[j + 2] = acc[j + 2] + p2;
                    acc[j + 3] = acc[j + 3] + p3;
                }
                if (i + 1 < NCH) tc_wait_ld(nxt);
            }
            tc_fence_before();
            mbar_arrive(&tmem_empty[s]);
        }
    }
    __syncthreads();
    const bool ok = *abort_flag == 0;
    if (ok) {
        // (L0 + L1) + (L2 + L3): the four lane chains of each output meet in shared memory
        if (warp < TC_EPI_WARPS) {
            const int q = warp & 3, half = warp >> 2;
#pragma unroll
            for (int j = 0; j < T::COLS; ++j) comb[(q * TC_MT + lane) * TC_COMB_STRIDE + half * T::COLS + j] = acc[j];
        }
        __syncthreads();
        for (int i = tid; i < TC_MT * NT; i += T::THREADS) {
            const int m = i / NT, n = i % NT;
            if (m < mr && n < nr) {
                const float c0 = comb[(0 * TC_MT + m) * TC_COMB_STRIDE + n], c1 = comb[(1 * TC_MT + m) * TC_COMB_STRIDE + n];
                const float c2 = comb[(2 * TC_MT + m) * TC_COMB_STRIDE + n], c3 = comb[(3 * TC_MT + m) * TC_COMB_STRIDE + n];
                Y[(long)(m0 + m) * y_stride + n0 + n] = (c0 + c1) + (c2 + c3);
            }
        }
    } else {
        // an expired wait: let this CTA's MMAs and copies finish (bounded) before its TMEM and
        // shared memory are released; each slot / stage has at most one outstanding phase
        if (tid == 32 * T::MMA_WARP)
            for (int g2 = max(0, g_issued - T::S); g2 < g_issued; ++g2)
                tc_wait(&mma_done[g2 % T::S], (uint32_t)(g2 / T::S) & 1u, err);
        if (tid == 32 * T::PROD_WARP) {
            for (int g2 = max(0, a_issued - T::S); g2 < a_issued; ++g2)
                tc_wait(&a_full[g2 % T::S], (uint32_t)(g2 / T::S) & 1u, err);
            for (int c = max(0, w_issued - TC_RS); c < w_issued; ++c)
                tc_wait(&raw_full[c % TC_RS], (uint32_t)(c / TC_RS) & 1u, err);
        }
        __syncwarp();
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TC_TMEM_COLS) : "memory");
    }
    asm volatile("griddepcontrol.launch_dependents;");
}

}  // namespace gtn
