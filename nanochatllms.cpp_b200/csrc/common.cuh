// Shared device helpers for the gten B200 kernels.
//
// Numerics contract: every kernel reproduces the reference CPU build's arithmetic bit for bit
// (iangitonga/nanochatllms.cpp, src/gten). The library is compiled with --fmad=false so that
// no multiply-add is contracted (the reference is built with -mavx and no FMA, so each
// multiply and add rounds separately); fmaf() is only written out where a fused operation is
// provably exact. Division and square root are IEEE round-to-nearest (nvcc's defaults).
#pragma once
#include <cuda_fp16.h>
#include <cstdint>

#include "../../include/gten_b200.h"

#define GTN_QBLK 32
#define GTN_Q8_BYTES 34  // quants.h:11-22: fp16 delta + 32 int8
#define GTN_Q4_BYTES 18  // quants.h:24-30: fp16 delta + 16 bytes (two nibbles each)

namespace gtn {

__host__ __device__ inline long row_bytes(int dt, int n) {
    switch (dt) {
        case GTN_Q8: return (long)((n + GTN_QBLK - 1) / GTN_QBLK) * GTN_Q8_BYTES;
        case GTN_Q4: return (long)(n / GTN_QBLK) * GTN_Q4_BYTES;
        case GTN_F16: return 2L * n;
        default: return 4L * n;
    }
}

// fp16 <-> fp32: hardware conversions; fp16 -> fp32 is exact and fp32 -> fp16 rounds to nearest
// even, as the reference's fp16_to_fp32 table and fp32_to_fp16 bit trick do (gten_types.h:69-109).
__device__ __forceinline__ float h2f(uint16_t h) { return __half2float(__ushort_as_half(h)); }
__device__ __forceinline__ uint16_t f2h(float f) { return __half_as_ushort(__float2half_rn(f)); }

__device__ __forceinline__ uint16_t ld_u16(const uint8_t* p) { return *reinterpret_cast<const uint16_t*>(p); }

// expf as the reference's math library evaluates it. The reference calls glibc's expf (silu,
// ops.cpp:733-772; softmax, ops.cpp:1064-1070), whose method is Szabolcs Nagy's table-driven
// exponential from Arm's optimized-routines (2017): with N = 32,
//   z = x * N / ln 2 (double),  k = round(z) (by adding 1.5 * 2^52),  r = z - k,
//   exp(x) = 2^(k/N) * (1 + c2 r + c1 r^2 + c0 r^3),  2^(k/N) = 2^floor(k/N) * tab[k mod N],
// evaluated in double and rounded once to float. tab[i] is the double nearest 2^(i/32), stored
// minus (i << 47) so that adding k << 47 to its bits also applies 2^floor(k/N); c0..c2 are the
// method's published minimax coefficients scaled by N^-3, N^-2, N^-1. glibc's x86-64 build for CPUs
// with FMA (the variant its loader selects on them) forms r = x * (N / ln 2) - k with one fused
// multiply-add, so r does so here. Against the host's expf this is bit-identical on all 2^32 float
// inputs (checked exhaustively); a correctly rounded exp differs from glibc's on 170,648 of them.
// The table sits in global memory and is read through the read-only cache: the threads of a warp
// index it with different k, which the constant cache would serve one address at a time.
__device__ static const unsigned long long k_expf_tab[32] = {
    0x3ff0000000000000ull, 0x3fefd9b0d3158574ull, 0x3fefb5586cf9890full, 0x3fef9301d0125b51ull,
    0x3fef72b83c7d517bull, 0x3fef54873168b9aaull, 0x3fef387a6e756238ull, 0x3fef1e9df51fdee1ull,
    0x3fef06fe0a31b715ull, 0x3feef1a7373aa9cbull, 0x3feedea64c123422ull, 0x3feece086061892dull,
    0x3feebfdad5362a27ull, 0x3feeb42b569d4f82ull, 0x3feeab07dd485429ull, 0x3feea47eb03a5585ull,
    0x3feea09e667f3bcdull, 0x3fee9f75e8ec5f74ull, 0x3feea11473eb0187ull, 0x3feea589994cce13ull,
    0x3feeace5422aa0dbull, 0x3feeb737b0cdc5e5ull, 0x3feec49182a3f090ull, 0x3feed503b23e255dull,
    0x3feee89f995ad3adull, 0x3feeff76f2fb5e47ull, 0x3fef199bdd85529cull, 0x3fef3720dcef9069ull,
    0x3fef5818dcfba487ull, 0x3fef7c97337b9b5full, 0x3fefa4afa2a490daull, 0x3fefd0765b6e4540ull,
};
__device__ __forceinline__ float expf_ref(float x) {
    const unsigned int ax = __float_as_uint(x) & 0x7fffffffu;
    if (ax >= 0x42b00000u) {                         // |x| >= 88, inf or nan
        if (__float_as_uint(x) == 0xff800000u) return 0.0f;  // exp(-inf)
        if (ax >= 0x7f800000u) return x + x;         // +inf, nan
        if (x > 0x1.62e42ep6f) return __int_as_float(0x7f800000);  // overflow
        if (x < -0x1.9fe368p6f) return 0.0f;         // underflow below 2^-150
    }
    const double inv_ln2n = 0x1.71547652b82fep+5, shift = 0x1.8p+52;
    const double xd = (double)x;
    const double z = __dmul_rn(inv_ln2n, xd);
    double kd = __dadd_rn(z, shift);
    const unsigned long long ki = (unsigned long long)__double_as_longlong(kd);
    kd = __dsub_rn(kd, shift);
    const double r = __fma_rn(inv_ln2n, xd, -kd);
    const double s = __longlong_as_double((long long)(__ldg(&k_expf_tab[ki & 31u]) + (ki << 47)));
    const double c0 = 0x1.c6af84b912394p-20, c1 = 0x1.ebfce50fac4f3p-13, c2 = 0x1.62e42ff0c52d6p-6;
    const double p = __dadd_rn(__dmul_rn(c0, r), c1);
    const double r2 = __dmul_rn(r, r);
    double y = __dadd_rn(__dmul_rn(c2, r), 1.0);
    y = __dadd_rn(__dmul_rn(p, r2), y);
    return __double2float_rn(__dmul_rn(y, s));
}

// fl(...fl(fl(0 + v[0]) + v[1])... + v[n-1]): the left-to-right fp32 sum of a shared-memory array
// v (16-byte aligned) by one thread, four elements per 128-bit load. The adds are one dependent
// chain either way; a single warp issues only about one instruction every two cycles, so a
// quarter of the loads shortens the loop (6.8 instead of 8.3 cycles per term for 2,048 squares;
// the softmax's sum of probabilities: TinyLlama's batch-1 decode step 0.2 % shorter).
__device__ __forceinline__ float serial_sum_smem(const float* v, int n) {
    const float4* v4 = reinterpret_cast<const float4*>(v);
    float s = 0.0f;
    int i = 0;
#pragma unroll 4
    for (; i + 4 <= n; i += 4) {
        const float4 q = v4[i >> 2];
        s = s + q.x;
        s = s + q.y;
        s = s + q.z;
        s = s + q.w;
    }
    for (; i < n; ++i) s = s + v[i];
    return s;
}

// Quantize one 32-element block held one element per lane (quants.cpp:16-30): absmax over the
// valid lanes, delta = absmax/127 (fp32, stored as fp16), scale = 1/delta of the UNROUNDED delta,
// q = roundf(x*scale) (half away from zero). Lanes >= n hold 0 and write nothing.
// Returns the quantized value; every lane receives the fp16 delta in *dh.
__device__ __forceinline__ int8_t warp_quant_block(float x, int lane, int n, uint16_t* dh) {
    // absmax as the reference's loop finds it (std::max from 0 skips NaN): non-negative floats
    // order like their bit patterns, so one warp max-reduction of the bits
    float a = lane < n ? fabsf(x) : 0.0f;
    a = a == a ? a : 0.0f;
    a = __uint_as_float(__reduce_max_sync(0xffffffffu, __float_as_uint(a)));
    const float delta = a / 127.0f;
    *dh = f2h(delta);
    const float scale = delta != 0.0f ? 1.0f / delta : 0.0f;
    return (int8_t)roundf(x * scale);
}

// Writes `n` (<= 32) floats, one per lane, as one Q8 block at `blk` (34 bytes).
__device__ __forceinline__ void warp_store_q8_block(float x, int lane, int n, uint8_t* blk) {
    uint16_t dh;
    const int8_t q = warp_quant_block(x, lane, n, &dh);
    if (lane == 0) *reinterpret_cast<uint16_t*>(blk) = dh;
    if (lane < n) blk[2 + lane] = (uint8_t)q;
}

// Reads element `i` of a row in dtype dt (Q8/Q4/F16/F32) as float (quants.cpp:33-138).
__device__ __forceinline__ float load_elem(const uint8_t* row, int dt, int i) {
    switch (dt) {
        case GTN_Q8: {
            const uint8_t* b = row + (i / GTN_QBLK) * GTN_Q8_BYTES;
            return (float)(int8_t)b[2 + (i % GTN_QBLK)] * h2f(ld_u16(b));
        }
        case GTN_Q4: {
            const uint8_t* b = row + (i / GTN_QBLK) * GTN_Q4_BYTES;
            const int j = i % GTN_QBLK;
            const uint8_t p = b[2 + (j & 15)];
            const int v = (j < 16 ? (p >> 4) : (p & 15)) - 7;
            return (float)v * h2f(ld_u16(b));
        }
        case GTN_F16: return h2f(reinterpret_cast<const uint16_t*>(row)[i]);
        default: return reinterpret_cast<const float*>(row)[i];
    }
}

// ---- TMA bulk copies with bounded mbarrier waits --------------------------------------------
// Every wait has an iteration limit; on expiry the kernel records GTN_DEVERR_TIMEOUT in the
// caller-visible error word and returns instead of spinning forever.
#define GTN_WAIT_LIMIT (1u << 26)
#define GTN_DEVERR_TIMEOUT 1u

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}
__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t phase) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(phase)
        : "memory");
    return ok != 0;
}
// Returns false (and flags *err) if the phase did not complete within the limit.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t phase, unsigned int* err) {
    for (uint32_t it = 0; it < GTN_WAIT_LIMIT; ++it)
        if (mbar_try_wait(bar, phase)) return true;
    if (err) atomicOr(err, GTN_DEVERR_TIMEOUT);
    return false;
}
// 1-D TMA bulk copy global -> shared, completion counted on `bar`. dst, src 16-byte aligned,
// bytes a multiple of 16. (No multicast: the source may be any GPU's memory.)
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ int dp4a(int a, int b, int c) { return __dp4a(a, b, c); }

// float(L) for |L| < 2^22 (every block lane sum: at most 8 * 128 * 128 in magnitude), bit-identical
// to the conversion instruction but on the full-rate integer and fp32 pipes: L + 0x4B400000 read as a
// float is 1.5 * 2^23 + L exactly (the binade [2^23, 2^24) has unit spacing), and subtracting
// 1.5 * 2^23 is exact. The conversion instruction issues at a fraction of the fp32 rate, and the
// block epilogues convert one lane sum per 8 multiply-adds.
__device__ __forceinline__ float lane_sum_f32(int L) { return __int_as_float(L + 0x4B400000) - 12582912.0f; }

}  // namespace gtn
