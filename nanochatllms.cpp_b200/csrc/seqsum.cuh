// Exact emulation of a sequential fp32 sum of non-negative terms, computed in parallel.
//
// The reference's RMSNorm accumulates sq = sq + x[i]*x[i] for i = 0..n-1 in fp32, one rounding
// per add (ops.cpp:830-836). Done by one thread that is a chain of n dependent adds. For
// non-negative terms the running sum S never decreases, so it moves through binades
// [2^e, 2^(e+1)) in order, and while S stays inside one binade every add rounds to a multiple of
// the same ulp u = 2^(e-23):
//     fl(S + p) = S + u * inc(p),  inc(p) = floor(p/u) + (frac(p/u) > 1/2)
// unless frac(p/u) == 1/2 exactly (a tie, decided by the parity of S/u). So a run of adds inside
// one binade is an exact integer sum of per-term increments, which can be summed in any order.
//
// Algorithm (one CTA): (1) terms p_i = fl(v_i * v_i); (2) a double-precision prefix scan predicts
// the binade e_i of the running sum after term i; (3) the first term of each predicted binade
// (its "head") is kept as a float, every other term adds inc(p_i) w.r.t. its binade's ulp to an
// integer total per binade; (4) one thread walks the binades in order: S = fl(S + p_head) (an
// exact IEEE add), checks that S really is in binade e, adds the binade's integer total and
// checks the result is still below 2^(e+1). A failed check (a mispredicted crossing), a tie, or
// a subnormal sum makes the CTA fall back to the plain sequential loop, so the result is always
// bit-identical to the serial sum.
#pragma once
#include <cstdint>

namespace gtn {

constexpr int SEQSUM_THREADS_MAX = 1024;
constexpr int SEQSUM_EXP_OFF = 150;     // slot = exponent + 150
constexpr int SEQSUM_EXP_SLOTS = 320;

struct SeqSumSmem {
    double scan[SEQSUM_THREADS_MAX / 32];
    int total[SEQSUM_EXP_SLOTS];
    int head[SEQSUM_EXP_SLOTS];
    int lo, hi;  // range of slots that received a head
    int bad;
    float result;
};

// Binade exponent of a positive double (floor(log2(q))).
__device__ __forceinline__ int binade_of(double q) {
    int e;
    frexp(q, &e);
    return e - 1;
}

__device__ __forceinline__ void seqsum_flush(SeqSumSmem& s, int e, int tot) {
    if (tot == 0) return;
    const int slot = e + SEQSUM_EXP_OFF;
    if (slot < 0 || slot >= SEQSUM_EXP_SLOTS) {
        s.bad = 1;
        return;
    }
    atomicAdd(&s.total[slot], tot);
}

// Returns fl(...fl(fl(0 + p_0) + p_1)... + p_{n-1}) with p_i = fl(v[i] * v[i]), for v in shared
// (or global) memory. All threads of the CTA must call it; it synchronizes the CTA.
__device__ __forceinline__ float seq_sum_squares(const float* v, int n, SeqSumSmem& s) {
    const int tid = threadIdx.x, nt = blockDim.x, lane = tid & 31, warp = tid >> 5;
    const int per = (n + nt - 1) / nt;
    const int i0 = min(n, tid * per), i1 = min(n, i0 + per);
    for (int i = tid; i < SEQSUM_EXP_SLOTS; i += nt) {
        s.total[i] = 0;
        s.head[i] = -1;
    }
    if (tid == 0) {
        s.bad = 0;
        s.lo = SEQSUM_EXP_SLOTS;
        s.hi = -1;
    }
    // (2) exclusive prefix of the per-thread chunk sums, in double
    double local = 0.0;
    for (int i = i0; i < i1; ++i) {
        const float p = v[i] * v[i];
        local += (double)p;
    }
    double incl = local;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const double t = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += t;
    }
    if (lane == 31) s.scan[warp] = incl;
    __syncthreads();
    if (warp == 0) {
        const int nw = nt >> 5;
        double w = lane < nw ? s.scan[lane] : 0.0;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const double t = __shfl_up_sync(0xffffffffu, w, o);
            if (lane >= o) w += t;
        }
        if (lane < nw) s.scan[lane] = w;
    }
    __syncthreads();
    double q = (warp > 0 ? s.scan[warp - 1] : 0.0) + (incl - local);  // terms before i0
    // (3) heads and per-binade integer totals (run-length accumulated per thread)
    int e_prev = q > 0.0 ? binade_of(q) : -1000;
    int cur_e = -1000, cur_tot = 0;
    for (int i = i0; i < i1; ++i) {
        const float p = v[i] * v[i];
        q += (double)p;
        if (q <= 0.0) continue;  // leading zero terms: the sum stays exactly 0
        const int e = binade_of(q);
        if (e != e_prev) {
            seqsum_flush(s, cur_e, cur_tot);
            cur_tot = 0;
            cur_e = e;
            const int slot = e + SEQSUM_EXP_OFF;
            if (slot < 0 || slot >= SEQSUM_EXP_SLOTS || atomicCAS(&s.head[slot], -1, i) != -1) {
                s.bad = 1;
            } else {
                atomicMin(&s.lo, slot);
                atomicMax(&s.hi, slot);
            }
        } else {
            if (e != cur_e) {
                seqsum_flush(s, cur_e, cur_tot);
                cur_tot = 0;
                cur_e = e;
            }
            const float x = p * ldexpf(1.0f, 23 - e);  // p/u, exact (power-of-two scaling)
            const float fl = floorf(x);
            const float fr = x - fl;
            if (fr == 0.5f || x >= 16777216.0f || e < -126) s.bad = 1;
            cur_tot += (int)fl + (fr > 0.5f ? 1 : 0);
        }
        e_prev = e;
    }
    seqsum_flush(s, cur_e, cur_tot);
    __syncthreads();
    // a total outside [lo, hi] belongs to a binade without a head: a misprediction
    for (int i = tid; i < SEQSUM_EXP_SLOTS; i += nt)
        if ((i < s.lo || i > s.hi) && s.total[i] != 0) s.bad = 1;
    __syncthreads();
    // (4) walk the binades in order, verifying every crossing
    if (tid == 0) {
        bool ok = !s.bad;
        float S = 0.0f;
        for (int slot = s.lo; ok && slot <= s.hi; ++slot) {
            const int h = s.head[slot];
            if (h < 0) {
                if (s.total[slot] != 0) ok = false;
                continue;
            }
            const int e = slot - SEQSUM_EXP_OFF;
            const float ph = v[h] * v[h];
            S = S + ph;
            int es;
            frexpf(S, &es);
            if (es - 1 != e || e < -126) {
                ok = false;
                break;
            }
            const long k = (long)(S * ldexpf(1.0f, 23 - e)) + (long)s.total[slot];
            if (k >= (1L << 24)) {
                ok = false;
                break;
            }
            S = ldexpf((float)k, e - 23);
        }
        if (!ok) {  // fallback: the reference's loop as is
            S = 0.0f;
            for (int i = 0; i < n; ++i) {
                const float p = v[i] * v[i];
                S = S + p;
            }
        }
        s.result = S;
    }
    __syncthreads();
    return s.result;
}

}  // namespace gtn
