// Exact emulation of a sequential fp32 sum of non-negative terms, computed in parallel.
//
// The reference's RMSNorm accumulates sq = sq + x[i]*x[i] for i = 0..n-1 in fp32, one rounding
// per add (ops.cpp:830-836). Done by one thread that is a chain of n dependent adds. For
// non-negative terms the running sum S never decreases, so it moves through binades
// [2^e, 2^(e+1)) in order, and while S stays inside one binade every add rounds to a multiple of
// the same ulp u = 2^(e-23):
//     fl(S + p) = S + u * inc,  inc = floor(p/u) + (frac(p/u) > 1/2)
// and when frac(p/u) == 1/2 exactly (a tie) round-half-even picks inc so that S/u + inc is even.
// So a run of adds inside one binade is an integer sum of per-term increments; only the ties
// depend on the running value, through its parity. For the ties j = 0, 1, ... of one binade let
// d_j be the parity of (the binade's increments up to and including tie j's floor); tie j rounds
// up iff (S_head/u + d_j + E_j) is odd, E_j being the round-ups before it. The parity of E_(j+1)
// equals c_j = (S_head/u + d_j) mod 2, so tie 0 rounds up iff c_0 is odd and tie j >= 1 iff
// d_j != d_(j-1): the binade's total round-ups are c_0 + sum_j (d_j xor d_(j-1)), which depends
// on the running value only through the parity of S_head/u.
//
// Algorithm (one CTA, every thread owns a contiguous chunk of terms, kept in registers):
//  (1) the exponent of the largest term fixes a fixed-point scale (the caller may supply it);
//  (2) an exact int64 prefix scan of floor(p_i * 2^F) predicts the binade of the running sum after
//      term i. Integer sums are associative, so every thread sees the same prediction at every
//      index;
//  (3) the first term of each predicted binade is its "head"; every other term gets its integer
//      increment w.r.t. its binade's ulp (integer arithmetic on the float's bits); ties are listed;
//  (4) an int64 prefix scan of the increments;
//  (5) per binade (in parallel): the increments from its head to the next head and the tie terms
//      above; then warp 0 walks the binades in order (their data in lane registers, fetched by
//      shuffles): S = fl(S + p_head) (an exact IEEE add) must land in binade e, then
//      S/u += increments + round-ups, which must stay below 2^24.
// Any failed check (a mispredicted crossing, a term below the fixed-point resolution, a subnormal
// binade, a non-finite term, more ties than the list holds) makes the CTA fall back to the plain
// sequential loop, so the result is always bit-identical to the serial sum.
#pragma once
#include <cstdint>

namespace gtn {

constexpr int SEQSUM_THREADS_MAX = 1024;
constexpr int SEQSUM_SLOTS = 64;      // binade slot = floor(log2(Q)), Q = the fixed-point sum
constexpr int SEQSUM_TIES_MAX = 128;
constexpr int SEQSUM_FRAC_BITS = 25;  // the largest term becomes < 2^(24 + 25)
constexpr int SEQSUM_PER_MAX = 8;     // terms per thread kept in registers

struct SeqSumSmem {
    long long wsum[2][SEQSUM_THREADS_MAX / 32];  // per-warp partials of the two scans
    long long cpre[SEQSUM_THREADS_MAX];          // per-thread exclusive prefix of the increments
    long long tot[SEQSUM_SLOTS];                 // per binade: increments from its head to the next head
    int head[SEQSUM_SLOTS];
    float phead[SEQSUM_SLOTS];
    int d0[SEQSUM_SLOTS];  // parity of the first tie (or -1: no tie)
    int x[SEQSUM_SLOTS];   // sum of d_j xor d_(j-1) over the binade's ties
    int tie[SEQSUM_TIES_MAX], tslot[SEQSUM_TIES_MAX];
    int sslot[SEQSUM_TIES_MAX], sd[SEQSUM_TIES_MAX];
    unsigned int mask[2];
    int ntie;
    int bad;
    unsigned int maxbits;
    float result;
};

// Exclusive prefix of x over the CTA (thread order), in int64, with per-warp partials in `wsum`
// (not read by a scan in flight); two CTA barriers.
__device__ __forceinline__ long long seqsum_exscan64(long long x, long long* wsum) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
    long long inc = x;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const long long t = __shfl_up_sync(0xffffffffu, inc, o);
        if (lane >= o) inc += t;
    }
    if (lane == 31) wsum[warp] = inc;
    __syncthreads();
    if (warp == 0) {
        long long w = lane < nw ? wsum[lane] : 0;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const long long t = __shfl_up_sync(0xffffffffu, w, o);
            if (lane >= o) w += t;
        }
        if (lane < nw) wsum[lane] = w;
    }
    __syncthreads();
    return (warp > 0 ? wsum[warp - 1] : 0) + inc - x;
}

// p = M * 2^(E - 23) for a finite non-negative float (M < 2^24; subnormals E = -126).
__device__ __forceinline__ void seqsum_split(float p, unsigned int& M, int& E) {
    const unsigned int b = __float_as_uint(p);
    const unsigned int ef = b >> 23;
    M = (b & 0x7fffffu) | (ef ? 0x800000u : 0u);
    E = ef ? (int)ef - 127 : -126;
}

// Largest of non-negative floats through their bit patterns (NaN maps above +inf).
__device__ __forceinline__ unsigned int seqsum_maxbits(float p) { return __float_as_uint(p); }

// Returns fl(...fl(fl(0 + p_0) + p_1)... + p_{n-1}) where p_i = term(i) >= 0 (a float computed
// the same way on every call). `incs`: n ints of scratch (shared memory). maxbits: the largest
// term's bit pattern if the caller knows it (from seqsum_maxbits), else 0. All threads of the
// CTA must call it (blockDim.x <= 1024, a multiple of 32, >= 64); it synchronizes the CTA.
template <class Term>
__device__ __forceinline__ float seq_sum_exact(Term term, int n, SeqSumSmem& s, int* incs, unsigned int maxbits = 0u) {
    const int tid = threadIdx.x, nt = blockDim.x, lane = tid & 31, warp = tid >> 5;
    const int per = (n + nt - 1) / nt;
    const int i0 = min(n, tid * per), i1 = min(n, i0 + per);
    // more than SEQSUM_PER_MAX terms per thread: the serial loop (cnt = 0 skips the parallel work)
    const int cnt = per <= SEQSUM_PER_MAX ? i1 - i0 : 0;
    float pv[SEQSUM_PER_MAX];
#pragma unroll
    for (int k = 0; k < SEQSUM_PER_MAX; ++k) pv[k] = k < cnt ? term(i0 + k) : 0.0f;
    if (tid < SEQSUM_SLOTS) {
        s.head[tid] = -1;
        s.d0[tid] = -1;
        s.x[tid] = 0;
    }
    if (tid == 0) {
        s.bad = n > (1 << 14) || per > SEQSUM_PER_MAX;  // n: keeps the fixed-point sum below 2^63
        s.ntie = 0;
        s.maxbits = maxbits;
    }
    if (maxbits == 0u) {
        __syncthreads();
        // (1) largest term (non-negative floats order like their bit patterns)
        unsigned int mb = 0u;
#pragma unroll
        for (int k = 0; k < SEQSUM_PER_MAX; ++k) mb = max(mb, __float_as_uint(pv[k]));  // pv >= +0
        mb = __reduce_max_sync(0xffffffffu, mb);
        if (lane == 0) atomicMax(&s.maxbits, mb);
    }
    __syncthreads();
    maxbits = s.maxbits;
    if (maxbits == 0u) return 0.0f;                   // every term is +0: the sum is exactly 0
    if (maxbits >= 0x7f800000u) s.bad = 1;            // inf / nan / a negative term
    const int emax = maxbits >= 0x800000u ? (int)(maxbits >> 23) - 127 : -126;
    // t_i = floor(p_i * 2^eoff), eoff = 23 + SEQSUM_FRAC_BITS - emax, i.e. with p = M * 2^(E-23):
    // t_i = M << (E - emax + SEQSUM_FRAC_BITS), truncated when the shift is negative.
    auto fixed = [&](float p) -> long long {
        unsigned int M;
        int E;
        seqsum_split(p, M, E);
        const int sh = E - emax + SEQSUM_FRAC_BITS;
        if (sh >= 0) return (long long)M << sh;  // sh <= 25
        return sh > -32 ? (long long)(M >> -sh) : 0LL;
    };
    // binade exponent of slot sl: Q = S * 2^eoff => e = sl - eoff
    const int eoff = 23 + SEQSUM_FRAC_BITS - emax;
    // (2) exact fixed-point prefix
    long long loc = 0;
#pragma unroll
    for (int k = 0; k < SEQSUM_PER_MAX; ++k) loc += fixed(pv[k]);  // pv[k >= cnt] = 0
    long long Q = seqsum_exscan64(loc, s.wsum[0]);
    // (3) heads, increments, ties
    int sl_prev = Q > 0 ? 63 - __clzll(Q) : -1;
    long long itot = 0;
#pragma unroll
    for (int k = 0; k < SEQSUM_PER_MAX; ++k) {
        if (k >= cnt) break;
        const int i = i0 + k;
        const float p = pv[k];
        Q += fixed(p);
        int inc = 0;
        if (Q == 0) {
            if (p != 0.0f) s.bad = 1;  // a non-zero term below the fixed-point resolution
        } else {
            const int sl = 63 - __clzll(Q);  // < 63 since Q < 2^63
            if (sl != sl_prev) {
                s.head[sl] = i;
            } else {
                const int e = sl - eoff;
                unsigned int M;
                int E;
                seqsum_split(p, M, E);
                const int sh = e - E;  // p / u = M * 2^-sh
                if (sh < 0 || e < -126) {
                    s.bad = 1;
                } else if (sh == 0) {
                    inc = (int)M;
                } else if (sh < 32) {
                    inc = (int)(M >> sh);
                    const unsigned int rem = M & ((1u << sh) - 1u), half = 1u << (sh - 1);
                    if (rem > half) {
                        ++inc;
                    } else if (rem == half) {
                        const int t = atomicAdd(&s.ntie, 1);
                        if (t < SEQSUM_TIES_MAX) {
                            s.tie[t] = i;
                            s.tslot[t] = sl;
                        } else {
                            s.bad = 1;
                        }
                    }
                }  // sh >= 32: p < u/2^8, the add does not change S
            }
            sl_prev = sl;
        }
        incs[i] = inc;
        itot += inc;
    }
    // (4) prefix of the increments: per-thread exclusive offsets in cpre
    const long long ip = seqsum_exscan64(itot, s.wsum[1]);
    s.cpre[tid] = ip;
    if (tid < SEQSUM_SLOTS) {
        const unsigned int bal = __ballot_sync(0xffffffffu, s.head[tid] >= 0);
        if (lane == 0) s.mask[warp] = bal;
    }
    __syncthreads();
    auto incl = [&](int i) -> long long {  // inclusive prefix of incs at i
        const int owner = i / per;
        long long r = s.cpre[owner];
        for (int j = owner * per; j <= i; ++j) r += incs[j];
        return r;
    };
    const int nties = min(s.ntie, SEQSUM_TIES_MAX);
    const unsigned long long mask = ((unsigned long long)s.mask[1] << 32) | s.mask[0];
    // (5a) per binade: increments from the head to the next head; tie parities in index order
    if (tid < SEQSUM_SLOTS) {
        const int h = s.head[tid];
        if (h >= 0) {
            const unsigned long long above = tid < 63 ? mask & (~0ULL << (tid + 1)) : 0ULL;
            const int hn = above ? s.head[__ffsll((long long)above) - 1] : n;
            s.tot[tid] = incl(hn - 1) - incl(h);
            s.phead[tid] = term(h);
        }
    }
    for (int k = tid - SEQSUM_SLOTS; k >= 0 && k < nties; k += nt) {  // rank sort of the ties
        const int i = s.tie[k];
        int r = 0;
        for (int j = 0; j < nties; ++j) r += s.tie[j] < i;
        const int sl = s.tslot[k];
        s.sslot[r] = sl;
        s.sd[r] = (int)((incl(i) - incl(s.head[sl])) & 1);
    }
    __syncthreads();
    for (int r = tid; r < nties; r += nt) {
        const int sl = s.sslot[r];
        if (r == 0 || s.sslot[r - 1] != sl) s.d0[sl] = s.sd[r];
        else atomicAdd(&s.x[sl], s.sd[r] ^ s.sd[r - 1]);
    }
    __syncthreads();
    // (5b) the walk: warp 0, binades in slot order, 32 at a time in lane registers
    if (warp == 0) {
        bool ok = !s.bad;
        float S = 0.0f;
        unsigned long long m = mask;
        while (ok && m) {
            // lane j takes the j-th remaining binade
            unsigned long long mm = m;
            int mine = -1;
            for (int j = 0; j < 32 && mm; ++j) {
                const int sl = __ffsll((long long)mm) - 1;
                mm &= mm - 1;
                if (j == lane) mine = sl;
            }
            const int cnt = min(32, __popcll(m));
            float ph = 0.0f;
            long long tt = 0;
            int dd = -1, xx = 0;
            if (mine >= 0) {
                ph = s.phead[mine];
                tt = s.tot[mine];
                dd = s.d0[mine];
                xx = s.x[mine];
            }
            for (int j = 0; j < cnt; ++j) {
                const int sl = __shfl_sync(0xffffffffu, mine, j);
                const float phj = __shfl_sync(0xffffffffu, ph, j);
                const long long ttj = __shfl_sync(0xffffffffu, tt, j);
                const int ddj = __shfl_sync(0xffffffffu, dd, j);
                const int xxj = __shfl_sync(0xffffffffu, xx, j);
                if (!ok) continue;
                const int e = sl - eoff;
                S = S + phj;
                const unsigned int b = __float_as_uint(S);
                if ((int)(b >> 23) - 127 != e || e < -126) {
                    ok = false;
                    continue;
                }
                long long Sb = (long long)((b & 0x7fffffu) | 0x800000u);  // S / u
                if (ddj >= 0) Sb += ((Sb + ddj) & 1) + xxj;
                Sb += ttj;
                if (Sb >= (1LL << 24)) {
                    ok = false;
                    continue;
                }
                S = __uint_as_float(((unsigned int)(e + 127) << 23) | ((unsigned int)Sb & 0x7fffffu));
            }
            m = mm;
        }
        if (lane == 0) {
            if (!ok) {  // fallback: the reference's loop as is
                S = 0.0f;
                for (int i = 0; i < n; ++i) {
                    const float p = term(i);
                    S = S + p;
                }
            }
            s.result = S;
        }
    }
    __syncthreads();
    return s.result;
}

// The sum of squares of v[0..n) (RMSNorm, ops.cpp:830-836: glibc powf(x, 2) == x*x exactly).
__device__ __forceinline__ float seq_sum_squares(const float* v, int n, SeqSumSmem& s, int* incs,
                                                 unsigned int maxbits = 0u) {
    return seq_sum_exact([v](int i) { return v[i] * v[i]; }, n, s, incs, maxbits);
}

}  // namespace gtn
