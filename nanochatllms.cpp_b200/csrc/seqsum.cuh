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
//      increment w.r.t. its binade's ulp (integer arithmetic on the float's bits) or is a tie;
//  (4) one int64 prefix scan of (increments + tie count * 2^48) gives every thread the increments
//      and the ties before its chunk, so heads record their increment prefix and ties land in
//      index order;
//  (5) one warp: per binade the increments from its head to the next head and the tie parities
//      d_j, packed into one 16-byte record per binade; then one thread walks the records in
//      order: S = fl(S + p_head) (an exact IEEE add) must land in binade e, then S/u +=
//      increments + round-ups, in 32-bit integers, which must stay below 2^24.
// Each scan takes one CTA barrier, the tail one and the result one more: four barriers when the
// caller supplies the largest term, six otherwise. (A walk that passed the binades between the
// lanes of a warp by shuffles ran about 1,100-1,700 cycles per binade on sm_100a; the
// single-thread walk over the records runs about 80.)
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
constexpr int SEQSUM_PER_MAX = 8;     // default terms per thread kept in registers

struct SeqSumSmem {
    long long wsum[2][SEQSUM_THREADS_MAX / 32];  // per-warp totals of the two scans
    long long hpre[SEQSUM_SLOTS];                // per binade: increments before its head
    int head[SEQSUM_SLOTS];
    float phead[SEQSUM_SLOTS];
    int d0[SEQSUM_SLOTS];  // parity of the first tie (or -1: no tie)
    int x[SEQSUM_SLOTS];   // sum of d_j xor d_(j-1) over the binade's ties
    int sslot[SEQSUM_TIES_MAX], sd[SEQSUM_TIES_MAX];  // ties in index order: binade, increment-prefix parity
    int4 walk[SEQSUM_SLOTS];  // the binades in order: head term, exponent bits, tie mask, increments
    int bad;
    unsigned int maxbits;
    float result;
};

// Exclusive prefix of x over the CTA (thread order), in int64, with one CTA barrier: every warp
// stores its total in `wsum`, then every warp sums the totals of the warps before its own (lane j
// takes warp j's, a butterfly adds them up). `wsum` must not be written again before the next CTA
// barrier.
__device__ __forceinline__ long long seqsum_exscan64(long long x, long long* wsum) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    long long inc = x;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const long long t = __shfl_up_sync(0xffffffffu, inc, o);
        if (lane >= o) inc += t;
    }
    if (lane == 31) wsum[warp] = inc;
    __syncthreads();
    long long pre = lane < warp ? wsum[lane] : 0;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) pre += __shfl_xor_sync(0xffffffffu, pre, o);
    return pre + inc - x;
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
// the same way on every call). `incs`: unused scratch (kept for callers' layouts). maxbits: the
// largest term's bit pattern if the caller knows it (from seqsum_maxbits), else 0. All threads of
// the CTA must call it (blockDim.x <= 1024, a multiple of 32, >= 64); it synchronizes the CTA.
// PER: terms per thread kept in registers (more per thread: the serial loop).
template <int PER = SEQSUM_PER_MAX, class Term>
__device__ __forceinline__ float seq_sum_exact(Term term, int n, SeqSumSmem& s, int* incs, unsigned int maxbits = 0u) {
    (void)incs;
    const int tid = threadIdx.x, nt = blockDim.x, lane = tid & 31, warp = tid >> 5;
    const int nw = (nt + 31) >> 5;
    const int per = (n + nt - 1) / nt;
    const int i0 = min(n, tid * per), i1 = min(n, i0 + per);
    // more than PER terms per thread: the serial loop (cnt = 0 skips the parallel work)
    const int cnt = per <= PER ? i1 - i0 : 0;
    float pv[PER];
#pragma unroll
    for (int k = 0; k < PER; ++k) pv[k] = k < cnt ? term(i0 + k) : 0.0f;
    if (tid < SEQSUM_SLOTS) {
        s.head[tid] = -1;
        s.d0[tid] = -1;
        s.x[tid] = 0;
    }
    if (tid == 0) {
        s.bad = n > (1 << 14) || per > PER;  // n: keeps the fixed-point sum below 2^63
        s.maxbits = 0u;
    }
    if (maxbits == 0u) {  // uniform over the CTA
        __syncthreads();
        // (1) largest term (non-negative floats order like their bit patterns)
        unsigned int mb = 0u;
#pragma unroll
        for (int k = 0; k < PER; ++k) mb = max(mb, __float_as_uint(pv[k]));  // pv >= +0
        mb = __reduce_max_sync(0xffffffffu, mb);
        if (lane == 0) atomicMax(&s.maxbits, mb);
        __syncthreads();
        maxbits = s.maxbits;
        if (maxbits == 0u) return 0.0f;  // every term is +0: the sum is exactly 0
    }
    // the shared state written above is next read after the first scan's barrier
    bool bad = maxbits >= 0x7f800000u;  // inf / nan / a negative term
    const int emax = maxbits >= 0x800000u ? (int)(maxbits >> 23) - 127 : -126;
    // binade exponent of slot sl: Q = S * 2^eoff => e = sl - eoff
    const int eoff = 23 + SEQSUM_FRAC_BITS - emax;
    // (2) t_i = floor(p_i * 2^eoff): with p = M * 2^(E-23), t_i = M << (E - emax + SEQSUM_FRAC_BITS),
    // truncated when the shift is negative; then the exact exclusive prefix over the CTA
    unsigned int Mv[PER];
    int Ev[PER];
    long long fx[PER], loc = 0;
#pragma unroll
    for (int k = 0; k < PER; ++k) {
        seqsum_split(pv[k], Mv[k], Ev[k]);
        const int sh = Ev[k] - emax + SEQSUM_FRAC_BITS;
        fx[k] = sh >= 0 ? (long long)Mv[k] << sh : (sh > -32 ? (long long)(Mv[k] >> -sh) : 0LL);  // sh <= 25
        loc += fx[k];  // pv[k >= cnt] = 0
    }
    const long long Q0 = seqsum_exscan64(loc, s.wsum[0]);
    // (3) per term: binade slot, head flag, increment, tie (independent once the slots are known)
    int slv[PER], inc[PER];
    bool hd[PER], tie[PER];
    {
        long long Q = Q0;
        int slp = Q0 > 0 ? 63 - __clzll(Q0) : -1;
#pragma unroll
        for (int k = 0; k < PER; ++k) {
            Q += fx[k];
            const bool valid = k < cnt;
            const int sk = Q > 0 ? 63 - __clzll(Q) : -1;  // < 63 since Q < 2^63
            bad |= valid && Q == 0 && pv[k] != 0.0f;      // a non-zero term below the resolution
            const bool live = valid && sk >= 0;
            hd[k] = live && sk != slp;
            const int e = sk - eoff, sh = e - Ev[k];  // p / u = M * 2^-sh
            const bool rest = live && !hd[k];
            bad |= rest && (sh < 0 || e < -126);
            const int shc = min(max(sh, 1), 31);
            const unsigned int rem = Mv[k] & ((1u << shc) - 1u), half = 1u << (shc - 1);
            int v = sh == 0 ? (int)Mv[k] : (int)(Mv[k] >> shc) + (rem > half ? 1 : 0);
            v = (sh < 0 || sh >= 32) ? 0 : v;  // sh >= 32: p < u/2^8, the add does not change S
            inc[k] = rest ? v : 0;
            tie[k] = rest && sh > 0 && sh < 32 && rem == half;
            slv[k] = valid ? sk : -1;
            slp = live ? sk : slp;
        }
    }
    if (bad) s.bad = 1;
    // (4) one scan of (increments + ties * 2^48): increments < 2^24 per term, ties <= 2^14
    long long itot = 0;
    int ntl = 0;
#pragma unroll
    for (int k = 0; k < PER; ++k) {
        itot += inc[k];
        ntl += tie[k] ? 1 : 0;
    }
    constexpr long long LOW48 = (1LL << 48) - 1;
    const long long P = seqsum_exscan64(itot + ((long long)ntl << 48), s.wsum[1]);
    long long cur = P & LOW48;
    int trank = (int)(P >> 48);
    // heads record their increment prefix; ties land in index order with the parity of the
    // increment prefix up to and including their own floor
#pragma unroll
    for (int k = 0; k < PER; ++k) {
        cur += inc[k];
        if (hd[k]) {
            s.head[slv[k]] = i0 + k;
            s.hpre[slv[k]] = cur;  // a head's own increment is 0
            s.phead[slv[k]] = pv[k];
        }
        if (tie[k]) {
            if (trank < SEQSUM_TIES_MAX) {
                s.sslot[trank] = slv[k];
                s.sd[trank] = (int)(cur & 1);
            }
            ++trank;
        }
    }
    __syncthreads();
    // (5) warp 0: the totals of the second scan, the binades present (64 slots as two ballots),
    // the ties per binade, then lane 0 walks the binades in order.
    if (warp == 0) {
        long long wt = lane < nw ? s.wsum[1][lane] : 0;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) wt += __shfl_xor_sync(0xffffffffu, wt, o);
        const long long total = wt & LOW48;
        const int ntie_all = (int)(wt >> 48);
        const unsigned long long mask = (unsigned long long)__ballot_sync(0xffffffffu, s.head[lane] >= 0) |
                                        ((unsigned long long)__ballot_sync(0xffffffffu, s.head[lane + 32] >= 0) << 32);
        // per binade: the first tie's parity d_0 (relative to the head's prefix) and the changes
        // d_j xor d_(j-1) between consecutive ties (the head's parity cancels in those)
        const int nties = min(ntie_all, SEQSUM_TIES_MAX);
        for (int r = lane; r < nties; r += 32) {
            const int sl = s.sslot[r];
            if (r == 0 || s.sslot[r - 1] != sl) s.d0[sl] = (s.sd[r] ^ (int)(s.hpre[sl] & 1)) & 1;
            else atomicAdd(&s.x[sl], (s.sd[r] ^ s.sd[r - 1]) & 1);
        }
        __syncwarp();
        // one record per binade present, in order (lanes j and j + 32 take slots j and j + 32):
        //   .x  the head term's bits
        //   .y  the binade's exponent field (e + 127) << 23, or ~0 when it is subnormal or
        //       beyond the largest finite binade
        //   .z  the first tie's parity d_0, or -1 without ties: the round-up on entry is
        //       ((S/u + d_0) & 1) & (d_0 >= 0 ? 1 : 0)
        //   .w  the increments up to the next head plus the later ties' round-ups, saturated at
        //       2^25 (the binade's integer S/u stays below 2^24, so more fails anyway)
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int sl = lane + 32 * h;
            if ((mask >> sl) & 1ULL) {
                const unsigned long long above = sl < 63 ? mask & (~0ULL << (sl + 1)) : 0ULL;
                const long long nxt = above ? s.hpre[__ffsll((long long)above) - 1] : total;
                const long long add = nxt - s.hpre[sl] + s.x[sl];
                const int e = sl - eoff;
                int4 w;
                w.x = __float_as_int(s.phead[sl]);
                w.y = e >= -126 && e <= 127 ? (e + 127) << 23 : -1;
                w.z = s.d0[sl];
                w.w = (int)min(add, (long long)(1 << 25));
                s.walk[__popcll(mask & ((1ULL << sl) - 1ULL))] = w;
            }
        }
        __syncwarp();
        if (lane == 0) {
            // the walk: S = fl(S + p_head) must land in binade e, then S/u += the round-up on
            // entry and the binade's increments, which must stay below 2^24
            const int nb = __popcll(mask);
            bool ok = !s.bad && ntie_all <= SEQSUM_TIES_MAX;
            float S = 0.0f;
#pragma unroll 4
            for (int r = 0; r < nb; ++r) {
                const int4 w = s.walk[r];
                S = S + __int_as_float(w.x);
                const int bS = __float_as_int(S);
                const int Sb = (bS & 0x7fffff) | 0x800000;  // S / u
                const int up = (Sb + w.z) & (w.z >= 0 ? 1 : 0);
                const int Sn = Sb + w.w + up;
                ok = ok && (bS & 0x7f800000) == w.y && Sn < (1 << 24);
                S = __int_as_float(w.y | (Sn & 0x7fffff));
            }
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
template <int PER = SEQSUM_PER_MAX>
__device__ __forceinline__ float seq_sum_squares(const float* v, int n, SeqSumSmem& s, int* incs,
                                                 unsigned int maxbits = 0u) {
    return seq_sum_exact<PER>([v](int i) { return v[i] * v[i]; }, n, s, incs, maxbits);
}

}  // namespace gtn
