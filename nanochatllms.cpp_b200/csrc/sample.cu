// Top-k / temperature sampling on the device with a seeded MT19937 (gtn_sample_topk, gtn_rng_*).
//
// Reference: topk_sample, sampler.cpp:63-128. Per step it divides every logit by temp in double,
// partial_sorts the top_k largest to the front (descending), replaces each by exp() and sums them in
// that order (double), divides by the sum, scatters the probabilities into a vocabulary-sized
// vector of zeros and draws from std::discrete_distribution with a std::mt19937. The distribution
// (libstdc++) sums its weights in index order, divides each by the sum, takes partial sums, forces
// the last one to 1.0 and returns the lower_bound of one generate_canonical<double> draw: two
// 32-bit outputs x0, x1 -> fl(x0 + x1 * 2^32) / 2^64 (mapped below 1). Zero weights add exactly
// nothing, so only the top_k entries in index order matter; an index without weight is returned
// only for a draw of exactly 0 (index 0) or a draw above the last partial sum (index n - 1).
//
// One CTA of 1024 threads: radix select of the top_k float keys (up to 4 passes of 8 bits over
// order-preserving unsigned keys, held in registers for vocabularies up to 32768), a gather of the
// selected keys (in index order among ties at the k-th place), bitonic sorts (by value, then by
// index), double exp and the divisions in parallel, the two ordered sums and the partial-sum search
// on one thread. MT19937 (Matsumoto & Nishimura 1998: n = 624, m = 397, the published twist and
// tempering constants) lives in device memory as 624 words and an index, seeded on the host like
// std::mt19937(seed); its twist runs block-parallel.
#include <cstring>
#include <vector>

#include "launch.cuh"

namespace gtn {

constexpr int MT_N = 624, MT_M = 397;
constexpr int TOPK_MAX = 1000, SAMPLE_THREADS = 1024, SAMPLE_BATCH = 8;

// MT19937 tempering of one state word.
__device__ __forceinline__ uint32_t mt_temper(uint32_t y) {
    y ^= y >> 11;
    y ^= (y << 7) & 0x9d2c5680u;
    y ^= (y << 15) & 0xefc60000u;
    y ^= y >> 18;
    return y;
}

__device__ __forceinline__ uint32_t mt_mix(uint32_t cur, uint32_t next, uint32_t far) {
    const uint32_t y = (cur & 0x80000000u) | (next & 0x7fffffffu);
    return far ^ (y >> 1) ^ ((y & 1u) ? 0x9908b0dfu : 0u);
}

// The MT19937 twist of the 624 state words, by the whole block. The sequential in-place loop
// x[k] = x[(k + 397) % 624] ^ f(x[k], x[(k + 1) % 624]) reads words it has already rewritten only
// through x[(k + 397) % 624] for k >= 227 (x[k - 227]) and x[0] for k = 623, so it runs as three
// parallel phases: k < 227, 227 <= k < 454, 454 <= k < 624 (every input read before any write).
__device__ void mt_twist_block(uint32_t* st) {
    const int t = threadIdx.x;
#pragma unroll
    for (int lo = 0; lo < MT_N; lo += 227) {
        const int hi = lo + 227 < 454 ? lo + 227 : (lo == 227 ? 454 : MT_N);
        const int k = lo + t;
        uint32_t v = 0u;
        if (k < hi) v = mt_mix(st[k], st[(k + 1) % MT_N], st[(k + MT_M) % MT_N]);
        __syncthreads();
        if (k < hi) st[k] = v;
        __syncthreads();
    }
}

// Order-preserving unsigned key of a float (NaN ranks lowest).
__device__ __forceinline__ uint32_t fkey(float f) {
    const uint32_t u = __float_as_uint(f);
    return f != f ? 0u : ((u & 0x80000000u) ? ~u : (u | 0x80000000u));
}

// In-place bitonic sort of the first P (a power of two, 256 < P <= SAMPLE_THREADS) keys in shared
// memory, ascending. Every thread of the block calls it.
__device__ void block_sort(unsigned long long* key, int P) {
    const int t = threadIdx.x;
    for (int size = 2; size <= P; size <<= 1) {
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
            __syncthreads();
            const int j = t ^ stride;
            if (t < P && j > t) {
                const bool up = (t & size) == 0;
                const unsigned long long a = key[t], b = key[j];
                if ((a > b) == up) {
                    key[t] = b;
                    key[j] = a;
                }
            }
        }
    }
    __syncthreads();
}

// The same network on the first 32 * E keys by one warp: element lane + 32 e in register x[e]
// (strides of 32 and more compare registers of a lane, shorter ones exchange between lanes).
template <int E>
__device__ void warp_sort(unsigned long long* key, int lane) {
    unsigned long long x[E];
#pragma unroll
    for (int e = 0; e < E; ++e) x[e] = key[lane + 32 * e];
#pragma unroll
    for (int size = 2; size <= 32 * E; size <<= 1) {
#pragma unroll
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
            if (stride >= 32) {
                const int es = stride >> 5;
#pragma unroll
                for (int e = 0; e < E; ++e) {
                    if ((e & es) == 0) {
                        const bool up = ((lane + 32 * e) & size) == 0;
                        const unsigned long long a = x[e], b = x[e | es];
                        const bool sw = (a > b) == up;
                        x[e] = sw ? b : a;
                        x[e | es] = sw ? a : b;
                    }
                }
            } else {
                const bool lower = (lane & stride) == 0;
#pragma unroll
                for (int e = 0; e < E; ++e) {
                    const unsigned long long y = __shfl_xor_sync(0xffffffffu, x[e], stride);
                    const bool up = ((lane + 32 * e) & size) == 0;
                    x[e] = (lower == up) ? (x[e] < y ? x[e] : y) : (x[e] < y ? y : x[e]);
                }
            }
        }
    }
#pragma unroll
    for (int e = 0; e < E; ++e) key[lane + 32 * e] = x[e];
}

// Ascending sort of the first P (a power of two) keys; every thread calls it.
__device__ __forceinline__ void sort_keys(unsigned long long* key, int P) {
    if (P <= 256) {
        if (threadIdx.x < 32) {
            if (P <= 64) warp_sort<2>(key, threadIdx.x);
            else if (P == 128) warp_sort<4>(key, threadIdx.x);
            else warp_sort<8>(key, threadIdx.x);
        }
        __syncthreads();
    } else {
        block_sort(key, P);
    }
}

__device__ __forceinline__ unsigned long long cand_key(uint32_t key, int j) {
    return ((unsigned long long)(~key) << 32) | (uint32_t)j;  // ascending = value descending, then index
}

struct SampleSel {  // the bin holding the rem-th largest key of a histogram pass
    unsigned int bin, rem, eqn;
};

// Histogram of NB = BPT * SAMPLE_THREADS bins; thread t owns the BPT bins NB-1-t*BPT-q (q < BPT), so
// counts accumulate from the top bin down. Finds the bin holding the rem-th largest key and the
// rank within it; every thread calls it.
template <int BPT>
__device__ void find_bin(const unsigned int* hist, uint32_t rem, unsigned int* wsum, SampleSel* out) {
    const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
    constexpr int NB = BPT * SAMPLE_THREADS;
    uint32_t c[BPT], tot = 0u;
#pragma unroll
    for (int q = 0; q < BPT; ++q) {
        c[q] = hist[NB - 1 - (t * BPT + q)];
        tot += c[q];
    }
    uint32_t incl = tot;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const uint32_t v = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += v;
    }
    if (lane == 31) wsum[warp] = incl;
    __syncthreads();
    uint32_t cum = incl - tot;
    for (int w = 0; w < warp; ++w) cum += wsum[w];
    if (cum < rem && rem <= cum + tot) {
#pragma unroll
        for (int q = 0; q < BPT; ++q) {
            if (cum + c[q] >= rem) {
                out->bin = (unsigned int)(NB - 1 - (t * BPT + q));
                out->rem = rem - cum;
                out->eqn = c[q];
                break;
            }
            cum += c[q];
        }
    }
    __syncthreads();
}

// The key of logit j from the shared cache or from global memory.
template <bool CACHED>
__device__ __forceinline__ uint32_t key_at(const uint32_t* kc, const float* logits, int j) {
    if constexpr (CACHED) return kc[j];
    else return fkey(__ldcg(logits + j));
}

// Every key >= T into an atomic slot of skey (the caller knows their number fits).
template <bool CACHED>
__device__ void gather_ge(const uint32_t* kc, const float* logits, int n, uint32_t T, unsigned long long* skey,
                          unsigned int* cnt) {
    const int tid = threadIdx.x;
    for (int base = 0; base < n; base += SAMPLE_THREADS * SAMPLE_BATCH) {
        uint32_t kb[SAMPLE_BATCH];
#pragma unroll
        for (int i = 0; i < SAMPLE_BATCH; ++i) {
            const int j = base + i * SAMPLE_THREADS + tid;
            kb[i] = j < n ? key_at<CACHED>(kc, logits, j) : 0u;
        }
#pragma unroll
        for (int i = 0; i < SAMPLE_BATCH; ++i) {
            const int j = base + i * SAMPLE_THREADS + tid;
            if (j < n && kb[i] >= T) skey[atomicAdd(cnt, 1u)] = cand_key(kb[i], j);
        }
    }
}

constexpr int SAMPLE_BINS1 = 4096;  // first digit: key bits 31..20

// grid 1, block SAMPLE_THREADS. k in [1, min(n, TOPK_MAX)], temp > 0; mt: the generator state.
// CACHED (n <= SAMPLE_CACHE keys, n * 4 bytes of dynamic shared memory): the keys are computed once
// into shared memory; otherwise each pass reads the logits (L2) in batches.
template <bool CACHED>
static __global__ void __launch_bounds__(SAMPLE_THREADS, 1) k_topk_sample(const float* __restrict__ logits, int n,
                                                                          float temp, int k, uint32_t* mt,
                                                                          SampleDst dst) {
    __shared__ union {
        unsigned int hist[SAMPLE_BINS1];  // selection
        struct {
            double sp[SAMPLE_THREADS], sq[SAMPLE_THREADS];
        } pr;                             // probabilities, after the selection
    } w;
    __shared__ unsigned long long skey[SAMPLE_THREADS];
    __shared__ unsigned int wsum[SAMPLE_THREADS / 32];
    __shared__ SampleSel sel;
    __shared__ unsigned int s_cnt, s_base, s_mti, s_first;
    __shared__ double s_sum, s_sum2, s_pr;
    extern __shared__ uint32_t kc[];  // CACHED: key of logit j at kc[j]
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    // the generator words this draw will use, fetched early (thread 0)
    uint32_t mti = 0u, w0 = 0u, w1 = 0u;
    if (tid == 0 && n >= 2) {
        mti = mt[MT_N];
        if (mti <= (uint32_t)MT_N - 2) {
            w0 = mt[mti];
            w1 = mt[mti + 1];
        } else if (mti == (uint32_t)MT_N - 1) {
            w0 = mt[mti];
        }
    }
    // (1) histogram of the top 12 key bits, fused with computing (and caching) the keys
    for (int i = tid; i < SAMPLE_BINS1; i += SAMPLE_THREADS) w.hist[i] = 0u;
    skey[tid] = ~0ull;  // padding sorts last
    if (tid == 0) s_cnt = 0u;
    __syncthreads();
    for (int base = 0; base < n; base += SAMPLE_THREADS * SAMPLE_BATCH) {
        float v[SAMPLE_BATCH];
#pragma unroll
        for (int i = 0; i < SAMPLE_BATCH; ++i) {
            const int j = base + i * SAMPLE_THREADS + tid;
            v[i] = j < n ? __ldcg(logits + j) : 0.0f;
        }
#pragma unroll
        for (int i = 0; i < SAMPLE_BATCH; ++i) {
            const int j = base + i * SAMPLE_THREADS + tid;
            if (j < n) {
                const uint32_t key = fkey(v[i]);
                if constexpr (CACHED) kc[j] = key;
                atomicAdd(&w.hist[key >> 20], 1u);
            }
        }
    }
    __syncthreads();
    find_bin<SAMPLE_BINS1 / SAMPLE_THREADS>(w.hist, (uint32_t)k, wsum, &sel);
    uint32_t T = sel.bin << 20, rem = sel.rem;
    const uint32_t n_ge = (uint32_t)k - rem + sel.eqn;  // keys >= T
    int n_sel;
    if (n_ge <= (uint32_t)SAMPLE_THREADS) {
        // (2a) every key >= T; the value sort below puts the k largest first (ties at the k-th place:
        // lowest indices first)
        gather_ge<CACHED>(kc, logits, n, T, skey, &s_cnt);
        n_sel = (int)n_ge;
    } else {
        // (2b) refine the boundary bin by 10-bit digits (bits 19..10, 9..0) until it is taken whole
        uint32_t mask = 0xfff00000u;
        for (int shift = 10; shift >= 0 && sel.eqn != rem; shift -= 10) {  // uniform
            w.hist[tid] = 0u;
            __syncthreads();
            for (int j = tid; j < n; j += SAMPLE_THREADS) {
                const uint32_t key = key_at<CACHED>(kc, logits, j);
                if ((key & mask) == T) atomicAdd(&w.hist[(key >> shift) & 1023u], 1u);
            }
            __syncthreads();
            find_bin<1>(w.hist, rem, wsum, &sel);
            T |= sel.bin << shift;
            rem = sel.rem;
            mask |= 1023u << shift;
        }
        if (sel.eqn == rem) {
            gather_ge<CACHED>(kc, logits, n, T, skey, &s_cnt);
        } else {  // a tie across the k-th place: keys above T, then the keys equal to T in index order
            if (tid == 0) s_base = 0u;
            __syncthreads();
            for (int base = 0; base < n; base += SAMPLE_THREADS) {
                const int j = base + tid;
                const uint32_t kj = j < n ? key_at<CACHED>(kc, logits, j) : 0u;
                const bool gt = j < n && kj > T, eq = j < n && kj == T;
                if (gt) skey[atomicAdd(&s_cnt, 1u)] = cand_key(kj, j);
                const unsigned int b = __ballot_sync(0xffffffffu, eq);
                if (lane == 0) wsum[warp] = __popc(b);
                __syncthreads();
                unsigned int before = s_base, total = 0u;
                for (int w2 = 0; w2 < SAMPLE_THREADS / 32; ++w2) {
                    if (w2 < warp) before += wsum[w2];
                    total += wsum[w2];
                }
                before += __popc(b & ((1u << lane) - 1u));
                if (eq && before < rem) skey[(uint32_t)k - rem + before] = cand_key(kj, j);
                __syncthreads();
                if (tid == 0) s_base += total;
                __syncthreads();
                const bool done = s_base >= rem && s_cnt >= (uint32_t)k - rem;
                __syncthreads();  // every thread has read s_cnt before the next pass adds to it
                if (done) break;  // uniform
            }
        }
        n_sel = k;
    }
    __syncthreads();
    int P = 1;
    while (P < n_sel) P <<= 1;
    // (3) value order (descending; ties by index); the first k entries are the selection. exp of
    // logit/temp in double and their sum in that order.
    sort_keys(skey, P);
    if (tid < k) {
        const int j = (int)(uint32_t)skey[tid];
        w.pr.sp[tid] = exp((double)__ldcg(logits + j) / (double)temp);
    }
    __syncthreads();
    if (tid == 0) {
        double s = 0.0;
#pragma unroll 8
        for (int t = 0; t < k; ++t) s += w.pr.sp[t];
        s_sum = s;
        s_mti = mti;
    }
    __syncthreads();
    // the probabilities of sampler.cpp:117-118; then index order (low word: position in value order)
    unsigned long long ik = ~0ull;
    if (tid < k) {
        w.pr.sp[tid] = w.pr.sp[tid] / s_sum;
        ik = ((unsigned long long)(uint32_t)skey[tid] << 32) | (uint32_t)tid;
    }
    __syncthreads();
    if (tid < P) skey[tid] = ik;
    __syncthreads();
    int P2 = 1;
    while (P2 < k) P2 <<= 1;
    sort_keys(skey, P2);
    if (tid < k) w.pr.sq[tid] = w.pr.sp[(uint32_t)skey[tid]];
    __syncthreads();
    if (tid == 0) {
        double s2 = 0.0;
#pragma unroll 8
        for (int t = 0; t < k; ++t) s2 += w.pr.sq[t];
        s_sum2 = s2;
    }
    __syncthreads();
    if (tid < k) w.pr.sq[tid] = w.pr.sq[tid] / s_sum2;  // std::discrete_distribution's normalized weights
    // (4) the generator: a twist of the state when this draw reaches its end
    const bool draw = n >= 2;  // a one-entry distribution returns 0 without drawing
    if (draw && s_mti >= (uint32_t)MT_N - 1) {  // uniform
        __syncthreads();
        mt_twist_block(mt);
    } else {
        __syncthreads();
    }
    // (5) std::discrete_distribution over the vocabulary, one draw: the first index whose partial sum
    // (in index order; the last one, of index n - 1, forced to 1) reaches the draw. The partial sums
    // are one ordered chain (thread 0); the search runs in parallel (they do not decrease).
    if (tid == 0) {
        s_first = (unsigned int)k;
        double pr = 0.0;
        if (draw) {
            uint32_t x0, x1;
            if (mti <= (uint32_t)MT_N - 2) {
                x0 = w0;
                x1 = w1;
                mt[MT_N] = mti + 2;
            } else if (mti == (uint32_t)MT_N - 1) {
                x0 = w0;
                x1 = mt[0];
                mt[MT_N] = 1;
            } else {
                x0 = mt[0];
                x1 = mt[1];
                mt[MT_N] = 2;
            }
            x0 = mt_temper(x0);
            x1 = mt_temper(x1);
            pr = ((double)x0 + (double)x1 * 4294967296.0) / 18446744073709551616.0;
            if (pr >= 1.0) pr = 1.0 - 1.1102230246251565e-16;  // the largest double below 1
            double c = 0.0;
#pragma unroll 8
            for (int t = 0; t < k; ++t) {
                c = c + w.pr.sq[t];
                w.pr.sq[t] = c;
            }
            if ((int)(skey[k - 1] >> 32) == n - 1) w.pr.sq[k - 1] = 1.0;
        }
        s_pr = pr;
    }
    __syncthreads();
    if (draw && s_pr > 0.0 && tid < k && w.pr.sq[tid] >= s_pr) atomicMin(&s_first, (unsigned int)tid);
    __syncthreads();
    if (tid == 0) {
        // lower_bound over the vocabulary: a draw of 0 stops at index 0 (cp[0] >= 0); past every
        // selected entry it stops at index n - 1 (cp[n - 1] = 1); one entry: 0 without drawing
        int ans = 0;
        if (draw && s_pr > 0.0) ans = s_first < (unsigned int)k ? (int)(skey[s_first] >> 32) : n - 1;
        if (dst.out) dst.out[0] = ans;
        if (dst.tok) {
            const int p = dst.pos[0];
            if (p + 1 < dst.max_ctx) {
                dst.tok[p + 1] = ans;
                dst.gen[p + 1] = ans;
                dst.pos[0] = p + 1;
            } else if (dst.err) {
                atomicOr(dst.err, 4u);
            }
        }
    }
}

constexpr int SAMPLE_CACHE = 49152;  // keys cached in shared memory (192 KB) up to this n

cudaError_t prepare_topk_sample(int n) {
    if (n > SAMPLE_CACHE) return cudaSuccess;
    return ensure_smem(k_topk_sample<true>, (size_t)SAMPLE_CACHE * sizeof(uint32_t));
}

cudaError_t launch_topk_sample(cudaStream_t st, const float* logits, int n, float temp, int k, uint32_t* mt,
                               SampleDst dst) {
    if (n <= SAMPLE_CACHE) {
        const cudaError_t e = prepare_topk_sample(n);
        if (e != cudaSuccess) return e;
        return launch_pdl(k_topk_sample<true>, dim3(1), dim3(SAMPLE_THREADS), sizeof(uint32_t) * (size_t)n, st,
                          logits, n, temp, k, mt, dst);
    }
    return launch_pdl(k_topk_sample<false>, dim3(1), dim3(SAMPLE_THREADS), 0, st, logits, n, temp, k, mt, dst);
}

}  // namespace gtn

using namespace gtn;

extern "C" {

int gtn_rng_create(uint32_t seed, gtn_rng** out) {
    if (!out) return fail(GTN_ERR_ARG, "rng_create: out is NULL");
    *out = nullptr;
    // std::mt19937(seed): x[0] = seed, x[i] = 1812433253 * (x[i-1] ^ (x[i-1] >> 30)) + i
    std::vector<uint32_t> st(MT_N + 1);
    st[0] = seed;
    for (int i = 1; i < MT_N; ++i) st[i] = 1812433253u * (st[i - 1] ^ (st[i - 1] >> 30)) + (uint32_t)i;
    st[MT_N] = MT_N;  // the first output twists
    gtn_rng* r = new gtn_rng();
    cudaGetDevice(&r->device);
    cudaError_t e = cudaMalloc(&r->state, sizeof(uint32_t) * (MT_N + 1));
    if (e == cudaSuccess)
        e = cudaMemcpy(r->state, st.data(), sizeof(uint32_t) * (MT_N + 1), cudaMemcpyHostToDevice);
    if (e != cudaSuccess) {
        if (r->state) cudaFree(r->state);
        delete r;
        return fail(e == cudaErrorMemoryAllocation ? GTN_ERR_OOM : GTN_ERR_CUDA, "rng_create: %s",
                    cudaGetErrorString(e));
    }
    *out = r;
    return GTN_OK;
}

int gtn_rng_free(gtn_rng* rng) {
    if (!rng) return GTN_OK;
    cudaFree(rng->state);
    delete rng;
    return GTN_OK;
}

int gtn_sample_topk(const float* logits, int n, float temp, int top_k, gtn_rng* rng, int32_t* out_index,
                    void* stream) {
    if (!logits || !out_index || !rng) return fail(GTN_ERR_ARG, "sample_topk: NULL argument");
    if (n < 1) return fail(GTN_ERR_ARG, "sample_topk: n %d", n);
    int dev = -1;
    cudaGetDevice(&dev);
    if (dev != rng->device)
        return fail(GTN_ERR_ARG, "sample_topk: rng lives on device %d, current device %d", rng->device, dev);
    if (!(temp > 0.0f)) return fail(GTN_ERR_ARG, "sample_topk: temp must be > 0");
    top_k = top_k < TOPK_MAX ? top_k : TOPK_MAX;  // sampler.cpp:66-67
    temp = temp < 2.0f ? temp : 2.0f;
    if (top_k < 1 || top_k > n) return fail(GTN_ERR_ARG, "sample_topk: top_k %d outside [1, %d]", top_k, n);
    SampleDst dst;
    dst.out = out_index;
    const cudaError_t e =
        launch_topk_sample(static_cast<cudaStream_t>(stream), logits, n, temp, top_k, rng->state, dst);
    if (e != cudaSuccess) return fail(GTN_ERR_CUDA, "sample_topk: %s", cudaGetErrorString(e));
    return GTN_OK;
}

}  // extern "C"
