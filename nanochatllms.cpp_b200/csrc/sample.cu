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
// One CTA of 1024 threads: radix select of the top_k float keys (4 passes of 8 bits over
// order-preserving unsigned keys), an in-order gather of the tied keys, bitonic sorts (by value,
// then by index), double exp in parallel, the two short sums and the draw on one thread. MT19937
// (Matsumoto & Nishimura 1998: n = 624, m = 397, the published twist and tempering constants)
// lives in device memory as 624 words and an index, seeded on the host like std::mt19937(seed).
#include <cstring>
#include <vector>

#include "launch.cuh"

struct gtn_rng {
    uint32_t* state = nullptr;  // device: 624 words, then the index of the next output
    int device = 0;
};

namespace gtn {

constexpr int MT_N = 624, MT_M = 397;
constexpr int TOPK_MAX = 1000, SAMPLE_THREADS = 1024;

// The next MT19937 output (one thread).
__device__ uint32_t mt_next(uint32_t* st) {
    uint32_t i = st[MT_N];
    if (i >= (uint32_t)MT_N) {
        for (int k = 0; k < MT_N; ++k) {
            const uint32_t y = (st[k] & 0x80000000u) | (st[(k + 1) % MT_N] & 0x7fffffffu);
            st[k] = st[(k + MT_M) % MT_N] ^ (y >> 1) ^ ((y & 1u) ? 0x9908b0dfu : 0u);
        }
        i = 0;
    }
    uint32_t y = st[i];
    st[MT_N] = i + 1;
    y ^= y >> 11;
    y ^= (y << 7) & 0x9d2c5680u;
    y ^= (y << 15) & 0xefc60000u;
    y ^= y >> 18;
    return y;
}

// Order-preserving unsigned key of a float (NaN ranks lowest).
__device__ __forceinline__ uint32_t fkey(float f) {
    const uint32_t u = __float_as_uint(f);
    return f != f ? 0u : ((u & 0x80000000u) ? ~u : (u | 0x80000000u));
}

// In-place bitonic sort of SAMPLE_THREADS (key, payload) pairs in shared memory, ascending by key.
__device__ void bitonic_sort(unsigned long long* key, int* pay) {
    const int t = threadIdx.x;
    for (int size = 2; size <= SAMPLE_THREADS; size <<= 1) {
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
            __syncthreads();
            const int j = t ^ stride;
            if (j > t) {
                const bool up = (t & size) == 0;
                const unsigned long long a = key[t], b = key[j];
                if ((a > b) == up) {
                    key[t] = b;
                    key[j] = a;
                    const int p = pay[t];
                    pay[t] = pay[j];
                    pay[j] = p;
                }
            }
        }
    }
    __syncthreads();
}

// grid 1, block SAMPLE_THREADS. k in [1, min(n, TOPK_MAX)], temp > 0; mt: the generator state.
static __global__ void __launch_bounds__(SAMPLE_THREADS) k_topk_sample(const float* __restrict__ logits, int n,
                                                                       float temp, int k, uint32_t* mt,
                                                                       int32_t* out) {
    __shared__ unsigned int hist[256];
    __shared__ unsigned int s_prefix, s_rem, s_cnt, s_base;
    __shared__ unsigned int wsum[SAMPLE_THREADS / 32];
    __shared__ unsigned long long skey[SAMPLE_THREADS];
    __shared__ int spay[SAMPLE_THREADS];
    __shared__ double sp[SAMPLE_THREADS];
    __shared__ double s_sum;
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    // (1) the k-th largest key by radix selection, 8 bits per pass from the top
    uint32_t prefix = 0u, mask = 0u, rem = (uint32_t)k;
    for (int shift = 24; shift >= 0; shift -= 8) {
        if (tid < 256) hist[tid] = 0u;
        __syncthreads();
        for (int j = tid; j < n; j += SAMPLE_THREADS) {
            const uint32_t key = fkey(logits[j]);
            if ((key & mask) == prefix) atomicAdd(&hist[(key >> shift) & 255u], 1u);
        }
        __syncthreads();
        if (tid == 0) {
            uint32_t cum = 0u;
            for (int b = 255; b >= 0; --b) {
                if (cum + hist[b] >= rem) {
                    s_prefix = prefix | ((uint32_t)b << shift);
                    s_rem = rem - cum;
                    break;
                }
                cum += hist[b];
            }
        }
        __syncthreads();
        prefix = s_prefix;
        rem = s_rem;
        mask |= 255u << shift;
    }
    const uint32_t T = prefix;  // keys above T: k - rem of them; keys equal to T: the first rem
    if (tid == 0) {
        s_cnt = 0u;
        s_base = 0u;
    }
    skey[tid] = ~0ull;  // padding sorts last
    __syncthreads();
    // (2) gather: every key above T, and the keys equal to T in index order until rem are taken
    for (int base = 0; base < n; base += SAMPLE_THREADS) {
        const int j = base + tid;
        const uint32_t key = j < n ? fkey(logits[j]) : 0u;
        const bool gt = j < n && key > T, eq = j < n && key == T;
        if (gt) skey[atomicAdd(&s_cnt, 1u)] = ((unsigned long long)(~key) << 32) | (uint32_t)j;
        const unsigned int b = __ballot_sync(0xffffffffu, eq);
        if (lane == 0) wsum[warp] = __popc(b);
        __syncthreads();
        unsigned int before = s_base, total = 0u;
        for (int w = 0; w < SAMPLE_THREADS / 32; ++w) {
            if (w < warp) before += wsum[w];
            total += wsum[w];
        }
        before += __popc(b & ((1u << lane) - 1u));
        if (eq && before < rem) skey[(uint32_t)k - rem + before] = ((unsigned long long)(~key) << 32) | (uint32_t)j;
        __syncthreads();
        if (tid == 0) s_base += total;
        __syncthreads();
        const bool done = s_base >= rem && s_cnt >= (uint32_t)k - rem;
        __syncthreads();  // every thread has read s_cnt before the next pass adds to it
        if (done) break;  // uniform
    }
    // (3) value order (descending; ties by index), exp of logit/temp in double, their sum in order
    bitonic_sort(skey, spay);
    if (tid < k) {
        const int j = (int)(uint32_t)skey[tid];
        sp[tid] = exp((double)logits[j] / (double)temp);
    }
    __syncthreads();
    if (tid == 0) {
        double s = 0.0;
        for (int t = 0; t < k; ++t) s += sp[t];
        s_sum = s;
    }
    __syncthreads();
    if (tid < k) sp[tid] = sp[tid] / s_sum;  // the probabilities of sampler.cpp:117-118
    // (4) index order (payload: position in value order)
    const unsigned long long ik = tid < k ? (unsigned long long)(uint32_t)skey[tid] : ~0ull;
    __syncthreads();
    skey[tid] = ik;
    spay[tid] = tid;
    bitonic_sort(skey, spay);
    // (5) std::discrete_distribution over the vocabulary, one draw
    if (tid == 0) {
        int ans = 0;
        if (n >= 2) {
            double s2 = 0.0;
            for (int t = 0; t < k; ++t) s2 += sp[spay[t]];
            const uint32_t x0 = mt_next(mt), x1 = mt_next(mt);
            double pr = ((double)x0 + (double)x1 * 4294967296.0) / 18446744073709551616.0;
            if (pr >= 1.0) pr = 1.0 - 1.1102230246251565e-16;  // the largest double below 1
            ans = n - 1;  // the last partial sum is forced to 1
            if (pr <= 0.0) {
                ans = 0;  // lower_bound: cp[0] >= 0
            } else {
                double c = 0.0;
                for (int t = 0; t < k; ++t) {
                    const int j = (int)(uint32_t)skey[t];
                    c = c + sp[spay[t]] / s2;
                    if (j == n - 1) c = 1.0;
                    if (c >= pr) {
                        ans = j;
                        break;
                    }
                }
            }
        }
        out[0] = ans;
    }
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
    if (!(temp > 0.0f)) return fail(GTN_ERR_ARG, "sample_topk: temp must be > 0");
    top_k = top_k < TOPK_MAX ? top_k : TOPK_MAX;  // sampler.cpp:66-67
    temp = temp < 2.0f ? temp : 2.0f;
    if (top_k < 1 || top_k > n) return fail(GTN_ERR_ARG, "sample_topk: top_k %d outside [1, %d]", top_k, n);
    const cudaError_t e = launch_pdl(k_topk_sample, dim3(1), dim3(SAMPLE_THREADS), 0,
                                     static_cast<cudaStream_t>(stream), logits, n, temp, top_k, rng->state,
                                     out_index);
    if (e != cudaSuccess) return fail(GTN_ERR_CUDA, "sample_topk: %s", cudaGetErrorString(e));
    return GTN_OK;
}

}  // extern "C"
