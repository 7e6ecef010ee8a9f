// Causal attention with GQA, bit-exact with the reference's qkv_attn (ops.cpp:1017-1220).
//
// For query row r (absolute position) and head h, with kv head g = h / (q_heads / kv_heads):
//   s_j = dot(q_r,h , k_j,g) * (1/sqrt(d_head))         j <= r (vec_dot_product, ops.cpp:1049)
//   m   = max_j s_j ; e_j = exp(s_j - m) ; S = sum_j e_j (sequential, j = 0..n-1)
//   P_j = e_j / S, stored in the activation dtype over the full row of n keys (Q8 blocks of 32
//         keys from key 0, partial last block; or fp16) and read back (ops.cpp:1084,1165)
//   o_c = dot_f32(P', V'[:, g*d + c]) with the 8-lane order of vec_dot_product_f32 (ops.cpp:245-289)
//   row r of the output written in the activation dtype (ops.cpp:1175).
// One CTA per (head, query row). Keys are scored in parallel; the softmax denominator is the
// reference's sequential fp32 sum (one thread); the probabilities are quantized per 32-key block
// by warps; P.V runs one thread per (channel, lane) over V tiles staged in shared memory.
#pragma once
#include "common.cuh"
#include "rowops.cuh"

namespace gtn {

constexpr int ATT_THREADS = 256;
constexpr int ATT_VTILE = 128;  // keys per V tile in shared memory

// Exact dot of two d-element head vectors in dtype dt (Q8: blocks of 32, 4 lanes; F16: 8 lanes).
__device__ __forceinline__ float head_dot(const uint8_t* q, const uint8_t* k, int dt, int d) {
    if (dt == GTN_Q8) {
        float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
        for (int b = 0; b < d / GTN_QBLK; ++b) {
            const uint8_t* qa = q + b * GTN_Q8_BYTES;
            const uint8_t* kb = k + b * GTN_Q8_BYTES;
            const float s = h2f(ld_u16(qa)) * h2f(ld_u16(kb));
            const int8_t* x = reinterpret_cast<const int8_t*>(qa + 2);
            const int8_t* y = reinterpret_cast<const int8_t*>(kb + 2);
#pragma unroll
            for (int l = 0; l < 4; ++l) {
                int L = 0;
#pragma unroll
                for (int c = 0; c < GTN_QBLK; c += 8)
                    L += (int)x[c + 2 * l] * y[c + 2 * l] + (int)x[c + 2 * l + 1] * y[c + 2 * l + 1];
                const float p = (float)L * s;
                acc[l] = acc[l] + p;
            }
        }
        return (acc[0] + acc[1]) + (acc[2] + acc[3]);
    } else {
        const uint16_t* x = reinterpret_cast<const uint16_t*>(q);
        const uint16_t* y = reinterpret_cast<const uint16_t*>(k);
        float acc[8];
#pragma unroll
        for (int l = 0; l < 8; ++l) acc[l] = 0.0f;
        for (int i = 0; i < (d / 8) * 8; i += 8) {
#pragma unroll
            for (int l = 0; l < 8; ++l) {
                const float p = h2f(x[i + l]) * h2f(y[i + l]);
                acc[l] = p + acc[l];
            }
        }
        float r = acc[0] + acc[1];
        for (int l = 2; l < 8; ++l) r = r + acc[l];
        for (int i = (d / 8) * 8; i < d; ++i) {
            const float p = h2f(x[i]) * h2f(y[i]);
            r = r + p;
        }
        return r;
    }
}

// q: rows of q_dim elements (row stride qs bytes, indexed by absolute position); k, v: cache rows
// of kv_dim (strides ks, vs bytes), rows 0..n-1 valid; out rows stride os (absolute positions).
// Rows r in [row0, row0 + gridDim.y) are computed; row r attends keys [0, r] and its probability
// row has n entries (keys > r are masked to 0). d <= 256.
// dynamic smem: attn_smem(n, dt, d).
static __global__ void __launch_bounds__(ATT_THREADS) k_attn(const uint8_t* q, long qs, const uint8_t* k, long ks,
                                                             const uint8_t* v, long vs, uint8_t* out, long os,
                                                             int dt, int n, int row0, int q_heads, int kv_heads,
                                                             int d) {
    asm volatile("griddepcontrol.wait;" ::: "memory");
    extern __shared__ __align__(16) uint8_t sm[];
    float* p = reinterpret_cast<float*>(sm);
    const long hb = row_bytes(dt, d);
    uint8_t* vt = sm + ((n * 4 + 15) / 16) * 16;
    float* part = reinterpret_cast<float*>(vt + (long)ATT_VTILE * hb);  // [8 lanes][d] partial sums
    __shared__ float red[ATT_THREADS / 32];
    __shared__ float s_stat[2];

    const int h = blockIdx.x, r = row0 + blockIdx.y;
    const int g = h / (q_heads / kv_heads);
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const float scale = 1.0f / sqrtf((float)d);
    const uint8_t* qh = q + (long)r * qs + (long)h * hb;

    // scores, keys 0..r; masked keys hold -inf (their exp is 0)
    float mx = -INFINITY;
    for (int j = tid; j < n; j += ATT_THREADS) {
        float sc = -INFINITY;
        if (j <= r) {
            const float dd = head_dot(qh, k + (long)j * ks + (long)g * hb, dt, d);
            sc = dd * scale;
        }
        p[j] = sc;
        mx = fmaxf(mx, sc);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if (lane == 0) red[warp] = mx;
    __syncthreads();
    if (tid == 0) {
        float m = red[0];
        for (int w = 1; w < ATT_THREADS / 32; ++w) m = fmaxf(m, red[w]);
        s_stat[0] = m;
    }
    __syncthreads();
    const float m = s_stat[0];
    for (int j = tid; j < n; j += ATT_THREADS) p[j] = j <= r ? exp_cr(p[j] - m) : 0.0f;
    __syncthreads();
    if (tid == 0) {
        float sum = 0.0f;
        for (int j = 0; j <= r; ++j) sum = sum + p[j];  // keys > r add +0.0f
        s_stat[1] = sum;
    }
    __syncthreads();
    const float sum = s_stat[1];
    // probabilities, stored and reloaded in the activation dtype
    for (int blk = warp; blk * GTN_QBLK < n; blk += ATT_THREADS / 32) {
        const int j = blk * GTN_QBLK + lane;
        const float pj = j < n ? p[j] / sum : 0.0f;
        float back;
        if (dt == GTN_Q8) {
            uint16_t dh;
            const int8_t qv = warp_quant_block(pj, lane, min(GTN_QBLK, n - blk * GTN_QBLK), &dh);
            back = (float)qv * h2f(dh);
        } else {
            back = h2f(f2h(pj));
        }
        __syncwarp();
        if (j < n) p[j] = back;
    }
    __syncthreads();

    // P.V: thread (c, l) for channel c < d and lane l < 8 accumulates keys 8i + l < n8 in order.
    const int n8 = (n / 8) * 8;
    const int npairs = d * 8;
    float acc[8];  // up to 8 (c, l) pairs per thread when d <= 256
    const int per = (npairs + ATT_THREADS - 1) / ATT_THREADS;
    for (int u = 0; u < 8; ++u) acc[u] = 0.0f;
    for (int t0 = 0; t0 < n; t0 += ATT_VTILE) {
        const int nt = min(ATT_VTILE, n - t0);
        const uint8_t* vsrc = v + (long)t0 * vs + (long)g * hb;
        for (int i = tid; i < nt * hb; i += ATT_THREADS) {
            const int jj = i / hb, bb = i % hb;
            vt[i] = vsrc[(long)jj * vs + bb];
        }
        __syncthreads();
        for (int u = 0; u < per; ++u) {
            const int pi = tid + u * ATT_THREADS;
            if (pi < npairs) {
                const int c = pi >> 3, l = pi & 7;
                float a = acc[u];
                // keys j = t0 + jj with j % 8 == l (t0 is a multiple of 8) and j < n8
                for (int jj = l; jj < nt && t0 + jj < n8; jj += 8) {
                    const float vv = load_elem(vt + (long)jj * hb, dt, c);
                    const float pr = p[t0 + jj] * vv;
                    a = pr + a;
                }
                acc[u] = a;
            }
        }
        __syncthreads();
    }
    for (int u = 0; u < per; ++u) {
        const int pi = tid + u * ATT_THREADS;
        if (pi < npairs) part[(pi & 7) * d + (pi >> 3)] = acc[u];
    }
    __syncthreads();
    // lanes left to right, then the tail keys n8..n-1 (vec_f32x8_sum + scalar loop)
    uint8_t* dst = out + (long)r * os + (long)h * hb;
    for (int blk = warp; blk * GTN_QBLK < d; blk += ATT_THREADS / 32) {
        const int c = blk * GTN_QBLK + lane;
        float y = 0.0f;
        if (c < d) {
            y = part[c] + part[d + c];
            for (int l = 2; l < 8; ++l) y = y + part[l * d + c];
            for (int j = n8; j < n; ++j) {
                const float vv = load_elem(v + (long)j * vs + (long)g * hb, dt, c);
                const float pr = p[j] * vv;
                y = y + pr;
            }
        }
        store_row_elem(dst, dt, blk, lane, d, y);
    }
}

inline size_t attn_smem(int n, int dt, int d) {
    return (size_t)((n * 4 + 15) / 16) * 16 + (size_t)ATT_VTILE * row_bytes(dt, d) + (size_t)8 * d * 4 + 16;
}

}  // namespace gtn
