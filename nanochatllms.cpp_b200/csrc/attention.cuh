// Causal attention with GQA, bit-exact with the reference's qkv_attn (ops.cpp:1017-1220).
//
// For query row r (absolute position) and head h, with kv head g = h / (q_heads / kv_heads):
//   s_j = dot(q_r,h , k_j,g) * (1/sqrt(d_head))         j <= r (vec_dot_product, ops.cpp:1049)
//   m   = max_j s_j ; e_j = exp(s_j - m) ; S = sum_j e_j (sequential, j = 0..n-1)
//   P_j = e_j / S, stored in the activation dtype over the full row of n keys (Q8 blocks of 32
//         keys from key 0, partial last block; or fp16) and read back (ops.cpp:1084,1165)
//   o_c = dot_f32(P', V'[:, g*d + c]) with the 8-lane order of vec_dot_product_f32 (ops.cpp:245-289)
//   row r of the output written in the activation dtype (ops.cpp:1175).
// One CTA per (head, query row). K and V rows are staged in shared-memory tiles with word copies;
// keys are scored one per thread (Q8 through dp4a lane words); the softmax denominator is the
// reference's sequential fp32 sum (one thread); the probabilities are quantized per 32-key block
// by warps; P.V runs one thread per (channel, lane pair) with the two lane chains interleaved.
#pragma once
#include "common.cuh"
#include "matmul.cuh"
#include "rowops.cuh"

namespace gtn {

constexpr int ATT_THREADS = 256;

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
                const float p = lane_sum_f32(L) * s;
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

// ---- shared pieces of the prefill/op-level kernel (k_attn) and the fused decode kernel ----------
// Shared-memory row stride of a head row staged by word copies: 4-byte multiple, odd in words (a
// thread per key reading the same offset of consecutive rows hits distinct banks).
__host__ __device__ inline int att_rs(long hb) {
    int rs = (int)((hb + 3) & ~3L);
    if (((rs >> 2) & 1) == 0) rs += 4;
    return rs;
}
// Row stride of the engine's head-major KV cache: the head row padded to 16 bytes, odd in 16-byte
// units (16-byte loads of consecutive rows by 8 threads hit distinct bank groups).
__host__ __device__ inline int att_kv_rs(long hb) {
    int r = (int)((hb + 15) & ~15L);
    if (((r >> 4) & 1) == 0) r += 16;
    return r;
}
// Largest staged row stride: word-copied rows (att_rs) or bulk-copied cache rows (att_kv_rs).
__host__ __device__ inline int att_rs_max(long hb) {
    const int a = att_rs(hb), b = att_kv_rs(hb);
    return a > b ? a : b;
}
// Keys per K / V tile: 512 for rows up to 100 bytes (Q8 heads), else 256.
__host__ __device__ inline int att_tile(long hb) { return att_rs_max(hb) <= 100 ? 512 : 256; }

// Shared memory of k_attn / k_fattn: [probabilities n floats][K tile][V tile][8 x d lane
// partials][q lane words].
struct AttSmem {
    float* p;
    uint8_t* kt;
    uint8_t* vt;
    float* part;
    LanePrep* qp;
    uint64_t* bars;  // [2] mbarriers (K tile, V tile), static shared memory of the kernel
    int* abort;      // set when a bounded wait expired
};
__device__ __forceinline__ AttSmem att_layout(uint8_t* sm, int n, long hb, int d, uint64_t* bars, int* abort) {
    AttSmem a;
    const size_t tb = (size_t)att_tile(hb) * att_rs_max(hb);
    a.p = reinterpret_cast<float*>(sm);
    a.kt = sm + ((n * 4 + 15) / 16) * 16;
    a.vt = a.kt + tb;
    a.part = reinterpret_cast<float*>(a.vt + tb);
    a.qp = reinterpret_cast<LanePrep*>(a.part + 8 * d);
    a.bars = bars;
    a.abort = abort;
    return a;
}
inline size_t attn_smem(int n, int dt, int d) {
    const long hb = row_bytes(dt, d);
    return (size_t)((n * 4 + 15) / 16) * 16 + (size_t)2 * att_tile(hb) * att_rs_max(hb) + (size_t)8 * d * 4 +
           (size_t)(d / GTN_QBLK) * 4 * sizeof(LanePrep) + 16;
}
// Thread 0 initializes the two tile barriers; the caller synchronizes the CTA afterwards.
__device__ __forceinline__ void att_init_bars(uint64_t* bars, int* abort) {
    if (threadIdx.x == 0) {
        mbar_init(&bars[0], 1);
        mbar_init(&bars[1], 1);
        fence_mbar_init();
        *abort = 0;
    }
}

// A cache whose head rows are 16-byte aligned with a 16-byte-multiple stride (the engine's
// head-major layout) is staged by one TMA bulk copy per tile; other layouts (the reference's
// [ctx][kv_dim] rows, 4-byte aligned) by 4-byte cp.async copies.
__device__ __forceinline__ bool att_bulk(const uint8_t* base, long stride, int hb) {
    return (reinterpret_cast<uintptr_t>(base) & 15) == 0 && stride == att_kv_rs(hb);
}

// Starts copying rows [j0, j0 + nt) of a strided cache (row j at base + j * stride, hb bytes) into
// shared rows of rs bytes. Bulk: thread 0 arms `bar` and issues one copy (rs == stride). Otherwise
// one cp.async group of 4-byte copies (all in flight at once), or synchronous byte copies for rows
// that are not word aligned. Row `jp` is replaced by `special` when the tile lands (att_land).
__device__ __forceinline__ void att_fetch(uint8_t* dst, int rs, const uint8_t* base, long stride, int j0, int nt,
                                          int hb, bool bulk, uint64_t* bar) {
    if (bulk) {
        if (threadIdx.x == 0 && nt > 0) {
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // earlier generic reads of dst
            mbar_arrive_expect_tx(bar, (uint32_t)(nt * stride));
            bulk_g2s(dst, base + (long)j0 * stride, (uint32_t)(nt * stride), bar);
        }
        return;
    }
    if ((hb & 3) == 0 && (stride & 3) == 0 && (reinterpret_cast<uintptr_t>(base) & 3) == 0) {
        const int wpr = hb >> 2;
        const int step_j = blockDim.x / wpr, step_w = blockDim.x - step_j * wpr;
        int jj = threadIdx.x / wpr, w = threadIdx.x - jj * wpr;
        while (jj < nt) {
            const uint32_t* src = reinterpret_cast<const uint32_t*>(base + (long)(j0 + jj) * stride) + w;
            uint32_t* d = reinterpret_cast<uint32_t*>(dst + (long)jj * rs) + w;
            asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(d)), "l"(src) : "memory");
            jj += step_j;
            w += step_w;
            if (w >= wpr) {
                w -= wpr;
                ++jj;
            }
        }
    } else {
        for (int i = threadIdx.x; i < nt * hb; i += blockDim.x) {
            const int jj = i / hb, bb = i - jj * hb;
            dst[(long)jj * rs + bb] = base[(long)(j0 + jj) * stride + bb];
        }
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
}
template <int N>
__device__ __forceinline__ void att_wait_group() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
// Completes a fetch: the bulk barrier's phase `par` (bounded; on expiry *abort is set and the
// error word flagged), or the cp.async groups down to one pending (keep_one: the other tile's
// group, committed later) or none; then overwrites row jp - j0 with `special` if it lies in the
// tile, and synchronizes the CTA.
__device__ __forceinline__ void att_land(uint8_t* dst, int rs, int j0, int nt, int hb, int jp, const uint8_t* special,
                                         bool bulk, bool keep_one, uint64_t* bar, uint32_t par, int* abort,
                                         unsigned int* err) {
    if (bulk) {
        if (nt > 0 && !*abort && !mbar_wait_bounded(bar, par, err)) *abort = 1;
    } else if (keep_one) {
        att_wait_group<1>();
    } else {
        att_wait_group<0>();
    }
    __syncthreads();
    if (jp >= j0 && jp < j0 + nt)
        for (int i = threadIdx.x; i < hb; i += blockDim.x) dst[(long)(jp - j0) * rs + i] = special[i];
    __syncthreads();
}

// Score dot of a staged key row with the query: Q8 through the lane words in qp (the order of
// head_dot / vec_dot_product_q8), fp16 through head_dot.
__device__ __forceinline__ float att_dot(const uint8_t* kr, const uint8_t* qraw, const LanePrep* qp, int dt, int d) {
    if (dt == GTN_Q8) {
        float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
        for (int b = 0; b < d / GTN_QBLK; ++b) {
            const uint8_t* kb = kr + b * GTN_Q8_BYTES;
            const float s = qp[b * 4].da * h2f(ld_u16(kb));
#pragma unroll
            for (int l = 0; l < 4; ++l) {
                const float pr = lane_sum_f32(q8_block_lane_dot(kb, l, qp[b * 4 + l])) * s;
                acc[l] = acc[l] + pr;
            }
        }
        return (acc[0] + acc[1]) + (acc[2] + acc[3]);
    }
    return head_dot(qraw, kr, dt, d);
}

// The same dot for a Q8 key row of two blocks (d = 64) at a 16-byte aligned shared address: five
// 16-byte loads (conflict-free across 8 consecutive rows of 80 bytes) and lane words extracted in
// registers.
__device__ __forceinline__ float att_dot_q8x2(const uint8_t* kr, const LanePrep* qp) {
    uint32_t w[20];
#pragma unroll
    for (int i = 0; i < 5; ++i) {
        const uint4 t = reinterpret_cast<const uint4*>(kr)[i];
        w[4 * i] = t.x;
        w[4 * i + 1] = t.y;
        w[4 * i + 2] = t.z;
        w[4 * i + 3] = t.w;
    }
    float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
    for (int b = 0; b < 2; ++b) {
        const int ob = b * GTN_Q8_BYTES;
        const float s = qp[b * 4].da * h2f((uint16_t)gv3_u16(w, ob));
#pragma unroll
        for (int l = 0; l < 4; ++l) {
            const int w0 = gv3_pair(w, ob + 2 + 2 * l, ob + 10 + 2 * l);
            const int w1 = gv3_pair(w, ob + 18 + 2 * l, ob + 26 + 2 * l);
            const LanePrep& a = qp[b * 4 + l];
            const float pr = lane_sum_f32(dp4a(w0, a.a0, dp4a(w1, a.a1, 0))) * s;
            acc[l] = acc[l] + pr;
        }
    }
    return (acc[0] + acc[1]) + (acc[2] + acc[3]);
}

// The fp16 dot (head_dot order: 8 lanes, separate mul / add roundings, lanes left to right) for
// d = 64 rows at a 16-byte aligned shared address: eight 16-byte loads of the key row; the query
// row is read from shared memory (broadcast).
__device__ __forceinline__ float att_dot_f16x64(const uint8_t* kr, const uint8_t* qraw) {
    const uint16_t* x = reinterpret_cast<const uint16_t*>(qraw);
    float acc[8];
#pragma unroll
    for (int l = 0; l < 8; ++l) acc[l] = 0.0f;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const uint4 t = reinterpret_cast<const uint4*>(kr)[i];
        const uint32_t w[4] = {t.x, t.y, t.z, t.w};
#pragma unroll
        for (int l = 0; l < 8; ++l) {
            const float kv = h2f((uint16_t)(w[l >> 1] >> ((l & 1) * 16)));
            const float p = h2f(x[8 * i + l]) * kv;
            acc[l] = p + acc[l];
        }
    }
    float r = acc[0] + acc[1];
#pragma unroll
    for (int l = 2; l < 8; ++l) r = r + acc[l];
    return r;
}

// P.V lane chains over a staged V tile (keys t0 + jj, jj < nt, rows of rs bytes): the chains of
// lanes l0 and l0 + 1 (keys = lane mod 8, keys < n8 only) for channel c, in key order. t0 is a
// multiple of 8.
__device__ __forceinline__ void att_pv_tile(const uint8_t* vt, int rs, int t0, int nt, int n8, const float* p, int dt,
                                            int c, int l0, float& accA, float& accB) {
    const int lim = min(nt, n8 - t0);
    int jj = l0;
    for (; jj + 25 < lim; jj += 32) {
        float va[4], vb[4], pa[4], pb[4];
#pragma unroll
        for (int s = 0; s < 4; ++s) {
            va[s] = load_elem(vt + (long)(jj + 8 * s) * rs, dt, c);
            vb[s] = load_elem(vt + (long)(jj + 8 * s + 1) * rs, dt, c);
            pa[s] = p[t0 + jj + 8 * s];
            pb[s] = p[t0 + jj + 8 * s + 1];
        }
#pragma unroll
        for (int s = 0; s < 4; ++s) {
            const float xa = pa[s] * va[s];
            accA = xa + accA;
            const float xb = pb[s] * vb[s];
            accB = xb + accB;
        }
    }
    for (; jj < lim; jj += 8) {
        const float xa = p[t0 + jj] * load_elem(vt + (long)jj * rs, dt, c);
        accA = xa + accA;
        if (jj + 1 < lim) {
            const float xb = p[t0 + jj + 1] * load_elem(vt + (long)(jj + 1) * rs, dt, c);
            accB = xb + accB;
        }
    }
}

// Softmax of p[0..n) (scores, -inf where masked; keys > last contribute exp = 0 and are not
// summed), the probabilities requantized in dtype dt per 32-key block and written back to p.
// `red` holds ATT_THREADS / 32 floats, `stat` 2.
__device__ __forceinline__ void att_softmax(float* p, int n, int last, float mx, int dt, float* red, float* stat) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    // the maximum as an order-preserving unsigned key (NaN ranks lowest, as a '>' scan skips it):
    // one warp max-reduction, then every thread combines the warps' keys
    const unsigned int ub = __float_as_uint(mx);
    unsigned int key = mx != mx ? 0u : ((ub & 0x80000000u) ? ~ub : (ub | 0x80000000u));
    key = __reduce_max_sync(0xffffffffu, key);
    unsigned int* redk = reinterpret_cast<unsigned int*>(red);
    if (lane == 0) redk[warp] = key;
    __syncthreads();
    unsigned int mk = 0u;
#pragma unroll
    for (int w = 0; w < ATT_THREADS / 32; ++w) mk = max(mk, redk[w]);
    const float m = __uint_as_float((mk & 0x80000000u) ? (mk ^ 0x80000000u) : ~mk);
    for (int j = tid; j < n; j += ATT_THREADS) p[j] = j <= last ? expf_ref(p[j] - m) : 0.0f;
    __syncthreads();
    if (tid == 0) stat[1] = serial_sum_smem(p, last + 1);  // keys > last add +0.0f
    __syncthreads();
    const float sum = stat[1];
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
}

// Keys whose probability can be non-zero: 0..last (keys above are masked, p = 0). The reference's
// P.V runs its 8 lane chains over keys < n8 = 8 * floor(n / 8) and a scalar tail over n8..n-1 of
// every key, masked ones included; a masked key adds 0 * v = +-0 to a chain or to the tail, which
// leaves an accumulator that started at +0 unchanged (round to nearest never makes it -0), so the
// chains stop at key min(n8, last + 1) and the tail at key last (identical unless V holds inf or
// NaN above the causal limit, where the reference's 0 * inf gives NaN).
// Rows of the V tile starting at key t0: T keys, or up to key e8 = min(n8, last + 1) where the
// chains stop; the tile that holds key e8 - 1 (tile 0 when e8 = 0) also takes the tail keys
// n8..last when they fit, so that att_out reads them from shared memory.
__device__ __forceinline__ int att_vtile_rows(int t0, int nk, int e8, int T) {
    return (e8 - t0 <= T && nk - t0 <= T) ? nk - t0 : min(T, e8 - t0);
}

// Scores (keys [0, last] of the cache, -inf above), softmax, and the P.V lane chains, leaving the 8
// lane partial sums in sm.part[l * d + c] (keys < n8). Key `jp` is read from kspecial / vspecial
// (shared memory) instead of the cache. The first V tile is copied while the scores are computed.
// Returns after a CTA barrier with no copy in flight; the last V tile stays in sm.vt (its first key
// in *vt0, its rows in *vnt) for att_out.
__device__ __forceinline__ void att_core(const uint8_t* k, long ks, const uint8_t* v, long vs, int hb, int n, int last,
                                         int jp, const uint8_t* kspecial, const uint8_t* vspecial,
                                         const uint8_t* qraw, const AttSmem& sm, int dt, int d, float* red,
                                         float* stat, unsigned int* err, int* vt0, int* vnt,
                                         bool prefetched = false) {
    const int tid = threadIdx.x;
    const int T = att_tile(hb);
    const bool kb = att_bulk(k, ks, hb), vb = att_bulk(v, vs, hb);
    const int krs = kb ? (int)ks : att_rs(hb), vrs = vb ? (int)vs : att_rs(hb);
    const bool kreg = d == 2 * GTN_QBLK && (krs & 15) == 0;  // 16-byte row loads (Q8 or fp16)
    const float scale = 1.0f / sqrtf((float)d);
    const int n8 = (n / 8) * 8, nk = min(n, last + 1), e8 = min(n8, nk);
    uint32_t kpar = 0, vpar = 0;
    float mx = -INFINITY;
    if (!prefetched) {  // else the caller issued exactly these two fetches (att_prefetch)
        att_fetch(sm.kt, krs, k, ks, 0, max(0, min(min(T, n), last + 1)), hb, kb, &sm.bars[0]);
        att_fetch(sm.vt, vrs, v, vs, 0, att_vtile_rows(0, nk, e8, T), hb, vb, &sm.bars[1]);
    }
    for (int t0 = 0; t0 < n; t0 += T) {
        const int nt = min(T, n - t0);
        const int nv = max(0, min(nt, last + 1 - t0));
        if (t0 > 0) {
            att_fetch(sm.kt, krs, k, ks, t0, nv, hb, kb, &sm.bars[0]);
            att_land(sm.kt, krs, t0, nv, hb, jp, kspecial, kb, false, &sm.bars[0], kpar, sm.abort, err);
        } else {  // V tile 0 may still be in flight (its cp.async group was committed after K's)
            att_land(sm.kt, krs, t0, nv, hb, jp, kspecial, kb, !vb, &sm.bars[0], kpar, sm.abort, err);
        }
        if (nv > 0) kpar ^= 1u;
        for (int jj = tid; jj < nt; jj += ATT_THREADS) {
            float sc = -INFINITY;
            if (jj < nv) {
                const uint8_t* kr = sm.kt + (long)jj * krs;
                const float dd = !kreg ? att_dot(kr, qraw, sm.qp, dt, d)
                                       : (dt == GTN_Q8 ? att_dot_q8x2(kr, sm.qp) : att_dot_f16x64(kr, qraw));
                sc = dd * scale;
            }
            sm.p[t0 + jj] = sc;
            mx = fmaxf(mx, sc);
        }
        __syncthreads();
    }
    att_softmax(sm.p, n, last, mx, dt, red, stat);
    const int units = d * 4;  // (channel, lane pair)
    float acc[2][2] = {{0.0f, 0.0f}, {0.0f, 0.0f}};  // d <= 128: at most 2 units per thread
    *vt0 = 0;
    *vnt = 0;
    for (int t0 = 0; t0 == 0 || t0 < e8; t0 += T) {
        const int nt = att_vtile_rows(t0, nk, e8, T);
        if (t0 > 0) att_fetch(sm.vt, vrs, v, vs, t0, nt, hb, vb, &sm.bars[1]);
        att_land(sm.vt, vrs, t0, nt, hb, jp, vspecial, vb, false, &sm.bars[1], vpar, sm.abort, err);
        if (nt > 0) vpar ^= 1u;
        *vt0 = t0;
        *vnt = nt;
#pragma unroll
        for (int u = 0; u < 2; ++u) {
            const int un = tid + u * ATT_THREADS;
            if (un < units) att_pv_tile(sm.vt, vrs, t0, nt, e8, sm.p, dt, un >> 2, 2 * (un & 3), acc[u][0], acc[u][1]);
        }
        __syncthreads();
    }
    att_wait_group<0>();
#pragma unroll
    for (int u = 0; u < 2; ++u) {
        const int un = tid + u * ATT_THREADS;
        if (un < units) {
            const int c = un >> 2, l0 = 2 * (un & 3);
            sm.part[l0 * d + c] = acc[u][0];
            sm.part[(l0 + 1) * d + c] = acc[u][1];
        }
    }
    if (*sm.abort && tid == 0) {
        // a bounded wait expired: wait (bounded again) for the copies that may still be in flight
        for (uint32_t i = 0; i < GTN_WAIT_LIMIT; ++i)
            if (mbar_try_wait(&sm.bars[0], kpar ^ 1u)) break;
        for (uint32_t i = 0; i < GTN_WAIT_LIMIT; ++i)
            if (mbar_try_wait(&sm.bars[1], vpar ^ 1u)) break;
    }
    __syncthreads();
}

// The first K and V tile fetches of att_core, issued early (e.g. before a kernel waits for the
// previous one: the cache rows below the new key do not depend on it).
__device__ __forceinline__ void att_prefetch(const uint8_t* k, long ks, const uint8_t* v, long vs, int hb, int n,
                                             int last, const AttSmem& sm) {
    const int T = att_tile(hb), n8 = (n / 8) * 8, nk = min(n, last + 1), e8 = min(n8, nk);
    const bool kb = att_bulk(k, ks, hb), vb = att_bulk(v, vs, hb);
    att_fetch(sm.kt, kb ? (int)ks : att_rs(hb), k, ks, 0, max(0, min(min(T, n), last + 1)), hb, kb, &sm.bars[0]);
    att_fetch(sm.vt, vb ? (int)vs : att_rs(hb), v, vs, 0, att_vtile_rows(0, nk, e8, T), hb, vb, &sm.bars[1]);
}

// Output row of one head: the lane partials summed left to right, then the tail keys n8..n-1
// (vec_f32x8_sum + the scalar loop of vec_dot_product_f32), written in dtype dt. Tail keys held by
// the last V tile (keys vt0 .. vt0 + vnt - 1 at vt, rows of vrs bytes) are read from it.
__device__ __forceinline__ void att_out(const float* part, const float* p, const uint8_t* v, long vs, int n, int last,
                                        int jp, const uint8_t* vspecial, int dt, int d, uint8_t* dst,
                                        const uint8_t* vt, int vrs, int vt0, int vnt) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int n8 = (n / 8) * 8;
    for (int blk = warp; blk * GTN_QBLK < d; blk += ATT_THREADS / 32) {
        const int c = blk * GTN_QBLK + lane;
        float y = 0.0f;
        if (c < d) {
            y = part[c] + part[d + c];
            for (int l = 2; l < 8; ++l) y = y + part[l * d + c];
            for (int j = n8; j < n && j <= last; ++j) {  // masked tail keys add +-0
                const uint8_t* vr = j - vt0 < vnt ? vt + (long)(j - vt0) * vrs : (j == jp ? vspecial : v + (long)j * vs);
                const float pr = p[j] * load_elem(vr, dt, c);
                y = y + pr;
            }
        }
        store_row_elem(dst, dt, blk, lane, d, y);
    }
}

// q: rows of q_dim elements (row stride qs bytes, indexed by absolute position); k, v: cache rows
// (row j of kv head g at k + g * khs + j * ks, likewise v), rows 0..n-1 valid; out rows stride os
// (absolute positions). Rows r in [row0, row0 + gridDim.y) are computed; row r attends keys
// [0, r] and its probability row has n entries (keys > r are masked to 0). d <= 128, a multiple
// of 32 for Q8. dynamic smem: attn_smem(n, dt, d).
static __global__ void __launch_bounds__(ATT_THREADS) k_attn(const uint8_t* q, long qs, const uint8_t* k, long ks,
                                                             long khs, const uint8_t* v, long vs, long vhs,
                                                             uint8_t* out, long os, int dt, int n, int row0,
                                                             int q_heads, int kv_heads, int d, unsigned int* err) {
    asm volatile("griddepcontrol.wait;" ::: "memory");
    extern __shared__ __align__(16) uint8_t sm[];
    __shared__ float red[ATT_THREADS / 32];
    __shared__ float s_stat[2];
    __shared__ __align__(8) uint64_t bars[2];
    __shared__ int abort_flag;
    const long hb = row_bytes(dt, d);
    const AttSmem L = att_layout(sm, n, hb, d, bars, &abort_flag);
    const int h = blockIdx.x, r = row0 + blockIdx.y;
    const int g = h / (q_heads / kv_heads);
    const uint8_t* qh = q + (long)r * qs + (long)h * hb;
    att_init_bars(bars, &abort_flag);
    if (dt == GTN_Q8) build_prep_q8(qh, 0, 0, 1, d / GTN_QBLK, L.qp);
    __syncthreads();
    int vt0, vnt;
    att_core(k + (long)g * khs, ks, v + (long)g * vhs, vs, (int)hb, n, r, -1, nullptr, nullptr, qh, L, dt, d, red,
             s_stat, err, &vt0, &vnt);
    const int vrs = att_bulk(v + (long)g * vhs, vs, (int)hb) ? (int)vs : att_rs(hb);
    att_out(L.part, L.p, v + (long)g * vhs, vs, n, r, -1, nullptr, dt, d, out + (long)r * os + (long)h * hb, L.vt,
            vrs, vt0, vnt);
}

}  // namespace gtn
