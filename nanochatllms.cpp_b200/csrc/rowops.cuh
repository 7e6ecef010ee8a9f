// Row-wise kernels of the gten ops API: elementwise ops, norms, RoPE, token embedding, the weight
// packer, the activation quantizer and the greedy argmax. Each reproduces the reference function
// it names bit for bit (see common.cuh for the numerics contract).
//
// Layout convention: a "row" is one tensor row in its dtype (Q8: ceil(n/32) 34-byte blocks;
// F16: n halves; F32: n floats). Writes in Q8 go through warp_store_q8_block, one warp per block,
// which is write_row_from_float / q8_quantize_row (ops.cpp:87-123, quants.cpp:140-158).
#pragma once
#include "common.cuh"
#include "seqsum.cuh"

namespace gtn {

// Stores the value `y` of element i = blk*32 + lane of a row in dtype dt.
__device__ __forceinline__ void store_row_elem(uint8_t* row, int dt, int blk, int lane, int n, float y) {
    const int i = blk * GTN_QBLK + lane;
    switch (dt) {
        case GTN_Q8: warp_store_q8_block(y, lane, min(GTN_QBLK, n - blk * GTN_QBLK), row + (long)blk * GTN_Q8_BYTES); break;
        case GTN_F16:
            if (i < n) reinterpret_cast<uint16_t*>(row)[i] = f2h(y);
            break;
        default:
            if (i < n) reinterpret_cast<float*>(row)[i] = y;
    }
}

enum { ROP_SILU = 0, ROP_MUL = 1, ROP_ADD = 2, ROP_SCALE = 3, ROP_BIAS = 4 };

// grid: (ceil(nblocks / 4), rows); block 128 (one warp per 32-element block).
//   silu  ops.cpp:750-753  x / (1 + exp(-x))
//   mul   ops.cpp:918-922  a * b
//   add   ops.cpp:166-205  a + b
//   scale ops.cpp:125-144  x * s
//   bias  ops.cpp:656-664  x + fp16(bias)
template <int OP>
static __global__ void k_rowop(const uint8_t* a, long as, const uint8_t* b, long bs, uint8_t* out, long os, int dt,
                               int n, int row0, float s, const uint16_t* bias) {
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const int row = row0 + blockIdx.y;
    const int blk = blockIdx.x * 4 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (blk * GTN_QBLK >= n) return;
    const int i = blk * GTN_QBLK + lane;
    const bool valid = i < n;
    const float x = valid ? load_elem(a + (long)row * as, dt, i) : 0.0f;
    float y;
    if (OP == ROP_SILU) {
        const float den = 1.0f + expf_ref(-x);
        y = x / den;
    } else if (OP == ROP_MUL) {
        y = x * (valid ? load_elem(b + (long)row * bs, dt, i) : 0.0f);
    } else if (OP == ROP_ADD) {
        y = x + (valid ? load_elem(b + (long)row * bs, dt, i) : 0.0f);
    } else if (OP == ROP_SCALE) {
        y = x * s;
    } else {
        y = x + (valid ? h2f(bias[i]) : 0.0f);
    }
    if (!valid) y = 0.0f;
    store_row_elem(out + (long)row * os, dt, blk, lane, n, y);
}

// RMSNorm / LayerNorm over one vector of n elements per CTA (2-D rows, or the heads of a 3-D
// [rows, heads, d] tensor for OpenELM's QK-norm). The sums are sequential fp32 sums in element
// order, as the reference computes them (one thread), the rest is element-parallel.
//   rms_norm_vec_f32 ops.cpp:830-846: x / (sqrt(sum(x^2)/n) + 1e-6) * w
//   vec_layer_norm_f32 ops.cpp:669-698: ((x - mean) / (sqrt(sum((x-mean)^2)/n) + 1e-5)) * w + b
// grid: (heads, rows); block 64 for the head norms (n = 64), 256 (512 for n > 1024) otherwise, and
// all threads reach the exact parallel sum (n > 256); dynamic smem 2n floats (values + the exact
// sum's scratch).
template <bool LAYER>
static __global__ void k_norm(const uint8_t* x, long xs, long hs, uint8_t* out, long os, long ohs, int dt, int n,
                              int row0, const uint16_t* w, const uint16_t* bvec) {
    asm volatile("griddepcontrol.wait;" ::: "memory");
    extern __shared__ float v[];
    __shared__ float stat[2];
    const int row = row0 + blockIdx.y, h = blockIdx.x;
    const uint8_t* src = x + (long)row * xs + (long)h * hs;
    for (int i = threadIdx.x; i < n; i += blockDim.x) v[i] = load_elem(src, dt, i);
    __syncthreads();
    if (!LAYER && n > 256) {
        // the sequential sum of squares, computed exactly in parallel (seqsum.cuh); short rows
        // (OpenELM's 64-wide head norms) take the serial loop below, which is faster there
        // the fewest terms per thread in registers that hold the row: the unrolled per-term work
        // is that much shorter (the decode step's cluster norm runs the 4-term form too)
        __shared__ SeqSumSmem ss;
        int* scratch = reinterpret_cast<int*>(v + n);
        const int per = (n + (int)blockDim.x - 1) / (int)blockDim.x;
        const float sq = per <= 4 ? seq_sum_squares<4>(v, n, ss, scratch)
                                  : (per <= 5 ? seq_sum_squares<5>(v, n, ss, scratch) : seq_sum_squares(v, n, ss, scratch));
        if (threadIdx.x == 0) {
            stat[0] = 0.0f;
            stat[1] = sqrtf(sq / (float)n);
        }
    } else if (threadIdx.x == 0) {
        if (LAYER) {
            float sum = 0.0f;
            for (int i = 0; i < n; ++i) sum = sum + v[i];
            const float mean = sum / (float)n;
            float ss = 0.0f;
            for (int i = 0; i < n; ++i) {
                const float d = v[i] - mean;
                const float d2 = d * d;
                ss = ss + d2;
            }
            stat[0] = mean;
            stat[1] = sqrtf(ss / (float)n);
        } else {
            float sq = 0.0f;
            for (int i = 0; i < n; ++i) {
                const float p = v[i] * v[i];  // glibc powf(x, 2.0f) == x*x for every float
                sq = sq + p;
            }
            stat[0] = 0.0f;
            stat[1] = sqrtf(sq / (float)n);
        }
    }
    __syncthreads();
    const float mean = stat[0], sd = stat[1];
    uint8_t* dst = out + (long)row * os + (long)h * ohs;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
    for (int blk = warp; blk * GTN_QBLK < n; blk += nw) {
        const int i = blk * GTN_QBLK + lane;
        float y = 0.0f;
        if (i < n) {
            if (LAYER) {
                const float d = v[i] - mean;
                const float t = d / (sd + 1e-05f);
                const float u = t * h2f(w[i]);
                y = u + h2f(bvec[i]);
            } else {
                const float t = v[i] / (sd + 1e-6f);
                y = t * h2f(w[i]);
            }
        }
        store_row_elem(dst, dt, blk, lane, n, y);
    }
}

// rotary_emb_impl (ops.cpp:775-821): position = row index; per head rotate pairs (j, j+half),
// j < half = rd/2, with cos/sin of m * pow(10000, -(2j/rd)) taken from `cs` (float2 per (pos, j),
// computed on the host with the same libm expression); the whole row is rewritten.
// grid: (heads, rows); block 32; d_head <= 256 and a multiple of 32.
static __global__ void k_rope(const uint8_t* in, long is, uint8_t* out, long os, int dt, int n_embd, int d_head,
                              int half, int row0, const float2* cs, int cs_stride) {
    asm volatile("griddepcontrol.wait;" ::: "memory");
    __shared__ float v[256];
    const int row = row0 + blockIdx.y, h = blockIdx.x, lane = threadIdx.x;
    const long hb = row_bytes(dt, d_head);
    const uint8_t* src = in + (long)row * is + (long)h * hb;
    for (int i = lane; i < d_head; i += 32) v[i] = load_elem(src, dt, i);
    __syncwarp();
    float o[8];
    const float2* c = cs + (long)row * cs_stride;
    for (int k = 0; k < d_head / 32; ++k) {
        const int i = k * 32 + lane;
        float y = v[i];
        if (i < half) {
            const float2 t = c[i];
            const float p0 = v[i] * t.x, p1 = v[i + half] * t.y;
            y = p0 - p1;
        } else if (i < 2 * half) {
            const float2 t = c[i - half];
            const float p2 = v[i - half] * t.y, p3 = v[i] * t.x;
            y = p2 + p3;
        }
        o[k] = y;
    }
    __syncwarp();
    uint8_t* dst = out + (long)row * os + (long)h * hb;
    for (int k = 0; k < d_head / 32; ++k) store_row_elem(dst, dt, k, lane, d_head, o[k]);
}

// token_embed / copy_row (ops.cpp:526-576). grid: (ceil(nblocks/4), rows); block 128.
// Token ids come from device memory, so each is range-checked here: an id outside [0, n_vocab)
// sets GTN_DEVERR_TOKEN in *err and row 0 is read instead (never out of bounds).
#define GTN_DEVERR_TOKEN 2u
static __global__ void k_embed(const uint8_t* w, long ws, int wdt, const int32_t* tokens, uint8_t* out, long os,
                               int odt, int n, int row0, int n_vocab, unsigned int* err) {
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const int row = row0 + blockIdx.y;
    const int blk = blockIdx.x * 4 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (blk * GTN_QBLK >= n) return;
    int tok = tokens[row];
    if (tok < 0 || tok >= n_vocab) {
        if (blk == 0 && lane == 0 && err) atomicOr(err, GTN_DEVERR_TOKEN);
        tok = 0;
    }
    const uint8_t* src = w + (long)tok * ws;
    uint8_t* dst = out + (long)row * os;
    if (wdt == GTN_Q4) {
        const int i = blk * GTN_QBLK + lane;
        const float x = i < n ? load_elem(src, GTN_Q4, i) : 0.0f;
        store_row_elem(dst, odt, blk, lane, n, x);
    } else {
        const long bb = wdt == GTN_Q8 ? GTN_Q8_BYTES : (wdt == GTN_F16 ? 64 : 128);
        const long off = blk * bb;
        const long end = min(off + bb, row_bytes(wdt, n));
        for (long j = off + lane; j < end; j += 32) dst[j] = src[j];
    }
}

// Weight packer (one thread per 32-element block), src/tinyllama/tinyllama_to_gten.py:24-91:
// delta = absmax / 127 (Q8) or / 7 (Q4) in IEEE fp32, inverse = 1 / delta where delta != 0,
// q = round-half-even(x * inverse) (torch.round), delta stored as fp16; Q4 adds 7 and packs
// byte j = (q[j] << 4) | (q[j+16] & 15).
template <bool Q4>
static __global__ void k_pack(const float* w, long nblocks, uint8_t* out) {
    const long b = (long)blockIdx.x * blockDim.x + threadIdx.x;
    if (b >= nblocks) return;
    const float4* src = reinterpret_cast<const float4*>(w + b * GTN_QBLK);
    float x[GTN_QBLK];
#pragma unroll
    for (int j = 0; j < GTN_QBLK / 4; ++j) {
        const float4 t = src[j];
        x[4 * j] = t.x; x[4 * j + 1] = t.y; x[4 * j + 2] = t.z; x[4 * j + 3] = t.w;
    }
    float absmax = 0.0f;
#pragma unroll
    for (int j = 0; j < GTN_QBLK; ++j) absmax = fmaxf(absmax, fabsf(x[j]));
    const float delta = absmax / (Q4 ? 7.0f : 127.0f);
    const float inv = delta != 0.0f ? 1.0f / delta : 0.0f;
    const uint16_t d = f2h(delta);
    // Blocks are 34 or 18 bytes, so every block starts on a 2-byte boundary: store 16-bit words.
    if (Q4) {
        uint16_t* o = reinterpret_cast<uint16_t*>(out + b * GTN_Q4_BYTES);
        o[0] = d;
#pragma unroll
        for (int j = 0; j < 16; j += 2) {
            const int a0 = (int)(rintf(x[j] * inv) + 7.0f), a1 = (int)(rintf(x[j + 16] * inv) + 7.0f);
            const int b0 = (int)(rintf(x[j + 1] * inv) + 7.0f), b1 = (int)(rintf(x[j + 17] * inv) + 7.0f);
            const unsigned lo = (unsigned)((a0 << 4) | (a1 & 15)) & 255u;
            const unsigned hi = (unsigned)((b0 << 4) | (b1 & 15)) & 255u;
            o[1 + j / 2] = (uint16_t)(lo | (hi << 8));
        }
    } else {
        uint16_t* o = reinterpret_cast<uint16_t*>(out + b * GTN_Q8_BYTES);
        o[0] = d;
#pragma unroll
        for (int j = 0; j < GTN_QBLK; j += 2) {
            const unsigned lo = (unsigned)(int)rintf(x[j] * inv) & 255u;
            const unsigned hi = (unsigned)(int)rintf(x[j + 1] * inv) & 255u;
            o[1 + j / 2] = (uint16_t)(lo | (hi << 8));
        }
    }
}

// Activation quantizer on fp32 rows (quants.cpp:140-158). grid (ceil(nblocks/4), rows); block 128.
static __global__ void k_quant_rows(const float* x, long xs, uint8_t* out, long os, int n) {
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const int row = blockIdx.y;
    const int blk = blockIdx.x * 4 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (blk * GTN_QBLK >= n) return;
    const int i = blk * GTN_QBLK + lane;
    const float v = i < n ? x[(long)row * xs + i] : 0.0f;
    store_row_elem(out + (long)row * os, GTN_Q8, blk, lane, n, v);
}

// fp32 rows (local index blockIdx.y) -> rows row0 + blockIdx.y of `out` in dtype dt
// (write_row_from_float, ops.cpp:87-123).
static __global__ void k_write_rows(const float* x, long xs, uint8_t* out, long os, int dt, int n, int row0) {
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const int row = row0 + blockIdx.y;
    const int blk = blockIdx.x * 4 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (blk * GTN_QBLK >= n) return;
    const int i = blk * GTN_QBLK + lane;
    const float v = i < n ? x[(long)blockIdx.y * xs + i] : 0.0f;
    store_row_elem(out + (long)row * os, dt, blk, lane, n, v);
}

// Copies M new rows of K or V (reference layout: row m at src + m * ss, kv head g at g * hb) into
// the engine's head-major cache (row p of head g at dst + g * hs + p * rs), rows p = p0 + m.
// grid (kv heads, M); block 32.
static __global__ void k_kv_scatter(const uint8_t* src, long ss, uint8_t* dst, long hs, long rs, int p0, int hb) {
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const int g = blockIdx.x, m = blockIdx.y;
    const uint8_t* s = src + (long)m * ss + (long)g * hb;
    uint8_t* d = dst + (long)g * hs + (long)(p0 + m) * rs;
    if ((((uintptr_t)s | (uintptr_t)d | (uintptr_t)hb) & 3) == 0) {
        for (int i = threadIdx.x; i < hb / 4; i += blockDim.x)
            reinterpret_cast<uint32_t*>(d)[i] = reinterpret_cast<const uint32_t*>(s)[i];
    } else {
        for (int i = threadIdx.x; i < hb; i += blockDim.x) d[i] = s[i];
    }
}

// Greedy argmax (sampler.cpp:30-41): first index of the maximum under strict '>' from -inf.
// One CTA of 1024 threads per row; each thread scans a contiguous slice in order, then a tree
// keeps the larger value and, on ties, the smaller index.
static __global__ void k_argmax(const float* x, int n, int32_t* out, long out_stride, long x_stride) {
    asm volatile("griddepcontrol.wait;" ::: "memory");
    __shared__ float bv[1024];
    __shared__ int bi[1024];
    const float* xr = x + (long)blockIdx.x * x_stride;
    const int t = threadIdx.x, nt = blockDim.x;
    float best = -INFINITY;
    int idx = 0x7fffffff;
    for (int j = t; j < n; j += nt) {  // coalesced; each thread keeps its first maximum
        const float v = xr[j];
        if (v > best) { best = v; idx = j; }
    }
    bv[t] = best;
    bi[t] = idx;
    __syncthreads();
    for (int s = nt / 2; s > 0; s >>= 1) {
        if (t < s) {
            const float v2 = bv[t + s];
            const int i2 = bi[t + s];
            if (v2 > bv[t] || (v2 == bv[t] && i2 < bi[t])) { bv[t] = v2; bi[t] = i2; }
        }
        __syncthreads();
    }
    if (t == 0) out[(long)blockIdx.x * out_stride] = bi[0] == 0x7fffffff ? 0 : bi[0];
}

}  // namespace gtn
