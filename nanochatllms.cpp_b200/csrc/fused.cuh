// Fused decode-step kernels (batch of B sequences, one new token each, device-side positions).
//
// The reference runs each decode step as ~20 ops per layer, requantizing every intermediate row
// (modules.cpp, tinyllama.cpp:35-40/88-97, zephyr.cpp:24-41, minicpm.cpp:42-69). Here one layer is
// five kernels, and every requantization point of the reference is kept inside them:
//   k_fgemv<RESNORM>  residual update  x = q(x_prev + q(y_prev))  [MiniCPM: q(q(y)*s)]
//                     then RMSNorm / LayerNorm -> q(.)  (the GEMV's activation), then the
//                     stacked q/k/v GEMV (fp32 out). Layer 0 takes the embedding row instead.
//   k_fattn           q(y_q) [+bias -> q] -> RoPE -> q; same for k; q(y_v) [+bias -> q]; writes the
//                     new K/V cache rows; causal attention over pos+1 keys -> q(att)
//   k_fgemv<COPY>     o-projection GEMV over q(att)
//   k_fgemv<RESNORM>  h = q(x + q(y_o)), norm -> q(.), gate/up GEMV
//   k_fgemv<SWIGLU>   q(silu(q(y_g))) * q(y_u) -> q(.), down GEMV
// and after the last layer k_fgemv<RESNORM> (final norm [MiniCPM: q(q(.)/9)], lm_head) and
// k_fargmax (greedy pick, appends the token, advances the position).
// Every CTA of a GEMV recomputes its prologue (the activation vector is small); block 0 writes the
// new residual row for the later kernels. All global writes happen after griddepcontrol.wait, and
// weights (read-only) are prefetched with TMA before it, so a kernel's weight stream overlaps the
// previous kernel under programmatic dependent launch.
#pragma once
#include <cooperative_groups.h>
#include "attention.cuh"
#include "matmul.cuh"
#include "rowops.cuh"

namespace gtn {

// Value of element blk*32+lane after a round trip through dtype adt (write_row_from_float +
// read_row_to_float, ops.cpp:41-123); optionally stores the bytes into `row` (nullptr: no store).
__device__ __forceinline__ float requant(float v, int lane, int nv, int adt, uint8_t* row, int blk) {
    if (adt == GTN_Q8) {
        uint16_t dh;
        const int8_t q = warp_quant_block(v, lane, nv, &dh);
        if (row) {
            uint8_t* b = row + (long)blk * GTN_Q8_BYTES;
            if (lane == 0) *reinterpret_cast<uint16_t*>(b) = dh;
            if (lane < nv) b[2 + lane] = (uint8_t)q;
        }
        return (float)q * h2f(dh);
    }
    if (adt == GTN_F16) {
        const uint16_t hv = f2h(v);
        if (row && lane < nv) reinterpret_cast<uint16_t*>(row)[blk * GTN_QBLK + lane] = hv;
        return h2f(hv);
    }
    if (row && lane < nv) reinterpret_cast<float*>(row)[blk * GTN_QBLK + lane] = v;
    return v;
}

enum { PRO_COPY = 0, PRO_RESNORM = 1, PRO_SWIGLU = 2 };

struct FArgs {
    int B;              // sequences in this launch (rows of the activation)
    const int* pos;     // [B] absolute position of each sequence's new token
    const int* active;  // [B] 0: an idle slot, skipped (its rows are not used); null: all active
    int adt;            // activation dtype (Q8 / F16)
    int K;              // activation width (GEMV input)
    // PRO_COPY: activation rows in global memory
    const uint8_t* xin; long xin_s;
    // PRO_RESNORM
    const uint8_t* xres; long xres_s;        // residual rows (adt)
    const float* yadd; long yadd_s;          // fp32 rows requantized and added to the residual (or null)
    int scale_y; float ys;                   // MiniCPM depth scale of the branch output
    uint8_t* xout; long xout_s;              // new residual rows, written by block 0 (or null)
    const uint8_t* emb; long emb_s; int emb_dt; const int32_t* tok; long tok_s; int n_vocab;
    int scale_emb; float es;                 // MiniCPM embedding scale (x12)
    const uint16_t* nw; const uint16_t* nb; int layer;  // norm gain / bias, LayerNorm if layer
    int post; float ps;                      // MiniCPM pre-lm_head scale (1/9)
    // PRO_SWIGLU: fp32 rows [gate | up], ffn columns each
    const float* gu; long gu_s;
    // GEMV
    const uint8_t* W; long ws; int N;
    float* Y; long ldy;
    unsigned int* err;
};

// Shared memory plan of k_fgemv: [mbarriers 128][weight stages][xq rows][prep][fp32 row buffer]
template <int WDT>
__host__ __device__ inline size_t fgemv_smem(int nw, int mt, int K, int adt, int pro) {
    const int nb = K / GTN_QBLK;
    size_t s = 128 + (size_t)MM_STAGES * nw * 8 * mm_q_tile_stride<WDT>();
    s += ((size_t)mt * row_bytes(adt, K) + 15) / 16 * 16;
    s += (size_t)mt * nb * 4 * sizeof(LanePrep);
    if (pro == PRO_RESNORM) s += (size_t)(mt + 1) * K * sizeof(float);  // values + the exact sum's scratch
    return s;
}

// Builds the MT activation rows of this launch in shared memory (xq), per the prologue kind.
template <int PRO, int MT, int PER = SEQSUM_PER_MAX>
__device__ __forceinline__ void fgemv_prologue(const FArgs& a, uint8_t* xq, float* sval, int m0, int mt) {
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, nwarps = blockDim.x >> 5;
    const int K = a.K, nbk = (K + GTN_QBLK - 1) / GTN_QBLK;
    const long xrb = row_bytes(a.adt, K);
    if (PRO == PRO_COPY) {
        for (int m = 0; m < mt; ++m) {
            const uint8_t* src = a.xin + (long)(m0 + m) * a.xin_s;
            uint8_t* dst = xq + (long)m * xrb;
            if ((((uintptr_t)src) & 3) == 0 && (xrb & 3) == 0) {
                for (int i = tid; i < xrb / 4; i += blockDim.x)
                    reinterpret_cast<uint32_t*>(dst)[i] = reinterpret_cast<const uint32_t*>(src)[i];
            } else {
                for (int i = tid; i < xrb; i += blockDim.x) dst[i] = src[i];
            }
        }
        return;
    }
    if (PRO == PRO_SWIGLU) {
        // ops.cpp:733-772 then 918-970: silu on the requantized gate, requantized, times the
        // requantized up projection, requantized (tinyllama.cpp:88-97).
        for (int m = 0; m < mt; ++m) {
            const float* g = a.gu + (long)(m0 + m) * a.gu_s;
            const float* u = g + K;
            for (int blk = warp; blk < nbk; blk += nwarps) {
                const int i = blk * GTN_QBLK + lane, nv = min(GTN_QBLK, K - blk * GTN_QBLK);
                const float gv = requant(i < K ? g[i] : 0.0f, lane, nv, a.adt, nullptr, blk);
                const float den = 1.0f + expf_ref(-gv);
                const float sv = requant(gv / den, lane, nv, a.adt, nullptr, blk);
                const float uv = requant(i < K ? u[i] : 0.0f, lane, nv, a.adt, nullptr, blk);
                requant(sv * uv, lane, nv, a.adt, xq + (long)m * xrb, blk);
            }
        }
        return;
    }
    // PRO_RESNORM: residual update, then the norm's sequential sums. Each warp takes blocks
    // warp, warp + nwarps, ... and loads up to RN of them before computing (the loads overlap).
    constexpr int RN = 4;
    __shared__ unsigned int wmax[32];  // per warp: largest r*r bit pattern (row 0)
    unsigned int mxb = 0u;
    for (int m = 0; m < mt; ++m) {
        float* sv = sval + (long)m * K;
        uint8_t* xo = (a.xout && blockIdx.x == 0) ? a.xout + (long)(m0 + m) * a.xout_s : nullptr;
        const uint8_t* xr = a.xres ? a.xres + (long)(m0 + m) * a.xres_s : nullptr;
        const float* y = a.yadd ? a.yadd + (long)(m0 + m) * a.yadd_s : nullptr;
        const uint8_t* er = nullptr;
        if (a.emb) {
            int t = a.tok[(long)(m0 + m) * a.tok_s + a.pos[m0 + m]];
            if (t < 0 || t >= a.n_vocab) {
                if (tid == 0 && blockIdx.x == 0 && a.err) atomicOr(a.err, GTN_DEVERR_TOKEN);
                t = 0;
            }
            er = a.emb + (long)t * a.emb_s;
        }
        for (int b0 = warp; b0 < nbk; b0 += RN * nwarps) {
            float ev[RN], xv[RN], yv[RN];
#pragma unroll
            for (int j = 0; j < RN; ++j) {
                const int blk = b0 + j * nwarps, i = blk * GTN_QBLK + lane;
                const bool ok = blk < nbk && i < K;
                ev[j] = ok && er ? load_elem(er, a.emb_dt, i) : 0.0f;
                xv[j] = ok && xr ? load_elem(xr, a.adt, i) : 0.0f;
                yv[j] = ok && y ? y[i] : 0.0f;
            }
#pragma unroll
            for (int j = 0; j < RN; ++j) {
                const int blk = b0 + j * nwarps;
                if (blk >= nbk) break;
                const int i = blk * GTN_QBLK + lane, nv = min(GTN_QBLK, K - blk * GTN_QBLK);
                float r;
                if (er) {
                    // token_embed (ops.cpp:526-545): Q8 / fp16 rows copied, Q4 rows requantized to Q8
                    const float e = ev[j];
                    if (a.emb_dt == a.adt) {
                        r = e;
                        if (xo && i < K) {
                            if (a.adt == GTN_Q8) {
                                const uint8_t* sb = er + (long)blk * GTN_Q8_BYTES;
                                uint8_t* db = xo + (long)blk * GTN_Q8_BYTES;
                                if (lane < 2) db[lane] = sb[lane];
                                db[2 + lane] = sb[2 + lane];
                            } else {
                                reinterpret_cast<uint16_t*>(xo)[i] = reinterpret_cast<const uint16_t*>(er)[i];
                            }
                        }
                        if (a.scale_emb) r = requant(r * a.es, lane, nv, a.adt, xo, blk);  // minicpm.cpp:96
                    } else {
                        r = requant(e, lane, nv, a.adt, a.scale_emb ? nullptr : xo, blk);
                        if (a.scale_emb) r = requant(r * a.es, lane, nv, a.adt, xo, blk);
                    }
                } else if (y) {
                    float o = requant(yv[j], lane, nv, a.adt, nullptr, blk);
                    if (a.scale_y) o = requant(o * a.ys, lane, nv, a.adt, nullptr, blk);  // minicpm.cpp:57-58
                    r = requant(xv[j] + o, lane, nv, a.adt, xo, blk);                     // ops::add
                } else {
                    r = xv[j];
                }
                if (i < K) {
                    sv[i] = r;
                    if (m == 0) mxb = max(mxb, seqsum_maxbits(r * r));
                }
            }
        }
    }
    mxb = __reduce_max_sync(0xffffffffu, mxb);
    if (lane == 0) wmax[warp] = mxb;
    __syncthreads();
    __shared__ float stat[MT][2];
    __shared__ SeqSumSmem ss;
    if (mt == 1 && !a.layer) {
        // one row: the exact parallel form of the sequential sum of squares (seqsum.cuh)
        unsigned int mb = lane < nwarps ? wmax[lane] : 0u;
        mb = __reduce_max_sync(0xffffffffu, mb);
        const float sq = seq_sum_squares<PER>(sval, K, ss, nullptr, mb);
        if (tid == 0) {
            stat[0][0] = 0.0f;
            stat[0][1] = sqrtf(sq / (float)K);
        }
    } else if (mt == 1) {
        // LayerNorm of one row (ops.cpp:669-698): the reference's serial mean, then the exact
        // parallel form of the sequential sum of squared deviations
        if (tid == 0) {
            float s0 = 0.0f;
            for (int i = 0; i < K; ++i) s0 = s0 + sval[i];
            stat[0][0] = s0 / (float)K;
        }
        __syncthreads();
        const float mean = stat[0][0];
        const float dev = seq_sum_exact<PER>(
            [sval, mean](int i) {
                const float d = sval[i] - mean;
                return d * d;
            },
            K, ss, nullptr);
        if (tid == 0) stat[0][1] = sqrtf(dev / (float)K);
    } else if (tid < mt) {
        const float* v = sval + (long)tid * K;
        if (a.layer) {
            float sum = 0.0f;
            for (int i = 0; i < K; ++i) sum = sum + v[i];
            const float mean = sum / (float)K;
            float ss = 0.0f;
            for (int i = 0; i < K; ++i) {
                const float d = v[i] - mean;
                const float d2 = d * d;
                ss = ss + d2;
            }
            stat[tid][0] = mean;
            stat[tid][1] = sqrtf(ss / (float)K);
        } else {
            float sq = 0.0f;
#pragma unroll 16
            for (int i = 0; i < K; ++i) {
                const float p = v[i] * v[i];
                sq = sq + p;
            }
            stat[tid][0] = 0.0f;
            stat[tid][1] = sqrtf(sq / (float)K);
        }
    }
    __syncthreads();
    for (int m = 0; m < mt; ++m) {
        const float* v = sval + (long)m * K;
        const float mean = stat[m][0], sd = stat[m][1];
        for (int b0 = warp; b0 < nbk; b0 += RN * nwarps) {
            float wv[RN], bv[RN];
#pragma unroll
            for (int j = 0; j < RN; ++j) {
                const int blk = b0 + j * nwarps, i = blk * GTN_QBLK + lane;
                const bool ok = blk < nbk && i < K;
                wv[j] = ok ? h2f(a.nw[i]) : 0.0f;
                bv[j] = ok && a.layer ? h2f(a.nb[i]) : 0.0f;
            }
#pragma unroll
            for (int j = 0; j < RN; ++j) {
                const int blk = b0 + j * nwarps;
                if (blk >= nbk) break;
                const int i = blk * GTN_QBLK + lane, nv = min(GTN_QBLK, K - blk * GTN_QBLK);
                float yv = 0.0f;
                if (i < K) {
                    if (a.layer) {
                        const float dd = v[i] - mean;
                        const float t = dd / (sd + 1e-05f);
                        const float u = t * wv[j];
                        yv = u + bv[j];
                    } else {
                        const float t = v[i] / (sd + 1e-6f);
                        yv = t * wv[j];
                    }
                }
                if (a.post) {
                    const float nq = requant(yv, lane, nv, a.adt, nullptr, blk);
                    requant(nq * a.ps, lane, nv, a.adt, xq + (long)m * xrb, blk);
                } else {
                    requant(yv, lane, nv, a.adt, xq + (long)m * xrb, blk);
                }
            }
        }
    }
}

// Fused GEMV: prologue (activation rows into shared memory) + the exact Q8/Q4 GEMV of k_mm_q.
// grid.x = ceil(N / (8*NW)); rows of the launch: B <= MT.
template <int WDT, int NW, int MT, int PRO>
__global__ void __launch_bounds__(NW * 32) k_fgemv(const FArgs a) {
    using C = MMCfg<WDT>;
    constexpr int ROWS = NW * 8;
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ int abort_flag;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem);
    const int tstride = mm_q_tile_stride<WDT>();
    uint8_t* stages = smem + 128;
    const int K = a.K, nb = K / GTN_QBLK;
    uint8_t* xq = stages + (size_t)MM_STAGES * ROWS * tstride;
    const size_t xq_bytes = ((size_t)MT * row_bytes(a.adt, K) + 15) / 16 * 16;
    LanePrep* prep = reinterpret_cast<LanePrep*>(xq + xq_bytes);
    float* sval = reinterpret_cast<float*>(prep + (size_t)MT * nb * 4);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int r_local = warp * 8 + (lane >> 2), l = lane & 3;
    const int row0 = blockIdx.x * ROWS;
    const int nrows = min(ROWS, a.N - row0);
    const int m0 = blockIdx.y * MT;
    const int mt = min(MT, a.B - m0);
    const int nkt = (nb + C::KT_BLOCKS - 1) / C::KT_BLOCKS;
    const uint8_t* W = a.W;
    const long w_stride = a.ws;

    auto issue = [&](int kt) {
        const int s = kt % MM_STAGES;
        const int b0 = kt * C::KT_BLOCKS;
        const int nbt = min(C::KT_BLOCKS, nb - b0);
        uint32_t total = 0;
        for (int r = 0; r < nrows; ++r) {
            const uintptr_t src = reinterpret_cast<uintptr_t>(W) + (uintptr_t)(row0 + r) * w_stride +
                                  (uintptr_t)b0 * C::BLK_BYTES;
            total += ((uint32_t)(src & 15) + nbt * C::BLK_BYTES + 15) & ~15u;
        }
        if (lane == 0) mbar_arrive_expect_tx(&bars[s], total);
        __syncwarp();
        for (int r = lane; r < nrows; r += 32) {
            const uintptr_t src = reinterpret_cast<uintptr_t>(W) + (uintptr_t)(row0 + r) * w_stride +
                                  (uintptr_t)b0 * C::BLK_BYTES;
            const uint32_t off = (uint32_t)(src & 15);
            bulk_g2s(stages + ((size_t)s * ROWS + r) * tstride, reinterpret_cast<const void*>(src - off),
                     (off + nbt * C::BLK_BYTES + 15) & ~15u, &bars[s]);
        }
    };

    if (tid == 0) {
        for (int s = 0; s < MM_STAGES; ++s) mbar_init(&bars[s], 1);
        fence_mbar_init();
        abort_flag = 0;
    }
    __syncthreads();
    if (warp == 0)
        for (int kt = 0; kt < min(MM_STAGES, nkt); ++kt) issue(kt);
    asm volatile("griddepcontrol.wait;" ::: "memory");
    fgemv_prologue<PRO, MT>(a, xq, sval, m0, mt);
    __syncthreads();
    build_prep_q8(xq, row_bytes(GTN_Q8, K), 0, mt, nb, prep);
    __syncthreads();

    float acc[MT];
#pragma unroll
    for (int m = 0; m < MT; ++m) acc[m] = 0.0f;
    for (int kt = 0; kt < nkt; ++kt) {
        const int s = kt % MM_STAGES;
        if (!abort_flag && !mbar_wait_bounded(&bars[s], (kt / MM_STAGES) & 1, a.err)) abort_flag = 1;
        const int b0 = kt * C::KT_BLOCKS;
        const int nbt = min(C::KT_BLOCKS, nb - b0);
        if (!abort_flag && r_local < nrows) {
            const uintptr_t src = reinterpret_cast<uintptr_t>(W) + (uintptr_t)(row0 + r_local) * w_stride +
                                  (uintptr_t)b0 * C::BLK_BYTES;
            const uint8_t* t = stages + ((size_t)s * ROWS + r_local) * tstride + (src & 15);
#pragma unroll 4
            for (int b = 0; b < nbt; ++b) {
                const uint8_t* p = t + b * C::BLK_BYTES;
                const float dw = h2f(ld_u16(p));
#pragma unroll
                for (int m = 0; m < MT; ++m) {
                    if (m < mt) {
                        const LanePrep av = prep[((size_t)m * nb + b0 + b) * 4 + l];
                        const int L = WDT == GTN_Q8 ? q8_block_lane_dot(p, l, av) : q4_block_lane_dot(p, l, av);
                        const float sc = av.da * dw;
                        const float pr = lane_sum_f32(L) * sc;
                        acc[m] = acc[m] + pr;
                    }
                }
            }
        }
        __syncthreads();
        if (warp == 0 && !abort_flag && kt + MM_STAGES < nkt) issue(kt + MM_STAGES);
    }
    asm volatile("griddepcontrol.launch_dependents;");
    if (abort_flag) {
        drain_stages(bars, nkt, tid);
        return;
    }
#pragma unroll
    for (int m = 0; m < MT; ++m) {
        const float t01 = acc[m] + __shfl_xor_sync(0xffffffffu, acc[m], 1);
        const float t = t01 + __shfl_xor_sync(0xffffffffu, t01, 2);
        if (l == 0 && r_local < nrows && m < mt) a.Y[(long)(m0 + m) * a.ldy + row0 + r_local] = t;
    }
}

// ---- residual update + norm on a cluster of PCL CTAs ------------------------------------------
// The residual update and norm of fgemv_prologue<PRO_RESNORM>, spread over a thread-block cluster so that the
// per-block requantizations (three per 32 elements) run on PCL SMs instead of one. CTA c updates
// the 32-blocks [c*E, (c+1)*E) of the residual row (E = ceil(blocks / PCL)) and stores the new
// values into the shared memory of every CTA of the cluster (distributed shared memory); after one
// cluster barrier every CTA holds the whole row and computes the norm's statistics itself:
//   RMSNorm    the exact sequential sum of squares (seq_sum_exact);
//   LayerNorm  the reference's serial mean, then the exact sequential sum of squared deviations;
// then normalizes its own blocks. grid (PCL, B), cluster (PCL, 1, 1), block PCL_THREADS, dynamic
// shared memory 2K floats (the row, then K ints of scratch for the sum).
constexpr int PCL = 8;
constexpr int PCL_THREADS = 512;
constexpr int PCL_PER = 5;  // terms per thread of the exact sum in registers (K <= 2560)

struct PclShared {
    unsigned int maxv[PCL];  // largest square per CTA, pushed by every CTA before the barrier
    unsigned int wmax[PCL_THREADS / 32];
    float mean;
    SeqSumSmem ss;
};

// One block of the residual update (as in fgemv_prologue<PRO_RESNORM>): returns the new residual
// value of element blk*32 + lane (already requantized), storing its block into xo if non-null.
__device__ __forceinline__ float resnorm_block(const FArgs& a, int blk, int lane, const uint8_t* er, float ev,
                                               float xv, float yv, bool has_y, uint8_t* xo) {
    const int K = a.K, i = blk * GTN_QBLK + lane, nv = min(GTN_QBLK, K - blk * GTN_QBLK);
    float r;
    if (er) {
        if (a.emb_dt == a.adt) {
            r = ev;
            if (xo && i < K) {
                if (a.adt == GTN_Q8) {
                    const uint8_t* sb = er + (long)blk * GTN_Q8_BYTES;
                    uint8_t* db = xo + (long)blk * GTN_Q8_BYTES;
                    if (lane < 2) db[lane] = sb[lane];
                    db[2 + lane] = sb[2 + lane];
                } else {
                    reinterpret_cast<uint16_t*>(xo)[i] = reinterpret_cast<const uint16_t*>(er)[i];
                }
            }
            if (a.scale_emb) r = requant(r * a.es, lane, nv, a.adt, xo, blk);  // minicpm.cpp:96
        } else {
            r = requant(ev, lane, nv, a.adt, a.scale_emb ? nullptr : xo, blk);
            if (a.scale_emb) r = requant(r * a.es, lane, nv, a.adt, xo, blk);
        }
    } else if (has_y) {
        float o = requant(yv, lane, nv, a.adt, nullptr, blk);
        if (a.scale_y) o = requant(o * a.ys, lane, nv, a.adt, nullptr, blk);  // minicpm.cpp:57-58
        r = requant(xv + o, lane, nv, a.adt, xo, blk);                        // ops::add
    } else {
        r = xv;
    }
    return r;
}

static __global__ void __launch_bounds__(PCL_THREADS) k_prep_cl(const FArgs a, uint8_t* act, long act_s) {
    // an idle slot: the whole cluster (one sequence) leaves before its first cluster barrier
    if (a.active && !__ldcg(a.active + blockIdx.y)) return;
    namespace cg = cooperative_groups;
    cg::cluster_group cl = cg::this_cluster();
    extern __shared__ float sv[];  // the row at global element indices, then K ints of scratch
    __shared__ PclShared S;
    // every CTA of the cluster has started before the first remote store: arrive now, wait below
    asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
    const int rank = (int)cl.block_rank();
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, nwarps = PCL_THREADS / 32;
    const int K = a.K, nbk = (K + GTN_QBLK - 1) / GTN_QBLK, E = (nbk + PCL - 1) / PCL;
    const int b0 = min(nbk, rank * E), b1 = min(nbk, b0 + E);
    const int e0 = b0 * GTN_QBLK, e1 = min(K, b1 * GTN_QBLK);
    {  // the norm weights do not depend on the previous kernel: warm L2 now
        const int lines = (e1 - e0) * 2 / 128 + 2;
        for (int i = tid; i < lines; i += PCL_THREADS) {
            const long off = min(2L * e0 + 128L * i, 2L * K - 2);
            asm volatile("prefetch.global.L2 [%0];" ::"l"(reinterpret_cast<const char*>(a.nw) + off));
            if (a.nb) asm volatile("prefetch.global.L2 [%0];" ::"l"(reinterpret_cast<const char*>(a.nb) + off));
        }
    }
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;");
    const int m = blockIdx.y;
    // ---- residual update of this CTA's blocks, stored into every CTA
    uint8_t* xo = a.xout ? a.xout + (long)m * a.xout_s : nullptr;  // every CTA writes its own blocks
    const uint8_t* xr = a.xres ? a.xres + (long)m * a.xres_s : nullptr;
    const float* y = a.yadd ? a.yadd + (long)m * a.yadd_s : nullptr;
    const uint8_t* er = nullptr;
    if (a.emb) {
        int t = a.tok[(long)m * a.tok_s + a.pos[m]];
        if (t < 0 || t >= a.n_vocab) {
            if (tid == 0 && rank == 0 && a.err) atomicOr(a.err, GTN_DEVERR_TOKEN);
            t = 0;
        }
        er = a.emb + (long)t * a.emb_s;
    }
    asm volatile("barrier.cluster.wait.aligned;" ::: "memory");
    unsigned int mxb = 0u;
    for (int blk = b0 + warp; blk < b1; blk += nwarps) {
        const int i = blk * GTN_QBLK + lane;
        const bool ok = i < K;
        const float ev = ok && er ? load_elem(er, a.emb_dt, i) : 0.0f;
        const float xv = ok && xr ? load_elem(xr, a.adt, i) : 0.0f;
        const float yv = ok && y ? y[i] : 0.0f;
        const float r = resnorm_block(a, blk, lane, er, ev, xv, yv, y != nullptr, xo);
        if (ok) {
#pragma unroll
            for (int q = 0; q < PCL; ++q) {
                float* d = q == rank ? sv : cl.map_shared_rank(sv, q);
                d[i] = r;
            }
            mxb = max(mxb, seqsum_maxbits(r * r));
        }
    }
    mxb = __reduce_max_sync(0xffffffffu, mxb);
    if (lane == 0) S.wmax[warp] = mxb;
    __syncthreads();
    if (warp == 0) {
        unsigned int mb = lane < nwarps ? S.wmax[lane] : 0u;
        mb = __reduce_max_sync(0xffffffffu, mb);
        if (lane < PCL) cl.map_shared_rank(&S, lane)->maxv[rank] = mb;
    }
    cl.sync();  // the whole row and every CTA's largest square are in place
    // ---- statistics, in every CTA (no remote access from here on)
    int* incs = reinterpret_cast<int*>(sv + K);
    float mean = 0.0f, sd;
    if (!a.layer) {
        unsigned int maxbits = 0u;
#pragma unroll
        for (int r = 0; r < PCL; ++r) maxbits = max(maxbits, S.maxv[r]);
        // four terms per thread where they fit (K <= 2048): the unrolled per-term work is a fifth
        // shorter than with PCL_PER
        const float sq = K <= 4 * PCL_THREADS ? seq_sum_squares<4>(sv, K, S.ss, incs, maxbits)
                                              : seq_sum_squares<PCL_PER>(sv, K, S.ss, incs, maxbits);
        sd = sqrtf(sq / (float)K);
    } else {
        if (tid == 0) {  // the signed sum of the mean: the reference's loop
            float s0 = 0.0f;
            for (int i = 0; i < K; ++i) s0 = s0 + sv[i];
            S.mean = s0 / (float)K;
        }
        __syncthreads();
        mean = S.mean;
        const auto dev2 = [mean](int i) {
            const float d = sv[i] - mean;
            return d * d;
        };
        const float ss = K <= 4 * PCL_THREADS ? seq_sum_exact<4>(dev2, K, S.ss, incs)
                                              : seq_sum_exact<PCL_PER>(dev2, K, S.ss, incs);
        sd = sqrtf(ss / (float)K);
    }
    // ---- norm of this CTA's blocks -> act
    uint8_t* xq = act + (long)m * act_s;
    for (int blk = b0 + warp; blk < b1; blk += nwarps) {
        const int i = blk * GTN_QBLK + lane, nv = min(GTN_QBLK, K - blk * GTN_QBLK);
        float yv = 0.0f;
        if (i < K) {
            if (a.layer) {
                const float dd = sv[i] - mean;
                const float t = dd / (sd + 1e-05f);
                const float u = t * h2f(a.nw[i]);
                yv = u + h2f(a.nb[i]);
            } else {
                const float t = sv[i] / (sd + 1e-6f);
                yv = t * h2f(a.nw[i]);
            }
        }
        if (a.post) {
            const float nq = requant(yv, lane, nv, a.adt, nullptr, blk);
            requant(nq * a.ps, lane, nv, a.adt, xq, blk);
        } else {
            requant(yv, lane, nv, a.adt, xq, blk);
        }
    }
}

// The SwiGLU activation is block-local, so it is spread over many CTAs: grid (ceil(blocks/32), B),
// block 1024 (one warp per 32-element block).
static __global__ void __launch_bounds__(1024) k_prep_swiglu(const FArgs a, uint8_t* act, long act_s) {
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;");
    const int K = a.K, nbk = (K + GTN_QBLK - 1) / GTN_QBLK;
    const int blk = blockIdx.x * 32 + (threadIdx.x >> 5), lane = threadIdx.x & 31, m = blockIdx.y;
    if (blk >= nbk) return;
    const float* g = a.gu + (long)m * a.gu_s;
    const float* u = g + K;
    const int i = blk * GTN_QBLK + lane, nv = min(GTN_QBLK, K - blk * GTN_QBLK);
    const float gv = requant(i < K ? g[i] : 0.0f, lane, nv, a.adt, nullptr, blk);
    const float den = 1.0f + expf_ref(-gv);
    const float sv = requant(gv / den, lane, nv, a.adt, nullptr, blk);
    const float uv = requant(i < K ? u[i] : 0.0f, lane, nv, a.adt, nullptr, blk);
    requant(sv * uv, lane, nv, a.adt, act + (long)m * act_s, blk);
}

// ---- attention with the q/k/v epilogue of the stacked projection ----------------------------
struct AArgs {
    int adt, q_heads, kv_heads, d;          // d = head size (64)
    const int* pos;                          // [B]
    const int* active;                       // [B] 0: idle slot (no cache write), or null
    const float* y; long ys;                 // stacked q|k|v fp32 rows
    const uint16_t *bq, *bk, *bv;            // Zephyr biases (or null)
    const uint16_t *qnw, *knw;               // OpenELM QK-norm gains [d] (or null)
    const float2* cs; int half;              // RoPE table [pos][half] (cos, sin), half = rd/2
    uint8_t* kc; uint8_t* vc; long kvs;      // cache of this layer: row stride kvs bytes
    long khs;                                // bytes between kv heads
    long seq_stride;                         // bytes between sequences
    uint8_t* out; long os;                   // attention output rows (adt)
    unsigned int* err;
};

// grid (q_heads, B); block ATT_THREADS. Decode attention of sequence b at position p = pos[b]
// (keys 0..p), preceded by the q/k/v epilogue of the stacked projection, one Linear output head
// each: requant (Linear) [-> + bias -> requant (bias_add_inplace)] [-> QK RMSNorm -> requant]
// [-> RoPE -> requant]. The epilogue runs one warp per (tensor, 32-block). The q-head 0 of each kv group writes the new K/V
// cache rows; key p is taken from this CTA's own epilogue values. Then att_core / att_out.
static __global__ void __launch_bounds__(ATT_THREADS) k_fattn(const AArgs a) {
    extern __shared__ __align__(16) uint8_t sm[];
    __shared__ __align__(16) uint8_t hrow[3][320];  // q, k, v head rows (adt), d <= 128
    __shared__ float tmp[3][128];
    __shared__ float red[ATT_THREADS / 32];
    __shared__ float s_stat[2];
    __shared__ __align__(8) uint64_t bars[2];
    __shared__ int abort_flag;
    const int h = blockIdx.x, b = blockIdx.y;
    if (a.active && !__ldcg(a.active + b)) return;  // an idle slot: no cache row, no output
    const int group = a.q_heads / a.kv_heads, g = h / group;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int d = a.d, nbh = d / GTN_QBLK;
    const long hb = row_bytes(a.adt, d);
    // The position was written by the previous step's last kernel, and the cache rows below it by
    // earlier steps: both are complete before this kernel starts, so the first K/V tiles are
    // fetched before waiting for the q/k/v projection (row p is replaced when the tiles land).
    const int p = __ldcg(a.pos + b), n = p + 1;  // L2 only: no L1 line of an earlier step
    uint8_t* kc = a.kc + (long)b * a.seq_stride + (long)g * a.khs;
    uint8_t* vc = a.vc + (long)b * a.seq_stride + (long)g * a.khs;
    const AttSmem L = att_layout(sm, n, hb, d, bars, &abort_flag);
    att_init_bars(bars, &abort_flag);
    att_prefetch(kc, a.kvs, vc, a.kvs, (int)hb, n, p, L);
    const bool rope = a.half > 0;
    float2 cs_first = make_float2(0.0f, 0.0f);  // this warp's first RoPE (cos, sin): a constant table
    if (rope && warp < 2 * nbh) {
        const int i = (warp % nbh) * GTN_QBLK + lane;
        if (i < 2 * a.half) cs_first = a.cs[(long)p * a.half + (i < a.half ? i : i - a.half)];
    }
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const float* yrow = a.y + (long)b * a.ys;
    const int qd = a.q_heads * d, kvd = a.kv_heads * d;
    // (1) Linear requant [+ bias requant], one warp per (tensor t, block k)
    for (int w = warp; w < 3 * nbh; w += ATT_THREADS / 32) {
        const int t = w / nbh, k = w - t * nbh, i = k * GTN_QBLK + lane;
        const int c0 = t == 0 ? h * d : (t == 1 ? qd + g * d : qd + kvd + g * d);
        const uint16_t* bias = t == 0 ? a.bq : (t == 1 ? a.bk : a.bv);
        float v = requant(yrow[c0 + i], lane, GTN_QBLK, a.adt, nullptr, 0);
        if (bias) v = requant(v + h2f(bias[(t == 0 ? h : g) * d + i]), lane, GTN_QBLK, a.adt, nullptr, 0);
        tmp[t][i] = v;
    }
    __syncthreads();
    if (a.qnw) {
        // OpenELM QK-norm (openelm.cpp:44-50 -> rms_norm 3-D, ops.cpp:830-846 and :862-885): per
        // head, the sequential fp32 sum of squares, sqrt of its mean, x / (rms + 1e-6) * w, requant
        if (tid < 2) {
            float ss = 0.0f;
            for (int i = 0; i < d; ++i) {
                const float x = tmp[tid][i];
                const float x2 = x * x;
                ss = ss + x2;
            }
            s_stat[tid] = sqrtf(ss / (float)d);
        }
        __syncthreads();
        for (int w = warp; w < 2 * nbh; w += ATT_THREADS / 32) {
            const int t = w / nbh, k = w - t * nbh, i = k * GTN_QBLK + lane;
            const float x = tmp[t][i] / (s_stat[t] + 1e-6f);
            const float y = x * h2f((t == 0 ? a.qnw : a.knw)[i]);
            tmp[t][i] = requant(y, lane, GTN_QBLK, a.adt, nullptr, 0);
        }
        __syncthreads();
    }
    // (2) RoPE (q, k) and the final requant into the head rows
    for (int w = warp; w < 3 * nbh; w += ATT_THREADS / 32) {
        const int t = w / nbh, k = w - t * nbh, i = k * GTN_QBLK + lane;
        float y = tmp[t][i];
        if (rope && t < 2) {
            const float2* c = a.cs + (long)p * a.half;
            if (i < a.half) {
                const float2 cs = w == warp ? cs_first : c[i];
                const float p0 = tmp[t][i] * cs.x, p1 = tmp[t][i + a.half] * cs.y;
                y = p0 - p1;
            } else if (i < 2 * a.half) {
                const float2 cs = w == warp ? cs_first : c[i - a.half];
                const float p2 = tmp[t][i - a.half] * cs.y, p3 = tmp[t][i] * cs.x;
                y = p2 + p3;
            }
        }
        requant(y, lane, GTN_QBLK, a.adt, hrow[t], k);
    }
    __syncthreads();
    if (h % group == 0) {
        for (int i = tid; i < hb; i += ATT_THREADS) {
            kc[(long)p * a.kvs + i] = hrow[1][i];
            vc[(long)p * a.kvs + i] = hrow[2][i];
        }
    }
    if (a.adt == GTN_Q8) build_prep_q8(hrow[0], 0, 0, 1, nbh, L.qp);
    __syncthreads();
    int vt0, vnt;
    att_core(kc, a.kvs, vc, a.kvs, (int)hb, n, p, p, hrow[1], hrow[2], hrow[0], L, a.adt, d, red, s_stat, a.err,
             &vt0, &vnt, true);
    asm volatile("griddepcontrol.launch_dependents;");
    const int vrs = att_bulk(vc, a.kvs, (int)hb) ? (int)a.kvs : att_rs(hb);
    att_out(L.part, L.p, vc, a.kvs, n, p, p, hrow[2], a.adt, d, a.out + (long)b * a.os + (long)h * hb, L.vt, vrs,
            vt0, vnt);
}

inline size_t fattn_smem(int n, int adt, int d) { return attn_smem(n, adt, d); }

// Greedy pick per sequence (sampler.cpp:30-41) + the decode loop's bookkeeping: the id becomes the
// input token of the next position and is recorded (and copied to next[b] if next is set); the
// position advances. Idle slots (active[b] == 0) are skipped. grid B; block 1024.
static __global__ void k_fargmax(const float* logits, long ls, int n, int32_t* tok, int32_t* gen, long tok_s,
                                 int* pos, int max_ctx, unsigned int* err, const int* active, int32_t* next) {
    if (active && !__ldcg(active + blockIdx.x)) return;
    asm volatile("griddepcontrol.wait;" ::: "memory");
    __shared__ float bv[1024];
    __shared__ int bi[1024];
    const int b = blockIdx.x;
    const float* xr = logits + (long)b * ls;
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
    if (t == 0) {
        const int id = bi[0] == 0x7fffffff ? 0 : bi[0];
        if (next) next[b] = id;
        const int p = pos[b];
        if (p + 1 < max_ctx) {
            tok[(long)b * tok_s + p + 1] = id;
            gen[(long)b * tok_s + p + 1] = id;
            pos[b] = p + 1;
        } else if (err) {
            atomicOr(err, 4u);
        }
    }
}

}  // namespace gtn
