/* Test infrastructure only: CPU restatement of the gten compute path of
 * iangitonga/nanochatllms.cpp. See gten_oracle.h for the contract.
 *
 * Build: oracle/Makefile (gcc -O2 -ffp-contract=off, OpenMP over output rows like the
 * reference's matmul). -ffp-contract=off matters: the reference is built with -mavx and no
 * -mfma, so every multiply and add is rounded separately; contraction would change results.
 * Transcendentals (expf, powf, sinf, cosf, sqrtf, roundf) are the same libm calls the reference
 * makes, so on the same host they return the same bits.
 */
#include "gten_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

#define QBLK 32
typedef struct __attribute__((packed)) { uint16_t d; int8_t q[QBLK]; } q8blk;     /* quants.h:11-22 */
typedef struct __attribute__((packed)) { uint16_t d; uint8_t q[QBLK / 2]; } q4blk; /* quants.h:24-30 */

static inline float bits_f(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }
static inline uint32_t f_bits(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }

long or_row_bytes(int dt, int n) {
    switch (dt) {
        case OR_Q8: return (long)((n + QBLK - 1) / QBLK) * (long)sizeof(q8blk);
        case OR_Q4: return (long)(n / QBLK) * (long)sizeof(q4blk);
        case OR_F16: return 2L * n;
        default: return 4L * n;
    }
}

/* gten_types.h:69-87 (fp16 -> fp32, exact for every half value; the reference caches it in a
 * 65536-entry table, gten_types.h:112-133). Restated from the IEEE binary16 definition. */
float or_fp16_to_fp32(uint16_t h) {
    const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    const uint32_t e = (h >> 10) & 0x1fu, m = h & 0x3ffu;
    if (e == 0) {
        const float v = ldexpf((float)m, -24);
        return sign ? -v : v;
    }
    if (e == 31) return bits_f(sign | 0x7f800000u | (m << 13));
    return bits_f(sign | ((e + 112u) << 23) | (m << 13));
}

/* gten_types.h:89-109 (fp32 -> fp16, round to nearest even; NaN -> 0x7e00). Also what F16C
 * _mm256_cvtps_ph(x, 0) does on the AVX paths (ops.cpp:97-107). */
uint16_t or_fp32_to_fp16(float f) {
    const uint32_t x = f_bits(f);
    const uint16_t sign = (uint16_t)((x >> 16) & 0x8000u);
    const uint32_t ax = x & 0x7fffffffu;
    if (ax >= 0x7f800000u) return sign | (ax > 0x7f800000u ? 0x7e00u : 0x7c00u);
    if (ax >= 0x477ff000u) return sign | 0x7c00u; /* >= 65520 rounds to inf */
    if (ax < 0x38800000u) {                        /* half subnormal range */
        const float q = nearbyintf(bits_f(ax) * 16777216.0f);
        return sign | (uint16_t)q;
    }
    uint32_t h = (((ax >> 23) - 112u) << 10) | ((ax & 0x7fffffu) >> 13);
    const uint32_t rem = ax & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h++;
    return sign | (uint16_t)h;
}

/* quants.cpp:16-30 q8_quantize_block: absmax, delta = absmax/127 (stored fp16), the reciprocal of
 * the UNROUNDED fp32 delta, roundf (half away from zero). Bytes past `n` are left untouched. */
static void q8_quantize_block(const float* x, q8blk* out, int n) {
    float absmax = 0.0f;
    for (int j = 0; j < n; j++) {
        const float a = fabsf(x[j]);
        absmax = (absmax < a) ? a : absmax; /* std::max */
    }
    const float delta = absmax / 127.0f;
    out->d = or_fp32_to_fp16(delta);
    const float scale = delta != 0.0f ? 1.0f / delta : 0.0f;
    for (int j = 0; j < n; j++) out->q[j] = (int8_t)roundf(x[j] * scale);
}

/* quants.cpp:140-158 */
void or_q8_quantize_row(const float* x, void* out, int n) {
    q8blk* o = (q8blk*)out;
    const int nb = n / QBLK;
    for (int b = 0; b < nb; b++) q8_quantize_block(x + b * QBLK, o + b, QBLK);
    if (n % QBLK) q8_quantize_block(x + nb * QBLK, o + nb, n % QBLK);
}

/* ops.cpp:41-84 read_row_to_float with quants.cpp:33-63 (Q8), :81-138 (Q4: byte j holds element
 * j in the high nibble and element j+16 in the low nibble, both +7 biased), :160-185. */
void or_read_row(const void* row, int dt, float* out, int n) {
    switch (dt) {
        case OR_Q8: {
            const q8blk* b = (const q8blk*)row;
            for (int i = 0; i < n; i++) {
                const float d = or_fp16_to_fp32(b[i / QBLK].d);
                out[i] = (float)b[i / QBLK].q[i % QBLK] * d;
            }
        } break;
        case OR_Q4: {
            const q4blk* b = (const q4blk*)row;
            for (int k = 0; k < n / QBLK; k++) {
                const float d = or_fp16_to_fp32(b[k].d);
                for (int j = 0; j < QBLK / 2; j++) {
                    const uint8_t p = b[k].q[j];
                    out[k * QBLK + j] = (float)((int)(p >> 4) - 7) * d;
                    out[k * QBLK + j + 16] = (float)((int)(p & 15) - 7) * d;
                }
            }
        } break;
        case OR_F16: {
            const uint16_t* h = (const uint16_t*)row;
            for (int i = 0; i < n; i++) out[i] = or_fp16_to_fp32(h[i]);
        } break;
        default: memcpy(out, row, sizeof(float) * (size_t)n);
    }
}

/* ops.cpp:87-123 write_row_from_float */
void or_write_row(const float* x, void* row, int dt, int n) {
    switch (dt) {
        case OR_Q8: or_q8_quantize_row(x, row, n); break;
        case OR_F16: {
            uint16_t* h = (uint16_t*)row;
            for (int i = 0; i < n; i++) h[i] = or_fp32_to_fp16(x[i]);
        } break;
        default: memcpy(row, x, sizeof(float) * (size_t)n);
    }
}

/* src/tinyllama/tinyllama_to_gten.py:24-51 q8_quantize: delta = absmax / 127 (IEEE fp32 division),
 * inverse = 1 / delta where delta != 0, q = torch.round(x * inverse) (half to even), delta stored
 * as fp16. Record layout per block: fp16 delta then 32 int8 (write_layer, :110-127). */
void or_pack_q8(const float* w, int rows, int cols, void* out) {
    q8blk* o = (q8blk*)out;
    const long nb = (long)rows * (cols / QBLK);
    for (long b = 0; b < nb; b++) {
        const float* x = w + b * QBLK;
        float absmax = 0.0f;
        for (int j = 0; j < QBLK; j++) absmax = fmaxf(absmax, fabsf(x[j]));
        const float delta = absmax / 127.0f;
        const float inv = delta != 0.0f ? 1.0f / delta : 0.0f;
        o[b].d = or_fp32_to_fp16(delta);
        for (int j = 0; j < QBLK; j++) o[b].q[j] = (int8_t)nearbyintf(x[j] * inv);
    }
}

/* src/tinyllama/tinyllama_to_gten.py:54-91 q4_quantize: delta = absmax / 7, q = round(x/delta) + 7
 * in [0, 14]; byte j = (q[j] << 4) | (q[j+16] & 0xF). */
void or_pack_q4(const float* w, int rows, int cols, void* out) {
    q4blk* o = (q4blk*)out;
    const long nb = (long)rows * (cols / QBLK);
    for (long b = 0; b < nb; b++) {
        const float* x = w + b * QBLK;
        float absmax = 0.0f;
        for (int j = 0; j < QBLK; j++) absmax = fmaxf(absmax, fabsf(x[j]));
        const float delta = absmax / 7.0f;
        const float inv = delta != 0.0f ? 1.0f / delta : 0.0f;
        o[b].d = or_fp32_to_fp16(delta);
        for (int j = 0; j < QBLK / 2; j++) {
            const uint8_t t0 = (uint8_t)(nearbyintf(x[j] * inv) + 7.0f);
            const uint8_t t1 = (uint8_t)(nearbyintf(x[j + 16] * inv) + 7.0f);
            o[b].q[j] = (uint8_t)((t0 << 4) | (t1 & 0x0f));
        }
    }
}

/* Lane l of the reference's 4-wide SSE accumulator owns elements {c+2l, c+2l+1 : c in
 * {0,8,16,24}} of every block (_mm_madd_epi16 on 8-element chunks, ops.cpp:320-348 and
 * ops.cpp:407-446). */
static inline void q8_lane_sums(const int8_t* a, const int8_t* w, int L[4]) {
    for (int l = 0; l < 4; l++) {
        int s = 0;
        for (int c = 0; c < QBLK; c += 8) s += (int)a[c + 2 * l] * w[c + 2 * l] + (int)a[c + 2 * l + 1] * w[c + 2 * l + 1];
        L[l] = s;
    }
}

static inline void q4_unpack(const q4blk* b, int8_t w[QBLK]) {
    for (int j = 0; j < QBLK / 2; j++) {
        w[j] = (int8_t)((int)(b->q[j] >> 4) - 7);
        w[j + 16] = (int8_t)((int)(b->q[j] & 15) - 7);
    }
}

/* ops.cpp:292-384 vec_dot_product_q8 and ops.cpp:387-490 vec_dot_product_q8_q4 (AVX paths):
 * per block exact int32 lane sums, converted to fp32, times fp16(da)*fp16(db), added lane-wise;
 * result (L0+L1)+(L2+L3) from two _mm_hadd_ps. order 1: one accumulator, block sums in order. */
static float dot_q8(const q8blk* a, const void* w, int wq4, int n, int order) {
    const int nb = n / QBLK;
    float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    float acc1 = 0.0f;
    for (int b = 0; b < nb; b++) {
        int8_t wv[QBLK];
        uint16_t wd;
        if (wq4) {
            const q4blk* wb = (const q4blk*)w + b;
            q4_unpack(wb, wv);
            wd = wb->d;
        } else {
            const q8blk* wb = (const q8blk*)w + b;
            memcpy(wv, wb->q, QBLK);
            wd = wb->d;
        }
        const float s = or_fp16_to_fp32(a[b].d) * or_fp16_to_fp32(wd);
        int L[4];
        q8_lane_sums(a[b].q, wv, L);
        if (order == 0) {
            for (int l = 0; l < 4; l++) {
                const float p = (float)L[l] * s;
                acc[l] = acc[l] + p;
            }
        } else {
            const float p = (float)(L[0] + L[1] + L[2] + L[3]) * s;
            acc1 = acc1 + p;
        }
    }
    if (order != 0) return acc1;
    return (acc[0] + acc[1]) + (acc[2] + acc[3]);
}

/* ops.cpp:208-289 vec_dot_product_f16/_f32 (AVX): 8 fp32 lanes, lane l sums x[8i+l]*y[8i+l]
 * (mul rounded, then add: simd_ops.h:71-73), lanes summed left to right (simd_ops.h:75-78),
 * then the scalar tail. */
static float dot_f(const void* a, const void* b, int n, int f16) {
    float acc[8] = {0};
    const int n8 = (n / 8) * 8;
    for (int i = 0; i < n8; i += 8) {
        for (int l = 0; l < 8; l++) {
            float x, y;
            if (f16) {
                x = or_fp16_to_fp32(((const uint16_t*)a)[i + l]);
                y = or_fp16_to_fp32(((const uint16_t*)b)[i + l]);
            } else {
                x = ((const float*)a)[i + l];
                y = ((const float*)b)[i + l];
            }
            const float p = x * y;
            acc[l] = p + acc[l];
        }
    }
    float dot = acc[0] + acc[1] + acc[2] + acc[3] + acc[4] + acc[5] + acc[6] + acc[7];
    for (int i = n8; i < n; i++) {
        float x, y;
        if (f16) {
            x = or_fp16_to_fp32(((const uint16_t*)a)[i]);
            y = or_fp16_to_fp32(((const uint16_t*)b)[i]);
        } else {
            x = ((const float*)a)[i];
            y = ((const float*)b)[i];
        }
        const float p = x * y;
        dot = dot + p;
    }
    return dot;
}

/* ops.cpp:493-523 vec_dot_product dispatch on the first operand's dtype */
float or_vec_dot(const void* a, int adt, const void* b, int bdt, int n, int order) {
    switch (adt) {
        case OR_Q8: return dot_q8((const q8blk*)a, b, bdt == OR_Q4, n, order);
        case OR_F16: return dot_f(a, b, n, 1);
        default: return dot_f(a, b, n, 0);
    }
}

/* ops.cpp:579-636 matmul_2d / matmul_2d_impl: rows [start_pos, n_ctx), out[c] = dot(x_r, W_c),
 * then write_row_from_float into the output dtype. out_1d: EmbeddingLinear's stride-0 fp32 row. */
void or_matmul_2d(const void* x, int xdt, int n_ctx, int n_embd, const void* w, int wdt, int n_out, void* out,
                  int odt, int start_pos, int out_1d, int order) {
    const long xs = or_row_bytes(xdt, n_embd), ws = or_row_bytes(wdt, n_embd);
    const long os = out_1d ? 0 : or_row_bytes(odt, n_out);
    float* buf = (float*)malloc(sizeof(float) * (size_t)n_out);
    for (int r = start_pos; r < n_ctx; r++) {
        const char* xr = (const char*)x + r * xs;
#pragma omp parallel for schedule(static)
        for (int c = 0; c < n_out; c++) buf[c] = or_vec_dot(xr, xdt, (const char*)w + (long)c * ws, wdt, n_embd, order);
        or_write_row(buf, (char*)out + r * os, odt, n_out);
    }
    free(buf);
}

/* ops.cpp:830-846 rms_norm_vec_f32: x / (sqrt(sum(x^2)/n) + 1e-6) * w, sequential fp32 sum;
 * std::pow(x, 2.0f) returns exactly x*x for every float on glibc (checked exhaustively). */
static void rms_vec(const float* x, const uint16_t* w, float* out, int n) {
    float sq = 0.0f;
    for (int i = 0; i < n; i++) sq += powf(x[i], 2.0f);
    const float mean = sq / (float)n;
    const float rms = sqrtf(mean);
    for (int i = 0; i < n; i++) {
        const float t = x[i] / (rms + 1e-6f);
        out[i] = t * or_fp16_to_fp32(w[i]);
    }
}

/* ops.cpp:849-915 (2-D path) */
void or_rms_norm(const void* x, int dt, int n_ctx, int n_embd, const uint16_t* w, void* out, int start_pos) {
    const long rs = or_row_bytes(dt, n_embd);
    float* a = (float*)malloc(sizeof(float) * 2 * (size_t)n_embd);
    for (int r = start_pos; r < n_ctx; r++) {
        or_read_row((const char*)x + r * rs, dt, a, n_embd);
        rms_vec(a, w, a + n_embd, n_embd);
        or_write_row(a + n_embd, (char*)out + r * rs, dt, n_embd);
    }
    free(a);
}

/* ops.cpp:856-882 (3-D path: per row, per head, over d_head; OpenELM QK-norm) */
void or_rms_norm_3d(const void* x, int dt, int n_ctx, int n_heads, int d_head, const uint16_t* w, void* out,
                    int start_pos) {
    const long rs = or_row_bytes(dt, n_heads * d_head), hs = or_row_bytes(dt, d_head);
    float a[2 * 512];
    for (int r = start_pos; r < n_ctx; r++)
        for (int h = 0; h < n_heads; h++) {
            or_read_row((const char*)x + r * rs + h * hs, dt, a, d_head);
            rms_vec(a, w, a + d_head, d_head);
            or_write_row(a + d_head, (char*)out + r * rs + h * hs, dt, d_head);
        }
}

/* ops.cpp:669-730 vec_layer_norm_f32: mean and population variance with sequential sums,
 * ((x - mean) / (sqrt(var) + 1e-5)) * w + b. */
void or_layer_norm(const void* x, int dt, int n_ctx, int n_embd, const uint16_t* w, const uint16_t* b, void* out,
                   int start_pos) {
    const long rs = or_row_bytes(dt, n_embd);
    float* a = (float*)malloc(sizeof(float) * 2 * (size_t)n_embd);
    for (int r = start_pos; r < n_ctx; r++) {
        or_read_row((const char*)x + r * rs, dt, a, n_embd);
        float sum = 0.0f;
        for (int i = 0; i < n_embd; i++) sum += a[i];
        const float mean = sum / (float)n_embd;
        float ss = 0.0f;
        for (int i = 0; i < n_embd; i++) {
            const float d = a[i] - mean;
            const float d2 = d * d;
            ss += d2;
        }
        const float var = ss / (float)n_embd;
        const float sd = sqrtf(var);
        for (int i = 0; i < n_embd; i++) {
            const float d = a[i] - mean;
            const float t = d / (sd + 1e-05f);
            const float u = t * or_fp16_to_fp32(w[i]);
            a[n_embd + i] = u + or_fp16_to_fp32(b[i]);
        }
        or_write_row(a + n_embd, (char*)out + r * rs, dt, n_embd);
    }
    free(a);
}

/* ops.cpp:775-821 rotary_emb_impl: position = row index; per head rotate pairs (j, j + rd/2) for
 * j < rd/2 with rd = int(d_head * rope_pct), theta = m * pow(10000, -(2j/rd)); the whole row is
 * rewritten in the input dtype (also dims >= rd, which are requantized). */
void or_rotary_emb(const void* inp, void* out, int dt, int n_ctx, int n_embd, int d_head, float rope_pct,
                   int start_pos) {
    const long rs = or_row_bytes(dt, n_embd);
    const int n_head = n_embd / d_head;
    const int rd = (int)((float)d_head * rope_pct);
    const float d = (float)rd;
    float* a = (float*)malloc(sizeof(float) * (size_t)n_embd);
    for (int i = start_pos; i < n_ctx; i++) {
        or_read_row((const char*)inp + i * rs, dt, a, n_embd);
        for (int h = 0; h < n_head; h++) {
            float* v = a + h * d_head;
            const float m = (float)i;
            const int half = rd / 2;
            for (int j = 0; j < half; j++) {
                const float x0 = v[j], x1 = v[j + half];
                const float e = -((2.0f * (float)j) / d);
                const float th = m * powf(10000.0f, e);
                const float c = cosf(th), s = sinf(th);
                const float p0 = x0 * c, p1 = x1 * s, p2 = x0 * s, p3 = x1 * c;
                v[j] = p0 - p1;
                v[j + half] = p2 + p3;
            }
        }
        or_write_row(a, (char*)out + i * rs, dt, n_embd);
    }
    free(a);
}

/* ops.cpp:733-772 silu: x / (1 + exp(-x)) */
void or_silu(const void* x, void* out, int dt, int n_ctx, int n_embd, int start_pos) {
    const long rs = or_row_bytes(dt, n_embd);
    float* a = (float*)malloc(sizeof(float) * (size_t)n_embd);
    for (int r = start_pos; r < n_ctx; r++) {
        or_read_row((const char*)x + r * rs, dt, a, n_embd);
        for (int j = 0; j < n_embd; j++) {
            const float den = 1.0f + expf(-a[j]);
            a[j] = a[j] / den;
        }
        or_write_row(a, (char*)out + r * rs, dt, n_embd);
    }
    free(a);
}

static void binop(const void* a, const void* b, void* out, int dt, int n_ctx, int n, int start_pos, int mul) {
    const long rs = or_row_bytes(dt, n);
    float* x = (float*)malloc(sizeof(float) * 2 * (size_t)n);
    for (int r = start_pos; r < n_ctx; r++) {
        or_read_row((const char*)a + r * rs, dt, x, n);
        or_read_row((const char*)b + r * rs, dt, x + n, n);
        for (int j = 0; j < n; j++) x[j] = mul ? x[j] * x[n + j] : x[j] + x[n + j];
        or_write_row(x, (char*)out + r * rs, dt, n);
    }
    free(x);
}

/* ops.cpp:918-970 multiply */
void or_multiply(const void* a, const void* b, void* out, int dt, int n_ctx, int n_embd, int start_pos) {
    binop(a, b, out, dt, n_ctx, n_embd, start_pos, 1);
}

/* ops.cpp:973-1014 add */
void or_add(const void* a, const void* b, void* out, int dt, int n_ctx, int n_embd, int start_pos) {
    binop(a, b, out, dt, n_ctx, n_embd, start_pos, 0);
}

/* ops.cpp:125-164 scale (in place) */
void or_scale(void* x, int dt, int n_ctx, int n_embd, float s, int start_pos) {
    const long rs = or_row_bytes(dt, n_embd);
    float* a = (float*)malloc(sizeof(float) * (size_t)n_embd);
    for (int r = start_pos; r < n_ctx; r++) {
        or_read_row((char*)x + r * rs, dt, a, n_embd);
        for (int j = 0; j < n_embd; j++) a[j] = a[j] * s;
        or_write_row(a, (char*)x + r * rs, dt, n_embd);
    }
    free(a);
}

/* ops.cpp:639-666 bias_add_inplace: reads the already-requantized row, adds the fp16 bias,
 * requantizes again. */
void or_bias_add_inplace(void* x, int dt, int n_ctx, int n_embd, const uint16_t* bias, int start_pos) {
    const long rs = or_row_bytes(dt, n_embd);
    float* a = (float*)malloc(sizeof(float) * (size_t)n_embd);
    for (int r = start_pos; r < n_ctx; r++) {
        or_read_row((char*)x + r * rs, dt, a, n_embd);
        for (int j = 0; j < n_embd; j++) a[j] = a[j] + or_fp16_to_fp32(bias[j]);
        or_write_row(a, (char*)x + r * rs, dt, n_embd);
    }
    free(a);
}

/* ops.cpp:526-576 token_embed / copy_row: Q8 and fp16 rows are copied, Q4 rows are dequantized
 * and requantized to Q8. */
void or_token_embed(const void* w, int wdt, int n_vocab, int n_embd, const int32_t* tokens, int n_ctx, void* out,
                    int odt, int start_pos) {
    (void)n_vocab;
    const long ws = or_row_bytes(wdt, n_embd), os = or_row_bytes(odt, n_embd);
    float* a = (float*)malloc(sizeof(float) * (size_t)n_embd);
    for (int i = start_pos; i < n_ctx; i++) {
        const char* src = (const char*)w + (long)tokens[i] * ws;
        if (wdt == OR_Q4) {
            or_read_row(src, OR_Q4, a, n_embd);
            or_write_row(a, (char*)out + i * os, OR_Q8, n_embd);
        } else {
            memcpy((char*)out + i * os, src, (size_t)ws);
        }
    }
    free(a);
}

/* ops.cpp:1017-1220 qkv_attn: causal softmax(q.k * 1/sqrt(d)) with the probabilities stored in the
 * activation dtype (Q8 blocks of 32 keys from key 0, or fp16), then P.V with the fp32 8-lane dot.
 * Restated with one separate probability row per (head, query) (the reference's qk buffer uses
 * element strides as byte offsets, ops.cpp:1033-1034,1083; callers size max_ctx so rows do not
 * overlap, and then the two agree). */
void or_qkv_attn(const void* q, const void* k, const void* v, int dt, int n_ctx, int n_head, int q_dim,
                 int kv_dim, void* qkv, int start_pos) {
    const int dh = q_dim / n_head;
    const int kvh = kv_dim / dh;
    const int group = n_head / kvh;
    const long qrs = or_row_bytes(dt, q_dim), krs = or_row_bytes(dt, kv_dim), hs = or_row_bytes(dt, dh);
    const float scale = 1.0f / sqrtf((float)dh);
    float* vt = (float*)malloc(sizeof(float) * (size_t)n_ctx * kv_dim); /* transpose_v, :1091-1132 */
    float* row = (float*)malloc(sizeof(float) * (size_t)kv_dim);
    for (int j = 0; j < n_ctx; j++) {
        or_read_row((const char*)v + j * krs, dt, row, kv_dim);
        for (int c = 0; c < kv_dim; c++) vt[(long)c * n_ctx + j] = row[c];
    }
    free(row);
    float* sc = (float*)malloc(sizeof(float) * (size_t)n_ctx);
    void* prow = malloc((size_t)or_row_bytes(dt, n_ctx) + 64);
    float* o = (float*)malloc(sizeof(float) * (size_t)q_dim);
    for (int r = start_pos; r < n_ctx; r++) {
        for (int h = 0; h < n_head; h++) {
            const char* qh = (const char*)q + r * qrs + h * hs;
            const int g = h / group;
            for (int j = 0; j <= r; j++) {
                const float d = or_vec_dot(qh, dt, (const char*)k + j * krs + g * hs, dt, dh, 0);
                sc[j] = d * scale;
            }
            for (int j = r + 1; j < n_ctx; j++) sc[j] = -INFINITY;
            float mx = -INFINITY;
            for (int j = 0; j < n_ctx; j++)
                if (sc[j] > mx) mx = sc[j];
            float sum = 0.0f;
            for (int j = 0; j < n_ctx; j++) {
                const float e = expf(sc[j] - mx);
                sc[j] = e;
                sum += e;
            }
            for (int j = 0; j < n_ctx; j++) sc[j] = sc[j] / sum;
            or_write_row(sc, prow, dt, n_ctx);
            or_read_row(prow, dt, sc, n_ctx); /* qkv_matmul reads the stored row back, :1165 */
            for (int c = 0; c < dh; c++) o[h * dh + c] = dot_f(sc, vt + (long)(g * dh + c) * n_ctx, n_ctx, 0);
        }
        or_write_row(o, (char*)qkv + r * qrs, dt, q_dim);
    }
    free(o);
    free(prow);
    free(sc);
    free(vt);
}

/* sampler.cpp:30-41: first index of the maximum (strict >, starting from -inf). */
int or_argmax(const float* x, int n) {
    float best = -INFINITY;
    int idx = 0;
    for (int j = 0; j < n; j++)
        if (x[j] > best) {
            best = x[j];
            idx = j;
        }
    return idx;
}

/* ------------------------------------------------------------------------------------------
 * Model wiring. Families: 0 llama (TinyLlama: RMSNorm, GQA, full RoPE, separate lm_head),
 * 1 zephyr (LayerNorm+bias, qkv bias, partial RoPE), 2 minicpm (tied embedding, scales),
 * 3 openelm (per-layer heads/FFN, QK RMSNorm, tied embedding).
 * ---------------------------------------------------------------------------------------- */
#define OR_MAX_LAYERS 64
typedef struct {
    const void *wq, *wk, *wv, *wo, *wg, *wu, *wd;
    const uint16_t *bq, *bk, *bv;
    const uint16_t *n1w, *n1b, *n2w, *n2b, *qnw, *knw;
    int nh, nkv, nffn;
    void *kc, *vc; /* KV cache rows [n_ctx, kv_dim] in the activation dtype */
} or_layer;

struct or_model {
    int family, wdt, adt, n_ctx, n_vocab, d, nl, dh;
    float rope_pct;
    const void* emb;
    const void* lm_head;
    const uint16_t *nfw, *nfb;
    or_layer L[OR_MAX_LAYERS];
};

static const int elm_sm_qh[] = {12, 12, 12, 12, 12, 16, 16, 16, 16, 16, 16, 16, 20, 20, 20, 20};
static const int elm_sm_kv[] = {3, 3, 3, 3, 3, 4, 4, 4, 4, 4, 4, 4, 5, 5, 5, 5};
static const int elm_sm_ff[] = {768, 1024, 1280, 1536, 1792, 2048, 2560, 2816, 3072, 3328, 3584, 3840, 4352, 4608, 4864, 5120};
static const int elm_md_qh[] = {12, 12, 12, 16, 16, 16, 16, 16, 16, 16, 20, 20, 20, 20, 20, 20, 24, 24, 24, 24};
static const int elm_md_kv[] = {3, 3, 3, 4, 4, 4, 4, 4, 4, 4, 5, 5, 5, 5, 5, 5, 6, 6, 6, 6};
static const int elm_md_ff[] = {768, 1024, 1280, 1536, 1792, 2304, 2560, 2816, 3072, 3328, 3584, 3840, 4096, 4352, 4608, 5120, 5376, 5632, 5888, 6144};
static const int elm_lg_qh[] = {16, 16, 16, 20, 20, 20, 20, 20, 20, 20, 24, 24, 24, 24, 24, 24, 24, 24, 28, 28, 28, 28, 28, 28, 32, 32, 32, 32};
static const int elm_lg_kv[] = {4, 4, 4, 5, 5, 5, 5, 5, 5, 5, 6, 6, 6, 6, 6, 6, 6, 6, 7, 7, 7, 7, 7, 7, 8, 8, 8, 8};
static const int elm_lg_ff[] = {1024, 1280, 1536, 1792, 2048, 2304, 2560, 2816, 3072, 3328, 3584, 3840, 4096, 4608, 4608, 5120, 5376, 5632, 5888, 6144, 6400, 6656, 6912, 7168, 7424, 7680, 7936, 8192};

/* Configs: tinyllama.h:12-24, zephyr.h:10-23, minicpm.h:9-24, openelm.h:26-51. */
or_model* or_model_new(int kind, int wdt, int n_ctx, const int* dims) {
    or_model* m = (or_model*)calloc(1, sizeof(or_model));
    m->wdt = wdt;
    m->adt = wdt == OR_F16 ? OR_F16 : OR_Q8; /* gten_types.h:40-42 */
    m->n_ctx = n_ctx;
    m->dh = 64;
    m->rope_pct = 1.0f;
    int nh = 0, nkv = 0, nff = 0;
    const int *qh = NULL, *kv = NULL, *ff = NULL;
    switch (kind) {
        case 0: m->family = 0; m->n_vocab = 32003; m->d = 2048; m->nl = 22; nh = 32; nkv = 4; nff = 5632; break;
        case 1: m->family = 1; m->n_vocab = 100352; m->d = 2048; m->nl = 24; nh = 32; nkv = 32; nff = 5632; m->rope_pct = 0.25f; break;
        case 2: m->family = 2; m->n_vocab = 122753; m->d = 2304; m->nl = 40; nh = 36; nkv = 36; nff = 5760; break;
        case 3: m->family = 3; m->n_vocab = 32000; m->d = 1280; m->nl = 16; qh = elm_sm_qh; kv = elm_sm_kv; ff = elm_sm_ff; break;
        case 4: m->family = 3; m->n_vocab = 32000; m->d = 1536; m->nl = 20; qh = elm_md_qh; kv = elm_md_kv; ff = elm_md_ff; break;
        case 5: m->family = 3; m->n_vocab = 32000; m->d = 2048; m->nl = 28; qh = elm_lg_qh; kv = elm_lg_kv; ff = elm_lg_ff; break;
        default:
            m->n_vocab = dims[0]; m->d = dims[1]; m->nl = dims[2]; nh = dims[3]; nkv = dims[4]; nff = dims[5];
            m->family = dims[6];
            if (m->family == 1) m->rope_pct = 0.25f;
    }
    if (m->nl > OR_MAX_LAYERS) { free(m); return NULL; }
    for (int l = 0; l < m->nl; l++) {
        m->L[l].nh = qh ? qh[l] : nh;
        m->L[l].nkv = kv ? kv[l] : nkv;
        m->L[l].nffn = ff ? ff[l] : nff;
        const long kvb = or_row_bytes(m->adt, m->L[l].nkv * m->dh) * n_ctx;
        m->L[l].kc = calloc(1, (size_t)kvb);
        m->L[l].vc = calloc(1, (size_t)kvb);
    }
    return m;
}

void or_model_free(or_model* m) {
    if (!m) return;
    for (int l = 0; l < m->nl; l++) {
        free(m->L[l].kc);
        free(m->L[l].vc);
    }
    free(m);
}

int or_model_n_vocab(const or_model* m) { return m->n_vocab; }

typedef struct { const char* p; const char* end; int err; } cursor;

/* utils.cpp:51-61 read_layer_header + utils.cpp:29-48 read_into_weight: int32 name length +
 * name, twice, then int32 payload size (checked) and the payload. */
static const void* next_rec(cursor* c, long expect) {
    for (int t = 0; t < 2; t++) {
        int32_t n;
        if (c->end - c->p < 4) { c->err = 1; return NULL; }
        memcpy(&n, c->p, 4);
        c->p += 4 + n;
    }
    int32_t sz;
    if (c->end - c->p < 4) { c->err = 1; return NULL; }
    memcpy(&sz, c->p, 4);
    c->p += 4;
    if (sz != expect || c->end - c->p < sz) { c->err = 2; return NULL; }
    const void* r = c->p;
    c->p += sz;
    return r;
}

/* Load orders: tinyllama.cpp:195-251, zephyr.cpp:79-150, minicpm.cpp:113-166, openelm.cpp:201-262 */
int or_model_load(or_model* m, const void* image, long nbytes) {
    cursor c = {(const char*)image, (const char*)image + nbytes, 0};
    int64_t magic;
    if (nbytes < 8) return -1;
    memcpy(&magic, c.p, 8);
    if (magic != 0x454c49464e455447LL) return -1;
    c.p += 8;
    const int d = m->d, wdt = m->wdt;
    m->emb = next_rec(&c, or_row_bytes(wdt, d) * m->n_vocab);
    for (int l = 0; l < m->nl; l++) {
        or_layer* L = &m->L[l];
        const int qd = L->nh * m->dh, kvd = L->nkv * m->dh;
        L->wq = next_rec(&c, or_row_bytes(wdt, d) * qd);
        if (m->family == 1) L->bq = (const uint16_t*)next_rec(&c, 2L * qd);
        L->wk = next_rec(&c, or_row_bytes(wdt, d) * kvd);
        if (m->family == 1) L->bk = (const uint16_t*)next_rec(&c, 2L * kvd);
        L->wv = next_rec(&c, or_row_bytes(wdt, d) * kvd);
        if (m->family == 1) L->bv = (const uint16_t*)next_rec(&c, 2L * kvd);
        L->wo = next_rec(&c, or_row_bytes(wdt, qd) * d);
        L->wg = next_rec(&c, or_row_bytes(wdt, d) * L->nffn);
        L->wu = next_rec(&c, or_row_bytes(wdt, d) * L->nffn);
        L->wd = next_rec(&c, or_row_bytes(wdt, L->nffn) * d);
        if (m->family == 3) {
            L->qnw = (const uint16_t*)next_rec(&c, 2L * m->dh);
            L->knw = (const uint16_t*)next_rec(&c, 2L * m->dh);
        }
        L->n1w = (const uint16_t*)next_rec(&c, 2L * d);
        if (m->family == 1) L->n1b = (const uint16_t*)next_rec(&c, 2L * d);
        L->n2w = (const uint16_t*)next_rec(&c, 2L * d);
        if (m->family == 1) L->n2b = (const uint16_t*)next_rec(&c, 2L * d);
    }
    m->nfw = (const uint16_t*)next_rec(&c, 2L * d);
    if (m->family == 1) m->nfb = (const uint16_t*)next_rec(&c, 2L * d);
    if (m->family == 0 || m->family == 1) m->lm_head = next_rec(&c, or_row_bytes(wdt, d) * m->n_vocab);
    else m->lm_head = m->emb; /* TiedEmbedding::forward_proj, modules.cpp:48-59 */
    return c.err ? -2 : 0;
}

static void norm_rows(const or_model* m, const void* x, const uint16_t* w, const uint16_t* b, void* out, int n,
                      int sp) {
    if (m->family == 1) or_layer_norm(x, m->adt, n, m->d, w, b, out, sp);
    else or_rms_norm(x, m->adt, n, m->d, w, out, sp);
}

/* Model::logits: tinyllama.cpp:122-138 (block :99-104, ffn :88-97), zephyr.cpp:36-76,
 * minicpm.cpp:52-110, openelm.cpp:33-58,103-146; attention modules.cpp:286-315. */
int or_model_logits(or_model* m, const int32_t* tokens, int n, int sp, float* logits) {
    if (n > m->n_ctx || sp < 0 || sp >= n) return -1;
    const int adt = m->adt, wdt = m->wdt, d = m->d, dh = m->dh;
    const long rd = or_row_bytes(adt, d);
    int maxq = 0, maxf = 0;
    for (int l = 0; l < m->nl; l++) {
        if (m->L[l].nh * dh > maxq) maxq = m->L[l].nh * dh;
        if (m->L[l].nffn > maxf) maxf = m->L[l].nffn;
    }
    const long rq = or_row_bytes(adt, maxq), rf = or_row_bytes(adt, maxf);
    char* x = (char*)calloc((size_t)n, (size_t)rd);
    char* a = (char*)calloc((size_t)n, (size_t)rd);
    char* h = (char*)calloc((size_t)n, (size_t)rd);
    char* o = (char*)calloc((size_t)n, (size_t)rd);
    char* q = (char*)calloc((size_t)n, (size_t)rq);
    char* qn = (char*)calloc((size_t)n, (size_t)rq);
    char* att = (char*)calloc((size_t)n, (size_t)rq);
    char* kn = (char*)calloc((size_t)n, (size_t)rq);
    char* g = (char*)calloc((size_t)n, (size_t)rf);
    char* u = (char*)calloc((size_t)n, (size_t)rf);
    const float depth = (float)(1.4f / sqrt(40.0)); /* minicpm.cpp:57: float / std::sqrt(int) */

    or_token_embed(m->emb, wdt, m->n_vocab, d, tokens, n, x, adt, sp);
    if (m->family == 2) or_scale(x, adt, n, d, 12.0f, sp); /* minicpm.cpp:96 */
    for (int l = 0; l < m->nl; l++) {
        or_layer* L = &m->L[l];
        const int qd = L->nh * dh, kvd = L->nkv * dh;
        norm_rows(m, x, L->n1w, L->n1b, a, n, sp);
        or_matmul_2d(a, adt, n, d, L->wq, wdt, qd, q, adt, sp, 0, 0);
        if (L->bq) or_bias_add_inplace(q, adt, n, qd, L->bq, sp);
        or_matmul_2d(a, adt, n, d, L->wk, wdt, kvd, L->kc, adt, sp, 0, 0);
        if (L->bk) or_bias_add_inplace(L->kc, adt, n, kvd, L->bk, sp);
        or_matmul_2d(a, adt, n, d, L->wv, wdt, kvd, L->vc, adt, sp, 0, 0);
        if (L->bv) or_bias_add_inplace(L->vc, adt, n, kvd, L->bv, sp);
        const void* qa = q;
        if (m->family == 3) {
            /* openelm.cpp:44-52: QK RMSNorm (3-D) then non-inplace RoPE. The key path writes the
             * rotated keys back into the cache rows (the reference keeps them in the RoPE
             * module's buffer; only rows >= start_pos change). */
            or_rms_norm_3d(q, adt, n, L->nh, dh, L->qnw, qn, sp);
            or_rms_norm_3d(L->kc, adt, n, L->nkv, dh, L->knw, kn, sp);
            or_rotary_emb(qn, q, adt, n, qd, dh, m->rope_pct, sp);
            or_rotary_emb(kn, L->kc, adt, n, kvd, dh, m->rope_pct, sp);
        } else {
            or_rotary_emb(q, q, adt, n, qd, dh, m->rope_pct, sp);
            or_rotary_emb(L->kc, L->kc, adt, n, kvd, dh, m->rope_pct, sp);
        }
        or_qkv_attn(qa, L->kc, L->vc, adt, n, L->nh, qd, kvd, att, sp);
        or_matmul_2d(att, adt, n, qd, L->wo, wdt, d, o, adt, sp, 0, 0);
        if (m->family == 2) or_scale(o, adt, n, d, depth, sp);
        or_add(x, o, h, adt, n, d, sp);
        norm_rows(m, h, L->n2w, L->n2b, a, n, sp);
        or_matmul_2d(a, adt, n, d, L->wg, wdt, L->nffn, g, adt, sp, 0, 0);
        or_matmul_2d(a, adt, n, d, L->wu, wdt, L->nffn, u, adt, sp, 0, 0);
        or_silu(g, g, adt, n, L->nffn, sp);
        or_multiply(g, u, g, adt, n, L->nffn, sp);
        or_matmul_2d(g, adt, n, L->nffn, L->wd, wdt, d, o, adt, sp, 0, 0);
        if (m->family == 2) or_scale(o, adt, n, d, depth, sp);
        or_add(h, o, x, adt, n, d, sp);
    }
    norm_rows(m, x, m->nfw, m->nfb, a, n, sp);
    if (m->family == 2) or_scale(a, adt, n, d, 1.0f / 9, sp); /* minicpm.cpp:104-105 */
    or_matmul_2d(a, adt, n, d, m->lm_head, wdt, m->n_vocab, logits, OR_F32, n - 1, 1, 0);
    free(x); free(a); free(h); free(o); free(q); free(qn); free(att); free(kn); free(g); free(u);
    return m->n_vocab;
}

/* sampler.cpp:11-53 without the EOS break */
int or_model_greedy(or_model* m, const int32_t* prompt, int n_prompt, int n_gen, int32_t* out_tokens) {
    int32_t* toks = (int32_t*)malloc(sizeof(int32_t) * (size_t)(n_prompt + n_gen));
    float* lg = (float*)malloc(sizeof(float) * (size_t)m->n_vocab);
    memcpy(toks, prompt, sizeof(int32_t) * (size_t)n_prompt);
    int n = n_prompt;
    int rc = 0;
    for (int i = 0; i < n_gen; i++) {
        const int sp = i == 0 ? 0 : n - 1;
        if (or_model_logits(m, toks, n, sp, lg) < 0) { rc = -1; break; }
        const int t = or_argmax(lg, m->n_vocab);
        out_tokens[i] = t;
        toks[n++] = t;
    }
    free(lg);
    free(toks);
    return rc;
}
