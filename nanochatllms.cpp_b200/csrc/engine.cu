// Model engine: the four reference model families (src/tinyllama, src/zephyr, src/minicpm,
// src/openelm) on the B200 kernels, behind gtn_model_* (include/gten_b200.h).
//
// HBM layout. All weights live in one arena in the reference's block format. Per layer the q/k/v
// weights are stacked row-wise into one [q_dim + 2*kv_dim, d] matrix and gate/up into one
// [2*ffn, d] matrix, so each is streamed by one matmul launch; rows keep the reference layout and
// the stacked outputs are split at multiples of 32 columns, so requantizing each slice equals
// requantizing each Linear's output (modules.cpp:89-104). Row strides are padded to 16 bytes
// where the reference row size is not a multiple of 16 (MiniCPM's 5760-wide down projection), and
// every tensor is followed by 64 bytes of padding, which the TMA tile reads may touch.
// The KV cache of layer l is the K/V Linear activation buffer of the reference (modules.cpp:78-87):
// [max_batch][max_ctx][kv_dim] rows in the activation dtype, post-RoPE keys.
// Activations of the rows being computed use local row indices 0..M-1.
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <cmath>
#include <cstring>
#include <memory>
#include <thread>
#include <vector>

#include "fused.cuh"
#include "launch.cuh"

namespace gtn {

struct Layer {
    int nh = 0, nkv = 0, nffn = 0;
    const uint8_t *wqkv = nullptr, *wo = nullptr, *wgu = nullptr, *wd = nullptr;
    long rs_d = 0, rs_q = 0, rs_f = 0;  // weight row strides for inputs of width d, q_dim, ffn
    const uint16_t *bq = nullptr, *bk = nullptr, *bv = nullptr;
    const uint16_t *n1w = nullptr, *n1b = nullptr, *n2w = nullptr, *n2b = nullptr, *qnw = nullptr, *knw = nullptr;
    uint8_t *kc = nullptr, *vc = nullptr;
};

}  // namespace gtn

struct gtn_model {
    int kind = 0, family = 0, wdt = 0, adt = 0, max_ctx = 0, max_batch = 0;
    int n_vocab = 0, d = 0, nl = 0, dh = 64;
    float rope_pct = 1.0f;
    int rd = 64;
    std::vector<gtn::Layer> L;
    uint8_t* arena = nullptr;
    size_t arena_bytes = 0;
    const uint8_t *emb = nullptr, *lm_head = nullptr;
    long emb_rs = 0;
    const uint16_t *nfw = nullptr, *nfb = nullptr;
    bool loaded = false;
    // activations, capacity max_rows local rows
    int max_rows = 0, max_q = 0, max_kv = 0, max_ffn = 0;
    uint8_t *x = nullptr, *a = nullptr, *h = nullptr, *o = nullptr, *q = nullptr, *qn = nullptr, *att = nullptr;
    uint8_t *g = nullptr, *u = nullptr, *kn = nullptr;
    uint8_t *kr = nullptr, *vr = nullptr;  // new K / V rows of a prefill, reference layout
    long kv_rs = 0;                        // KV cache row stride (att_kv_rs: one padded head row)
    float* y = nullptr;
    gtn::TcScratch tcs;  // expanded activation image of the tensor-core GEMM (Q8/Q4 weights)
    float* logits = nullptr;
    int32_t* tok = nullptr;
    int32_t* next = nullptr;
    int32_t* gen = nullptr;
    float2* rope = nullptr;
    cudaStream_t st = nullptr;
    std::vector<void*> allocs;
    // fused decode step (Q8/Q4 weights, families 0-2): per-sequence device positions, residual
    // rows (x after attention input, h after attention), stacked projection outputs
    bool fused = false;
    int* pos = nullptr;
    uint8_t *rx = nullptr, *rh = nullptr, *datt = nullptr, *act = nullptr;
    long act_s = 0;
    float *yqkv = nullptr, *yo = nullptr, *ygu = nullptr, *yd = nullptr;
    long ldqkv = 0, ldgu = 0;
    cudaGraphExec_t graph = nullptr;
    int graph_B = 0;
    long graph_kernels = 0;
    // top-k sampling of gtn_model_generate_topk (s_mt null: greedy); the captured step is keyed on it
    uint32_t* s_mt = nullptr;
    float s_temp = 1.0f;
    int s_topk = 1;
    uint32_t* graph_mt = nullptr;
    float graph_temp = 0.0f;
    int graph_topk = 0;
    int* pos_host = nullptr;  // pinned staging for position uploads
    // continuous batching: slot s holds one sequence between gtn_slot_start and gtn_slot_finish;
    // active[] (device, staged in active_host) tells the decode step which slots to run
    int* active = nullptr;
    int* active_host = nullptr;
    std::vector<int> slot_pos;  // host: position of each active slot's last token (-1: free)
    bool slot_mode = false;     // the captured step runs every slot under the active mask
    bool graph_slots = false;
    // pinned staging of the model upload (allocated by the first load): one buffer, event and
    // stream per upload worker
    uint8_t* stage[8] = {};
    cudaEvent_t stage_ev[8] = {};
    cudaStream_t stage_st[8] = {};
};

namespace gtn {

static const int elm_sm_qh[] = {12, 12, 12, 12, 12, 16, 16, 16, 16, 16, 16, 16, 20, 20, 20, 20};
static const int elm_sm_kv[] = {3, 3, 3, 3, 3, 4, 4, 4, 4, 4, 4, 4, 5, 5, 5, 5};
static const int elm_sm_ff[] = {768, 1024, 1280, 1536, 1792, 2048, 2560, 2816, 3072, 3328, 3584, 3840, 4352, 4608, 4864, 5120};
static const int elm_md_qh[] = {12, 12, 12, 16, 16, 16, 16, 16, 16, 16, 20, 20, 20, 20, 20, 20, 24, 24, 24, 24};
static const int elm_md_kv[] = {3, 3, 3, 4, 4, 4, 4, 4, 4, 4, 5, 5, 5, 5, 5, 5, 6, 6, 6, 6};
static const int elm_md_ff[] = {768, 1024, 1280, 1536, 1792, 2304, 2560, 2816, 3072, 3328, 3584, 3840, 4096, 4352, 4608, 5120, 5376, 5632, 5888, 6144};
static const int elm_lg_qh[] = {16, 16, 16, 20, 20, 20, 20, 20, 20, 20, 24, 24, 24, 24, 24, 24, 24, 24, 28, 28, 28, 28, 28, 28, 32, 32, 32, 32};
static const int elm_lg_kv[] = {4, 4, 4, 5, 5, 5, 5, 5, 5, 5, 6, 6, 6, 6, 6, 6, 6, 6, 7, 7, 7, 7, 7, 7, 8, 8, 8, 8};
static const int elm_lg_ff[] = {1024, 1280, 1536, 1792, 2048, 2304, 2560, 2816, 3072, 3328, 3584, 3840, 4096, 4608, 4608, 5120, 5376, 5632, 5888, 6144, 6400, 6656, 6912, 7168, 7424, 7680, 7936, 8192};

static long pad16(long b) { return (b + 15) & ~15L; }

static int cuda_st(cudaError_t e, const char* what) {
    if (e == cudaSuccess) return GTN_OK;
    return fail(e == cudaErrorMemoryAllocation ? GTN_ERR_OOM : GTN_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

#define ECHK(expr, what)                       \
    do {                                       \
        const int rc_ = cuda_st((expr), what); \
        if (rc_ != GTN_OK) return rc_;         \
    } while (0)

template <typename T>
static int dalloc(gtn_model* m, T** p, size_t bytes) {
    void* v = nullptr;
    ECHK(cudaMalloc(&v, bytes ? bytes : 16), "cudaMalloc");
    m->allocs.push_back(v);
    *p = reinterpret_cast<T*>(v);
    return GTN_OK;
}

// Record reader (utils.cpp:29-61): int32 name length + name, twice, then int32 payload size.
struct Reader {
    const uint8_t* p;
    const uint8_t* end;
    int err = 0;
    const uint8_t* next(long expect) {
        if (err) return nullptr;
        for (int t = 0; t < 2; ++t) {
            int32_t n;
            if (end - p < 4) { err = 1; return nullptr; }
            memcpy(&n, p, 4);
            if (n < 0 || end - p < 4 + (long)n) { err = 1; return nullptr; }
            p += 4 + n;
        }
        int32_t sz;
        if (end - p < 4) { err = 1; return nullptr; }
        memcpy(&sz, p, 4);
        p += 4;
        if (sz != expect || end - p < sz) { err = 2; return nullptr; }
        const uint8_t* r = p;
        p += sz;
        return r;
    }
};

static void free_all(gtn_model* m) {
    for (void* p : m->allocs) cudaFree(p);
    m->allocs.clear();
}

}  // namespace gtn

using namespace gtn;

extern "C" {

int gtn_model_create(int kind, int wdtype, int max_ctx, int max_batch, const int32_t* dims, gtn_model** out) {
    if (!out) return fail(GTN_ERR_ARG, "model_create: out is NULL");
    *out = nullptr;
    if (wdtype != GTN_F16 && wdtype != GTN_Q8 && wdtype != GTN_Q4) return fail(GTN_ERR_ARG, "model_create: wdtype");
    if (max_ctx <= 0 || max_batch <= 0) return fail(GTN_ERR_ARG, "model_create: max_ctx/max_batch");
    std::unique_ptr<gtn_model> m(new gtn_model());
    m->kind = kind;
    m->wdt = wdtype;
    m->adt = wdtype == GTN_F16 ? GTN_F16 : GTN_Q8;  // gten_types.h:40-42
    m->max_ctx = max_ctx;
    m->max_batch = max_batch;
    int nh = 0, nkv = 0, nff = 0;
    const int *qh = nullptr, *kv = nullptr, *ff = nullptr;
    switch (kind) {  // tinyllama.h:12-24, zephyr.h:10-23, minicpm.h:9-24, openelm.h:26-51
        case GTN_MODEL_TINYLLAMA: m->family = 0; m->n_vocab = 32003; m->d = 2048; m->nl = 22; nh = 32; nkv = 4; nff = 5632; break;
        case GTN_MODEL_ZEPHYR: m->family = 1; m->n_vocab = 100352; m->d = 2048; m->nl = 24; nh = 32; nkv = 32; nff = 5632; m->rope_pct = 0.25f; break;
        case GTN_MODEL_MINICPM: m->family = 2; m->n_vocab = 122753; m->d = 2304; m->nl = 40; nh = 36; nkv = 36; nff = 5760; break;
        case GTN_MODEL_OPENELM_SM: m->family = 3; m->n_vocab = 32000; m->d = 1280; m->nl = 16; qh = elm_sm_qh; kv = elm_sm_kv; ff = elm_sm_ff; break;
        case GTN_MODEL_OPENELM_MD: m->family = 3; m->n_vocab = 32000; m->d = 1536; m->nl = 20; qh = elm_md_qh; kv = elm_md_kv; ff = elm_md_ff; break;
        case GTN_MODEL_OPENELM_LG: m->family = 3; m->n_vocab = 32000; m->d = 2048; m->nl = 28; qh = elm_lg_qh; kv = elm_lg_kv; ff = elm_lg_ff; break;
        case GTN_MODEL_CUSTOM:
            if (!dims) return fail(GTN_ERR_ARG, "model_create: custom model needs dims");
            m->n_vocab = dims[0]; m->d = dims[1]; m->nl = dims[2]; nh = dims[3]; nkv = dims[4]; nff = dims[5];
            m->family = dims[6];
            if (m->family < 0 || m->family > 3) return fail(GTN_ERR_ARG, "model_create: family %d", m->family);
            if (m->family == 1) m->rope_pct = 0.25f;
            if (m->n_vocab <= 0 || m->d <= 0 || m->d % 64 || m->nl <= 0 || nh <= 0 || nkv <= 0 || nh % nkv ||
                nff <= 0 || nff % 32)
                return fail(GTN_ERR_ARG, "model_create: invalid custom dims");
            break;
        default: return fail(GTN_ERR_ARG, "model_create: kind %d", kind);
    }
    m->rd = (int)((float)m->dh * m->rope_pct);
    m->L.resize(m->nl);
    for (int l = 0; l < m->nl; ++l) {
        m->L[l].nh = qh ? qh[l] : nh;
        m->L[l].nkv = kv ? kv[l] : nkv;
        m->L[l].nffn = ff ? ff[l] : nff;
        m->max_q = std::max(m->max_q, m->L[l].nh * m->dh);
        m->max_kv = std::max(m->max_kv, m->L[l].nkv * m->dh);
        m->max_ffn = std::max(m->max_ffn, m->L[l].nffn);
    }
    ECHK(cudaStreamCreateWithFlags(&m->st, cudaStreamNonBlocking), "stream");
    // activations: up to max_ctx rows (prefill of a full context)
    m->max_rows = max_ctx;
    const int adt = m->adt;
    const long R = m->max_rows;
    int rc = GTN_OK;
    rc |= dalloc(m.get(), &m->x, R * row_bytes(adt, m->d));
    rc |= dalloc(m.get(), &m->a, R * row_bytes(adt, m->d));
    rc |= dalloc(m.get(), &m->h, R * row_bytes(adt, m->d));
    rc |= dalloc(m.get(), &m->o, R * row_bytes(adt, m->d));
    rc |= dalloc(m.get(), &m->q, R * row_bytes(adt, m->max_q));
    rc |= dalloc(m.get(), &m->qn, R * row_bytes(adt, m->max_q));
    rc |= dalloc(m.get(), &m->att, R * row_bytes(adt, m->max_q));
    rc |= dalloc(m.get(), &m->kn, R * row_bytes(adt, m->max_kv));
    rc |= dalloc(m.get(), &m->kr, R * row_bytes(adt, m->max_kv));
    rc |= dalloc(m.get(), &m->vr, R * row_bytes(adt, m->max_kv));
    rc |= dalloc(m.get(), &m->g, R * row_bytes(adt, m->max_ffn));
    rc |= dalloc(m.get(), &m->u, R * row_bytes(adt, m->max_ffn));
    const long ywidth = std::max<long>(m->max_q + 2L * m->max_kv, 2L * m->max_ffn);
    rc |= dalloc(m.get(), &m->y, sizeof(float) * R * ywidth);
    if (m->wdt == GTN_Q8 || m->wdt == GTN_Q4) {
        // k_gemm_tc's activation image: up to 512 rows per pass (prefill chunks, batched steps)
        const int rows = std::min(512, std::max(m->max_rows, max_batch));
        const int kmax = std::max(m->d, std::max(m->max_q, m->max_ffn));
        m->tcs.bytes = gtn::tc_aimg_bytes(rows, kmax);
        rc |= dalloc(m.get(), &m->tcs.p, m->tcs.bytes);
    }
    rc |= dalloc(m.get(), &m->logits, sizeof(float) * (size_t)m->n_vocab * max_batch);
    // token ids per sequence: max_ctx + 1 slots (the last generated id is recorded, never fed back)
    rc |= dalloc(m.get(), &m->tok, sizeof(int32_t) * (size_t)(max_ctx + 1) * max_batch);
    rc |= dalloc(m.get(), &m->next, sizeof(int32_t) * (size_t)max_batch);
    rc |= dalloc(m.get(), &m->gen, sizeof(int32_t) * (size_t)(max_ctx + 1) * max_batch);
    // KV cache, head-major: [sequence][kv head][position][head row padded to 16 bytes, odd in
    // 16-byte units], so that a run of positions of one head is one contiguous, 16-byte aligned
    // range (one TMA bulk copy) whose rows load without bank conflicts
    m->kv_rs = att_kv_rs(row_bytes(adt, m->dh));
    for (int l = 0; l < m->nl && rc == GTN_OK; ++l) {
        const long kvb = (long)max_batch * m->L[l].nkv * max_ctx * m->kv_rs;
        rc |= dalloc(m.get(), &m->L[l].kc, kvb);
        rc |= dalloc(m.get(), &m->L[l].vc, kvb);
    }
    m->fused = m->dh == 64;
    if (rc == GTN_OK && m->fused) {
        const long B = max_batch;
        m->ldqkv = m->max_q + 2L * m->max_kv;
        m->ldgu = 2L * m->max_ffn;
        rc |= dalloc(m.get(), &m->pos, sizeof(int) * B);
        rc |= dalloc(m.get(), &m->rx, B * row_bytes(adt, m->d));
        rc |= dalloc(m.get(), &m->rh, B * row_bytes(adt, m->d));
        rc |= dalloc(m.get(), &m->datt, B * row_bytes(adt, m->max_q));
        m->act_s = (std::max(row_bytes(adt, m->d), row_bytes(adt, m->max_ffn)) + 15) / 16 * 16;
        rc |= dalloc(m.get(), &m->act, B * m->act_s);
        rc |= dalloc(m.get(), &m->yqkv, sizeof(float) * B * m->ldqkv);
        rc |= dalloc(m.get(), &m->yo, sizeof(float) * B * m->d);
        rc |= dalloc(m.get(), &m->ygu, sizeof(float) * B * m->ldgu);
        rc |= dalloc(m.get(), &m->yd, sizeof(float) * B * m->d);
        if (rc == GTN_OK && cudaMallocHost((void**)&m->pos_host, sizeof(int) * B) != cudaSuccess) rc = GTN_ERR_OOM;
        rc |= dalloc(m.get(), &m->active, sizeof(int) * B);
        if (rc == GTN_OK && cudaMallocHost((void**)&m->active_host, sizeof(int) * B) != cudaSuccess) rc = GTN_ERR_OOM;
        if (rc == GTN_OK) {
            for (int b = 0; b < B; ++b) m->active_host[b] = 0;
            m->slot_pos.assign(B, -1);
        }
    }
    if (rc == GTN_OK && m->rd > 0) {
        auto tab = rope_table_host(max_ctx, m->rd);
        rc = dalloc(m.get(), &m->rope, tab.size() * sizeof(float2));
        if (rc == GTN_OK)
            rc = cuda_st(cudaMemcpy(m->rope, tab.data(), tab.size() * sizeof(float2), cudaMemcpyHostToDevice),
                         "rope table");
    }
    if (rc != GTN_OK) {
        free_all(m.get());
        cudaStreamDestroy(m->st);
        return rc == GTN_ERR_OOM || (rc & GTN_ERR_OOM) ? GTN_ERR_OOM : rc;
    }
    *out = m.release();
    return GTN_OK;
}

void gtn_model_free(gtn_model* m) {
    if (!m) return;
    if (m->st) cudaStreamSynchronize(m->st);
    if (m->graph) cudaGraphExecDestroy(m->graph);
    if (m->pos_host) cudaFreeHost(m->pos_host);
    if (m->active_host) cudaFreeHost(m->active_host);
    for (int i = 0; i < 8; ++i) {
        if (m->stage[i]) cudaFreeHost(m->stage[i]);
        if (m->stage_ev[i]) cudaEventDestroy(m->stage_ev[i]);
        if (m->stage_st[i]) cudaStreamDestroy(m->stage_st[i]);
    }
    free_all(m);
    if (m->arena) cudaFree(m->arena);
    if (m->st) cudaStreamDestroy(m->st);
    delete m;
}

int gtn_model_n_vocab(const gtn_model* m) { return m ? m->n_vocab : 0; }

}  // extern "C"

namespace gtn {

struct LoadPiece {
    const uint8_t* src;  // host bytes of the record (rows of rb bytes, back to back)
    long rows, rb;
    long off;            // arena offset; rows land at a stride of pad16(rb) when rows > 1
};

constexpr int LOAD_WORKERS = 8;
constexpr size_t LOAD_STAGE_BYTES = 8u << 20;

struct LoadChunk {
    const LoadPiece* p;
    long a, b;  // rows [a, b) of a padded piece, or bytes [a, b) of an unpadded one
};

// Host -> arena upload: the records are cut into chunks of at most LOAD_STAGE_BYTES and worker w
// takes chunks w, w + W, ...: it copies the chunk into its pinned buffer (rows placed at the
// arena's padded stride, pad bytes zero), issues the asynchronous copy on its own stream and,
// before refilling the buffer, waits for the event recorded behind that copy. W single-threaded
// host copies run side by side while the copy engines drain the buffers already filled.
// With fd >= 0 the record bytes are read from that file (src - base is the file offset) straight
// into the pinned buffers instead of copied from memory.
static int upload_pieces(gtn_model* m, const std::vector<LoadPiece>& pieces, int fd = -1,
                         const uint8_t* base = nullptr) {
    for (int i = 0; i < LOAD_WORKERS; ++i) {
        if (!m->stage[i]) ECHK(cudaHostAlloc((void**)&m->stage[i], LOAD_STAGE_BYTES, cudaHostAllocDefault), "model_load: staging");
        if (!m->stage_ev[i]) ECHK(cudaEventCreateWithFlags(&m->stage_ev[i], cudaEventDisableTiming), "model_load: staging");
        if (!m->stage_st[i]) ECHK(cudaStreamCreateWithFlags(&m->stage_st[i], cudaStreamNonBlocking), "model_load: staging");
    }
    std::vector<LoadChunk> chunks;
    for (const LoadPiece& p : pieces) {
        const long stride = p.rows > 1 ? pad16(p.rb) : p.rb;
        if (stride == p.rb) {
            const long total = p.rows * p.rb;
            for (long x = 0; x < total; x += (long)LOAD_STAGE_BYTES)
                chunks.push_back({&p, x, std::min(total, x + (long)LOAD_STAGE_BYTES)});
        } else {
            const long per = std::max(1L, (long)LOAD_STAGE_BYTES / stride);
            for (long r = 0; r < p.rows; r += per) chunks.push_back({&p, r, std::min(p.rows, r + per)});
        }
    }
    // the arena clear (model stream) comes before every upload copy
    ECHK(cudaStreamSynchronize(m->st), "model_load");
    int dev = 0;
    ECHK(cudaGetDevice(&dev), "model_load");
    std::vector<cudaError_t> err(LOAD_WORKERS, cudaSuccess);
    auto work = [&](int w) {
        cudaError_t e = cudaSetDevice(dev);
        uint8_t* st = m->stage[w];
        bool pending = false;
        for (size_t c = (size_t)w; c < chunks.size() && e == cudaSuccess; c += LOAD_WORKERS) {
            const LoadChunk& k = chunks[c];
            const LoadPiece& p = *k.p;
            if (pending) e = cudaEventSynchronize(m->stage_ev[w]);
            if (e != cudaSuccess) break;
            const long stride = p.rows > 1 ? pad16(p.rb) : p.rb;
            size_t len;
            uint8_t* dst;
            // the chunk's source bytes are contiguous: bytes [a, b), or rows [a, b) of rb bytes
            const long s0 = stride == p.rb ? k.a : k.a * p.rb;
            const size_t raw = (size_t)(stride == p.rb ? k.b - k.a : (k.b - k.a) * p.rb);
            if (fd >= 0) {
                size_t got = 0;
                while (got < raw) {
                    const ssize_t r = pread(fd, st + got, raw - got, (off_t)(p.src - base + s0 + (long)got));
                    if (r <= 0) break;
                    got += (size_t)r;
                }
                if (got != raw) {
                    e = cudaErrorInvalidValue;
                    break;
                }
            } else {
                memcpy(st, p.src + s0, raw);
            }
            if (stride == p.rb) {
                len = raw;
                dst = m->arena + p.off + k.a;
            } else {  // spread the rows to the padded stride, last row first (in place)
                for (long r = k.b - k.a - 1; r >= 0; --r) {
                    memmove(st + r * stride, st + r * p.rb, (size_t)p.rb);
                    memset(st + r * stride + p.rb, 0, (size_t)(stride - p.rb));
                }
                len = (size_t)((k.b - k.a) * stride);
                dst = m->arena + p.off + k.a * stride;
            }
            e = cudaMemcpyAsync(dst, st, len, cudaMemcpyHostToDevice, m->stage_st[w]);
            if (e == cudaSuccess) e = cudaEventRecord(m->stage_ev[w], m->stage_st[w]);
            pending = true;
        }
        const cudaError_t e2 = cudaStreamSynchronize(m->stage_st[w]);
        err[w] = e != cudaSuccess ? e : e2;
    };
    std::vector<std::thread> th;
    for (int w = 1; w < LOAD_WORKERS; ++w) th.emplace_back(work, w);
    work(0);
    for (auto& t : th) t.join();
    for (int w = 0; w < LOAD_WORKERS; ++w) ECHK(err[w], "model_load: upload");
    return GTN_OK;
}

}  // namespace gtn

extern "C" {

static int load_image(gtn_model* m, const void* host_image, size_t nbytes, int fd);

// load_from_ckpt from a path (the reference opens the .gten file itself, utils.cpp:29-61): the
// file is mapped to parse the record headers; the payload bytes are read from the file straight
// into the pinned upload buffers.
int gtn_model_load_file(gtn_model* m, const char* path) {
    if (!m || !path) return fail(GTN_ERR_ARG, "model_load_file: arguments");
    const int fd = open(path, O_RDONLY);
    if (fd < 0) return fail(GTN_ERR_ARG, "model_load_file: cannot open %s", path);
    struct stat sb;
    if (fstat(fd, &sb) != 0 || sb.st_size < 8) {
        close(fd);
        return fail(GTN_ERR_FORMAT, "model_load_file: %s is not a .gten file", path);
    }
    const size_t n = (size_t)sb.st_size;
    void* map = mmap(nullptr, n, PROT_READ, MAP_PRIVATE, fd, 0);
    if (map == MAP_FAILED) {
        close(fd);
        return fail(GTN_ERR_ARG, "model_load_file: cannot map %s", path);
    }
    const int rc = load_image(m, map, n, fd);
    munmap(map, n);
    close(fd);
    return rc;
}

// load_from_ckpt: tinyllama.cpp:195-251, zephyr.cpp:79-150, minicpm.cpp:113-166, openelm.cpp:201-262.
int gtn_model_load(gtn_model* m, const void* host_image, size_t nbytes) {
    return load_image(m, host_image, nbytes, -1);
}

static int load_image(gtn_model* m, const void* host_image, size_t nbytes, int fd) {
    if (!m || !host_image) return fail(GTN_ERR_ARG, "model_load: arguments");
    const uint8_t* img = (const uint8_t*)host_image;
    int64_t magic = 0;
    if (nbytes < 8) return fail(GTN_ERR_FORMAT, "model_load: truncated header");
    memcpy(&magic, img, 8);
    if (magic != 0x454c49464e455447LL) return fail(GTN_ERR_FORMAT, "model_load: bad magic");
    Reader rd{img + 8, img + nbytes};
    const int d = m->d, wdt = m->wdt, dh = m->dh;
    const bool fam1 = m->family == 1, fam3 = m->family == 3;
    // First pass: locate records and size the arena.
    std::vector<LoadPiece> pieces;
    long off = 0;
    auto place = [&](const uint8_t* src, long rows, long rb) -> long {
        const long o = off;
        pieces.push_back({src, rows, rb, o});
        off += pad16(rows * pad16(rb)) + 64;
        return o;
    };
    // stacked tensors: consecutive pieces share one padded row stride
    auto place_rows = [&](const uint8_t* src, long rows, long rb) -> long {
        const long o = off;
        pieces.push_back({src, rows, rb, o});
        off += rows * pad16(rb);
        return o;
    };
    auto end_stack = [&]() { off = pad16(off) + 64; };
    const long rbd = row_bytes(wdt, d);
    struct LOff { long qkv, o, gu, dn, bq, bk, bv, n1w, n1b, n2w, n2b, qnw, knw; };
    std::vector<LOff> lo(m->nl);
    const uint8_t* emb = rd.next(rbd * m->n_vocab);
    if (!emb) return fail(GTN_ERR_FORMAT, "model_load: embedding record (%d)", rd.err);
    const long emb_off = place(emb, m->n_vocab, rbd);
    for (int l = 0; l < m->nl; ++l) {
        Layer& Ly = m->L[l];
        const int qd = Ly.nh * dh, kvd = Ly.nkv * dh;
        const uint8_t *bq = nullptr, *bk = nullptr, *bv = nullptr;
        const uint8_t* wq = rd.next(rbd * qd);
        if (fam1) bq = rd.next(2L * qd);
        const uint8_t* wk = rd.next(rbd * kvd);
        if (fam1) bk = rd.next(2L * kvd);
        const uint8_t* wv = rd.next(rbd * kvd);
        if (fam1) bv = rd.next(2L * kvd);
        const uint8_t* wo = rd.next(row_bytes(wdt, qd) * d);
        const uint8_t* wg = rd.next(rbd * Ly.nffn);
        const uint8_t* wu = rd.next(rbd * Ly.nffn);
        const uint8_t* wdn = rd.next(row_bytes(wdt, Ly.nffn) * d);
        const uint8_t *qnw = nullptr, *knw = nullptr;
        if (fam3) {
            qnw = rd.next(2L * dh);
            knw = rd.next(2L * dh);
        }
        const uint8_t* n1w = rd.next(2L * d);
        const uint8_t* n1b = fam1 ? rd.next(2L * d) : nullptr;
        const uint8_t* n2w = rd.next(2L * d);
        const uint8_t* n2b = fam1 ? rd.next(2L * d) : nullptr;
        if (rd.err) return fail(GTN_ERR_FORMAT, "model_load: layer %d records (%d)", l, rd.err);
        lo[l].qkv = place_rows(wq, qd, rbd);
        place_rows(wk, kvd, rbd);
        place_rows(wv, kvd, rbd);
        end_stack();
        lo[l].o = place(wo, d, row_bytes(wdt, qd));
        lo[l].gu = place_rows(wg, Ly.nffn, rbd);
        place_rows(wu, Ly.nffn, rbd);
        end_stack();
        lo[l].dn = place(wdn, d, row_bytes(wdt, Ly.nffn));
        lo[l].bq = fam1 ? place(bq, 1, 2L * qd) : -1;
        lo[l].bk = fam1 ? place(bk, 1, 2L * kvd) : -1;
        lo[l].bv = fam1 ? place(bv, 1, 2L * kvd) : -1;
        lo[l].qnw = fam3 ? place(qnw, 1, 2L * dh) : -1;
        lo[l].knw = fam3 ? place(knw, 1, 2L * dh) : -1;
        lo[l].n1w = place(n1w, 1, 2L * d);
        lo[l].n1b = fam1 ? place(n1b, 1, 2L * d) : -1;
        lo[l].n2w = place(n2w, 1, 2L * d);
        lo[l].n2b = fam1 ? place(n2b, 1, 2L * d) : -1;
    }
    const uint8_t* nfw = rd.next(2L * d);
    const uint8_t* nfb = fam1 ? rd.next(2L * d) : nullptr;
    const uint8_t* lmh = (m->family == 0 || m->family == 1) ? rd.next(rbd * m->n_vocab) : nullptr;
    if (rd.err) return fail(GTN_ERR_FORMAT, "model_load: final records (%d)", rd.err);
    const long nfw_off = place(nfw, 1, 2L * d);
    const long nfb_off = fam1 ? place(nfb, 1, 2L * d) : -1;
    const long lmh_off = lmh ? place(lmh, m->n_vocab, rbd) : -1;

    m->loaded = false;
    if (m->arena && m->arena_bytes < (size_t)off) {  // a reload of the same model reuses the arena
        cudaFree(m->arena);
        m->arena = nullptr;
    }
    if (!m->arena) {
        ECHK(cudaMalloc((void**)&m->arena, (size_t)off), "model_load: arena");
        m->arena_bytes = (size_t)off;
    }
    ECHK(cudaMemsetAsync(m->arena, 0, (size_t)off, m->st), "model_load: arena clear");
    {
        const int rc = upload_pieces(m, pieces, fd, img);
        if (rc != GTN_OK) return rc;
    }
    uint8_t* A = m->arena;
    m->emb = A + emb_off;
    m->emb_rs = pad16(rbd);
    for (int l = 0; l < m->nl; ++l) {
        Layer& Ly = m->L[l];
        Ly.wqkv = A + lo[l].qkv;
        Ly.wo = A + lo[l].o;
        Ly.wgu = A + lo[l].gu;
        Ly.wd = A + lo[l].dn;
        Ly.rs_d = pad16(rbd);
        Ly.rs_q = pad16(row_bytes(wdt, Ly.nh * dh));
        Ly.rs_f = pad16(row_bytes(wdt, Ly.nffn));
        Ly.bq = fam1 ? (const uint16_t*)(A + lo[l].bq) : nullptr;
        Ly.bk = fam1 ? (const uint16_t*)(A + lo[l].bk) : nullptr;
        Ly.bv = fam1 ? (const uint16_t*)(A + lo[l].bv) : nullptr;
        Ly.qnw = fam3 ? (const uint16_t*)(A + lo[l].qnw) : nullptr;
        Ly.knw = fam3 ? (const uint16_t*)(A + lo[l].knw) : nullptr;
        Ly.n1w = (const uint16_t*)(A + lo[l].n1w);
        Ly.n1b = fam1 ? (const uint16_t*)(A + lo[l].n1b) : nullptr;
        Ly.n2w = (const uint16_t*)(A + lo[l].n2w);
        Ly.n2b = fam1 ? (const uint16_t*)(A + lo[l].n2b) : nullptr;
    }
    m->nfw = (const uint16_t*)(A + nfw_off);
    m->nfb = fam1 ? (const uint16_t*)(A + nfb_off) : nullptr;
    m->lm_head = lmh ? A + lmh_off : m->emb;  // TiedEmbedding::forward_proj (modules.cpp:48-59)
    m->loaded = true;
    return GTN_OK;
}

}  // extern "C"

namespace gtn {

static cudaError_t rows_op(int op, const uint8_t* a, long as, const uint8_t* b, long bs, uint8_t* out, long os,
                           int dt, int n, int M, float s, const uint16_t* bias, cudaStream_t st) {
    const dim3 grid(((n + 31) / 32 + 3) / 4, M);
    switch (op) {
        case ROP_SILU: return launch_pdl(k_rowop<ROP_SILU>, grid, dim3(128), 0, st, a, as, b, bs, out, os, dt, n, 0, s, bias);
        case ROP_MUL: return launch_pdl(k_rowop<ROP_MUL>, grid, dim3(128), 0, st, a, as, b, bs, out, os, dt, n, 0, s, bias);
        case ROP_ADD: return launch_pdl(k_rowop<ROP_ADD>, grid, dim3(128), 0, st, a, as, b, bs, out, os, dt, n, 0, s, bias);
        case ROP_SCALE: return launch_pdl(k_rowop<ROP_SCALE>, grid, dim3(128), 0, st, a, as, b, bs, out, os, dt, n, 0, s, bias);
        default: return launch_pdl(k_rowop<ROP_BIAS>, grid, dim3(128), 0, st, a, as, b, bs, out, os, dt, n, 0, s, bias);
    }
}

static cudaError_t norm_rows(const gtn_model* m, const uint8_t* x, uint8_t* out, const uint16_t* w, const uint16_t* b,
                             int M, cudaStream_t st) {
    const long rs = row_bytes(m->adt, m->d);
    const size_t smem = 2 * sizeof(float) * m->d;  // values + the exact sum's scratch
    const cudaError_t e = m->family == 1 ? ensure_smem(k_norm<true>, smem) : ensure_smem(k_norm<false>, smem);
    if (e != cudaSuccess) return e;
    if (m->family == 1)
        return launch_pdl(k_norm<true>, dim3(1, M), dim3(512), smem, st, x, rs, 0L, out, rs, 0L, m->adt, m->d, 0, w, b);
    return launch_pdl(k_norm<false>, dim3(1, M), dim3(512), smem, st, x, rs, 0L, out, rs, 0L, m->adt, m->d, 0, w,
                      (const uint16_t*)nullptr);
}

// fp32 columns [c0, c0+n) of Y (row stride ldy) -> rows of `out` in dtype dt (stride os).
static cudaError_t write_cols(const float* Y, long ldy, int c0, int n, uint8_t* out, long os, int dt, int M,
                              cudaStream_t st) {
    return launch_pdl(k_write_rows, dim3(((n + 31) / 32 + 3) / 4, M), dim3(128), 0, st, Y + c0, ldy, out, os, dt, n, 0);
}

// Rows [sp, n) of sequence `seq` (tokens already on the device at m->tok + seq*max_ctx).
// Writes the last row's fp32 logits to m->logits + seq*n_vocab and its argmax to m->next[seq].
// Model::logits, e.g. tinyllama.cpp:122-138 with blocks :99-104 and ffn :88-97; zephyr.cpp:36-76;
// minicpm.cpp:52-110; openelm.cpp:33-58,103-146; SelfAttention::forward modules.cpp:286-315.
static int forward(gtn_model* m, int seq, int n, int sp) {
    cudaStream_t st = m->st;
    const int adt = m->adt, d = m->d, dh = m->dh, M = n - sp;
    const long rd_ = row_bytes(adt, d);
    const float depth = (float)(1.4f / std::sqrt(40.0));  // minicpm.cpp:57
    cudaError_t e = cudaSuccess;
#define GK(expr)                                            \
    do {                                                    \
        e = (expr);                                         \
        if (e != cudaSuccess) return cuda_st(e, #expr);     \
    } while (0)
    const int32_t* toks = m->tok + (long)seq * (m->max_ctx + 1) + sp;
    GK(launch_pdl(k_embed, dim3(((d + 31) / 32 + 3) / 4, M), dim3(128), 0, st, m->emb, m->emb_rs, m->wdt, toks, m->x,
                  rd_, adt, d, 0, m->n_vocab, device_error_word()));
    if (m->family == 2) GK(rows_op(ROP_SCALE, m->x, rd_, nullptr, 0, m->x, rd_, adt, d, M, 12.0f, nullptr, st));
    for (int l = 0; l < m->nl; ++l) {
        Layer& Ly = m->L[l];
        const int qd = Ly.nh * dh, kvd = Ly.nkv * dh, nqkv = qd + 2 * kvd;
        const long rq = row_bytes(adt, qd), rkv = row_bytes(adt, kvd), rf = row_bytes(adt, Ly.nffn);
        const long khs = (long)m->max_ctx * m->kv_rs;  // bytes between kv heads in the cache
        uint8_t* kc = Ly.kc + (long)seq * Ly.nkv * khs;
        uint8_t* vc = Ly.vc + (long)seq * Ly.nkv * khs;
        // the new rows in reference layout, local row 0 = position sp (rope kernels index rows by
        // absolute position, so they get bases shifted by -sp rows)
        uint8_t* kr = m->kr;
        uint8_t* vr = m->vr;
        GK(norm_rows(m, m->x, m->a, Ly.n1w, Ly.n1b, M, st));
        GK(matmul_f32(m->a, rd_, adt, M, Ly.wqkv, Ly.rs_d, m->wdt, nqkv, d, m->y, nqkv, st, true, m->tcs));
        GK(write_cols(m->y, nqkv, 0, qd, m->q, rq, adt, M, st));
        GK(write_cols(m->y, nqkv, qd, kvd, kr, rkv, adt, M, st));
        GK(write_cols(m->y, nqkv, qd + kvd, kvd, vr, rkv, adt, M, st));
        if (Ly.bq) {
            GK(rows_op(ROP_BIAS, m->q, rq, nullptr, 0, m->q, rq, adt, qd, M, 0.0f, Ly.bq, st));
            GK(rows_op(ROP_BIAS, kr, rkv, nullptr, 0, kr, rkv, adt, kvd, M, 0.0f, Ly.bk, st));
            GK(rows_op(ROP_BIAS, vr, rkv, nullptr, 0, vr, rkv, adt, kvd, M, 0.0f, Ly.bv, st));
        }
        const int half = m->rd / 2;
        const long hb = row_bytes(adt, dh);
        if (m->family == 3) {
            // openelm.cpp:44-52: QK RMSNorm over heads, then RoPE into the cache / query buffer.
            GK(launch_pdl(k_norm<false>, dim3(Ly.nh, M), dim3(64), 2 * sizeof(float) * dh, st, (const uint8_t*)m->q, rq,
                          hb, m->qn, rq, hb, adt, dh, 0, Ly.qnw, (const uint16_t*)nullptr));
            GK(launch_pdl(k_norm<false>, dim3(Ly.nkv, M), dim3(64), 2 * sizeof(float) * dh, st,
                          (const uint8_t*)kr, rkv, hb, m->kn, rkv, hb, adt, dh, 0, Ly.knw, (const uint16_t*)nullptr));
            // the rope kernels index rows by absolute position; local buffers get bases shifted by -sp rows
            GK(launch_pdl(k_rope, dim3(Ly.nh, M), dim3(32), 0, st, (const uint8_t*)(m->qn - (long)sp * rq), rq,
                          m->q - (long)sp * rq, rq, adt, qd, dh, half, sp, (const float2*)m->rope, half));
            GK(launch_pdl(k_rope, dim3(Ly.nkv, M), dim3(32), 0, st, (const uint8_t*)(m->kn - (long)sp * rkv), rkv,
                          kr - (long)sp * rkv, rkv, adt, kvd, dh, half, sp, (const float2*)m->rope, half));
        } else if (half > 0) {
            GK(launch_pdl(k_rope, dim3(Ly.nh, M), dim3(32), 0, st, (const uint8_t*)(m->q - (long)sp * rq), rq,
                          m->q - (long)sp * rq, rq, adt, qd, dh, half, sp, (const float2*)m->rope, half));
            GK(launch_pdl(k_rope, dim3(Ly.nkv, M), dim3(32), 0, st, (const uint8_t*)(kr - (long)sp * rkv), rkv,
                          kr - (long)sp * rkv, rkv, adt, kvd, dh, half, sp, (const float2*)m->rope, half));
        }
        GK(launch_pdl(k_kv_scatter, dim3(Ly.nkv, M), dim3(32), 0, st, (const uint8_t*)kr, rkv, kc, khs, m->kv_rs, sp,
                      (int)hb));
        GK(launch_pdl(k_kv_scatter, dim3(Ly.nkv, M), dim3(32), 0, st, (const uint8_t*)vr, rkv, vc, khs, m->kv_rs, sp,
                      (int)hb));
        const size_t asmem = attn_smem(n, adt, dh);
        GK(ensure_smem(k_attn, asmem));
        GK(launch_pdl(k_attn, dim3(Ly.nh, M), dim3(ATT_THREADS), asmem, st, (const uint8_t*)(m->q - (long)sp * rq),
                      rq, (const uint8_t*)kc, m->kv_rs, khs, (const uint8_t*)vc, m->kv_rs, khs,
                      m->att - (long)sp * rq, rq, adt, n, sp, Ly.nh, Ly.nkv, dh, device_error_word()));
        GK(matmul_f32(m->att, rq, adt, M, Ly.wo, Ly.rs_q, m->wdt, d, qd, m->y, d, st, true, m->tcs));
        GK(write_cols(m->y, d, 0, d, m->o, rd_, adt, M, st));
        if (m->family == 2) GK(rows_op(ROP_SCALE, m->o, rd_, nullptr, 0, m->o, rd_, adt, d, M, depth, nullptr, st));
        GK(rows_op(ROP_ADD, m->x, rd_, m->o, rd_, m->h, rd_, adt, d, M, 0.0f, nullptr, st));
        GK(norm_rows(m, m->h, m->a, Ly.n2w, Ly.n2b, M, st));
        GK(matmul_f32(m->a, rd_, adt, M, Ly.wgu, Ly.rs_d, m->wdt, 2 * Ly.nffn, d, m->y, 2L * Ly.nffn, st, true, m->tcs));
        GK(write_cols(m->y, 2L * Ly.nffn, 0, Ly.nffn, m->g, rf, adt, M, st));
        GK(write_cols(m->y, 2L * Ly.nffn, Ly.nffn, Ly.nffn, m->u, rf, adt, M, st));
        GK(rows_op(ROP_SILU, m->g, rf, nullptr, 0, m->g, rf, adt, Ly.nffn, M, 0.0f, nullptr, st));
        GK(rows_op(ROP_MUL, m->g, rf, m->u, rf, m->g, rf, adt, Ly.nffn, M, 0.0f, nullptr, st));
        GK(matmul_f32(m->g, rf, adt, M, Ly.wd, Ly.rs_f, m->wdt, d, Ly.nffn, m->y, d, st, true, m->tcs));
        GK(write_cols(m->y, d, 0, d, m->o, rd_, adt, M, st));
        if (m->family == 2) GK(rows_op(ROP_SCALE, m->o, rd_, nullptr, 0, m->o, rd_, adt, d, M, depth, nullptr, st));
        GK(rows_op(ROP_ADD, m->h, rd_, m->o, rd_, m->x, rd_, adt, d, M, 0.0f, nullptr, st));
    }
    // final norm and lm_head on the last row only (the other rows' logits are never read).
    uint8_t* xl = m->x + (long)(M - 1) * rd_;
    GK(norm_rows(m, xl, m->a, m->nfw, m->nfb, 1, st));
    if (m->family == 2) GK(rows_op(ROP_SCALE, m->a, rd_, nullptr, 0, m->a, rd_, adt, d, 1, 1.0f / 9, nullptr, st));
    float* lg = m->logits + (long)seq * m->n_vocab;
    GK(matmul_f32(m->a, rd_, adt, 1, m->lm_head, m->emb_rs, m->wdt, m->n_vocab, d, lg, m->n_vocab, st));
    GK(launch_pdl(k_argmax, dim3(1), dim3(1024), 0, st, (const float*)lg, m->n_vocab, m->next + seq, 0L, 0L));
#undef GK
    return GTN_OK;
}

static int check_dev_err() {
    const unsigned int v = take_device_error();
    if (v)
        return fail(GTN_ERR_DEVICE, "device-side error code %u (1: a bounded wait expired, 2: token id out of range)",
                    v);
    return GTN_OK;
}

// ---- fused decode step ---------------------------------------------------------------------
// With `dry` set, only the shared-memory attributes of the kernels are configured (so that the
// step can then be captured into a CUDA graph with no non-stream calls inside the capture).
static long g_step_kernels = 0;

template <int WDT, int NW, int MT, int PRO>
static cudaError_t fg_launch(const FArgs& a, cudaStream_t st, bool dry) {
    const size_t smem = fgemv_smem<WDT>(NW, MT, a.K, a.adt, PRO);
    if (dry) return ensure_smem(k_fgemv<WDT, NW, MT, PRO>, smem);
    ++g_step_kernels;
    const dim3 grid((a.N + NW * 8 - 1) / (NW * 8), (a.B + MT - 1) / MT);
    return launch_pdl(k_fgemv<WDT, NW, MT, PRO>, grid, dim3(NW * 32), smem, st, a);
}

template <int WDT, int PRO>
static cudaError_t fg_mt(const FArgs& a, cudaStream_t st, bool dry) {
    const bool big = a.N > 4096;
    if (a.B <= 1) return big ? fg_launch<WDT, 4, 1, PRO>(a, st, dry) : fg_launch<WDT, 1, 1, PRO>(a, st, dry);
    if (a.B <= 2) return big ? fg_launch<WDT, 4, 2, PRO>(a, st, dry) : fg_launch<WDT, 1, 2, PRO>(a, st, dry);
    if (a.B <= 4) return big ? fg_launch<WDT, 4, 4, PRO>(a, st, dry) : fg_launch<WDT, 1, 4, PRO>(a, st, dry);
    return big ? fg_launch<WDT, 4, 8, PRO>(a, st, dry) : fg_launch<WDT, 1, 8, PRO>(a, st, dry);
}

// Residual update + norm of every sequence into m->act: one cluster of PCL CTAs per sequence (the
// row and the sum's scratch: 2K floats of shared memory).
static cudaError_t prep_resnorm(const gtn_model* m, const FArgs& a, bool dry) {
    const size_t csmem = 2 * sizeof(float) * (size_t)a.K;
    if (dry) return ensure_smem(k_prep_cl, csmem);
    ++g_step_kernels;
    return launch_pdl_cluster(k_prep_cl, dim3(PCL, a.B), dim3(PCL_THREADS), csmem, m->st, PCL, a, m->act, m->act_s);
}

// A GEMV whose activation needs a prologue runs it once into m->act (residual + norm: k_prep_cl;
// SwiGLU: k_prep_swiglu); the GEMV then reads that row. (Computing the prologue inside every GEMV
// CTA instead was measured slower: each of ~300 CTAs then redoes every block's requantizations and
// the norm on 8 warps, 20-28 us per GEMV against 8 us for the cluster. Doing the SwiGLU in the
// gate/up GEMV's epilogue, per 32-block by the CTA that completes it, was measured no faster than
// the separate kernel.)
static cudaError_t fgemv(const gtn_model* m, const FArgs& a, int pro, bool dry) {
    FArgs g = a;
    if (pro != PRO_COPY) {
        cudaError_t e;
        if (pro == PRO_RESNORM) {
            e = prep_resnorm(m, a, dry);
        } else if (!dry) {
            ++g_step_kernels;
            const int nbk = (a.K + GTN_QBLK - 1) / GTN_QBLK;
            e = launch_pdl(k_prep_swiglu, dim3((nbk + 31) / 32, a.B), dim3(1024), 0, m->st, a, m->act, m->act_s);
        } else {
            e = cudaSuccess;
        }
        if (e != cudaSuccess) return e;
        g.xin = m->act;
        g.xin_s = m->act_s;
    }
    if (m->wdt == GTN_F16) {  // fp16 weights and activations: the exact 8-lane CUDA-core kernel
        if (!dry) ++g_step_kernels;
        return gemm_f16(g.xin, g.xin_s, g.B, g.W, g.ws, g.N, g.K, g.Y, g.ldy, m->st, dry);
    }
    if (gemv_q_fits(g.B, m->wdt, g.K)) {
        if (!dry) ++g_step_kernels;
        return gemv_q(g.xin, g.xin_s, g.B, g.W, g.ws, m->wdt, g.N, g.K, g.Y, g.ldy, m->st, dry);
    }
    if (gemm_q_fits(g.W, g.ws, g.B, m->wdt, g.K, m->tcs)) {  // batches of 5 or more sequences
        if (!dry) g_step_kernels += tc_fits(g.W, g.ws, g.B, m->wdt, g.K, m->tcs) ? 2 : 1;
        return gemm_q(g.xin, g.xin_s, g.B, g.W, g.ws, m->wdt, g.N, g.K, g.Y, g.ldy, m->st, dry, m->tcs);
    }
    if (m->wdt == GTN_Q8) return fg_mt<GTN_Q8, PRO_COPY>(g, m->st, dry);
    return fg_mt<GTN_Q4, PRO_COPY>(g, m->st, dry);
}

// One greedy decode step for sequences 0..B-1 at positions m->pos[b] (their input tokens are at
// m->tok[b*max_ctx + pos[b]]): the reference's block sequence (tinyllama.cpp:99-104 and the
// siblings) as five kernels per layer, then the lm_head GEMV and the greedy pick.
// The decode loop's bookkeeping for a sampled id of sequence 0 (as k_fargmax does for greedy ids).
static SampleDst sample_dst(gtn_model* m, unsigned int* err) {
    SampleDst sd;
    sd.tok = m->tok;
    sd.gen = m->gen;
    sd.pos = m->pos;
    sd.max_ctx = m->max_ctx + 1;
    sd.err = err;
    return sd;
}

static int decode_step(gtn_model* m, int B, bool dry) {
    cudaStream_t st = m->st;
    const int adt = m->adt, d = m->d, dh = m->dh;
    const float depth = (float)(1.4f / std::sqrt(40.0));  // minicpm.cpp:57
    const bool cpm = m->family == 2;
    unsigned int* err = device_error_word();
    cudaError_t e = cudaSuccess;
#define SK(expr)                                              \
    do {                                                      \
        e = (expr);                                           \
        if (e != cudaSuccess) return cuda_st(e, #expr);       \
    } while (0)
    const int* act_mask = m->slot_mode ? m->active : nullptr;
    FArgs base{};
    base.B = B;
    base.pos = m->pos;
    base.active = act_mask;
    base.adt = adt;
    base.err = err;
    for (int l = 0; l < m->nl; ++l) {
        Layer& Ly = m->L[l];
        const int qd = Ly.nh * dh, kvd = Ly.nkv * dh, nqkv = qd + 2 * kvd;
        const long rkv = row_bytes(adt, kvd);
        FArgs q = base;
        q.K = d;
        if (l == 0) {
            q.emb = m->emb; q.emb_s = m->emb_rs; q.emb_dt = m->wdt; q.tok = m->tok; q.tok_s = m->max_ctx + 1;
            q.n_vocab = m->n_vocab; q.scale_emb = cpm; q.es = 12.0f;
        } else {
            q.xres = m->rh; q.xres_s = row_bytes(adt, d); q.yadd = m->yd; q.yadd_s = d;
            q.scale_y = cpm; q.ys = depth;
        }
        q.xout = m->rx; q.xout_s = row_bytes(adt, d);
        q.nw = Ly.n1w; q.nb = Ly.n1b; q.layer = m->family == 1;
        q.W = Ly.wqkv; q.ws = Ly.rs_d; q.N = nqkv; q.Y = m->yqkv; q.ldy = m->ldqkv;
        SK(fgemv(m, q, PRO_RESNORM, dry));

        AArgs at{};
        at.adt = adt; at.q_heads = Ly.nh; at.kv_heads = Ly.nkv; at.d = dh; at.pos = m->pos;
        at.y = m->yqkv; at.ys = m->ldqkv; at.bq = Ly.bq; at.bk = Ly.bk; at.bv = Ly.bv;
        at.qnw = Ly.qnw; at.knw = Ly.knw;
        at.cs = m->rope; at.half = m->rd / 2; at.kc = Ly.kc; at.vc = Ly.vc; at.kvs = m->kv_rs;
        at.khs = (long)m->max_ctx * m->kv_rs; at.seq_stride = (long)Ly.nkv * at.khs;
        at.out = m->datt; at.os = row_bytes(adt, m->max_q); at.err = err; at.active = act_mask;
        const size_t asm_ = fattn_smem(m->max_ctx, adt, dh);
        if (dry) {
            SK(ensure_smem(k_fattn, asm_));
        } else {
            ++g_step_kernels;
            SK(launch_pdl(k_fattn, dim3(Ly.nh, B), dim3(ATT_THREADS), asm_, st, at));
        }

        FArgs o = base;
        o.K = qd; o.xin = m->datt; o.xin_s = row_bytes(adt, m->max_q);
        o.W = Ly.wo; o.ws = Ly.rs_q; o.N = d; o.Y = m->yo; o.ldy = d;
        SK(fgemv(m, o, PRO_COPY, dry));

        FArgs gu = base;
        gu.K = d; gu.xres = m->rx; gu.xres_s = row_bytes(adt, d); gu.yadd = m->yo; gu.yadd_s = d;
        gu.scale_y = cpm; gu.ys = depth; gu.xout = m->rh; gu.xout_s = row_bytes(adt, d);
        gu.nw = Ly.n2w; gu.nb = Ly.n2b; gu.layer = m->family == 1;
        gu.W = Ly.wgu; gu.ws = Ly.rs_d; gu.N = 2 * Ly.nffn; gu.Y = m->ygu; gu.ldy = m->ldgu;
        SK(fgemv(m, gu, PRO_RESNORM, dry));

        FArgs dn = base;
        dn.K = Ly.nffn; dn.gu = m->ygu; dn.gu_s = m->ldgu;
        dn.W = Ly.wd; dn.ws = Ly.rs_f; dn.N = d; dn.Y = m->yd; dn.ldy = d;
        SK(fgemv(m, dn, PRO_SWIGLU, dry));
    }
    FArgs hd = base;
    hd.K = d; hd.xres = m->rh; hd.xres_s = row_bytes(adt, d); hd.yadd = m->yd; hd.yadd_s = d;
    hd.scale_y = cpm; hd.ys = depth;
    hd.nw = m->nfw; hd.nb = m->nfb; hd.layer = m->family == 1; hd.post = cpm; hd.ps = 1.0f / 9;
    hd.W = m->lm_head; hd.ws = m->emb_rs; hd.N = m->n_vocab; hd.Y = m->logits; hd.ldy = m->n_vocab;
    SK(fgemv(m, hd, PRO_RESNORM, dry));
    if (dry) {
        SK(prepare_topk_sample(m->n_vocab));
    } else {
        ++g_step_kernels;
        if (m->s_mt)
            SK(launch_topk_sample(st, m->logits, m->n_vocab, m->s_temp, m->s_topk, m->s_mt, sample_dst(m, err)));
        else
            SK(launch_pdl(k_fargmax, dim3(B), dim3(1024), 0, st, (const float*)m->logits, (long)m->n_vocab,
                          m->n_vocab, m->tok, m->gen, (long)m->max_ctx + 1, m->pos, m->max_ctx + 1, err, act_mask,
                          m->slot_mode ? m->next : (int32_t*)nullptr));
    }
#undef SK
    return GTN_OK;
}

// Captures decode_step(B) into a CUDA graph (once per B) and launches it.
static int run_step(gtn_model* m, int B) {
    if (!m->graph || m->graph_B != B || m->graph_mt != m->s_mt || m->graph_temp != m->s_temp ||
        m->graph_topk != m->s_topk || m->graph_slots != m->slot_mode) {
        if (m->graph) {
            cudaGraphExecDestroy(m->graph);
            m->graph = nullptr;
        }
        int rc = decode_step(m, B, true);
        if (rc != GTN_OK) return rc;
        cudaGraph_t g = nullptr;
        ECHK(cudaStreamBeginCapture(m->st, cudaStreamCaptureModeThreadLocal), "graph capture");
        g_step_kernels = 0;
        rc = decode_step(m, B, false);
        const cudaError_t ec = cudaStreamEndCapture(m->st, &g);
        if (rc != GTN_OK) {
            if (g) cudaGraphDestroy(g);
            return rc;
        }
        ECHK(ec, "graph capture end");
        const cudaError_t ei = cudaGraphInstantiate(&m->graph, g, 0);
        cudaGraphDestroy(g);
        ECHK(ei, "graph instantiate");
        m->graph_B = B;
        m->graph_slots = m->slot_mode;
        m->graph_mt = m->s_mt;
        m->graph_temp = m->s_temp;
        m->graph_topk = m->s_topk;
        m->graph_kernels = g_step_kernels;
    }
    ECHK(cudaGraphLaunch(m->graph, m->st), "graph launch");
    for (long i = 0; i < m->graph_kernels; ++i) count_launch();
    return GTN_OK;
}

// Sets pos[b] = p for b < B (from pinned host memory, ordered on the model's stream).
static int set_positions(gtn_model* m, int B, int p) {
    ECHK(cudaStreamSynchronize(m->st), "positions");
    for (int b = 0; b < B; ++b) m->pos_host[b] = p;
    ECHK(cudaMemcpyAsync(m->pos, m->pos_host, sizeof(int) * B, cudaMemcpyHostToDevice, m->st), "positions");
    return GTN_OK;
}

// Greedy generation for sequences 0..B-1 whose n_prompt prompt tokens are already in m->tok
// (row b at b*max_ctx): per-sequence prefill with the op-by-op path (it fills the KV cache and
// the last row's logits), the greedy pick, then n_gen-1 fused decode steps replayed from a CUDA
// graph. The generated ids land in m->gen[b*max_ctx + n_prompt + i].
static int generate_fused(gtn_model* m, int B, int n_prompt, int n_gen) {
    m->slot_mode = false;
    for (int b = 0; b < B; ++b) {
        const int rc = forward(m, b, n_prompt, 0);
        if (rc != GTN_OK) return rc;
    }
    int rc = set_positions(m, B, n_prompt - 1);
    if (rc != GTN_OK) return rc;
    if (m->s_mt) {
        ECHK(launch_topk_sample(m->st, m->logits, m->n_vocab, m->s_temp, m->s_topk, m->s_mt,
                                sample_dst(m, device_error_word())),
             "first token");
    } else {
        ECHK(launch_pdl(k_fargmax, dim3(B), dim3(1024), 0, m->st, (const float*)m->logits, (long)m->n_vocab,
                        m->n_vocab, m->tok, m->gen, (long)m->max_ctx + 1, m->pos, m->max_ctx + 1,
                        device_error_word(), (const int*)nullptr, (int32_t*)nullptr),
             "first token");
    }
    for (int i = 1; i < n_gen; ++i) {
        rc = run_step(m, B);
        if (rc != GTN_OK) return rc;
    }
    return GTN_OK;
}

// Greedy loop on the device (sampler.cpp:19-53 without the EOS stop): the prompt is already in
// m->tok; each step's argmax becomes the next input token and is appended to `out` (device).
static int generate_dev(gtn_model* m, int n_prompt, int n_gen, int32_t* out) {
    if (m->fused) {
        const int rc = generate_fused(m, 1, n_prompt, n_gen);
        if (rc != GTN_OK) return rc;
        ECHK(cudaMemcpyAsync(out, m->gen + n_prompt, sizeof(int32_t) * n_gen, cudaMemcpyDeviceToDevice, m->st),
             "out");
        return GTN_OK;
    }
    int n = n_prompt;
    for (int i = 0; i < n_gen; ++i) {
        const int rc = forward(m, 0, n, i == 0 ? 0 : n - 1);
        if (rc != GTN_OK) return rc;
        if (m->s_mt) {  // the sampled id replaces the argmax in m->next
            SampleDst sd;
            sd.out = m->next;
            ECHK(launch_topk_sample(m->st, m->logits, m->n_vocab, m->s_temp, m->s_topk, m->s_mt, sd), "sample");
        }
        if (i + 1 < n_gen)
            ECHK(cudaMemcpyAsync(m->tok + n, m->next, sizeof(int32_t), cudaMemcpyDeviceToDevice, m->st), "next");
        ECHK(cudaMemcpyAsync(out + i, m->next, sizeof(int32_t), cudaMemcpyDeviceToDevice, m->st), "out");
        ++n;
    }
    return GTN_OK;
}

// Sequences started with gtn_slot_start and not finished own their slots' KV rows and positions.
static bool slots_busy(const gtn_model* m) {
    for (int p : m->slot_pos)
        if (p >= 0) return true;
    return false;
}

}  // namespace gtn

extern "C" {

int gtn_model_logits(gtn_model* m, const int32_t* tokens, int n_tokens, int start_pos, float* logits) {
    if (!m || !m->loaded || !tokens || !logits) return fail(GTN_ERR_ARG, "model_logits: arguments");
    if (n_tokens > m->max_ctx) return fail(GTN_ERR_ARG, "model_logits: %d tokens exceed max_ctx %d", n_tokens, m->max_ctx);
    if (slots_busy(m)) return fail(GTN_ERR_ARG, "model_logits: slots are in use (gtn_slot_finish them first)");
    if (start_pos < 0 || start_pos >= n_tokens) return fail(GTN_ERR_ARG, "model_logits: start_pos");
    for (int i = 0; i < n_tokens; ++i)
        if (tokens[i] < 0 || tokens[i] >= m->n_vocab) return fail(GTN_ERR_ARG, "model_logits: token id %d", tokens[i]);
    ECHK(cudaMemcpyAsync(m->tok, tokens, sizeof(int32_t) * n_tokens, cudaMemcpyHostToDevice, m->st), "tokens");
    const int rc = forward(m, 0, n_tokens, start_pos);
    if (rc != GTN_OK) return rc;
    ECHK(cudaMemcpyAsync(logits, m->logits, sizeof(float) * m->n_vocab, cudaMemcpyDeviceToHost, m->st), "logits");
    ECHK(cudaStreamSynchronize(m->st), "model_logits");
    return check_dev_err();
}

int gtn_model_generate(gtn_model* m, const int32_t* prompt, int n_prompt, int n_gen, int32_t* out_tokens) {
    if (!m || !m->loaded || !prompt || !out_tokens || n_prompt <= 0 || n_gen <= 0)
        return fail(GTN_ERR_ARG, "model_generate: arguments");
    if (n_prompt + n_gen - 1 > m->max_ctx) return fail(GTN_ERR_ARG, "model_generate: exceeds max_ctx");
    if (slots_busy(m)) return fail(GTN_ERR_ARG, "model_generate: slots are in use (gtn_slot_finish them first)");
    for (int i = 0; i < n_prompt; ++i)
        if (prompt[i] < 0 || prompt[i] >= m->n_vocab) return fail(GTN_ERR_ARG, "model_generate: token id %d", prompt[i]);
    ECHK(cudaMemcpyAsync(m->tok, prompt, sizeof(int32_t) * n_prompt, cudaMemcpyHostToDevice, m->st), "prompt");
    // generated ids collect on the device and come back in one copy
    if (m->fused) {
        const int rc = generate_fused(m, 1, n_prompt, n_gen);
        if (rc != GTN_OK) return rc;
        ECHK(cudaMemcpyAsync(out_tokens, m->gen + n_prompt, sizeof(int32_t) * n_gen, cudaMemcpyDeviceToHost, m->st),
             "out");
    } else {
        int32_t* tmp = m->gen + 0;
        const int rc = generate_dev(m, n_prompt, n_gen, tmp);
        if (rc != GTN_OK) return rc;
        ECHK(cudaMemcpyAsync(out_tokens, tmp, sizeof(int32_t) * n_gen, cudaMemcpyDeviceToHost, m->st), "out");
    }
    ECHK(cudaStreamSynchronize(m->st), "model_generate");
    return check_dev_err();
}

int gtn_model_generate_topk(gtn_model* m, const int32_t* prompt, int n_prompt, int n_gen, float temp, int top_k,
                            gtn_rng* rng, int32_t* out_tokens) {
    if (!m || !m->loaded || !rng) return fail(GTN_ERR_ARG, "model_generate_topk: arguments");
    int dev = -1;
    cudaGetDevice(&dev);
    if (dev != rng->device)
        return fail(GTN_ERR_ARG, "model_generate_topk: rng lives on device %d, current device %d", rng->device, dev);
    if (!(temp > 0.0f)) return fail(GTN_ERR_ARG, "model_generate_topk: temp must be > 0");
    top_k = top_k < 1000 ? top_k : 1000;  // sampler.cpp:66-67
    temp = temp < 2.0f ? temp : 2.0f;
    if (top_k < 1 || top_k > m->n_vocab)
        return fail(GTN_ERR_ARG, "model_generate_topk: top_k %d outside [1, %d]", top_k, m->n_vocab);
    m->s_mt = rng->state;
    m->s_temp = temp;
    m->s_topk = top_k;
    const int rc = gtn_model_generate(m, prompt, n_prompt, n_gen, out_tokens);
    m->s_mt = nullptr;
    return rc;
}

int gtn_model_generate_batch(gtn_model* m, const int32_t* prompts, int batch, int n_prompt, int n_gen,
                             int32_t* out_tokens) {
    if (!m || !m->loaded || !prompts || !out_tokens || batch <= 0 || n_prompt <= 0 || n_gen <= 0)
        return fail(GTN_ERR_ARG, "model_generate_batch: arguments");
    if (batch > m->max_batch) return fail(GTN_ERR_ARG, "model_generate_batch: batch %d > max_batch %d", batch, m->max_batch);
    if (n_prompt + n_gen - 1 > m->max_ctx) return fail(GTN_ERR_ARG, "model_generate_batch: exceeds max_ctx");
    if (slots_busy(m)) return fail(GTN_ERR_ARG, "model_generate_batch: slots are in use");
    if (!m->fused) return fail(GTN_ERR_ARG, "model_generate_batch: needs a model with 64-wide heads");
    for (long i = 0; i < (long)batch * n_prompt; ++i)
        if (prompts[i] < 0 || prompts[i] >= m->n_vocab) return fail(GTN_ERR_ARG, "model_generate_batch: token id %d", prompts[i]);
    const long ts = m->max_ctx + 1;
    ECHK(cudaMemcpy2DAsync(m->tok, sizeof(int32_t) * ts, prompts, sizeof(int32_t) * n_prompt, sizeof(int32_t) * n_prompt,
                           batch, cudaMemcpyHostToDevice, m->st),
         "prompts");
    const int rc = generate_fused(m, batch, n_prompt, n_gen);
    if (rc != GTN_OK) return rc;
    ECHK(cudaMemcpy2DAsync(out_tokens, sizeof(int32_t) * n_gen, m->gen + n_prompt, sizeof(int32_t) * ts,
                           sizeof(int32_t) * n_gen, batch, cudaMemcpyDeviceToHost, m->st),
         "out");
    ECHK(cudaStreamSynchronize(m->st), "model_generate_batch");
    return check_dev_err();
}

int gtn_model_generate_device(gtn_model* m, const int32_t* prompt, int n_prompt, int n_gen, int32_t* out_tokens) {
    if (!m || !m->loaded || !prompt || !out_tokens || n_prompt <= 0 || n_gen <= 0)
        return fail(GTN_ERR_ARG, "model_generate_device: arguments");
    if (n_prompt + n_gen - 1 > m->max_ctx) return fail(GTN_ERR_ARG, "model_generate_device: exceeds max_ctx");
    if (slots_busy(m)) return fail(GTN_ERR_ARG, "model_generate_device: slots are in use");
    ECHK(cudaMemcpyAsync(m->tok, prompt, sizeof(int32_t) * n_prompt, cudaMemcpyDeviceToDevice, m->st), "prompt");
    return generate_dev(m, n_prompt, n_gen, out_tokens);
}

int gtn_slot_start(gtn_model* m, const int32_t* prompt, int n_prompt, int* slot, int32_t* first_id) {
    if (!m || !m->loaded || !prompt || n_prompt <= 0 || !slot) return fail(GTN_ERR_ARG, "slot_start: arguments");
    if (!m->fused) return fail(GTN_ERR_ARG, "slot_start: needs a model with 64-wide heads");
    if (n_prompt > m->max_ctx) return fail(GTN_ERR_ARG, "slot_start: %d prompt tokens exceed max_ctx %d", n_prompt, m->max_ctx);
    for (int i = 0; i < n_prompt; ++i)
        if (prompt[i] < 0 || prompt[i] >= m->n_vocab) return fail(GTN_ERR_ARG, "slot_start: token id %d", prompt[i]);
    int s = -1;
    for (int b = 0; b < m->max_batch && s < 0; ++b)
        if (m->slot_pos[b] < 0) s = b;
    if (s < 0) return fail(GTN_ERR_ARG, "slot_start: all %d slots are busy", m->max_batch);
    const long ts = m->max_ctx + 1;
    ECHK(cudaMemcpyAsync(m->tok + (long)s * ts, prompt, sizeof(int32_t) * n_prompt, cudaMemcpyHostToDevice, m->st),
         "slot_start: prompt");
    int rc = forward(m, s, n_prompt, 0);  // the prompt's KV rows of slot s and its last logits
    if (rc != GTN_OK) return rc;
    m->pos_host[s] = n_prompt - 1;
    ECHK(cudaMemcpyAsync(m->pos + s, m->pos_host + s, sizeof(int), cudaMemcpyHostToDevice, m->st), "slot_start");
    ECHK(launch_pdl(k_fargmax, dim3(1), dim3(1024), 0, m->st, (const float*)(m->logits + (long)s * m->n_vocab),
                    (long)m->n_vocab, m->n_vocab, m->tok + (long)s * ts, m->gen + (long)s * ts, ts, m->pos + s,
                    m->max_ctx + 1, device_error_word(), (const int*)nullptr, m->next + s),
         "slot_start: first token");
    int32_t id = 0;
    ECHK(cudaMemcpyAsync(&id, m->next + s, sizeof(int32_t), cudaMemcpyDeviceToHost, m->st), "slot_start");
    ECHK(cudaStreamSynchronize(m->st), "slot_start");
    rc = check_dev_err();
    if (rc != GTN_OK) return rc;
    m->slot_pos[s] = n_prompt;
    *slot = s;
    if (first_id) *first_id = id;
    return GTN_OK;
}

int gtn_slots_step(gtn_model* m, int32_t* ids) {
    if (!m || !m->loaded || !ids) return fail(GTN_ERR_ARG, "slots_step: arguments");
    if (!m->fused) return fail(GTN_ERR_ARG, "slots_step: needs a model with 64-wide heads");
    int nact = 0;
    for (int b = 0; b < m->max_batch; ++b) {
        const int p = m->slot_pos[b];
        m->active_host[b] = p >= 0;
        if (p < 0) continue;
        ++nact;
        if (p >= m->max_ctx) return fail(GTN_ERR_ARG, "slots_step: slot %d has reached max_ctx %d", b, m->max_ctx);
    }
    for (int b = 0; b < m->max_batch; ++b) ids[b] = -1;
    if (nact == 0) return GTN_OK;
    ECHK(cudaMemcpyAsync(m->active, m->active_host, sizeof(int) * m->max_batch, cudaMemcpyHostToDevice, m->st),
         "slots_step: mask");
    m->slot_mode = true;
    int rc = run_step(m, m->max_batch);
    if (rc != GTN_OK) return rc;
    ECHK(cudaMemcpyAsync(m->pos_host, m->next, sizeof(int32_t) * m->max_batch, cudaMemcpyDeviceToHost, m->st),
         "slots_step: ids");
    ECHK(cudaStreamSynchronize(m->st), "slots_step");
    rc = check_dev_err();
    if (rc != GTN_OK) return rc;
    for (int b = 0; b < m->max_batch; ++b) {
        if (m->slot_pos[b] < 0) continue;
        ids[b] = m->pos_host[b];
        ++m->slot_pos[b];
    }
    return GTN_OK;
}

int gtn_slot_finish(gtn_model* m, int slot) {
    if (!m || slot < 0 || slot >= m->max_batch) return fail(GTN_ERR_ARG, "slot_finish: slot %d", slot);
    if (m->slot_pos[slot] < 0) return fail(GTN_ERR_ARG, "slot_finish: slot %d is not in use", slot);
    m->slot_pos[slot] = -1;
    m->active_host[slot] = 0;
    return GTN_OK;
}

void* gtn_model_stream(gtn_model* m) { return m ? (void*)m->st : nullptr; }

int gtn_model_check(gtn_model* m) {
    if (!m) return fail(GTN_ERR_ARG, "model_check: NULL");
    ECHK(cudaStreamSynchronize(m->st), "model_check");
    return check_dev_err();
}

}  // extern "C"
