// The reference's kernel C-ABI (reference csrc/ops.h:24-74, bound by sardyne/capi.py:79-102) on
// the GPU. Arguments are host pointers, as in the reference: each call stages its inputs into
// device memory on a per-thread stream, runs the CUDA kernels, and copies the results back.
// Weight matrices registered with sdy_weights_register stay resident in the device layout and
// are read in place — the counterpart of the reference reading weights from its mmap.
#include "common.cuh"
#include "fp_ops.cuh"
#include "sardyne_b200.h"

#include <stdarg.h>
#include <string.h>

#include <atomic>
#include <map>
#include <mutex>
#include <vector>

namespace sdy {

// ------------------------------------------------------------------------------ errors

static thread_local std::string tl_error;
static std::atomic<uint64_t> g_launches{0};

void set_error(const char *fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    if (tl_error.empty()) fprintf(stderr, "sardyne_b200: %s\n", buf);
    tl_error = buf;
}
const char *last_error() { return tl_error.c_str(); }
void clear_error() { tl_error.clear(); }
bool cuda_check(cudaError_t e, const char *what, const char *file, int line) {
    if (e == cudaSuccess) return true;
    set_error("%s failed: %s (%s:%d)", what, cudaGetErrorString(e), file, line);
    return false;
}
void note_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }
bool pdl_enabled() {
    static const bool on = getenv("SARDYNE_NO_PDL") == nullptr;
    return on;
}

// ------------------------------------------------------------------------------ staging

struct DevBuf {
    void *p = nullptr;
    size_t cap = 0;
    void *get(size_t n) {
        if (n == 0) n = 16;
        if (n > cap) {
            if (p) cudaFree(p);
            size_t want = std::max(n, cap + cap / 2);
            if (!SDY_CUDA(cudaMalloc(&p, want))) { p = nullptr; cap = 0; return nullptr; }
            cap = want;
        }
        return p;
    }
};

// One per (host thread, device): the reference lets several threads call op_* at once on
// different row ranges (csrc/model_llama.c:569-574), so nothing here is shared between threads.
struct Stage {
    int dev = 0;
    cudaStream_t st = nullptr;
    DevBuf b[6];
};

static Stage *stage() {
    static thread_local std::map<int, Stage *> stages;
    int dev = 0;
    if (!SDY_CUDA(cudaGetDevice(&dev))) return nullptr;
    auto it = stages.find(dev);
    if (it != stages.end()) return it->second;
    Stage *s = new Stage();
    s->dev = dev;
    if (!SDY_CUDA(cudaStreamCreateWithFlags(&s->st, cudaStreamNonBlocking))) { delete s; return nullptr; }
    stages[dev] = s;
    return s;
}

static bool sync(Stage *s) { return SDY_CUDA(cudaStreamSynchronize(s->st)); }

// ------------------------------------------------------------------------------ resident weights

struct Resident {
    const uint8_t *host;
    size_t bytes;
    int dev;
    QMat m;
    uint8_t *slabs;
};
static std::mutex g_reg_mu;
static std::vector<Resident> g_reg;

// Finds a registered matrix holding host row `w` of (type, n_in) on this device.
static bool resident_lookup(const void *w, int type, int n_in, int dev, QMat *m, int64_t *row) {
    std::lock_guard<std::mutex> lk(g_reg_mu);
    const uint8_t *p = (const uint8_t *)w;
    for (const Resident &r : g_reg) {
        if (r.dev != dev || r.m.type != type || r.m.n_in != n_in) continue;
        if (p < r.host || p >= r.host + r.bytes) continue;
        size_t rb = row_bytes(type, n_in);
        if ((size_t)(p - r.host) % rb) continue;
        *m = r.m;
        *row = (int64_t)((size_t)(p - r.host) / rb);
        return true;
    }
    return false;
}

// Device view of host rows [row0, row1) of w: either the resident copy or a staged upload.
// *first is the QMat row that holds host row row0.
static bool weights_view(Stage *s, const void *w, int type, int n_in, int64_t row0, int64_t row1, QMat *m,
                         int64_t *first) {
    int64_t base;
    if (resident_lookup(w, type, n_in, s->dev, m, &base) && base + row1 <= m->n_rows) {
        *first = base + row0;
        return true;
    }
    size_t rb = row_bytes(type, n_in);
    int64_t n = row1 - row0;
    uint8_t *raw = (uint8_t *)s->b[0].get(rb * n);
    QMat q;
    q.type = type;
    q.n_in = n_in;
    q.nb = n_in / block_elems(type);
    q.n_rows = n;
    uint8_t *slabs = (uint8_t *)s->b[1].get(q.bytes());
    if (!raw || !slabs) return false;
    if (!SDY_CUDA(cudaMemcpyAsync(raw, (const uint8_t *)w + rb * row0, rb * n, cudaMemcpyHostToDevice, s->st)))
        return false;
    repack_to_slabs(raw, type, n, n_in, slabs, s->st);
    q.slabs = slabs;
    *m = q;
    *first = 0;
    return true;
}

static void fill_nan(float *out, size_t n) {
    for (size_t i = 0; i < n; i++) out[i] = __builtin_nanf("");
}

}  // namespace sdy

using namespace sdy;

// ------------------------------------------------------------------------------ C-ABI

extern "C" {

const char *engine_version(void) { return "0.0.1"; }

const char *sdy_last_error(void) { return last_error(); }
void sdy_clear_error(void) { clear_error(); }
uint64_t sdy_kernel_launches(void) { return g_launches.load(); }
uint32_t sdy_kernel_status(void) { return qgemm_status() | qmatvec_status(); }

void sdy_kernel_clear_status(void) {
    qgemm_clear_status();
    qmatvec_clear_status();
}

static int g_simd = 1;
int op_simd(void) { return g_simd; }
int op_set_simd(int enable) {
    g_simd = enable ? 1 : 0;
    return g_simd;
}

size_t op_row_size(int type, int n) { return row_bytes(type, n); }

int sdy_weights_register(const void *host, int wtype, int64_t n_rows, int32_t n_in) {
    if (!host || n_rows <= 0 || !is_quant_weight(wtype) || n_in <= 0 || n_in % block_elems(wtype)) {
        set_error("sdy_weights_register: bad arguments (type %d, %lld rows of %d)", wtype, (long long)n_rows, n_in);
        return -1;
    }
    Stage *s = stage();
    if (!s) return -1;
    QMat q;
    q.type = wtype;
    q.n_in = n_in;
    q.nb = n_in / block_elems(wtype);
    q.n_rows = n_rows;
    size_t rb = row_bytes(wtype, n_in);
    uint8_t *slabs = nullptr, *raw = nullptr;
    if (!SDY_CUDA(cudaMalloc(&slabs, q.bytes()))) return -1;
    if (!SDY_CUDA(cudaMalloc(&raw, rb * n_rows))) { cudaFree(slabs); return -1; }
    bool ok = SDY_CUDA(cudaMemcpyAsync(raw, host, rb * n_rows, cudaMemcpyHostToDevice, s->st));
    if (ok) repack_to_slabs(raw, wtype, n_rows, n_in, slabs, s->st);
    ok = ok && sync(s);
    cudaFree(raw);
    if (!ok) { cudaFree(slabs); return -1; }
    q.slabs = slabs;
    std::lock_guard<std::mutex> lk(g_reg_mu);
    g_reg.push_back(Resident{(const uint8_t *)host, rb * n_rows, s->dev, q, slabs});
    return 0;
}

int sdy_weights_unregister(const void *host) {
    std::lock_guard<std::mutex> lk(g_reg_mu);
    for (size_t i = 0; i < g_reg.size(); i++) {
        if (g_reg[i].host == host) {
            cudaFree(g_reg[i].slabs);
            g_reg.erase(g_reg.begin() + i);
            return 0;
        }
    }
    return -1;
}

void op_quantize_rows(int vtype, const float *x, void *xq, int n_in, int t0, int t1) {
    int n = t1 - t0;
    if (n <= 0) return;
    if ((vtype != T_Q8_0 && vtype != T_Q8_K) || n_in % block_elems(vtype)) {
        set_error("op_quantize_rows: bad type %d / n_in %d", vtype, n_in);
        return;
    }
    Stage *s = stage();
    if (!s) return;
    size_t xb = (size_t)n * n_in * 4, rb = row_bytes(vtype, n_in);
    float *dx = (float *)s->b[2].get(xb);
    void *dq = s->b[3].get(xq_bytes(vtype, n_in, n));
    uint8_t *draw = (uint8_t *)s->b[4].get(rb * n);
    if (!dx || !dq || !draw) return;
    XQ q = xq_carve(dq, vtype, n_in, n);
    if (!SDY_CUDA(cudaMemcpyAsync(dx, x + (size_t)t0 * n_in, xb, cudaMemcpyHostToDevice, s->st))) return;
    quantize_rows(vtype, dx, n_in, n, n_in, q, s->st);
    xq_export(q, draw, s->st);
    SDY_CUDA(cudaMemcpyAsync((uint8_t *)xq + rb * t0, draw, rb * n, cudaMemcpyDeviceToHost, s->st));
    sync(s);
}

// Shared by op_matmul_q_rows / op_vec_dot_q / op_matmul: activations already in XQ form on the
// device; computes rows [row0, row1) of every token into host out[t*n_out + j].
static void run_qmatvec(Stage *s, const XQ &q, const void *w, int wtype, int n_tok, int n_in, int n_out, int row0,
                        int row1, float *out) {
    QMat m;
    int64_t first;
    if (!weights_view(s, w, wtype, n_in, row0, row1, &m, &first)) return;
    int64_t n = row1 - row0;
    float *dout = (float *)s->b[5].get((size_t)n * n_tok * 4);
    if (!dout) return;
    qmatvec(m, q, dout, n, first, first + n, first, s->st);
    SDY_CUDA(cudaMemcpy2DAsync(out + row0, (size_t)n_out * 4, dout, (size_t)n * 4, (size_t)n * 4, n_tok,
                               cudaMemcpyDeviceToHost, s->st));
    sync(s);
}

void op_matmul_q_rows(float *out, const void *xq, const void *w, int wtype, int n_tok, int n_in, int n_out, int row0,
                      int row1) {
    if (row1 <= row0 || n_tok <= 0) return;
    if (!is_quant_weight(wtype) || n_in % block_elems(wtype)) {
        set_error("op_matmul_q_rows: unsupported type %d / n_in %d", wtype, n_in);
        return;
    }
    Stage *s = stage();
    if (!s) return;
    int vt = vec_dot_type(wtype);
    size_t xr = row_bytes(vt, n_in) * n_tok;
    uint8_t *draw = (uint8_t *)s->b[4].get(xr);
    void *dq = s->b[3].get(xq_bytes(vt, n_in, n_tok));
    if (!draw || !dq) return;
    XQ q = xq_carve(dq, vt, n_in, n_tok);
    if (!SDY_CUDA(cudaMemcpyAsync(draw, xq, xr, cudaMemcpyHostToDevice, s->st))) return;
    xq_import(vt, draw, n_tok, n_in, q, s->st);
    run_qmatvec(s, q, w, wtype, n_tok, n_in, n_out, row0, row1, out);
}

float op_vec_dot_q(int wtype, const void *w, const void *xq, int n) {
    float r = __builtin_nanf("");
    op_matmul_q_rows(&r, xq, w, wtype, 1, n, 1, 0, 1);
    return r;
}

void op_matmul_rows(float *out, const float *x, const void *w, int wtype, int n_tok, int n_in, int n_out, int row0,
                    int row1) {
    if (row1 <= row0 || n_tok <= 0) return;
    if (!is_float_weight(wtype)) {
        set_error("op_matmul_rows: type %d is not F32/F16/BF16", wtype);
        return;
    }
    Stage *s = stage();
    if (!s) return;
    int64_t n = row1 - row0;
    size_t es = block_bytes(wtype), wb = (size_t)n * n_in * es, xb = (size_t)n_tok * n_in * 4;
    void *dw = s->b[0].get(wb);
    float *dx = (float *)s->b[2].get(xb);
    float *dout = (float *)s->b[5].get((size_t)n * n_tok * 4);
    if (!dw || !dx || !dout) return;
    SDY_CUDA(cudaMemcpyAsync(dw, (const uint8_t *)w + (size_t)row0 * n_in * es, wb, cudaMemcpyHostToDevice, s->st));
    SDY_CUDA(cudaMemcpyAsync(dx, x, xb, cudaMemcpyHostToDevice, s->st));
    fmatmul(dx, n_in, dw, wtype, n_tok, n_in, 0, n, dout, n, 0, s->st);
    SDY_CUDA(cudaMemcpy2DAsync(out + row0, (size_t)n_out * 4, dout, (size_t)n * 4, (size_t)n * 4, n_tok,
                               cudaMemcpyDeviceToHost, s->st));
    sync(s);
}

void op_matmul(float *out, const float *x, const void *w, int wtype, int n_tok, int n_in, int n_out) {
    if (n_tok <= 0 || n_out <= 0) return;
    if (is_float_weight(wtype)) {
        op_matmul_rows(out, x, w, wtype, n_tok, n_in, n_out, 0, n_out);
        return;
    }
    if (!is_quant_weight(wtype) || n_in % block_elems(wtype)) {
        set_error("op_matmul: unsupported type %d / n_in %d", wtype, n_in);
        return;
    }
    Stage *s = stage();
    if (!s) return;
    int vt = vec_dot_type(wtype);
    size_t xb = (size_t)n_tok * n_in * 4;
    float *dx = (float *)s->b[2].get(xb);
    void *dq = s->b[3].get(xq_bytes(vt, n_in, n_tok));
    if (!dx || !dq) return;
    XQ q = xq_carve(dq, vt, n_in, n_tok);
    if (!SDY_CUDA(cudaMemcpyAsync(dx, x, xb, cudaMemcpyHostToDevice, s->st))) return;
    const int gmin = gemm_min_tokens();
    if (gmin <= 0 || n_tok < gmin) {
        // below the tensor-core route: one launch, every CTA quantizing its tokens' rows itself
        // (the same bytes as quantize_rows), so a call is copy in, one kernel, copy out
        QMat m;
        int64_t first;
        if (!weights_view(s, w, wtype, n_in, 0, n_out, &m, &first)) return;
        // a pinned (page-locked, mapped) output buffer is written by the kernel itself, during
        // the kernel, instead of by a copy after it
        cudaPointerAttributes at{};
        const bool direct = cudaPointerGetAttributes(&at, out) == cudaSuccess && at.type == cudaMemoryTypeHost &&
                            at.devicePointer != nullptr;
        if (!direct) cudaGetLastError();  // a plain host pointer: not an error
        float *dout = direct ? (float *)at.devicePointer : (float *)s->b[5].get((size_t)n_out * n_tok * 4);
        if (!dout) return;
        const ActIn act{dx, n_in};
        qmatvec(m, q, dout, n_out, first, first + n_out, first, s->st, nullptr, &act);
        if (!direct)
            SDY_CUDA(cudaMemcpyAsync(out, dout, (size_t)n_out * n_tok * 4, cudaMemcpyDeviceToHost, s->st));
        sync(s);
        return;
    }
    quantize_rows(vt, dx, n_in, n_tok, n_in, q, s->st);
    run_qmatvec(s, q, w, wtype, n_tok, n_in, n_out, 0, n_out, out);
}

void op_row_to_f32(const void *row, int type, float *out, size_t n) {
    if (n == 0) return;
    Stage *s = stage();
    if (!s) return;
    float *dout = (float *)s->b[5].get(n * 4);
    if (!dout) return;
    if (is_float_weight(type)) {
        size_t b = n * block_bytes(type);
        void *d = s->b[0].get(b);
        if (!d) return;
        SDY_CUDA(cudaMemcpyAsync(d, row, b, cudaMemcpyHostToDevice, s->st));
        convert_to_f32(d, type, dout, (int64_t)n, s->st);
    } else if (is_quant_weight(type) && n % block_elems(type) == 0) {
        QMat m;
        int64_t first;
        if (!weights_view(s, row, type, (int)n, 0, 1, &m, &first)) return;
        dequant_rows(m, nullptr, 1, first, dout, (int64_t)n, s->st);
    } else {
        set_error("op_row_to_f32: unsupported type %d / n %zu", type, n);
        fill_nan(out, n);
        return;
    }
    SDY_CUDA(cudaMemcpyAsync(out, dout, n * 4, cudaMemcpyDeviceToHost, s->st));
    sync(s);
}

void op_f16_to_f32_n(const uint16_t *x, float *out, size_t n) { op_row_to_f32(x, T_F16, out, n); }

uint16_t op_f32_to_f16(float f) {
    Stage *s = stage();
    if (!s) return 0x7E00;
    float *d = (float *)s->b[2].get(16);
    uint16_t *h = (uint16_t *)s->b[5].get(16);
    uint16_t r = 0x7E00;
    if (!d || !h) return r;
    SDY_CUDA(cudaMemcpyAsync(d, &f, 4, cudaMemcpyHostToDevice, s->st));
    f32_to_f16(d, h, 1, s->st);
    SDY_CUDA(cudaMemcpyAsync(&r, h, 2, cudaMemcpyDeviceToHost, s->st));
    sync(s);
    return r;
}

// Host-pointer wrappers of the fp32 kernels: stage, run, copy back.
static float *upload(Stage *s, int slot, const float *h, size_t n) {
    float *d = (float *)s->b[slot].get(n * 4);
    if (d && h) SDY_CUDA(cudaMemcpyAsync(d, h, n * 4, cudaMemcpyHostToDevice, s->st));
    return d;
}
static void download(Stage *s, float *h, const float *d, size_t n) {
    SDY_CUDA(cudaMemcpyAsync(h, d, n * 4, cudaMemcpyDeviceToHost, s->st));
    sync(s);
}

void engine_add_f32(const float *a, const float *b, float *out, size_t n) {
    if (!n) return;
    Stage *s = stage();
    if (!s) return;
    float *da = upload(s, 0, a, n), *db = upload(s, 1, b, n), *dc = upload(s, 2, nullptr, n);
    if (!da || !db || !dc) return;
    add(dc, da, db, (int64_t)n, s->st);
    download(s, out, dc, n);
}

float op_dot_f32(const float *a, const float *b, int n) {
    float r = __builtin_nanf("");
    if (n <= 0) return 0.0f;
    Stage *s = stage();
    if (!s) return r;
    float *da = upload(s, 0, a, n), *db = upload(s, 1, b, n), *dr = upload(s, 2, nullptr, 1);
    if (!da || !db || !dr) return r;
    dot(da, db, n, dr, s->st);
    download(s, &r, dr, 1);
    return r;
}

void op_axpy(float *y, float a, const float *x, int n) {
    if (n <= 0) return;
    Stage *s = stage();
    if (!s) return;
    float *dy = upload(s, 0, y, n), *dx = upload(s, 1, x, n);
    if (!dy || !dx) return;
    axpy(dy, a, dx, n, s->st);
    download(s, y, dy, n);
}

void op_rmsnorm(float *out, const float *x, const float *w, int n, float eps) {
    if (n <= 0) return;
    Stage *s = stage();
    if (!s) return;
    float *dx = upload(s, 0, x, n), *dw = upload(s, 1, w, n), *dout = upload(s, 2, nullptr, n);
    if (!dx || !dw || !dout) return;
    rmsnorm(dout, n, dx, n, dw, n, 1, eps, s->st);
    download(s, out, dout, n);
}

void op_softmax(float *x, int n) {
    if (n <= 0) return;
    Stage *s = stage();
    if (!s) return;
    float *dx = upload(s, 0, x, n);
    if (!dx) return;
    softmax(dx, n, n, 1, s->st);
    download(s, x, dx, n);
}

void op_silu_mul(float *gate, const float *up, int n) {
    if (n <= 0) return;
    Stage *s = stage();
    if (!s) return;
    float *dg = upload(s, 0, gate, n), *du = upload(s, 1, up, n);
    if (!dg || !du) return;
    silu_mul(dg, du, n, s->st);
    download(s, gate, dg, n);
}

void op_rope_table(float *cos_out, float *sin_out, int n_pos, int head_dim, float theta) {
    size_t n = (size_t)n_pos * (head_dim / 2);
    if (!n) return;
    Stage *s = stage();
    if (!s) return;
    float *dc = upload(s, 0, nullptr, n), *ds = upload(s, 1, nullptr, n);
    if (!dc || !ds) return;
    rope_table(dc, ds, n_pos, head_dim, theta, s->st);
    SDY_CUDA(cudaMemcpyAsync(cos_out, dc, n * 4, cudaMemcpyDeviceToHost, s->st));
    download(s, sin_out, ds, n);
}

void op_rope(float *x, int n_heads, int head_dim, const float *c, const float *sn, int interleaved) {
    size_t n = (size_t)n_heads * head_dim, h = (size_t)head_dim / 2;
    if (!n) return;
    Stage *s = stage();
    if (!s) return;
    float *dx = upload(s, 0, x, n), *dc = upload(s, 1, c, h), *ds = upload(s, 2, sn, h);
    if (!dx || !dc || !ds) return;
    rope(dx, (int64_t)n, 1, n_heads, head_dim, dc, ds, 0, nullptr, interleaved, s->st);
    download(s, x, dx, n);
}

void op_attention(float *out, const float *q, const float *k_cache, const float *v_cache, int n_head, int n_kv_head,
                  int head_dim, int n_kv, int stride, float *scores) {
    (void)scores;  // the reference's per-call work buffer; the GPU uses its own
    if (n_head <= 0 || n_kv <= 0) return;
    Stage *s = stage();
    if (!s) return;
    size_t qn = (size_t)n_head * head_dim, cn = (size_t)n_kv_head * stride * head_dim;
    float *dq = upload(s, 0, q, qn), *dk = upload(s, 1, k_cache, cn), *dv = upload(s, 2, v_cache, cn);
    float *dout = upload(s, 3, nullptr, qn), *dsc = upload(s, 4, nullptr, (size_t)n_head * stride);
    if (!dq || !dk || !dv || !dout || !dsc) return;
    attention(dout, dq, (int64_t)qn, dk, dv, 1, n_head, n_kv_head, head_dim, 0, nullptr, stride, dsc, n_kv, s->st);
    download(s, out, dout, qn);
}

// ---------------------------------------------------------------------------- device-pointer API

struct sdy_qmat_s {
    QMat m;
    uint8_t *slabs;
};

void *sdy_qmat_upload(const void *host, int wtype, int64_t n_rows, int32_t n_in) {
    if (!host || n_rows <= 0 || !is_quant_weight(wtype) || n_in <= 0 || n_in % block_elems(wtype)) {
        set_error("sdy_qmat_upload: bad arguments (type %d, %lld rows of %d)", wtype, (long long)n_rows, n_in);
        return nullptr;
    }
    Stage *s = stage();
    if (!s) return nullptr;
    sdy_qmat_s *h = new sdy_qmat_s();
    h->m.type = wtype;
    h->m.n_in = n_in;
    h->m.nb = n_in / block_elems(wtype);
    h->m.n_rows = n_rows;
    size_t rb = row_bytes(wtype, n_in);
    uint8_t *raw = nullptr;
    bool ok = SDY_CUDA(cudaMalloc(&h->slabs, h->m.bytes())) && SDY_CUDA(cudaMalloc(&raw, rb * n_rows)) &&
              SDY_CUDA(cudaMemcpyAsync(raw, host, rb * n_rows, cudaMemcpyHostToDevice, s->st));
    if (ok) repack_to_slabs(raw, wtype, n_rows, n_in, h->slabs, s->st);
    ok = ok && sync(s);
    if (raw) cudaFree(raw);
    if (!ok) {
        if (h->slabs) cudaFree(h->slabs);
        delete h;
        return nullptr;
    }
    h->m.slabs = h->slabs;
    return h;
}

void sdy_qmat_free(void *h) {
    if (!h) return;
    cudaFree(((sdy_qmat_s *)h)->slabs);
    delete (sdy_qmat_s *)h;
}

size_t sdy_qmat_bytes(const void *h) { return h ? ((const sdy_qmat_s *)h)->m.bytes() : 0; }

}  // extern "C"

const QMat *sdy::qmat_of(const void *h) { return h ? &((const sdy_qmat_s *)h)->m : nullptr; }

extern "C" {

size_t sdy_xq_bytes(int vtype, int n_in, int n_tok) { return xq_bytes(vtype, n_in, n_tok); }

int sdy_quantize_rows_dev(int vtype, const float *d_x, int n_tok, int n_in, void *d_xq, void *stream) {
    clear_error();
    if ((vtype != T_Q8_0 && vtype != T_Q8_K) || n_in <= 0 || n_in % block_elems(vtype) || n_tok <= 0) {
        set_error("sdy_quantize_rows_dev: bad type %d / n_in %d / n_tok %d", vtype, n_in, n_tok);
        return -1;
    }
    XQ q = xq_carve(d_xq, vtype, n_in, n_tok);
    quantize_rows(vtype, d_x, n_in, n_tok, n_in, q, (cudaStream_t)stream);
    return last_error()[0] ? -1 : 0;
}

int sdy_qmatvec_dev(const void *h, const void *d_xq, int n_tok, float *d_out, int64_t ldo, int64_t row0,
                    int64_t row1, void *stream) {
    clear_error();
    const sdy_qmat_s *w = (const sdy_qmat_s *)h;
    if (!w || row0 < 0 || row1 > w->m.n_rows || row1 < row0 || n_tok <= 0) {
        set_error("sdy_qmatvec_dev: bad arguments");
        return -1;
    }
    XQ q = xq_carve((void *)d_xq, vec_dot_type(w->m.type), w->m.n_in, n_tok);
    qmatvec(w->m, q, d_out, ldo, row0, row1, row0, (cudaStream_t)stream);
    return last_error()[0] ? -1 : 0;
}

int sdy_qmatvec_batch_dev(int n, const void *const *hs, const void *const *d_xq, float *const *d_out, void *stream) {
    clear_error();
    if (n < 1 || n > 8 || !hs || !d_xq || !d_out) {
        set_error("sdy_qmatvec_batch_dev: 1..8 products with their weights, activations and outputs");
        return -1;
    }
    const QMat *w[8];
    XQ q[8];
    const XQ *qp[8];
    for (int i = 0; i < n; i++) {
        const sdy_qmat_s *h = (const sdy_qmat_s *)hs[i];
        if (!h || !d_xq[i] || !d_out[i]) {
            set_error("sdy_qmatvec_batch_dev: product %d: null argument", i);
            return -1;
        }
        w[i] = &h->m;
        q[i] = xq_carve((void *)d_xq[i], vec_dot_type(h->m.type), h->m.n_in, 1);
        qp[i] = &q[i];
    }
    qmatvec_batch(n, w, qp, d_out, (cudaStream_t)stream);
    return last_error()[0] ? -1 : 0;
}

int sdy_qmatvec_batch_f32_dev(int n, const void *const *hs, const float *const *d_x, float *const *d_out,
                              void *stream) {
    clear_error();
    if (n < 1 || n > 8 || !hs || !d_x || !d_out) {
        set_error("sdy_qmatvec_batch_f32_dev: 1..8 products with their weights, inputs and outputs");
        return -1;
    }
    const QMat *w[8];
    XQ q[8];
    const XQ *qp[8];
    ActIn act[8];
    for (int i = 0; i < n; i++) {
        const sdy_qmat_s *h = (const sdy_qmat_s *)hs[i];
        if (!h || !d_x[i] || !d_out[i]) {
            set_error("sdy_qmatvec_batch_f32_dev: product %d: null argument", i);
            return -1;
        }
        if (((uintptr_t)d_x[i] & 15) || h->m.n_in % 256) {
            set_error("sdy_qmatvec_batch_f32_dev: product %d: input must be 16-byte aligned, rows of whole "
                      "superblocks", i);
            return -1;
        }
        w[i] = &h->m;
        q[i] = xq_carve(nullptr, vec_dot_type(h->m.type), h->m.n_in, 1);  // geometry only
        qp[i] = &q[i];
        act[i] = ActIn{d_x[i], h->m.n_in};
    }
    qmatvec_batch(n, w, qp, d_out, (cudaStream_t)stream, act);
    return last_error()[0] ? -1 : 0;
}

int sdy_qmatvec_batch_f32_gather_dev(int n, const void *const *hs, const float *const *d_x, const int64_t *out_off,
                                     int64_t count, void *const *bases, int32_t rank, int32_t world, void *stream) {
    clear_error();
    if (n < 1 || n > 8 || !hs || !d_x || !out_off || count <= 0 || !bases || world < 1 || world > 8 || rank < 0 ||
        rank >= world) {
        set_error("sdy_qmatvec_batch_f32_gather_dev: bad arguments (1..8 products, 1 <= world <= 8)");
        return -1;
    }
    for (int q = 0; q < world; q++)
        if (!bases[q]) {
            set_error("sdy_qmatvec_batch_f32_gather_dev: buffer of rank %d missing", q);
            return -1;
        }
    // the layout of sdy_allgather_p2p: world * count floats, then the flag words
    const size_t F = align_up((size_t)world * count * 4, 256);
    PeerGatherTail tail;
    tail.rank = rank;
    tail.world = world;
    for (int q = 0; q < world; q++) {
        tail.flags[q] = (unsigned *)((uint8_t *)bases[q] + F);
        if (q != rank) tail.delta[tail.n_peer++] = (int64_t)((uint8_t *)bases[q] - (uint8_t *)bases[rank]);
    }
    tail.done = (unsigned *)((uint8_t *)bases[rank] + F + 128);
    tail.round = (unsigned *)((uint8_t *)bases[rank] + F + 132);
    float *out[8];
    for (int i = 0; i < n; i++) {
        const sdy_qmat_s *h = (const sdy_qmat_s *)hs[i];
        if (!h || out_off[i] < 0 || out_off[i] + h->m.n_rows > count) {
            set_error("sdy_qmatvec_batch_f32_gather_dev: product %d: rows past this rank's %lld-float slice", i,
                      (long long)count);
            return -1;
        }
        out[i] = (float *)bases[rank] + (size_t)rank * count + out_off[i];
    }
    const QMat *w[8];
    XQ q[8];
    const XQ *qp[8];
    ActIn act[8];
    for (int i = 0; i < n; i++) {
        const sdy_qmat_s *h = (const sdy_qmat_s *)hs[i];
        if (!d_x[i] || ((uintptr_t)d_x[i] & 15) || h->m.n_in % 256) {
            set_error("sdy_qmatvec_batch_f32_gather_dev: product %d: input must be 16-byte aligned, rows of whole "
                      "superblocks", i);
            return -1;
        }
        w[i] = &h->m;
        q[i] = xq_carve(nullptr, vec_dot_type(h->m.type), h->m.n_in, 1);
        qp[i] = &q[i];
        act[i] = ActIn{d_x[i], h->m.n_in};
    }
    qmatvec_batch(n, w, qp, out, (cudaStream_t)stream, act, world > 1 ? &tail : nullptr);
    return last_error()[0] ? -1 : 0;
}

}  // extern "C"
