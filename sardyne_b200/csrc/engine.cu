// The reference's model runtime (reference csrc/model_llama.c, API csrc/engine.h:43-72) on the GPU.
//
// engine_model_load reads the GGUF with the gguf_* reader, checks the configuration exactly as
// the reference does (same accepted files, same error messages), and uploads every weight
// matrix once: quantized matrices are repacked into the slab layout (3D expert tensors one
// expert at a time, each padded to whole 8-row groups), float matrices stay as they are, norms
// and biases become f32. engine_ctx_new allocates the device KV cache, the RoPE tables and all
// activation buffers in one arena. engine_eval runs the forward (model_llama.c:757-832) as a
// sequence of CUDA kernels on the context's stream and copies only the logits back.
#include "common.cuh"
#include "fp_ops.cuh"
#include "sardyne_b200.h"

#include <stdarg.h>
#include <string.h>

#include <string>
#include <vector>

namespace sdy {

namespace {

constexpr int MAX_SEQ_LIMIT = 1 << 20;
constexpr int MAX_BATCH_LIMIT = 4096;

void put_err(char *err, size_t len, const char *fmt, ...) {
    if (!err || !len) return;
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(err, len, fmt, ap);
    va_end(ap);
}

// A weight tensor on the device: [n_expert or 1][n_out][n_in].
struct DMat {
    int type = -1;
    int n_in = 0;
    int64_t n_out = 0;
    int n_expert = 0;      // 0: a plain matrix
    QMat q;                // quantized: slabs (each expert padded to gpe groups)
    int64_t gpe = 0;       // groups per expert
    const void *f = nullptr;  // float weights, raw [n_expert][n_out][n_in]
    bool quant() const { return is_quant_weight(type); }
};

struct DLayer {
    float *attn_norm = nullptr, *ffn_norm = nullptr, *bq = nullptr, *bk = nullptr, *bv = nullptr;
    float *q_norm = nullptr, *k_norm = nullptr;
    DMat wq, wk, wv, wo, gate, up, down, gate_inp;
};

const char *LAYER_SUFFIXES[] = {
    "attn_norm.weight", "attn_q.weight", "attn_q.bias", "attn_k.weight", "attn_k.bias", "attn_v.weight",
    "attn_v.bias", "attn_q_norm.weight", "attn_k_norm.weight", "attn_output.weight", "ffn_norm.weight",
    "ffn_gate.weight", "ffn_up.weight", "ffn_down.weight", "ffn_gate_inp.weight", "ffn_gate_exps.weight",
    "ffn_up_exps.weight", "ffn_down_exps.weight",
};

// Tensor names the runtime knows (model_llama.c:128-154): anything else is a model variant it
// cannot run, and loading fails.
bool known_tensor(const char *name, int n_layer) {
    if (!strcmp(name, "token_embd.weight") || !strcmp(name, "output_norm.weight") || !strcmp(name, "output.weight"))
        return true;
    if (strncmp(name, "blk.", 4)) return false;
    const char *p = name + 4;
    if (*p < '0' || *p > '9') return false;
    long idx = 0;
    while (*p >= '0' && *p <= '9') {
        idx = idx * 10 + (*p - '0');
        if (idx >= n_layer) return false;
        p++;
    }
    if (*p++ != '.') return false;
    for (const char *s : LAYER_SUFFIXES)
        if (!strcmp(p, s)) return true;
    return false;
}

bool type_supported(uint32_t t) { return is_quant_weight((int)t) || is_float_weight((int)t); }

}  // namespace
}  // namespace sdy

using namespace sdy;

struct engine_model {
    gguf_file *gf = nullptr;
    engine_model_info info{};
    int dev = 0;
    DMat tok_embd, output;
    float *output_norm = nullptr;
    std::vector<DLayer> layers;
    std::vector<void *> allocs;
    cudaStream_t st = nullptr;
    uint8_t *raw = nullptr;  // upload bounce buffer (load time only)
    size_t raw_cap = 0;
};

struct engine_ctx {
    const engine_model *m = nullptr;
    int max_seq = 0, n_batch = 0, logits_all = 0, n_past = 0, n_logits = 0, n_threads = 0;
    cudaStream_t st = nullptr;
    void *arena = nullptr;
    float *k_cache = nullptr, *v_cache = nullptr, *rope_cos = nullptr, *rope_sin = nullptr;
    float *x = nullptr, *xb = nullptr, *q = nullptr, *k = nullptr, *v = nullptr, *att = nullptr, *hb = nullptr,
          *hb2 = nullptr, *logits = nullptr, *scores = nullptr;
    float *moe_probs = nullptr, *moe_w = nullptr, *moe_g = nullptr, *moe_u = nullptr, *moe_y = nullptr,
          *moe_sum = nullptr;
    int32_t *moe_top = nullptr, *tok_ids = nullptr;
    void *xq_buf[2] = {nullptr, nullptr};  // [0] Q8_0, [1] Q8_K activations
    const float *xq_src[2] = {nullptr, nullptr};
    int xq_n[2] = {0, 0}, xq_in[2] = {0, 0};
    XQ xq[2];
    float *h_logits = nullptr;  // pinned host copy returned by engine_logits
    char err[256] = {0};
};

namespace sdy {
namespace eng {

// ------------------------------------------------------------------------------ metadata

struct Meta {
    const gguf_file *gf;
    std::string arch;
    char *err;
    size_t len;
    int64_t key(const char *suffix) const {
        std::string k = arch + "." + suffix;
        return gguf_find_kv(gf, k.c_str());
    }
    // Required (def < 0) or defaulted integer in 1..2^30; -1 on error (model_llama.c:92-105).
    int64_t integer(const char *suffix, int64_t def) const {
        int64_t i = key(suffix);
        uint64_t v;
        if (i < 0) {
            if (def < 0) put_err(err, len, "metadato mancante: %s.%s", arch.c_str(), suffix);
            return def;
        }
        if (gguf_kv_get_u64(gf, i, &v) || v == 0 || v > (1u << 30)) {
            put_err(err, len, "metadato non valido: %s.%s", arch.c_str(), suffix);
            return -1;
        }
        return (int64_t)v;
    }
    int real(const char *suffix, double def, float *out) const {
        int64_t i = key(suffix);
        double v = def;
        if (i < 0 && def < 0) {
            put_err(err, len, "metadato mancante: %s.%s", arch.c_str(), suffix);
            return -1;
        }
        if (i >= 0 && gguf_kv_get_f64(gf, i, &v)) {
            put_err(err, len, "metadato non valido: %s.%s", arch.c_str(), suffix);
            return -1;
        }
        if (!(v > 0.0) || v > 1e12) {
            put_err(err, len, "valore non valido per %s.%s", arch.c_str(), suffix);
            return -1;
        }
        *out = (float)v;
        return 0;
    }
};

const gguf_tensor *find(const gguf_file *gf, const char *name) {
    int64_t i = gguf_find_tensor(gf, name);
    return i < 0 ? nullptr : gguf_get_tensor(gf, (uint64_t)i);
}

// Same checks and messages as the reference's read_config (model_llama.c:225-319).
int read_config(engine_model *m, char *err, size_t len) {
    const gguf_file *gf = m->gf;
    uint64_t n;
    const char *arch = gguf_kv_get_str(gf, gguf_find_kv(gf, "general.architecture"), &n);
    if (!arch || n == 0 || n >= 32) {
        put_err(err, len, "general.architecture mancante o non valido");
        return -1;
    }
    Meta mt{gf, std::string(arch, n), err, len};
    engine_model_info *in = &m->info;
    if (mt.arch == "llama") in->rope_interleaved = 1;
    else if (mt.arch == "qwen2" || mt.arch == "qwen3" || mt.arch == "qwen3moe") in->rope_interleaved = 0;
    else {
        put_err(err, len, "architettura %s non supportata", mt.arch.c_str());
        return -1;
    }
    const char *scaling = gguf_kv_get_str(gf, mt.key("rope.scaling.type"), &n);
    if ((scaling && !(n == 4 && !memcmp(scaling, "none", 4))) || find(gf, "rope_freqs.weight")) {
        put_err(err, len, "rope scaling (anche 'llama3' via rope_freqs.weight) non supportato");
        return -1;
    }
    int64_t v;
    if ((v = mt.integer("embedding_length", -1)) < 0) return -1;
    in->dim = (int32_t)v;
    if ((v = mt.integer("block_count", -1)) < 0) return -1;
    in->n_layer = (int32_t)v;
    if ((v = mt.integer("feed_forward_length", -1)) < 0) return -1;
    in->ffn_dim = (int32_t)v;
    if (mt.arch == "qwen3moe") {
        if ((v = mt.integer("expert_count", -1)) < 0) return -1;
        in->n_expert = (int32_t)v;
        if ((v = mt.integer("expert_used_count", -1)) < 0) return -1;
        in->n_expert_used = (int32_t)v;
        if (in->n_expert_used > in->n_expert) {
            put_err(err, len, "expert_used_count=%d oltre expert_count=%d", in->n_expert_used, in->n_expert);
            return -1;
        }
        if ((v = mt.integer("expert_feed_forward_length", in->ffn_dim / in->n_expert_used)) <= 0) {
            if (v == 0) put_err(err, len, "dimensione degli esperti nulla");
            return -1;
        }
        in->ffn_exp_dim = (int32_t)v;
        if (in->n_expert_used > 64) {  // moe_combine_kernel orders at most 64 slots per token
            put_err(err, len, "expert_used_count=%d oltre il massimo di 64 di questa build", in->n_expert_used);
            return -1;
        }
    }
    if ((v = mt.integer("attention.head_count", -1)) < 0) return -1;
    in->n_head = (int32_t)v;
    if ((v = mt.integer("attention.head_count_kv", in->n_head)) < 0) return -1;
    in->n_kv_head = (int32_t)v;
    if ((v = mt.integer("attention.key_length", in->dim / in->n_head)) <= 0) {
        if (v == 0) put_err(err, len, "head_dim nullo");
        return -1;
    }
    in->head_dim = (int32_t)v;
    if (mt.integer("attention.value_length", in->head_dim) != in->head_dim) {
        put_err(err, len, "key_length diverso da value_length");
        return -1;
    }
    if (mt.integer("rope.dimension_count", in->head_dim) != in->head_dim) {
        put_err(err, len, "RoPE parziale (rope.dimension_count < head_dim) non supportata");
        return -1;
    }
    if ((v = mt.integer("context_length", 2048)) < 0) return -1;
    in->max_pos = (int32_t)v;
    if (mt.real("attention.layer_norm_rms_epsilon", -1.0, &in->norm_eps)) return -1;
    if (mt.real("rope.freq_base", 10000.0, &in->rope_theta)) return -1;
    if (in->n_head % in->n_kv_head || in->head_dim % 2) {
        put_err(err, len, "teste o head_dim non validi (n_head %% n_kv_head, head_dim pari)");
        return -1;
    }
    const gguf_tensor *emb = find(gf, "token_embd.weight");
    if (!emb || emb->n_dims != 2 || emb->ne[1] == 0 || emb->ne[1] > (1u << 30)) {
        put_err(err, len, "token_embd.weight mancante o non valido");
        return -1;
    }
    in->n_vocab = (int32_t)emb->ne[1];
    in->tied_embeddings = find(gf, "output.weight") == nullptr;
    in->qkv_bias = find(gf, "blk.0.attn_q.bias") != nullptr;
    in->qk_norm = find(gf, "blk.0.attn_q_norm.weight") != nullptr;
    for (uint64_t i = 0; i < gguf_n_tensors(gf); i++) {
        const char *name = gguf_get_tensor(gf, i)->name;
        if (!known_tensor(name, in->n_layer)) {
            put_err(err, len, "tensore non supportato: %s", name);
            return -1;
        }
    }
    return 0;
}

// ------------------------------------------------------------------------------ upload

void *dalloc(engine_model *m, size_t bytes) {
    void *p = nullptr;
    if (!SDY_CUDA(cudaMalloc(&p, bytes ? bytes : 16))) return nullptr;
    m->allocs.push_back(p);
    return p;
}

uint8_t *bounce(engine_model *m, size_t bytes) {
    if (bytes > m->raw_cap) {
        if (m->raw) cudaFree(m->raw);
        m->raw = nullptr;
        m->raw_cap = 0;
        if (!SDY_CUDA(cudaMalloc(&m->raw, bytes))) return nullptr;
        m->raw_cap = bytes;
    }
    return m->raw;
}

// A tensor [n_expert][n_out][n_in] (n_expert 0: a matrix) of a supported type (model_llama.c:163-185).
int get_tensor(engine_model *m, const char *name, int n_in, int64_t n_out, int n_expert, DMat *out, char *err,
               size_t len) {
    const gguf_tensor *t = find(m->gf, name);
    if (!t) {
        put_err(err, len, "tensore mancante: %s", name);
        return -1;
    }
    if (t->n_dims != (n_expert ? 3u : 2u) || t->ne[0] != (uint64_t)n_in || t->ne[1] != (uint64_t)n_out ||
        (n_expert && t->ne[2] != (uint64_t)n_expert)) {
        put_err(err, len, "%s: dimensioni [%llu, %llu, %llu], attese [%d, %lld, %d]", name,
                (unsigned long long)t->ne[0], (unsigned long long)t->ne[1], (unsigned long long)t->ne[2], n_in,
                (long long)n_out, n_expert ? n_expert : 1);
        return -1;
    }
    if (!type_supported(t->type)) {
        put_err(err, len,
                "%s: tipo %s non supportato dal runtime (supportati: F32, F16, BF16, Q8_0, Q4_0, Q5_0, Q4_K, Q6_K)",
                name, gguf_type_name(t->type));
        return -1;
    }
    DMat d;
    d.type = (int)t->type;
    d.n_in = n_in;
    d.n_out = n_out;
    d.n_expert = n_expert;
    int ne = n_expert ? n_expert : 1;
    if (d.quant()) {
        d.q.type = d.type;
        d.q.n_in = n_in;
        d.q.nb = n_in / block_elems(d.type);
        d.q.n_rows = n_out;
        d.gpe = d.q.n_groups();
        size_t per = d.q.bytes();
        uint8_t *slabs = (uint8_t *)dalloc(m, per * ne);
        uint8_t *raw = bounce(m, t->nbytes);
        if (!slabs || !raw) goto oom;
        if (!SDY_CUDA(cudaMemcpyAsync(raw, t->data, t->nbytes, cudaMemcpyHostToDevice, m->st))) goto oom;
        size_t rb = row_bytes(d.type, n_in);
        for (int e = 0; e < ne; e++)
            repack_to_slabs(raw + (size_t)e * n_out * rb, d.type, n_out, n_in, slabs + per * e, m->st);
        d.q.slabs = slabs;
        d.q.n_rows = n_out;
    } else {
        void *f = dalloc(m, t->nbytes);
        if (!f || !SDY_CUDA(cudaMemcpyAsync(f, t->data, t->nbytes, cudaMemcpyHostToDevice, m->st))) goto oom;
        d.f = f;
    }
    if (!SDY_CUDA(cudaStreamSynchronize(m->st))) goto oom;
    *out = d;
    return 0;
oom:
    put_err(err, len, "%s: caricamento sulla GPU fallito (%s)", name, last_error());
    return -1;
}

// A vector of n elements converted to f32 on the device.
int get_vector(engine_model *m, const char *name, int n, float **out, char *err, size_t len) {
    const gguf_tensor *t = find(m->gf, name);
    if (!t) {
        put_err(err, len, "tensore mancante: %s", name);
        return -1;
    }
    if (t->n_dims != 1 || t->ne[0] != (uint64_t)n) {
        put_err(err, len, "%s: dimensione %llu, attesa %d", name, (unsigned long long)t->ne[0], n);
        return -1;
    }
    if (!type_supported(t->type) || is_quant_weight((int)t->type)) {
        put_err(err, len, "%s: tipo %s non supportato", name, gguf_type_name(t->type));
        return -1;
    }
    float *d = (float *)dalloc(m, (size_t)n * 4);
    uint8_t *raw = bounce(m, t->nbytes);
    if (!d || !raw || !SDY_CUDA(cudaMemcpyAsync(raw, t->data, t->nbytes, cudaMemcpyHostToDevice, m->st))) {
        put_err(err, len, "%s: caricamento sulla GPU fallito (%s)", name, last_error());
        return -1;
    }
    convert_to_f32(raw, (int)t->type, d, n, m->st);
    if (!SDY_CUDA(cudaStreamSynchronize(m->st))) return -1;
    *out = d;
    return 0;
}

// ------------------------------------------------------------------------------ small kernels

// x[t] = row tok[t] of a float table (F32/F16/BF16).
__global__ void embed_float_kernel(const void *table, int type, const int32_t *ids, int dim, float *x) {
    int t = blockIdx.x;
    size_t base = (size_t)ids[t] * dim;
    for (int i = threadIdx.x; i < dim; i += blockDim.x) {
        float v;
        if (type == T_F32) v = ((const float *)table)[base + i];
        else if (type == T_F16) v = __half2float(((const __half *)table)[base + i]);
        else v = __uint_as_float((uint32_t)((const uint16_t *)table)[base + i] << 16);
        x[(size_t)t * dim + i] = v;
    }
}

// K and V of n tokens into the cache [n_kv_head][max_seq][hd] at positions pos0.. (model_llama.c:796-799).
__global__ void kv_store_kernel(const float *k, const float *v, int kv_dim, int hd, int max_seq, int pos0, float *kc,
                                float *vc) {
    int t = blockIdx.y;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < kv_dim; i += gridDim.x * blockDim.x) {
        int h = i / hd, j = i % hd;
        size_t dst = ((size_t)h * max_seq + pos0 + t) * hd + j;
        kc[dst] = k[(size_t)t * kv_dim + i];
        vc[dst] = v[(size_t)t * kv_dim + i];
    }
}

// Router selection per token (model_llama.c:653-666): the k most probable experts, ties to the
// lowest index, weights renormalised by their float sum.
__global__ void topk_kernel(const float *probs, int n_tok, int ne, int k, int32_t *top, float *w) {
    int t = blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= n_tok) return;
    const float *p = probs + (size_t)t * ne;
    int32_t *tp = top + (size_t)t * k;
    int n = 0;
    for (int e = 0; e < ne; e++) {
        int pos = n;
        while (pos > 0 && p[e] > p[tp[pos - 1]]) pos--;
        if (pos == k) continue;
        for (int j = n < k ? n : k - 1; j > pos; j--) tp[j] = tp[j - 1];
        tp[pos] = e;
        if (n < k) n++;
    }
    float sum = 0.0f;
    for (int i = 0; i < k; i++) sum = __fadd_rn(sum, p[tp[i]]);
    for (int i = 0; i < k; i++) w[(size_t)t * k + i] = __fdiv_rn(p[tp[i]], sum);
}

// out[t] = sum over t's k slots, in ascending expert order (the order moe_ffn adds them,
// model_llama.c:734-750), of w * y[slot].
__global__ void moe_combine_kernel(const float *y, const int32_t *top, const float *w, int k, int dim, float *out) {
    int t = blockIdx.y;
    int order[64];
    for (int i = 0; i < k; i++) order[i] = i;
    for (int i = 1; i < k; i++) {  // insertion sort of the slots by expert id (k is small)
        int s = order[i], j = i;
        while (j > 0 && top[(size_t)t * k + order[j - 1]] > top[(size_t)t * k + s]) { order[j] = order[j - 1]; j--; }
        order[j] = s;
    }
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < dim; i += gridDim.x * blockDim.x) {
        float acc = 0.0f;
        for (int j = 0; j < k; j++) {
            int s = order[j];
            acc = __fadd_rn(acc, __fmul_rn(w[(size_t)t * k + s], y[((size_t)t * k + s) * dim + i]));
        }
        out[(size_t)t * dim + i] = acc;
    }
}

// Float-weight experts: out[s][r] = E[top[s]][r] . x[s / tok_div], one thread per row, in the
// reference's scalar dot order (four accumulators, csrc/ops.c:155-167).
__global__ void fmatmul_gather_kernel(const void *w, int type, int n_in, int64_t rows, const int32_t *top,
                                      const float *x, int64_t ldx, int tok_div, float *out, int64_t ldo) {
    int s = blockIdx.y;
    int64_t r = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    if (r >= rows) return;
    size_t base = ((size_t)top[s] * rows + r) * n_in;
    const float *xv = x + (size_t)(s / tok_div) * ldx;
    auto wv = [&](int i) -> float {
        if (type == T_F32) return ((const float *)w)[base + i];
        if (type == T_F16) return __half2float(((const __half *)w)[base + i]);
        return __uint_as_float((uint32_t)((const uint16_t *)w)[base + i] << 16);
    };
    float s0 = 0.0f, s1 = 0.0f, s2 = 0.0f, s3 = 0.0f;
    int i = 0;
    for (; i + 4 <= n_in; i += 4) {
        s0 = __fadd_rn(s0, __fmul_rn(xv[i], wv(i)));
        s1 = __fadd_rn(s1, __fmul_rn(xv[i + 1], wv(i + 1)));
        s2 = __fadd_rn(s2, __fmul_rn(xv[i + 2], wv(i + 2)));
        s3 = __fadd_rn(s3, __fmul_rn(xv[i + 3], wv(i + 3)));
    }
    for (; i < n_in; i++) s0 = __fadd_rn(s0, __fmul_rn(xv[i], wv(i)));
    out[(size_t)s * ldo + r] = __fadd_rn(__fadd_rn(s0, s1), __fadd_rn(s2, s3));
}

// ------------------------------------------------------------------------------ forward

// Quantized activations of x for weight type wtype, reused while the input is unchanged
// (model_llama.c:590-611).
const XQ &activations(engine_ctx *c, const float *x, int n, int n_in, int wtype) {
    int vt = vec_dot_type(wtype), s = vt == T_Q8_K ? 1 : 0;
    if (c->xq_src[s] != x || c->xq_n[s] != n || c->xq_in[s] != n_in) {
        c->xq[s] = xq_carve(c->xq_buf[s], vt, n_in, n);
        quantize_rows(vt, x, n_in, n, n_in, c->xq[s], c->st);
        c->xq_src[s] = x;
        c->xq_n[s] = n;
        c->xq_in[s] = n_in;
    }
    return c->xq[s];
}

// out = x . W^T for n tokens (model_llama.c:592-611). new_input: x changed since the last call.
void matmul(engine_ctx *c, float *out, const float *x, const DMat &w, int n, bool new_input) {
    if (new_input) c->xq_src[0] = c->xq_src[1] = nullptr;
    if (!w.quant()) {
        fmatmul(x, w.n_in, w.f, w.type, n, w.n_in, 0, w.n_out, out, w.n_out, 0, c->st);
        return;
    }
    const XQ &xq = activations(c, x, n, w.n_in, w.type);
    qmatvec(w.q, xq, out, w.n_out, 0, w.n_out, 0, c->st);
}

// Gathered experts: out[s] = E[top[s]] . x[s / tok_div] for n_slots slots.
void matmul_experts(engine_ctx *c, float *out, const float *x, int n_x, const DMat &w, int n_slots, int tok_div,
                    bool new_input) {
    if (new_input) c->xq_src[0] = c->xq_src[1] = nullptr;
    if (!w.quant()) {
        dim3 grid((unsigned)((w.n_out + 255) / 256), n_slots);
        fmatmul_gather_kernel<<<grid, 256, 0, c->st>>>(w.f, w.type, w.n_in, w.n_out, c->moe_top, x, w.n_in, tok_div,
                                                        out, w.n_out);
        SDY_LAUNCHED();
        return;
    }
    const XQ &xq = activations(c, x, n_x, w.n_in, w.type);
    qmatvec_gather(w.q, w.gpe, w.n_expert, xq, tok_div, c->moe_top, n_slots, w.n_out, out, w.n_out, c->st);
}

void moe_ffn(engine_ctx *c, const DLayer &L, int n) {
    const engine_model_info &in = c->m->info;
    const int dim = in.dim, fe = in.ffn_exp_dim, ne = in.n_expert, k = in.n_expert_used;
    matmul(c, c->moe_probs, c->xb, L.gate_inp, n, true);
    softmax(c->moe_probs, ne, ne, n, c->st);
    topk_kernel<<<(n + 127) / 128, 128, 0, c->st>>>(c->moe_probs, n, ne, k, c->moe_top, c->moe_w);
    SDY_LAUNCHED();
    matmul_experts(c, c->moe_g, c->xb, n, L.gate, n * k, k, true);
    matmul_experts(c, c->moe_u, c->xb, n, L.up, n * k, k, false);
    silu_mul(c->moe_g, c->moe_u, (int64_t)n * k * fe, c->st);
    matmul_experts(c, c->moe_y, c->moe_g, n * k, L.down, n * k, 1, true);
    moe_combine_kernel<<<dim3((dim + 255) / 256, n), 256, 0, c->st>>>(c->moe_y, c->moe_top, c->moe_w, k, dim,
                                                                     c->moe_sum);
    SDY_LAUNCHED();
}

void embed(engine_ctx *c, int n) {
    const engine_model *m = c->m;
    const DMat &e = m->tok_embd;
    if (e.quant()) dequant_rows(e.q, c->tok_ids, n, 0, c->x, m->info.dim, c->st);
    else {
        embed_float_kernel<<<n, 256, 0, c->st>>>(e.f, e.type, c->tok_ids, m->info.dim, c->x);
        SDY_LAUNCHED();
    }
}

// n <= n_batch tokens at n_past; logits of the last out_rows tokens (model_llama.c:757-832).
void forward(engine_ctx *c, int n, int out_rows) {
    const engine_model *m = c->m;
    const engine_model_info &in = m->info;
    const int dim = in.dim, hd = in.head_dim, q_dim = in.n_head * hd, kv_dim = in.n_kv_head * hd;
    const int pos0 = c->n_past;
    const size_t layer_stride = (size_t)in.n_kv_head * c->max_seq * hd;
    embed(c, n);
    for (int l = 0; l < in.n_layer; l++) {
        const DLayer &L = m->layers[l];
        float *kc = c->k_cache + l * layer_stride, *vc = c->v_cache + l * layer_stride;
        rmsnorm(c->xb, dim, c->x, dim, L.attn_norm, dim, n, in.norm_eps, c->st);
        matmul(c, c->q, c->xb, L.wq, n, true);
        matmul(c, c->k, c->xb, L.wk, n, false);
        matmul(c, c->v, c->xb, L.wv, n, false);
        if (L.bq) {
            add_bias(c->q, q_dim, L.bq, q_dim, n, c->st);
            add_bias(c->k, kv_dim, L.bk, kv_dim, n, c->st);
            add_bias(c->v, kv_dim, L.bv, kv_dim, n, c->st);
        }
        if (L.q_norm) {
            rmsnorm(c->q, hd, c->q, hd, L.q_norm, hd, n * in.n_head, in.norm_eps, c->st);
            rmsnorm(c->k, hd, c->k, hd, L.k_norm, hd, n * in.n_kv_head, in.norm_eps, c->st);
        }
        rope(c->q, q_dim, n, in.n_head, hd, c->rope_cos, c->rope_sin, pos0, nullptr, in.rope_interleaved, c->st);
        rope(c->k, kv_dim, n, in.n_kv_head, hd, c->rope_cos, c->rope_sin, pos0, nullptr, in.rope_interleaved, c->st);
        kv_store_kernel<<<dim3((kv_dim + 255) / 256, n), 256, 0, c->st>>>(c->k, c->v, kv_dim, hd, c->max_seq, pos0, kc,
                                                                         vc);
        SDY_LAUNCHED();
        attention(c->att, c->q, kc, vc, n, in.n_head, in.n_kv_head, hd, pos0, c->max_seq, c->scores, 0, c->st);
        matmul(c, c->xb, c->att, L.wo, n, true);
        add(c->x, c->x, c->xb, (int64_t)n * dim, c->st);
        rmsnorm(c->xb, dim, c->x, dim, L.ffn_norm, dim, n, in.norm_eps, c->st);
        const float *ffn_out = c->xb;
        if (in.n_expert) {
            moe_ffn(c, L, n);
            ffn_out = c->moe_sum;
        } else {
            matmul(c, c->hb, c->xb, L.gate, n, true);
            matmul(c, c->hb2, c->xb, L.up, n, false);
            silu_mul(c->hb, c->hb2, (int64_t)n * in.ffn_dim, c->st);
            matmul(c, c->xb, c->hb, L.down, n, true);
        }
        add(c->x, c->x, ffn_out, (int64_t)n * dim, c->st);
    }
    if (out_rows > 0) {
        rmsnorm(c->xb, dim, c->x + (size_t)(n - out_rows) * dim, dim, m->output_norm, dim, out_rows, in.norm_eps,
                c->st);
        matmul(c, c->logits, c->xb, m->output, out_rows, true);
    }
}

}  // namespace eng
}  // namespace sdy

using namespace sdy::eng;

// ------------------------------------------------------------------------------ C-ABI

extern "C" {

void engine_model_free(engine_model *m) {
    if (!m) return;
    cudaSetDevice(m->dev);
    for (void *p : m->allocs) cudaFree(p);
    if (m->raw) cudaFree(m->raw);
    if (m->st) cudaStreamDestroy(m->st);
    gguf_close(m->gf);
    delete m;
}

void engine_model_get_info(const engine_model *m, engine_model_info *out) {
    if (m && out) *out = m->info;
}

engine_model *engine_model_load(const char *path, char *err, size_t err_len) {
    if (err && err_len) err[0] = '\0';
    engine_model *m = new engine_model();
    cudaGetDevice(&m->dev);
    if (!(m->gf = gguf_open(path, err, err_len)) || read_config(m, err, err_len)) {
        engine_model_free(m);
        return nullptr;
    }
    if (!SDY_CUDA(cudaStreamCreateWithFlags(&m->st, cudaStreamNonBlocking))) {
        put_err(err, err_len, "GPU non disponibile: %s", last_error());
        engine_model_free(m);
        return nullptr;
    }
    const engine_model_info &in = m->info;
    const int dim = in.dim, q_dim = in.n_head * in.head_dim, kv_dim = in.n_kv_head * in.head_dim;
    m->layers.resize(in.n_layer);
    bool ok = !get_tensor(m, "token_embd.weight", dim, in.n_vocab, 0, &m->tok_embd, err, err_len) &&
              !get_vector(m, "output_norm.weight", dim, &m->output_norm, err, err_len);
    if (ok) {
        if (in.tied_embeddings) m->output = m->tok_embd;
        else ok = !get_tensor(m, "output.weight", dim, in.n_vocab, 0, &m->output, err, err_len);
    }
    for (int l = 0; ok && l < in.n_layer; l++) {
        DLayer &L = m->layers[l];
        auto nm = [&](const char *suffix) {
            static thread_local char buf[96];
            snprintf(buf, sizeof buf, "blk.%d.%s", l, suffix);
            return buf;
        };
        ok = !get_vector(m, nm("attn_norm.weight"), dim, &L.attn_norm, err, err_len) &&
             !get_vector(m, nm("ffn_norm.weight"), dim, &L.ffn_norm, err, err_len) &&
             !get_tensor(m, nm("attn_q.weight"), dim, q_dim, 0, &L.wq, err, err_len) &&
             !get_tensor(m, nm("attn_k.weight"), dim, kv_dim, 0, &L.wk, err, err_len) &&
             !get_tensor(m, nm("attn_v.weight"), dim, kv_dim, 0, &L.wv, err, err_len) &&
             !get_tensor(m, nm("attn_output.weight"), q_dim, dim, 0, &L.wo, err, err_len);
        if (!ok) break;
        if (in.n_expert) {
            int ne = in.n_expert, fe = in.ffn_exp_dim;
            ok = !get_tensor(m, nm("ffn_gate_inp.weight"), dim, ne, 0, &L.gate_inp, err, err_len) &&
                 !get_tensor(m, nm("ffn_gate_exps.weight"), dim, fe, ne, &L.gate, err, err_len) &&
                 !get_tensor(m, nm("ffn_up_exps.weight"), dim, fe, ne, &L.up, err, err_len) &&
                 !get_tensor(m, nm("ffn_down_exps.weight"), fe, dim, ne, &L.down, err, err_len);
        } else {
            ok = !get_tensor(m, nm("ffn_gate.weight"), dim, in.ffn_dim, 0, &L.gate, err, err_len) &&
                 !get_tensor(m, nm("ffn_up.weight"), dim, in.ffn_dim, 0, &L.up, err, err_len) &&
                 !get_tensor(m, nm("ffn_down.weight"), in.ffn_dim, dim, 0, &L.down, err, err_len);
        }
        if (ok && in.qkv_bias)
            ok = !get_vector(m, nm("attn_q.bias"), q_dim, &L.bq, err, err_len) &&
                 !get_vector(m, nm("attn_k.bias"), kv_dim, &L.bk, err, err_len) &&
                 !get_vector(m, nm("attn_v.bias"), kv_dim, &L.bv, err, err_len);
        if (ok && in.qk_norm)
            ok = !get_vector(m, nm("attn_q_norm.weight"), in.head_dim, &L.q_norm, err, err_len) &&
                 !get_vector(m, nm("attn_k_norm.weight"), in.head_dim, &L.k_norm, err, err_len);
    }
    if (m->raw) {
        cudaFree(m->raw);
        m->raw = nullptr;
        m->raw_cap = 0;
    }
    if (!ok) {
        engine_model_free(m);
        return nullptr;
    }
    return m;
}

engine_ctx *engine_ctx_new(const engine_model *m, int32_t max_seq, int32_t n_batch, int32_t logits_all,
                           int32_t n_threads, char *err, size_t err_len) {
    if (err && err_len) err[0] = '\0';
    if (!m) {
        put_err(err, err_len, "modello NULL");
        return nullptr;
    }
    if (max_seq < 1 || max_seq > MAX_SEQ_LIMIT || max_seq > m->info.max_pos) {
        put_err(err, err_len, "max_seq=%d non valido (1..%d)", max_seq,
                m->info.max_pos < MAX_SEQ_LIMIT ? m->info.max_pos : MAX_SEQ_LIMIT);
        return nullptr;
    }
    if (n_batch < 1 || n_batch > MAX_BATCH_LIMIT) {
        put_err(err, err_len, "n_batch=%d non valido (1..%d)", n_batch, MAX_BATCH_LIMIT);
        return nullptr;
    }
    if (n_threads < 0 || n_threads > 256) {
        put_err(err, err_len, "n_threads=%d non valido (0..256)", n_threads);
        return nullptr;
    }
    cudaSetDevice(m->dev);
    engine_ctx *c = new engine_ctx();
    c->m = m;
    c->max_seq = max_seq;
    c->n_batch = n_batch;
    c->logits_all = logits_all != 0;
    c->n_threads = n_threads;
    const engine_model_info &in = m->info;
    const size_t B = n_batch, S = max_seq, hd = in.head_dim;
    const size_t q_dim = (size_t)in.n_head * hd, kv_dim = (size_t)in.n_kv_head * hd;
    const size_t kv = (size_t)in.n_layer * in.n_kv_head * S * hd;
    const size_t ffn = in.n_expert ? in.ffn_exp_dim : in.ffn_dim;
    const size_t K = in.n_expert ? in.n_expert_used : 0, slots = B * K;
    size_t max_in = std::max<size_t>(std::max<size_t>(in.dim, q_dim), ffn);
    // Arena layout: one pass to size, one to assign.
    struct Item { void **dst; size_t bytes; };
    std::vector<Item> items = {
        {(void **)&c->k_cache, kv * 4}, {(void **)&c->v_cache, kv * 4},
        {(void **)&c->rope_cos, S * hd / 2 * 4}, {(void **)&c->rope_sin, S * hd / 2 * 4},
        {(void **)&c->x, B * in.dim * 4}, {(void **)&c->xb, B * in.dim * 4}, {(void **)&c->q, B * q_dim * 4},
        {(void **)&c->k, B * kv_dim * 4}, {(void **)&c->v, B * kv_dim * 4}, {(void **)&c->att, B * q_dim * 4},
        {(void **)&c->hb, B * ffn * 4}, {(void **)&c->hb2, B * ffn * 4},
        {(void **)&c->scores, B * in.n_head * S * 4},
        {(void **)&c->logits, (c->logits_all ? B : 1) * in.n_vocab * 4},
        {(void **)&c->tok_ids, B * 4},
    };
    if (in.n_expert) {
        items.push_back({(void **)&c->moe_probs, B * in.n_expert * 4});
        items.push_back({(void **)&c->moe_w, slots * 4});
        items.push_back({(void **)&c->moe_top, slots * 4});
        items.push_back({(void **)&c->moe_g, slots * ffn * 4});
        items.push_back({(void **)&c->moe_u, slots * ffn * 4});
        items.push_back({(void **)&c->moe_y, slots * in.dim * 4});
        items.push_back({(void **)&c->moe_sum, B * in.dim * 4});
    }
    size_t xq_cap = 0;
    for (int vt : {T_Q8_0, T_Q8_K}) {
        int be = block_elems(vt);
        for (size_t nin : {(size_t)in.dim, q_dim, ffn})
            if (nin % be == 0) xq_cap = std::max(xq_cap, xq_bytes(vt, (int)nin, (int)B));
        if (in.n_expert && ffn % be == 0) xq_cap = std::max(xq_cap, xq_bytes(vt, (int)ffn, (int)slots));
    }
    (void)max_in;
    items.push_back({&c->xq_buf[0], xq_cap});
    items.push_back({&c->xq_buf[1], xq_cap});
    size_t total = 0;
    for (auto &it : items) total += align_up(it.bytes, 256);
    if (!SDY_CUDA(cudaMalloc(&c->arena, total))) {
        put_err(err, err_len, "memoria GPU esaurita (%.1f MB per contesto e KV cache)", total / 1e6);
        delete c;
        return nullptr;
    }
    uint8_t *p = (uint8_t *)c->arena;
    for (auto &it : items) {
        *it.dst = p;
        p += align_up(it.bytes, 256);
    }
    size_t lbytes = (c->logits_all ? B : 1) * in.n_vocab * 4;
    if (!SDY_CUDA(cudaStreamCreateWithFlags(&c->st, cudaStreamNonBlocking)) ||
        !SDY_CUDA(cudaMallocHost(&c->h_logits, lbytes))) {
        put_err(err, err_len, "inizializzazione del contesto fallita: %s", last_error());
        engine_ctx_free(c);
        return nullptr;
    }
    rope_table(c->rope_cos, c->rope_sin, max_seq, in.head_dim, in.rope_theta, c->st);
    if (!SDY_CUDA(cudaStreamSynchronize(c->st))) {
        put_err(err, err_len, "inizializzazione del contesto fallita: %s", last_error());
        engine_ctx_free(c);
        return nullptr;
    }
    return c;
}

int32_t engine_ctx_n_threads(const engine_ctx *c) { return c ? c->n_threads : 0; }

void engine_ctx_free(engine_ctx *c) {
    if (!c) return;
    if (c->st) cudaStreamDestroy(c->st);
    if (c->arena) cudaFree(c->arena);
    if (c->h_logits) cudaFreeHost(c->h_logits);
    delete c;
}

int engine_eval(engine_ctx *c, const int32_t *tokens, int32_t n) {
    if (!c) return -1;
    c->err[0] = '\0';
    if (!tokens || n < 1) {
        snprintf(c->err, sizeof c->err, "nessun token in ingresso");
        return -1;
    }
    if (c->logits_all && n > c->n_batch) {
        snprintf(c->err, sizeof c->err, "con logits_all servono al massimo n_batch=%d token per chiamata", c->n_batch);
        return -1;
    }
    if (n > c->max_seq - c->n_past) {
        snprintf(c->err, sizeof c->err, "contesto pieno: %d + %d > max_seq=%d", c->n_past, n, c->max_seq);
        return -1;
    }
    for (int i = 0; i < n; i++) {
        if (tokens[i] < 0 || tokens[i] >= c->m->info.n_vocab) {
            snprintf(c->err, sizeof c->err, "token %d fuori dal vocabolario [0, %d)", tokens[i], c->m->info.n_vocab);
            return -1;
        }
    }
    cudaSetDevice(c->m->dev);
    clear_error();
    const int saved = c->n_past;
    int out_rows = 0;
    for (int done = 0; done < n;) {
        int chunk = std::min(n - done, c->n_batch);
        bool last = done + chunk == n;
        out_rows = last ? (c->logits_all ? chunk : 1) : 0;
        SDY_CUDA(cudaMemcpyAsync(c->tok_ids, tokens + done, (size_t)chunk * 4, cudaMemcpyHostToDevice, c->st));
        forward(c, chunk, out_rows);
        c->n_past += chunk;
        done += chunk;
    }
    size_t lb = (size_t)out_rows * c->m->info.n_vocab * 4;
    SDY_CUDA(cudaMemcpyAsync(c->h_logits, c->logits, lb, cudaMemcpyDeviceToHost, c->st));
    SDY_CUDA(cudaStreamSynchronize(c->st));
    if (last_error()[0]) {
        c->n_past = saved;
        snprintf(c->err, sizeof c->err, "errore GPU: %s", last_error());
        return -1;
    }
    c->n_logits = c->logits_all ? n : 1;
    return 0;
}

const float *engine_logits(const engine_ctx *c) { return c && c->n_logits ? c->h_logits : nullptr; }
int32_t engine_n_logits(const engine_ctx *c) { return c ? c->n_logits : 0; }
int32_t engine_n_past(const engine_ctx *c) { return c ? c->n_past : 0; }
const char *engine_last_error(const engine_ctx *c) { return c ? c->err : "contesto NULL"; }

void engine_reset(engine_ctx *c) {
    if (!c) return;
    c->n_past = 0;
    c->n_logits = 0;
}

int engine_truncate(engine_ctx *c, int32_t n) {
    if (!c) return -1;
    if (n < 0 || n > c->n_past) {
        snprintf(c->err, sizeof c->err, "posizione %d fuori da [0, %d]", n, c->n_past);
        return -1;
    }
    c->n_past = n;
    c->n_logits = 0;
    return 0;
}

}  // extern "C"
