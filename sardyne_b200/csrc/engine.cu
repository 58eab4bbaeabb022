// The reference's model runtime (reference csrc/model_llama.c, API csrc/engine.h:43-72) on the GPU.
//
// engine_model_load reads the GGUF with the gguf_* reader, checks the configuration exactly as
// the reference does (same accepted files, same error messages), and uploads every weight
// matrix once in the slab layout. Projections that share an input and a quantized type are
// stored as one device matrix (q|k|v, gate|up; for MoE gate|up of every expert), so each runs as
// one launch. engine_ctx_new allocates the device KV cache, the RoPE tables and all activation
// buffers in one arena. engine_eval runs the forward (model_llama.c:757-832) as CUDA kernels on
// the context's stream; a single-token step is captured once as a CUDA graph and replayed (the
// token id and its position are read from device memory), and only the logits come back.
#include "common.cuh"
#include "fp_ops.cuh"
#include "fused.cuh"
#include "sardyne_b200.h"

#include <dlfcn.h>
#include <nccl.h>
#include <stdarg.h>
#include <stdlib.h>
#include <string.h>

#include <algorithm>
#include <iterator>
#include <string>
#include <string_view>
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

// NCCL, opened on first use (only sharded models need it): the process's already loaded
// libnccl.so.2 when there is one (e.g. torch's), else the system's.
struct Nccl {
    ncclResult_t (*get_unique_id)(ncclUniqueId *) = nullptr;
    ncclResult_t (*comm_init_rank)(ncclComm_t *, int, ncclUniqueId, int) = nullptr;
    ncclResult_t (*all_reduce)(const void *, void *, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                               cudaStream_t) = nullptr;
    ncclResult_t (*all_gather)(const void *, void *, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
    const char *(*error_string)(ncclResult_t) = nullptr;
};
const Nccl *nccl() {
    static const Nccl n = [] {  // resolved once (thread-safe static initialisation)
        Nccl r;
        void *h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (h) {
            r.get_unique_id = (decltype(r.get_unique_id))dlsym(h, "ncclGetUniqueId");
            r.comm_init_rank = (decltype(r.comm_init_rank))dlsym(h, "ncclCommInitRank");
            r.all_reduce = (decltype(r.all_reduce))dlsym(h, "ncclAllReduce");
            r.all_gather = (decltype(r.all_gather))dlsym(h, "ncclAllGather");
            r.comm_destroy = (decltype(r.comm_destroy))dlsym(h, "ncclCommDestroy");
            r.error_string = (decltype(r.error_string))dlsym(h, "ncclGetErrorString");
        }
        return r;
    }();
    return n.get_unique_id && n.comm_init_rank && n.all_reduce && n.all_gather && n.comm_destroy && n.error_string
               ? &n
               : nullptr;
}

// Process-wide shard configuration for the next engine_model_load (sdy_engine_set_shard).
struct ShardCfg {
    int rank = 0, world = 1;
    ncclUniqueId id{};
};
ShardCfg g_shard;

// Rows [b, e) of n for `rank` of `world`, in whole units of `align` rows.
void shard_range(int64_t n, int world, int rank, int64_t align, int64_t *b, int64_t *e) {
    const int64_t units = (n + align - 1) / align;
    *b = std::min<int64_t>(n, units * rank / world * align);
    *e = std::min<int64_t>(n, units * (rank + 1) / world * align);
}

// A weight tensor on the device: [n_expert or 1][n_out][n_in].
struct DMat {
    int type = -1;
    int n_in = 0;
    int64_t n_out = 0;        // rows (per expert)
    int n_expert = 0;         // 0: a plain matrix
    QMat q;                   // quantized: slabs (each expert padded to gpe groups)
    int64_t gpe = 0;          // groups per expert
    const void *f = nullptr;  // float weights, raw [n_expert][n_out][n_in]
    bool quant() const { return is_quant_weight(type); }
};

// Projections sharing one input: each part fills output columns [col, col + m.n_out).
struct Part {
    DMat m;
    int col = 0;
};
struct Proj {
    std::vector<Part> parts;
    int width = 0;
};

struct DLayer {
    float *attn_norm = nullptr, *ffn_norm = nullptr, *bq = nullptr, *bk = nullptr, *bv = nullptr;
    float *q_norm = nullptr, *k_norm = nullptr;
    Proj qkv, gateup;
    DMat wo, down, gate_inp;
};

// The per-layer tensors the loader reads, by role. Their GGUF names ("blk.<i>.<name>") are the
// file format's; the set is the one the reference runtime accepts (model_llama.c:128-154).
enum LayerTensor {
    LT_ATTN_NORM, LT_Q, LT_Q_BIAS, LT_K, LT_K_BIAS, LT_V, LT_V_BIAS, LT_Q_NORM, LT_K_NORM, LT_WO, LT_FFN_NORM,
    LT_GATE, LT_UP, LT_DOWN, LT_ROUTER, LT_GATE_EXPS, LT_UP_EXPS, LT_DOWN_EXPS, LT_COUNT
};
constexpr std::string_view kLayerTensorName[LT_COUNT] = {
    "attn_norm.weight", "attn_q.weight", "attn_q.bias", "attn_k.weight", "attn_k.bias", "attn_v.weight",
    "attn_v.bias", "attn_q_norm.weight", "attn_k_norm.weight", "attn_output.weight", "ffn_norm.weight",
    "ffn_gate.weight", "ffn_up.weight", "ffn_down.weight", "ffn_gate_inp.weight", "ffn_gate_exps.weight",
    "ffn_up_exps.weight", "ffn_down_exps.weight",
};
constexpr std::string_view kModelTensorName[] = {"token_embd.weight", "output_norm.weight", "output.weight"};

std::string layer_tensor(int layer, LayerTensor t) {
    return "blk." + std::to_string(layer) + "." + std::string(kLayerTensorName[t]);
}

// True when the loader has a use for a tensor of this name in a model of n_layer layers: a
// model-level name, or "blk.<i>.<layer tensor>" with i < n_layer in decimal digits (leading
// zeros allowed). Any other tensor marks an architecture variant this runtime cannot run.
bool runtime_reads(std::string_view name, int n_layer) {
    for (std::string_view top : kModelTensorName)
        if (name == top) return true;
    constexpr std::string_view prefix = "blk.";
    if (name.substr(0, prefix.size()) != prefix) return false;
    name.remove_prefix(prefix.size());
    const size_t ndig = name.find_first_not_of("0123456789");
    if (ndig == 0 || ndig == std::string_view::npos || name[ndig] != '.') return false;
    uint64_t layer = 0;  // saturates far above any layer count
    for (char ch : name.substr(0, ndig)) layer = std::min<uint64_t>(layer * 10 + (uint64_t)(ch - '0'), 1ull << 32);
    if (layer >= (uint64_t)n_layer) return false;
    const std::string_view rest = name.substr(ndig + 1);
    return std::find(std::begin(kLayerTensorName), std::end(kLayerTensorName), rest) != std::end(kLayerTensorName);
}

bool type_supported(uint32_t t) { return is_quant_weight((int)t) || is_float_weight((int)t); }

}  // namespace
}  // namespace sdy

using namespace sdy;

struct engine_model {
    gguf_file *gf = nullptr;
    engine_model_info info{};
    int dev = 0;
    // Sharding across `world` processes, one GPU each (sdy_engine_set_shard before loading): the
    // router is replicated; this rank holds dense FFN rows [f0, f1) of gate and up, output rows
    // [d0, d1) of down (and of the attention output matrix when attention is split, below),
    // experts [e0, e1) and vocabulary rows [v0, v1) of the output matrix. Every cross-rank
    // exchange assembles parts that the ranks computed disjointly (exchange(): over peer memory at
    // single-token sizes, else an NCCL all-reduce of buffers that are zero outside each rank's
    // part), so results equal the one-GPU forward bit for bit.
    int rank = 0, world = 1;
    ncclComm_t comm = nullptr;
    int64_t f0 = 0, f1 = 0, d0 = 0, d1 = 0, e0 = 0, e1 = 0, v0 = 0, v1 = 0;
    // Tensor-parallel attention (world > 1 where the heads split evenly enough): this rank holds
    // query heads [h0, h1) and KV heads [k0, k1) (q/k/v rows, their biases, its KV cache) and rows
    // [d0, d1) of the attention output matrix; attn_tp false: attention replicated on every rank.
    bool attn_tp = false;
    int h0 = 0, h1 = 0, k0 = 0, k1 = 0;
    DMat tok_embd, output;
    float *output_norm = nullptr;
    std::vector<DLayer> layers;
    std::vector<void *> allocs;
    cudaStream_t st = nullptr;
    uint8_t *raw = nullptr;  // upload bounce buffer (load time only)
    size_t raw_cap = 0;
};

// Quantized activations of one buffer, reused while the buffer is unchanged (model_llama.c:590-611).
struct ActCache {
    const float *src = nullptr;
    int64_t ld = 0;
    int n = 0, n_in = 0;
};

struct engine_ctx {
    const engine_model *m = nullptr;
    int max_seq = 0, n_batch = 0, logits_all = 0, n_past = 0, n_logits = 0, n_threads = 0;
    int qkv_ld = 0, gu_ld = 0;
    cudaStream_t st = nullptr;
    // Side branch of a single-token step: the next layer's weights are pulled into L2 there while
    // this layer's kernels run on st (forked and joined with the two events).
    cudaStream_t side = nullptr;
    cudaEvent_t ev_fork = nullptr, ev_join = nullptr;
    bool forked = false;
    void *arena = nullptr;
    float *k_cache = nullptr, *v_cache = nullptr, *rope_cos = nullptr, *rope_sin = nullptr;
    float *x = nullptr, *xb = nullptr, *qkv = nullptr, *att = nullptr, *hgu = nullptr, *tmp = nullptr,
          *logits = nullptr, *scores = nullptr;
    float *moe_probs = nullptr, *moe_w = nullptr, *moe_gu = nullptr, *moe_y = nullptr;
    int32_t *moe_count = nullptr;  // per-token router counters (router_topk)
    unsigned *md_sync = nullptr;   // fused MoE decode block: 3 barrier words + 1 status word
    // greedy choice on the device: per-block candidates, the counter, the chosen id (and its
    // pinned host copy)
    float *am_v = nullptr;
    int *am_i = nullptr;
    unsigned *am_count = nullptr;
    int32_t *am_out = nullptr, *h_am_out = nullptr;
    unsigned *h_md_status = nullptr;  // pinned copy of the status word, read after each eval
    int32_t *grp_off = nullptr, *grp_slot = nullptr, *grp_tiles = nullptr;  // slots by expert (prefill GEMM)
    // Sharded models: all-reduce sources, zero outside this rank's columns (hsend: FFN activations
    // [B][ffn_dim], xsend: residual [B][dim], lsend: logits), and the gathered FFN activations.
    float *hsend = nullptr, *hfull = nullptr, *xsend = nullptr, *lsend = nullptr;
    // Heads split across ranks: this rank's attention output (prefill: [B][local heads * hd]) and
    // the all-reduce source of the gathered one (zero outside this rank's columns).
    float *att_loc = nullptr, *attsend = nullptr;
    // Single-token exchanges over NVLink peer memory (peer_gather) instead of NCCL: this rank's
    // exchange buffer, the peers' as mapped here, the pinned copy of its status word; px_failed
    // once a wait ran out (the ranks' rounds may then disagree, so the context refuses work).
    PeerExchange px;
    bool px_on = false, px_failed = false;
    unsigned *h_px_status = nullptr;
    int32_t *moe_top = nullptr;
    int32_t *tokpos = nullptr;    // device: [0] position of the first token, [1..] token ids
    int32_t *h_tokpos = nullptr;  // pinned staging of the same
    void *xq_buf[2] = {nullptr, nullptr};  // [0] Q8_0, [1] Q8_K activations
    XQ xq[2];
    ActCache xc[2];
    float *h_logits = nullptr;             // pinned host copy returned by engine_logits
    // The single-token forward as a chain of graphs of a few layers each, replayed each decode step:
    // launching a graph costs host time per node, so the GPU starts on the first segment while
    // the host still launches the later ones.
    std::vector<cudaGraphExec_t> step_graphs;
    int graph_state = 0;  // 0: next single-token step runs eagerly, 2: capture next, 1: captured, -1: off
    bool capturing = false;
    bool capture_ok = true;
    char err[256] = {0};
};

namespace sdy {
namespace eng {

// ------------------------------------------------------------------------------ metadata

const gguf_tensor *find(const gguf_file *gf, const char *name) {
    int64_t i = gguf_find_tensor(gf, name);
    return i < 0 ? nullptr : gguf_get_tensor(gf, (uint64_t)i);
}

// The model header, checked as a table. Each row is one "<arch>.<key>" entry and the
// engine_model_info field it fills; rows run in order and the first failure is reported. The
// files accepted and the messages of the refused ones are the reference runtime's
// (model_llama.c:225-319), because callers and tests match those texts.
using I = engine_model_info;
using IntField = int32_t I::*;
using RealField = float I::*;

struct HeaderRow {
    const char *key;
    bool moe_only;
    IntField int_field;    // integer entry in 1..2^30, stored here ...
    RealField real_field;  // ... or real entry in (0, 1e12], stored here
    // Value taken when the key is absent, from the fields read so far (nullptr: required).
    double (*absent)(const I &);
    const char *zero_msg;  // failure when the absent-key value is 0
    IntField must_equal;   // the entry must equal this field (and is not stored) ...
    const char *unequal;   // ... else this failure, whatever made it differ
    // Checked once the row is read: a failure message, or nullptr.
    const char *(*rule)(const I &, char *buf, size_t len);
};

const char *used_within_count(const I &in, char *buf, size_t len) {
    if (in.n_expert_used <= in.n_expert) return nullptr;
    snprintf(buf, len, "expert_used_count=%d oltre expert_count=%d", in.n_expert_used, in.n_expert);
    return buf;
}
const char *used_within_combine(const I &in, char *buf, size_t len) {
    if (in.n_expert_used <= 64) return nullptr;  // moe_combine_kernel orders at most 64 slots per token
    snprintf(buf, len, "expert_used_count=%d oltre il massimo di 64 di questa build", in.n_expert_used);
    return buf;
}
const char *heads_consistent(const I &in, char *, size_t) {
    const bool ok = in.n_head % in.n_kv_head == 0 && in.head_dim % 2 == 0;
    return ok ? nullptr : "teste o head_dim non validi (n_head % n_kv_head, head_dim pari)";
}
double experts_share_ffn(const I &in) { return in.ffn_dim / in.n_expert_used; }
double kv_heads_default(const I &in) { return in.n_head; }
double head_dim_default(const I &in) { return in.dim / in.n_head; }
double same_as_head_dim(const I &in) { return in.head_dim; }
double context_default(const I &) { return 2048; }
double theta_default(const I &) { return 10000; }

const HeaderRow kHeaderRows[] = {
    {"embedding_length", false, &I::dim, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr},
    {"block_count", false, &I::n_layer, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr},
    {"feed_forward_length", false, &I::ffn_dim, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr},
    {"expert_count", true, &I::n_expert, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr},
    {"expert_used_count", true, &I::n_expert_used, nullptr, nullptr, nullptr, nullptr, nullptr, used_within_count},
    {"expert_feed_forward_length", true, &I::ffn_exp_dim, nullptr, experts_share_ffn,
     "dimensione degli esperti nulla", nullptr, nullptr, used_within_combine},
    {"attention.head_count", false, &I::n_head, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr},
    {"attention.head_count_kv", false, &I::n_kv_head, nullptr, kv_heads_default, nullptr, nullptr, nullptr, nullptr},
    {"attention.key_length", false, &I::head_dim, nullptr, head_dim_default, "head_dim nullo", nullptr, nullptr,
     nullptr},
    {"attention.value_length", false, nullptr, nullptr, same_as_head_dim, nullptr, &I::head_dim,
     "key_length diverso da value_length", nullptr},
    {"rope.dimension_count", false, nullptr, nullptr, same_as_head_dim, nullptr, &I::head_dim,
     "RoPE parziale (rope.dimension_count < head_dim) non supportata", nullptr},
    {"context_length", false, &I::max_pos, nullptr, context_default, nullptr, nullptr, nullptr, nullptr},
    {"attention.layer_norm_rms_epsilon", false, nullptr, &I::norm_eps, nullptr, nullptr, nullptr, nullptr, nullptr},
    {"rope.freq_base", false, nullptr, &I::rope_theta, theta_default, nullptr, nullptr, nullptr, heads_consistent},
};

// One row: reads (or defaults) its entry and stores or compares it. nullptr, or the failure.
const char *check_row(const gguf_file *gf, const std::string &arch, const HeaderRow &r, I *in, char *buf,
                      size_t len) {
    const std::string key = arch + "." + r.key;
    const int64_t at = gguf_find_kv(gf, key.c_str());
    const bool is_int = r.real_field == nullptr;
    double v = 0;
    const char *fail = nullptr;
    if (at < 0 && !r.absent) {
        snprintf(buf, len, "metadato mancante: %s", key.c_str());
        fail = buf;
    } else if (at < 0) {
        v = r.absent(*in);
        if (is_int && v == 0 && r.zero_msg) fail = r.zero_msg;
    } else if (is_int) {
        uint64_t u = 0;
        if (gguf_kv_get_u64(gf, at, &u) || u == 0 || u > (1u << 30)) {
            snprintf(buf, len, "metadato non valido: %s", key.c_str());
            fail = buf;
        }
        v = (double)u;
    } else if (gguf_kv_get_f64(gf, at, &v)) {
        snprintf(buf, len, "metadato non valido: %s", key.c_str());
        fail = buf;
    }
    if (!fail && !is_int && (!(v > 0.0) || v > 1e12)) {
        snprintf(buf, len, "valore non valido per %s", key.c_str());
        fail = buf;
    }
    if (r.must_equal) return fail || (int64_t)v != in->*r.must_equal ? r.unequal : nullptr;
    if (fail) return fail;
    if (is_int) in->*r.int_field = (int32_t)v;
    else in->*r.real_field = (float)v;
    return r.rule ? r.rule(*in, buf, len) : nullptr;
}

// Header and tensor-name checks of a GGUF before anything is uploaded.
int read_config(engine_model *m, char *err, size_t len) {
    const gguf_file *gf = m->gf;
    I *in = &m->info;
    uint64_t n = 0;
    const char *arch_s = gguf_kv_get_str(gf, gguf_find_kv(gf, "general.architecture"), &n);
    if (!arch_s || n == 0 || n >= 32) {
        put_err(err, len, "general.architecture mancante o non valido");
        return -1;
    }
    const std::string arch(arch_s, n);
    // llama rotates interleaved pairs; the qwen families rotate the two halves of a head
    static const std::pair<const char *, int> kArchs[] = {{"llama", 1}, {"qwen2", 0}, {"qwen3", 0}, {"qwen3moe", 0}};
    const auto *a = std::find_if(std::begin(kArchs), std::end(kArchs), [&](auto &p) { return arch == p.first; });
    if (a == std::end(kArchs)) {
        put_err(err, len, "architettura %s non supportata", arch.c_str());
        return -1;
    }
    in->rope_interleaved = a->second;
    const bool moe = arch == "qwen3moe";
    const char *scaling = gguf_kv_get_str(gf, gguf_find_kv(gf, (arch + ".rope.scaling.type").c_str()), &n);
    const bool plain_rope = !scaling || std::string_view(scaling, n) == "none";
    if (!plain_rope || find(gf, "rope_freqs.weight")) {
        put_err(err, len, "rope scaling (anche 'llama3' via rope_freqs.weight) non supportato");
        return -1;
    }
    char buf[192];
    for (const HeaderRow &r : kHeaderRows) {
        if (r.moe_only && !moe) continue;
        if (const char *fail = check_row(gf, arch, r, in, buf, sizeof buf)) {
            put_err(err, len, "%s", fail);
            return -1;
        }
    }
    const gguf_tensor *emb = find(gf, "token_embd.weight");
    if (!emb || emb->n_dims != 2 || emb->ne[1] == 0 || emb->ne[1] > (1u << 30)) {
        put_err(err, len, "token_embd.weight mancante o non valido");
        return -1;
    }
    in->n_vocab = (int32_t)emb->ne[1];
    in->tied_embeddings = find(gf, "output.weight") == nullptr;
    in->qkv_bias = find(gf, layer_tensor(0, LT_Q_BIAS).c_str()) != nullptr;
    in->qk_norm = find(gf, layer_tensor(0, LT_Q_NORM).c_str()) != nullptr;
    for (uint64_t i = 0; i < gguf_n_tensors(gf); i++) {
        const char *name = gguf_get_tensor(gf, i)->name;
        if (!runtime_reads(name, in->n_layer)) {
            put_err(err, len, "tensore non supportato: %s", name);
            return -1;
        }
    }
    return 0;
}

// The attention heads of rank `rank` of `world`: whole KV heads with their query heads when every
// rank can have one (world <= n_kv_head); otherwise, when the query heads divide evenly and each
// rank's share lies within one KV head, that KV head is computed by every rank that shares it.
// Any other shape keeps attention replicated (*tp false).
void attention_split(const engine_model_info &in, int world, int rank, bool *tp, int *h0, int *h1, int *k0, int *k1,
                     bool allow = true) {
    *tp = false;
    *h0 = 0, *h1 = in.n_head, *k0 = 0, *k1 = in.n_kv_head;
    if (world <= 1 || !allow) return;
    const int n_rep = in.n_head / in.n_kv_head;
    if (world <= in.n_kv_head) {
        int64_t b, e;
        shard_range(in.n_kv_head, world, rank, 1, &b, &e);
        *k0 = (int)b, *k1 = (int)e, *h0 = *k0 * n_rep, *h1 = *k1 * n_rep;
        *tp = true;
    } else if (world % in.n_kv_head == 0 && in.n_head % world == 0 && n_rep % (world / in.n_kv_head) == 0) {
        const int per = in.n_head / world;
        *h0 = rank * per, *h1 = *h0 + per, *k0 = *h0 / n_rep, *k1 = *k0 + 1;
        *tp = true;
    }
    if (*tp && ((*h1 - *h0) * in.head_dim % GROUP_ROWS || (*k1 - *k0) * in.head_dim % GROUP_ROWS)) {
        *tp = false;  // q/k/v row slices must be whole 8-row groups
        *h0 = 0, *h1 = in.n_head, *k0 = 0, *k1 = in.n_kv_head;
    }
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

// Checks a tensor [n_expert][n_out][n_in] (n_expert 0: a matrix) of a supported type
// (model_llama.c:163-185).
const gguf_tensor *check_tensor(engine_model *m, const char *name, int n_in, int64_t n_out, int n_expert, char *err,
                                size_t len) {
    const gguf_tensor *t = find(m->gf, name);
    if (!t) {
        put_err(err, len, "tensore mancante: %s", name);
        return nullptr;
    }
    if (t->n_dims != (n_expert ? 3u : 2u) || t->ne[0] != (uint64_t)n_in || t->ne[1] != (uint64_t)n_out ||
        (n_expert && t->ne[2] != (uint64_t)n_expert)) {
        put_err(err, len, "%s: dimensioni [%llu, %llu, %llu], attese [%d, %lld, %d]", name,
                (unsigned long long)t->ne[0], (unsigned long long)t->ne[1], (unsigned long long)t->ne[2], n_in,
                (long long)n_out, n_expert ? n_expert : 1);
        return nullptr;
    }
    if (!type_supported(t->type)) {
        put_err(err, len,
                "%s: tipo %s non supportato dal runtime (supportati: F32, F16, BF16, Q8_0, Q4_0, Q5_0, Q4_K, Q6_K)",
                name, gguf_type_name(t->type));
        return nullptr;
    }
    return t;
}

// Uploads tensors of one type that share n_in as ONE device matrix: expert e (or the single
// matrix) holds rows [starts[0], starts[0] + rows[0]) of ts[0], then those of ts[1], ... Of a
// tensor with experts, experts e_begin .. e_begin + n_expert - 1 are taken (n_expert 0: a plain
// matrix). Quantized rows are repacked into slabs.
int upload_group(engine_model *m, const std::vector<const gguf_tensor *> &ts, const std::vector<int64_t> &rows,
                 const std::vector<int64_t> &starts, int n_in, int64_t e_begin, int n_expert, DMat *out, char *err,
                 size_t len) {
    DMat d;
    d.type = (int)ts[0]->type;
    d.n_in = n_in;
    d.n_expert = n_expert;
    int64_t total = 0;
    for (int64_t r : rows) total += r;
    d.n_out = total;
    const int ne = n_expert ? n_expert : 1;
    const size_t rb = row_bytes(d.type, n_in);
    uint8_t *raw = bounce(m, (size_t)ne * total * rb);
    bool ok = raw != nullptr;
    for (int e = 0; ok && e < ne; e++) {
        size_t off = (size_t)e * total * rb;
        for (size_t i = 0; ok && i < ts.size(); i++) {
            const size_t full = (size_t)ts[i]->ne[1];
            const uint8_t *src = (const uint8_t *)ts[i]->data + ((size_t)(e_begin + e) * full + starts[i]) * rb;
            ok = SDY_CUDA(cudaMemcpyAsync(raw + off, src, rows[i] * rb, cudaMemcpyHostToDevice, m->st));
            off += rows[i] * rb;
        }
    }
    if (ok && d.quant()) {
        d.q.type = d.type;
        d.q.n_in = n_in;
        d.q.nb = n_in / block_elems(d.type);
        d.q.n_rows = total;
        d.gpe = d.q.n_groups();
        const size_t per = d.q.bytes();
        uint8_t *slabs = (uint8_t *)dalloc(m, per * ne);
        ok = slabs != nullptr;
        for (int e = 0; ok && e < ne; e++)
            repack_to_slabs(raw + (size_t)e * total * rb, d.type, total, n_in, slabs + per * e, m->st);
        d.q.slabs = slabs;
    } else if (ok) {
        void *f = dalloc(m, (size_t)ne * total * rb);
        ok = f && SDY_CUDA(cudaMemcpyAsync(f, raw, (size_t)ne * total * rb, cudaMemcpyDeviceToDevice, m->st));
        d.f = f;
    }
    ok = ok && SDY_CUDA(cudaStreamSynchronize(m->st));
    if (!ok) {
        put_err(err, len, "%s: caricamento sulla GPU fallito (%s)", ts[0]->name, last_error());
        return -1;
    }
    *out = d;
    return 0;
}

// Rows [r0, r1) (r1 < 0: all) of experts [e_begin, e_end) (e_end < 0: all) of a checked tensor.
int get_tensor(engine_model *m, const char *name, int n_in, int64_t n_out, int n_expert, DMat *out, char *err,
               size_t len, int64_t r0 = 0, int64_t r1 = -1, int64_t e_begin = 0, int64_t e_end = -1) {
    const gguf_tensor *t = check_tensor(m, name, n_in, n_out, n_expert, err, len);
    if (!t) return -1;
    if (r1 < 0) r1 = n_out;
    if (e_end < 0) e_end = n_expert;
    return upload_group(m, {t}, {r1 - r0}, {r0}, n_in, e_begin, n_expert ? (int)(e_end - e_begin) : 0, out, err, len);
}

// A projection from one input: consecutive tensors of the same quantized type whose row counts
// are whole 8-row groups share one device matrix (one launch); the others stay separate. Rows
// [r0, r1) of every tensor (r1 < 0: all), experts [e_begin, e_end) (e_end < 0: all).
// slices: per tensor (first row, row count), overriding [r0, r1).
int get_proj(engine_model *m, const std::vector<std::string> &names, const std::vector<int64_t> &rows, int n_in,
             int n_expert, Proj *out, char *err, size_t len, int64_t r0 = 0, int64_t r1 = -1, int64_t e_begin = 0,
             int64_t e_end = -1, const std::vector<std::pair<int64_t, int64_t>> *slices = nullptr) {
    std::vector<const gguf_tensor *> ts;
    std::vector<int64_t> cnt, st;
    for (size_t i = 0; i < names.size(); i++) {
        const gguf_tensor *t = check_tensor(m, names[i].c_str(), n_in, rows[i], n_expert, err, len);
        if (!t) return -1;
        ts.push_back(t);
        if (slices) {
            st.push_back((*slices)[i].first);
            cnt.push_back((*slices)[i].second);
        } else {
            cnt.push_back(r1 < 0 ? rows[i] : r1 - r0);
            st.push_back(r1 < 0 ? 0 : r0);
        }
    }
    if (e_end < 0) e_end = n_expert;
    const int ne = n_expert ? (int)(e_end - e_begin) : 0;
    Proj p;
    int col = 0;
    for (size_t i = 0; i < ts.size();) {
        size_t j = i + 1;
        const bool fusable = is_quant_weight((int)ts[i]->type) && cnt[i] % GROUP_ROWS == 0;
        while (fusable && j < ts.size() && ts[j]->type == ts[i]->type && cnt[j] % GROUP_ROWS == 0) j++;
        Part part;
        part.col = col;
        if (upload_group(m, std::vector<const gguf_tensor *>(ts.begin() + i, ts.begin() + j),
                         std::vector<int64_t>(cnt.begin() + i, cnt.begin() + j),
                         std::vector<int64_t>(st.begin() + i, st.begin() + j), n_in, e_begin, ne, &part.m, err, len))
            return -1;
        col += (int)part.m.n_out;
        p.parts.push_back(part);
        i = j;
    }
    p.width = col;
    *out = p;
    return 0;
}

// A vector of n elements converted to f32 on the device (elements [first, first + count) of it
// when count > 0).
int get_vector(engine_model *m, const char *name, int n, float **out, char *err, size_t len, int first = 0,
               int count = 0) {
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
    if (count <= 0) first = 0, count = n;
    const size_t esz = block_bytes((int)t->type), bytes = (size_t)count * esz;
    float *d = (float *)dalloc(m, (size_t)count * 4);
    uint8_t *raw = bounce(m, bytes);
    if (!d || !raw ||
        !SDY_CUDA(cudaMemcpyAsync(raw, (const uint8_t *)t->data + (size_t)first * esz, bytes, cudaMemcpyHostToDevice,
                                  m->st))) {
        put_err(err, len, "%s: caricamento sulla GPU fallito (%s)", name, last_error());
        return -1;
    }
    convert_to_f32(raw, (int)t->type, d, count, m->st);
    if (!SDY_CUDA(cudaStreamSynchronize(m->st))) return -1;
    *out = d;
    return 0;
}

// ------------------------------------------------------------------------------ small kernels

// x[t] = row tok[t] of a float table (F32/F16/BF16).
__global__ void embed_float_kernel(const void *table, int type, const int32_t *ids, int dim, float *x) {
    pdl_wait();
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

// Router selection per token for a quantized router (model_llama.c:653-666): the k most
// probable experts, ties to the lowest index, weights renormalised by their float sum.
__global__ void topk_kernel(const float *probs, int n_tok, int ne, int k, int32_t *top, float *w) {
    pdl_wait();
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

// Float-weight experts: out[s*ldo + r] = E[top[s]][r] . x[s / tok_div], one thread per row, in
// the reference's scalar dot order (four accumulators, csrc/ops.c:155-167).
__global__ void fmatmul_gather_kernel(const void *w, int type, int n_in, int64_t rows, const int32_t *top,
                                      int expert0, int n_expert, const float *x, int64_t ldx, int tok_div, float *out,
                                      int64_t ldo) {
    pdl_wait();
    int s = blockIdx.y;
    int64_t r = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    const int e = top[s] - expert0;  // this matrix holds experts expert0 .. expert0 + n_expert - 1
    if (r >= rows || e < 0 || e >= n_expert) return;
    size_t base = ((size_t)e * rows + r) * n_in;
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

// Greedy choice on the device: the index of the largest logit, the first one on ties and the first
// NaN if there is one (numpy.argmax, which the reference's greedy loop applies to the host logits,
// sardyne/runtime.py:115-140). ARGMAX_CTAS blocks take strided elements; the last block to finish
// (a counter it leaves at zero) reduces their candidates.
constexpr int ARGMAX_CTAS = 32, ARGMAX_THREADS = 512;
struct Cand {
    float v;
    int i;
};
__device__ __forceinline__ Cand better(Cand a, Cand b) {  // a before b in the scan order when equal
    const bool an = a.v != a.v, bn = b.v != b.v;
    if (an || bn) return an && (!bn || a.i < b.i) ? a : b;
    return (b.v > a.v || (b.v == a.v && b.i < a.i)) ? b : a;
}
__device__ Cand block_best(Cand c, Cand *part) {
    for (int o = 16; o; o >>= 1) {
        Cand d{__shfl_xor_sync(0xffffffffu, c.v, o), __shfl_xor_sync(0xffffffffu, c.i, o)};
        c = better(c, d);
    }
    const int w = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
    __syncthreads();
    if (lane == 0) part[w] = c;
    __syncthreads();
    c = lane < nw ? part[lane] : Cand{-INFINITY, 0x7fffffff};
    for (int o = 16; o; o >>= 1) {
        Cand d{__shfl_xor_sync(0xffffffffu, c.v, o), __shfl_xor_sync(0xffffffffu, c.i, o)};
        c = better(c, d);
    }
    return c;
}
__global__ void __launch_bounds__(ARGMAX_THREADS) argmax_kernel(const float *x, int n, float *cand_v, int *cand_i,
                                                                unsigned *counter, int32_t *out) {
    pdl_wait();
    __shared__ Cand part[32];
    __shared__ int last;
    Cand c{-INFINITY, 0x7fffffff};
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) c = better(c, Cand{x[i], i});
    c = block_best(c, part);
    if (threadIdx.x == 0) {
        cand_v[blockIdx.x] = c.v;
        cand_i[blockIdx.x] = c.i;
        __threadfence();
        last = atomicAdd(counter, 1u) == gridDim.x - 1;
    }
    __syncthreads();
    if (!last) return;
    __threadfence();
    c = threadIdx.x < gridDim.x ? Cand{__ldcg(cand_v + threadIdx.x), __ldcg(cand_i + threadIdx.x)}
                                : Cand{-INFINITY, 0x7fffffff};
    c = block_best(c, part);
    if (threadIdx.x == 0) {
        *out = c.i;
        *counter = 0;
    }
}

// ------------------------------------------------------------------------------ forward

int act_slot(int vt) { return vt == T_Q8_K ? 1 : 0; }

// Quantized activations of x (n rows of n_in, row stride ldx) for weights of type wtype.
const XQ &activations(engine_ctx *c, const float *x, int64_t ldx, int n, int n_in, int wtype) {
    const int vt = vec_dot_type(wtype), s = act_slot(vt);
    ActCache &k = c->xc[s];
    if (k.src != x || k.ld != ldx || k.n != n || k.n_in != n_in) {
        c->xq[s] = xq_carve(c->xq_buf[s], vt, n_in, n);
        quantize_rows(vt, x, ldx, n, n_in, c->xq[s], c->st);
        k = ActCache{x, ldx, n, n_in};
    }
    return c->xq[s];
}

void forget_activations(engine_ctx *c) { c->xc[0] = c->xc[1] = ActCache(); }

// Reserves the XQ slots a producer kernel (norm or SiLU fused with quantization) fills for
// (x, n, n_in), for the activation types the given matrices consume.
void want_activations(engine_ctx *c, const std::vector<const DMat *> &mats, const float *x, int64_t ldx, int n,
                      int n_in, const XQ **q8k, const XQ **q80) {
    forget_activations(c);
    *q8k = *q80 = nullptr;
    for (const DMat *d : mats) {
        if (!d->quant()) continue;
        const int vt = vec_dot_type(d->type), s = act_slot(vt);
        if (c->xc[s].src) continue;
        c->xq[s] = xq_carve(c->xq_buf[s], vt, n_in, n);
        c->xc[s] = ActCache{x, ldx, n, n_in};
        (vt == T_Q8_K ? *q8k : *q80) = &c->xq[s];
    }
}

// out[t*ldo + j] = x[t] . W[j] (+ residual), W a plain matrix.
void matmul(engine_ctx *c, float *out, int64_t ldo, const float *x, int64_t ldx, const DMat &w, int n,
            const float *residual = nullptr) {
    if (!w.quant()) {
        float *dst = residual ? c->tmp : out;
        const int64_t ld = residual ? w.n_out : ldo;
        fmatmul(x, ldx, w.f, w.type, n, w.n_in, 0, w.n_out, dst, ld, 0, c->st);
        if (residual)  // x + W.a as the reference's `x[i] += xb[i]`
            for (int t = 0; t < n; t++)
                add(out + (size_t)t * ldo, residual + (size_t)t * ldo, c->tmp + (size_t)t * ld, w.n_out, c->st);
        return;
    }
    const XQ &xq = activations(c, x, ldx, n, w.n_in, w.type);
    qmatvec(w.q, xq, out, ldo, 0, w.n_out, 0, c->st, residual);
}

void project(engine_ctx *c, const Proj &p, float *out, int64_t ldo, const float *x, int64_t ldx, int n) {
    for (const Part &part : p.parts) matmul(c, out + part.col, ldo, x, ldx, part.m, n);
}

// Decode-step fusion of elementwise producers into their consumers: a single-token step whose
// norm (or SwiGLU gate, or plain activation) feeds quantized matrices lets the consuming kernel
// prepare and quantize its input itself (ActIn) instead of a separate kernel writing the
// quantized activations (SARDYNE_NO_FUSED_NORM: off). Used where ONE kernel consumes the input:
// each consumer pays the preparation in its prologue (about as long as the separate kernel on
// the critical path), so the parts of a projection go in one launch (qmatvec2) when their types
// differ.
bool fusion_enabled() {
    static const bool off = getenv("SARDYNE_NO_FUSED_NORM") != nullptr;
    return !off;
}
bool fused_norm_ok(int n, const std::vector<const DMat *> &mats) {
    if (!fusion_enabled() || n != 1) return false;
    if (mats.size() == 1) return mats[0]->quant();
    return mats.size() == 2 && mats[0]->quant() && mats[1]->quant() && mats[0]->n_in == mats[1]->n_in &&
           qmatvec2_supported(mats[0]->type, mats[1]->type);
}

// out = W . act for quantized W, the input prepared inside the matvec (+ residual).
void matmul_act(engine_ctx *c, float *out, int64_t ldo, const DMat &w, const ActIn &act, int n,
                const float *residual = nullptr) {
    const XQ geo = xq_carve(nullptr, vec_dot_type(w.type), w.n_in, n);  // geometry only
    qmatvec(w.q, geo, out, ldo, 0, w.n_out, 0, c->st, residual, &act);
}

void project_act(engine_ctx *c, const Proj &p, float *out, int64_t ldo, const ActIn &act, int n) {
    forget_activations(c);
    if (p.parts.size() == 2) {
        const DMat &a = p.parts[0].m, &b = p.parts[1].m;
        const XQ geo = xq_carve(nullptr, vec_dot_type(a.type), a.n_in, n);
        qmatvec2(a.q, out + p.parts[0].col, b.q, out + p.parts[1].col, geo, c->st, &act);
        return;
    }
    for (const Part &part : p.parts) matmul_act(c, out + part.col, ldo, part.m, act, n);
}

// Experts: out[s*ldo + part.col + r] = E[top[s]][r] . x[s / tok_div] for every part.
void project_experts(engine_ctx *c, const Proj &p, float *out, int64_t ldo, const float *x, int64_t ldx, int n_x,
                     int n_slots, int tok_div, const ActIn *act = nullptr) {
    for (const Part &part : p.parts) {
        const DMat &w = part.m;
        if (!w.quant()) {
            dim3 grid((unsigned)((w.n_out + 255) / 256), n_slots);
            launch(fmatmul_gather_kernel, grid, 256, 0, c->st, w.f, w.type, w.n_in, w.n_out, c->moe_top,
                   (int)c->m->e0, w.n_expert, x, ldx, tok_div, out + part.col, ldo);
            SDY_LAUNCHED();
            continue;
        }
        if (act) {
            const XQ geo = xq_carve(nullptr, vec_dot_type(w.type), w.n_in, n_x);  // geometry only
            qmatvec_gather(w.q, w.gpe, w.n_expert, geo, tok_div, c->moe_top, n_slots, w.n_out, out + part.col, ldo,
                           c->st, (int)c->m->e0, act);
            continue;
        }
        const XQ &xq = activations(c, x, ldx, n_x, w.n_in, w.type);
        qmatvec_gather(w.q, w.gpe, w.n_expert, xq, tok_div, c->moe_top, n_slots, w.n_out, out + part.col, ldo, c->st,
                       (int)c->m->e0);
    }
}

// recv = sum over ranks of send (count floats). Every element has one nonzero contributor, so
// the sum is that value exactly, whatever order NCCL adds in.
void all_reduce(engine_ctx *c, const float *send, float *recv, size_t count) {
    const ncclResult_t r = nccl()->all_reduce(send, recv, count, ncclFloat32, ncclSum, c->m->comm, c->st);
    if (r != ncclSuccess) set_error("ncclAllReduce: %s", nccl()->error_string(r));
}

// Whether the exchange of rows x ld floats goes over peer memory (the single-token sizes; the same
// answer on every rank, which all run the same steps).
bool peer_exchange(const engine_ctx *c, int rows, int64_t ld) { return c->px_on && (int64_t)rows * ld <= c->px.cap; }

// recv = the rows x ld floats of which every rank computed columns [lo, hi) of each row in its own
// send (rows of this rank's experts only, with `top`), the rest of send zero: over peer memory
// where peer_exchange() says so, else as an NCCL all-reduce.
void exchange(engine_ctx *c, const float *send, float *recv, int rows, int64_t ld, int64_t lo, int64_t hi,
              const int32_t *top = nullptr) {
    if (peer_exchange(c, rows, ld))
        peer_gather(c->px, send, recv, rows, ld, lo, hi, top, (int)c->m->e0, (int)c->m->e1, c->st);
    else
        all_reduce(c, send, recv, (size_t)rows * ld);
}

// L2 prefetch in single-token steps (SARDYNE_L2_PREFETCH = off | layer | experts | all): the next
// layer's matrices, and the chosen experts' down matrices. Default: all on MoE models, none on
// dense ones. Measured: the down prefetch gains ~1% on the Qwen3-30B-A3B shape and the next
// layer's (non-expert, ~12 MB) matrices another 1%; on the Qwen2.5-3B shape the next layer's
// ~47 MB cost 5% (their reads compete with the current layer's).
enum { PF_LAYER = 1, PF_EXPERTS = 2, PF_DEFAULT = -1 };
int prefetch_mode(const engine_model_info &in) {
    static const int mode = [] {
        const char *v = getenv("SARDYNE_L2_PREFETCH");
        if (!v) return (int)PF_DEFAULT;
        return !strcmp(v, "off") ? 0 : !strcmp(v, "layer") ? PF_LAYER : !strcmp(v, "experts") ? PF_EXPERTS
                                                                                  : PF_LAYER | PF_EXPERTS;
    }();
    if (mode == PF_DEFAULT) return in.n_expert ? PF_LAYER | PF_EXPERTS : 0;
    return mode;
}

// The side stream continues from the work queued on st so far; the layer loop joins it back.
void fork_side(engine_ctx *c) {
    SDY_CUDA(cudaEventRecord(c->ev_fork, c->st));
    SDY_CUDA(cudaStreamWaitEvent(c->side, c->ev_fork, 0));
    c->forked = true;
}

// Fork: layer L's weights (all but the experts, which the router prefetches once chosen) into L2
// on the side stream; the branch is joined at the end of the current layer.
void prefetch_layer(engine_ctx *c, const DLayer &L) {
    L2Ranges r;
    auto add = [&](const DMat &w) {
        if (w.n_expert) return;
        if (w.quant()) r.add(w.q.slabs, w.q.bytes());
        else if (w.f) r.add(w.f, (size_t)w.n_out * w.n_in * block_bytes(w.type));
    };
    for (const Part &p : L.qkv.parts) add(p.m);
    add(L.wo);
    add(L.gate_inp);
    for (const Part &p : L.gateup.parts) add(p.m);
    add(L.down);
    fork_side(c);
    l2_prefetch(r, c->side);
    SDY_CUDA(cudaEventRecord(c->ev_join, c->side));
}

// A single-token MoE step can take its ffn norm inside the float router and the gate|up expert
// kernels (two consumers, each normalising x itself) with SARDYNE_MOE_NORM=fused. Off by default:
// measured on the Qwen3-30B-A3B shape the router's prologue costs more than the norm kernel
// (327 against 336 tok/s).
bool moe_norm_fused(int n, const DLayer &L, const engine_model_info &in) {
    if (!router_topk_supported(in.dim, in.n_expert, in.n_expert_used, n, true)) return false;
    static const bool fused = [] {
        const char *v = getenv("SARDYNE_MOE_NORM");
        return v && !strcmp(v, "fused");
    }();
    if (!fused || !fusion_enabled() || n != 1 || L.gate_inp.quant()) return false;
    for (const Part &p : L.gateup.parts)
        if (!p.m.quant()) return false;
    return true;
}

// A single-token MoE block as one kernel (moe_decode.cu) with SARDYNE_MOE_DECODE=on; by default
// the separate norm, router, expert and combine kernels, measured faster so far. One GPU only:
// sharded experts need the exchange of the expert outputs before the combine.
bool moe_decode_ok(const engine_ctx *c, const DLayer &L, int n) {
    static const bool off = [] {
        const char *v = getenv("SARDYNE_MOE_DECODE");
        return !(v && !strcmp(v, "on"));
    }();
    const engine_model_info &in = c->m->info;
    if (off || n != 1 || c->m->world > 1 || !fusion_enabled() || L.gateup.parts.size() != 1 || L.gate_inp.quant() ||
        !L.down.quant())
        return false;
    const DMat &gu = L.gateup.parts[0].m;
    return gu.quant() && gu.n_out == 2 * in.ffn_exp_dim &&
           moe_decode_supported(gu.type, L.down.type, L.gate_inp.type, in.dim, in.ffn_exp_dim, in.n_expert,
                                in.n_expert_used);
}

bool moe_block_decode(engine_ctx *c, const DLayer &L) {
    const engine_model_info &in = c->m->info;
    const DMat &gu = L.gateup.parts[0].m;
    MoeDecode a;
    a.x = c->x;
    a.norm_w = L.ffn_norm;
    a.eps = in.norm_eps;
    a.dim = in.dim;
    a.router = L.gate_inp.f;
    a.rtype = L.gate_inp.type;
    a.ne = in.n_expert;
    a.k = in.n_expert_used;
    a.gu_slabs = gu.q.slabs;
    a.gpe_gu = gu.gpe;
    a.fe = in.ffn_exp_dim;
    a.dn_slabs = L.down.q.slabs;
    a.gpe_dn = L.down.gpe;
    a.logits = c->moe_probs;
    a.top = c->moe_top;
    a.wts = c->moe_w;
    a.gu = c->moe_gu;
    a.y = c->moe_y;
    a.bar = c->md_sync;
    a.status = c->md_sync + 3;
    if (!moe_decode(a, gu.type, L.down.type, c->st)) return false;
    return true;
}

// nin: the step's ffn norm is fused into the router and the gate|up experts (x = the residual).
void moe_ffn(engine_ctx *c, const DLayer &L, int n, const ActIn *nin = nullptr) {
    const engine_model_info &in = c->m->info;
    const int dim = in.dim, fe = in.ffn_exp_dim, ne = in.n_expert, k = in.n_expert_used;
    const DMat &r = L.gate_inp;
    if (nin) {
        router_topk(nin->x, dim, r.f, r.type, dim, ne, k, n, c->moe_top, c->moe_w, c->moe_probs, c->moe_count, c->st,
                    nin->w, nin->eps);
    } else if (!r.quant() && router_topk_supported(dim, ne, k, n, false)) {
        router_topk(c->xb, dim, r.f, r.type, dim, ne, k, n, c->moe_top, c->moe_w, c->moe_probs, c->moe_count,
                    c->st);
    } else {
        matmul(c, c->moe_probs, ne, c->xb, dim, r, n);
        softmax(c->moe_probs, ne, ne, n, c->st);
        launch(topk_kernel, (n + 127) / 128, 128, 0, c->st, c->moe_probs, n, ne, k, c->moe_top, c->moe_w);
        SDY_LAUNCHED();
    }
    const int slots = n * k, gu = 2 * fe;
    if (n == 1 && (prefetch_mode(in) & PF_EXPERTS) && L.down.quant()) {
        // the chosen experts' down matrices into L2 while their gate|up products run
        ExpertPrefetch ep;
        ep.base[0] = L.down.q.slabs;
        ep.bytes[0] = (size_t)L.down.gpe * L.down.q.nb * slab_bytes(L.down.type);
        ep.e0 = (int)c->m->e0;
        ep.n_local = L.down.n_expert;
        fork_side(c);
        expert_prefetch(ep, c->moe_top, k, c->side);
        SDY_CUDA(cudaEventRecord(c->ev_join, c->side));
    }
    // Many tokens: experts as grouped tensor-core GEMMs over the slots sorted by expert.
    bool grouped = !nin && gemm_min_tokens() > 0 && n >= gemm_min_tokens() && L.down.quant() &&
                   qgemm_supported(L.down.type, L.down.n_in);
    for (const Part &part : L.gateup.parts)
        grouped = grouped && part.m.quant() && qgemm_supported(part.m.type, part.m.n_in);
    const int ne_local = L.down.n_expert;
    if (grouped) {
        moe_group(c->moe_top, slots, (int)c->m->e0, ne_local, GEMM_TILE_TOKENS, c->grp_off, c->grp_slot,
                  c->grp_tiles, c->st);
        for (const Part &part : L.gateup.parts) {
            const XQ &xq = activations(c, c->xb, dim, n, dim, part.m.type);
            qgemm_grouped(part.m.q, part.m.gpe, ne_local, xq, k, c->grp_off, c->grp_slot, c->grp_tiles, slots,
                          part.m.n_out, c->moe_gu + part.col, gu, c->st);
        }
    } else {
        project_experts(c, L.gateup, c->moe_gu, gu, c->xb, dim, n, slots, k, nin);
    }
    // Expert products one slot at a time: the down kernels apply the SwiGLU gate to their own input.
    const bool silu_fused = !grouped && fusion_enabled() && L.down.quant();
    if (!silu_fused) {
        const XQ *q8k, *q80;
        want_activations(c, {&L.down}, c->moe_gu, gu, slots, fe, &q8k, &q80);
        silu_quant(c->moe_gu, gu, c->moe_gu + fe, gu, fe, slots, q8k, q80, c->st);
    }
    Proj down;
    down.parts.push_back(Part{L.down, 0});
    const bool sharded = c->m->world > 1;
    const bool over_peers = sharded && peer_exchange(c, slots, dim);
    if (sharded && !over_peers)  // other ranks' slots zero for the all-reduce
        SDY_CUDA(cudaMemsetAsync(c->moe_y, 0, (size_t)slots * dim * 4, c->st));
    if (grouped) {
        const XQ &xq = activations(c, c->moe_gu, gu, slots, fe, L.down.type);
        qgemm_grouped(L.down.q, L.down.gpe, ne_local, xq, 1, c->grp_off, c->grp_slot, c->grp_tiles, slots,
                      L.down.n_out, c->moe_y, dim, c->st);
    } else {
        ActIn gate;
        gate.x = c->moe_gu;
        gate.ldx = gu;
        gate.u = c->moe_gu + fe;
        gate.ldu = gu;
        project_experts(c, down, c->moe_y, dim, c->moe_gu, gu, slots, slots, 1, silu_fused ? &gate : nullptr);
    }
    if (sharded) exchange(c, c->moe_y, c->moe_y, slots, dim, 0, dim, c->moe_top);  // each slot from its expert's rank
    moe_combine(c->moe_y, dim, c->moe_top, c->moe_w, k, dim, n, c->x, dim, c->st);
}

void embed(engine_ctx *c, int n) {
    const engine_model *m = c->m;
    const DMat &e = m->tok_embd;
    const int32_t *ids = c->tokpos + 1;
    if (e.quant()) dequant_rows(e.q, ids, n, 0, c->x, m->info.dim, c->st);
    else {
        launch(embed_float_kernel, n, 256, 0, c->st, e.f, e.type, ids, m->info.dim, c->x);
        SDY_LAUNCHED();
    }
}

std::vector<const DMat *> mats_of(const Proj &p) {
    std::vector<const DMat *> v;
    for (const Part &q : p.parts) v.push_back(&q.m);
    return v;
}

// n <= n_batch tokens at the position stored in tokpos[0]; logits of the last out_rows tokens
// (model_llama.c:757-832).
void maybe_segment(engine_ctx *c, int layer);

void forward(engine_ctx *c, int n, int out_rows) {
    const engine_model *m = c->m;
    const engine_model_info &in = m->info;
    const int dim = in.dim, hd = in.head_dim, q_dim = in.n_head * hd;
    // this rank's heads (all of them unless attention is split across ranks)
    const int hq = m->h1 - m->h0, hkv = m->k1 - m->k0, q_loc = hq * hd, kv_loc = hkv * hd;
    const size_t layer_stride = (size_t)hkv * c->max_seq * hd;
    const int64_t QL = c->qkv_ld;
    const XQ *q8k, *q80;
    embed(c, n);
    for (int l = 0; l < in.n_layer; l++) {
        maybe_segment(c, l);
        const DLayer &L = m->layers[l];
        if (n == 1 && l + 1 < in.n_layer && (prefetch_mode(in) & PF_LAYER)) prefetch_layer(c, m->layers[l + 1]);
        float *kc = c->k_cache + l * layer_stride, *vc = c->v_cache + l * layer_stride;
        // attention: x = x + Wo . Attn(RoPE(Wq.norm(x)), RoPE(Wk.norm(x)), Wv.norm(x))
        if (fused_norm_ok(n, mats_of(L.qkv))) {
            project_act(c, L.qkv, c->qkv, QL, ActIn{c->x, dim, L.attn_norm, in.norm_eps}, n);
        } else {
            want_activations(c, mats_of(L.qkv), c->xb, dim, n, dim, &q8k, &q80);
            rmsnorm_quant(c->x, dim, L.attn_norm, dim, n, in.norm_eps, c->xb, dim, q8k, q80, c->st);
            project(c, L.qkv, c->qkv, QL, c->xb, dim, n);
        }
        PostQKV p{};
        p.q = c->qkv;
        p.k = c->qkv + q_loc;
        p.v = c->qkv + q_loc + kv_loc;
        p.ldq = p.ldk = p.ldv = QL;
        p.bq = L.bq;
        p.bk = L.bk;
        p.bv = L.bv;
        p.q_norm = L.q_norm;
        p.k_norm = L.k_norm;
        p.n_head = hq;
        p.n_kv_head = hkv;
        p.hd = hd;
        p.eps = in.norm_eps;
        p.cos = c->rope_cos;
        p.sin = c->rope_sin;
        p.pos_dev = c->tokpos;
        p.interleaved = in.rope_interleaved;
        p.kc = kc;
        p.vc = vc;
        p.max_seq = c->max_seq;
        if (m->attn_tp) {
            // this rank's heads, then every rank's head outputs gathered (an all-reduce of buffers
            // in which each column has one nonzero contributor), then this rank's rows [d0, d1) of
            // x + Wo . att, gathered likewise: every value is the one-GPU value
            float *aout = n == 1 ? c->attsend + (size_t)m->h0 * hd : c->att_loc;
            attention(aout, c->qkv, QL, kc, vc, n, hq, hkv, hd, 0, c->tokpos, c->max_seq, c->scores, 0, c->st, &p);
            if (n > 1)
                SDY_CUDA(cudaMemcpy2DAsync(c->attsend + (size_t)m->h0 * hd, (size_t)q_dim * 4, c->att_loc,
                                           (size_t)q_loc * 4, (size_t)q_loc * 4, n, cudaMemcpyDeviceToDevice, c->st));
            exchange(c, c->attsend, c->att, n, q_dim, (int64_t)m->h0 * hd, (int64_t)m->h1 * hd);
            forget_activations(c);
            if (n == 1 && fusion_enabled() && L.wo.quant())
                matmul_act(c, c->xsend + m->d0, dim, L.wo, ActIn{c->att, q_dim}, n, c->x + m->d0);
            else
                matmul(c, c->xsend + m->d0, dim, c->att, q_dim, L.wo, n, c->x + m->d0);
            exchange(c, c->xsend, c->x, n, dim, m->d0, m->d1);
        } else {
            attention(c->att, c->qkv, QL, kc, vc, n, hq, hkv, hd, 0, c->tokpos, c->max_seq, c->scores, 0, c->st, &p);
            forget_activations(c);
            if (n == 1 && fusion_enabled() && L.wo.quant())  // the attention output quantized in the prologue
                matmul_act(c, c->x, dim, L.wo, ActIn{c->att, q_dim}, n, c->x);
            else
                matmul(c, c->x, dim, c->att, q_dim, L.wo, n, c->x);
        }
        // MLP: x = x + down(silu(gate.norm(x)) * up.norm(x)), or its MoE
        const ActIn ffn_nin{c->x, dim, L.ffn_norm, in.norm_eps};
        if (in.n_expert && moe_decode_ok(c, L, n) && moe_block_decode(c, L)) {
            // norm, router, experts and combine in one kernel
        } else if (in.n_expert) {
            std::vector<const DMat *> need = mats_of(L.gateup);
            if (L.gate_inp.quant()) need.push_back(&L.gate_inp);
            if (moe_norm_fused(n, L, in)) {
                moe_ffn(c, L, n, &ffn_nin);
            } else {
                want_activations(c, need, c->xb, dim, n, dim, &q8k, &q80);
                rmsnorm_quant(c->x, dim, L.ffn_norm, dim, n, in.norm_eps, c->xb, dim, q8k, q80, c->st);
                moe_ffn(c, L, n);
            }
        } else {
            const int F = in.ffn_dim, GU = c->gu_ld;
            if (fused_norm_ok(n, mats_of(L.gateup))) {
                project_act(c, L.gateup, c->hgu, GU, ffn_nin, n);
            } else {
                want_activations(c, mats_of(L.gateup), c->xb, dim, n, dim, &q8k, &q80);
                rmsnorm_quant(c->x, dim, L.ffn_norm, dim, n, in.norm_eps, c->xb, dim, q8k, q80, c->st);
                project(c, L.gateup, c->hgu, GU, c->xb, dim, n);
            }
            if (m->world > 1) {
                // this rank's gate/up rows [f0, f1) -> its columns of the SiLU product, gathered to
                // every rank; its rows [d0, d1) of down -> its columns of x, gathered likewise
                const int nf = (int)(m->f1 - m->f0);
                silu_scatter(c->hgu, GU, c->hgu + nf, GU, nf, n, c->hsend + m->f0, F, c->st);
                exchange(c, c->hsend, c->hfull, n, F, m->f0, m->f1);
                forget_activations(c);
                matmul(c, c->xsend + m->d0, dim, c->hfull, F, L.down, n, c->x + m->d0);
                exchange(c, c->xsend, c->x, n, dim, m->d0, m->d1);
            } else {
                want_activations(c, {&L.down}, c->hgu, GU, n, F, &q8k, &q80);
                silu_quant(c->hgu, GU, c->hgu + F, GU, F, n, q8k, q80, c->st);
                matmul(c, c->x, dim, c->hgu, GU, L.down, n, c->x);
            }
        }
        if (c->forked) SDY_CUDA(cudaStreamWaitEvent(c->st, c->ev_join, 0));  // the side branch rejoins
        c->forked = false;
    }
    if (out_rows > 0) {
        // final norm and vocabulary projection for the requested rows only
        const float *xs = c->x + (size_t)(n - out_rows) * dim;
        float *lout = m->world > 1 ? c->lsend + m->v0 : c->logits;  // sharded: this rank's vocabulary rows
        if (fused_norm_ok(out_rows, {&m->output})) {
            forget_activations(c);
            matmul_act(c, lout, in.n_vocab, m->output, ActIn{xs, dim, m->output_norm, in.norm_eps}, out_rows);
        } else {
            want_activations(c, {&m->output}, c->xb, dim, out_rows, dim, &q8k, &q80);
            rmsnorm_quant(xs, dim, m->output_norm, dim, out_rows, in.norm_eps, c->xb, dim, q8k, q80, c->st);
            matmul(c, lout, in.n_vocab, c->xb, dim, m->output, out_rows);
        }
        if (m->world > 1) exchange(c, c->lsend, c->logits, out_rows, in.n_vocab, m->v0, m->v1);
    }
    forget_activations(c);
}

// One engine step of `chunk` tokens: staged token ids and position, then the forward. The
// single-token forward runs eagerly once, is captured as a CUDA graph on the next single-token
// step, and is replayed from then on (positions and ids are read from device memory).
void drop_graphs(engine_ctx *c) {
    for (cudaGraphExec_t e : c->step_graphs) cudaGraphExecDestroy(e);
    c->step_graphs.clear();
}

// Ends the capture in progress, instantiates it as the next segment and, unless `last`, opens the
// next capture. Failures are recorded in c->capture_ok.
void capture_segment(engine_ctx *c, bool last) {
    cudaGraph_t g = nullptr;
    bool ok = SDY_CUDA(cudaStreamEndCapture(c->st, &g)) && g;
    cudaGraphExec_t e = nullptr;
    ok = ok && SDY_CUDA(cudaGraphInstantiate(&e, g, 0));
    if (g) cudaGraphDestroy(g);
    if (ok) c->step_graphs.push_back(e);
    c->capture_ok = c->capture_ok && ok;
    if (!last && c->capture_ok)
        c->capture_ok = SDY_CUDA(cudaStreamBeginCapture(c->st, cudaStreamCaptureModeThreadLocal));
}

// Segment boundary inside forward(): every GRAPH_LAYERS layers while capturing.
constexpr int GRAPH_LAYERS = 4;
void maybe_segment(engine_ctx *c, int layer) {
    if (c->capturing && c->capture_ok && layer > 0 && layer % GRAPH_LAYERS == 0) capture_segment(c, false);
}

// One engine step of `chunk` tokens: staged token ids and position, then the forward. The
// single-token forward runs eagerly once, is captured as CUDA graphs on the next single-token
// step, and is replayed from then on (positions and ids are read from device memory).
void step(engine_ctx *c, const int32_t *tokens, int chunk, int out_rows) {
    c->h_tokpos[0] = c->n_past;
    memcpy(c->h_tokpos + 1, tokens, (size_t)chunk * 4);
    SDY_CUDA(cudaMemcpyAsync(c->tokpos, c->h_tokpos, (size_t)(chunk + 1) * 4, cudaMemcpyHostToDevice, c->st));
    if (chunk != 1 || out_rows != 1 || c->graph_state < 0) {
        forward(c, chunk, out_rows);
        return;
    }
    if (c->graph_state == 1) {
        for (cudaGraphExec_t e : c->step_graphs) SDY_CUDA(cudaGraphLaunch(e, c->st));
        return;
    }
    if (c->graph_state == 0) {
        forward(c, 1, 1);
        c->graph_state = 2;
        return;
    }
    c->capture_ok = SDY_CUDA(cudaStreamBeginCapture(c->st, cudaStreamCaptureModeThreadLocal));
    if (c->capture_ok) {
        c->capturing = true;
        forward(c, 1, 1);
        c->capturing = false;
        if (c->capture_ok) capture_segment(c, true);
    }
    if (c->capture_ok) {
        c->graph_state = 1;
        for (cudaGraphExec_t e : c->step_graphs) SDY_CUDA(cudaGraphLaunch(e, c->st));
    } else {  // capture unavailable: stay eager for this context
        cudaStreamCaptureStatus st = cudaStreamCaptureStatusNone;
        if (cudaStreamIsCapturing(c->st, &st) == cudaSuccess && st != cudaStreamCaptureStatusNone) {
            cudaGraph_t g = nullptr;
            cudaStreamEndCapture(c->st, &g);
            if (g) cudaGraphDestroy(g);
        }
        drop_graphs(c);
        clear_error();
        cudaGetLastError();
        c->graph_state = -1;
        forward(c, 1, 1);
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
    if (m->comm) nccl()->comm_destroy(m->comm);
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
    m->rank = g_shard.rank;
    m->world = g_shard.world;
    shard_range(in.ffn_dim, m->world, m->rank, GROUP_ROWS, &m->f0, &m->f1);
    shard_range(dim, m->world, m->rank, GROUP_ROWS, &m->d0, &m->d1);
    shard_range(in.n_expert, m->world, m->rank, 1, &m->e0, &m->e1);
    shard_range(in.n_vocab, m->world, m->rank, GROUP_ROWS, &m->v0, &m->v1);
    // SARDYNE_ATTN_TP=off: attention replicated on every rank (two exchanges less per layer:
    // lower batch-1 latency, but every rank holds all q/k/v/o rows and the whole KV cache)
    static const bool tp_off = [] {
        const char *v = getenv("SARDYNE_ATTN_TP");
        return v && !strcmp(v, "off");
    }();
    attention_split(in, m->world, m->rank, &m->attn_tp, &m->h0, &m->h1, &m->k0, &m->k1, !tp_off);
    if (m->world > 1) {
        const Nccl *nc = nccl();
        ncclResult_t r = nc ? nc->comm_init_rank(&m->comm, m->world, g_shard.id, m->rank) : ncclSystemError;
        if (r != ncclSuccess) {
            put_err(err, err_len, "NCCL non disponibile per il rank %d di %d: %s", m->rank, m->world,
                    nc ? nc->error_string(r) : "libnccl.so.2 mancante");
            m->comm = nullptr;
            engine_model_free(m);
            return nullptr;
        }
    }
    m->layers.resize(in.n_layer);
    // q / k / v rows this rank holds (all of them unless attention is split by heads)
    const int hd = in.head_dim;
    const std::vector<std::pair<int64_t, int64_t>> qkv_rows = {
        {(int64_t)m->h0 * hd, (int64_t)(m->h1 - m->h0) * hd},
        {(int64_t)m->k0 * hd, (int64_t)(m->k1 - m->k0) * hd},
        {(int64_t)m->k0 * hd, (int64_t)(m->k1 - m->k0) * hd}};
    bool ok = !get_tensor(m, "token_embd.weight", dim, in.n_vocab, 0, &m->tok_embd, err, err_len) &&
              !get_vector(m, "output_norm.weight", dim, &m->output_norm, err, err_len);
    if (ok) {
        const char *oname = in.tied_embeddings ? "token_embd.weight" : "output.weight";
        if (m->world > 1) ok = !get_tensor(m, oname, dim, in.n_vocab, 0, &m->output, err, err_len, m->v0, m->v1);
        else if (in.tied_embeddings) m->output = m->tok_embd;
        else ok = !get_tensor(m, oname, dim, in.n_vocab, 0, &m->output, err, err_len);
    }
    for (int l = 0; ok && l < in.n_layer; l++) {
        DLayer &L = m->layers[l];
        auto nm = [&](LayerTensor t) { return layer_tensor(l, t); };
        ok = !get_vector(m, nm(LT_ATTN_NORM).c_str(), dim, &L.attn_norm, err, err_len) &&
             !get_vector(m, nm(LT_FFN_NORM).c_str(), dim, &L.ffn_norm, err, err_len) &&
             !get_proj(m, {nm(LT_Q), nm(LT_K), nm(LT_V)}, {q_dim, kv_dim, kv_dim}, dim, 0, &L.qkv, err, err_len, 0,
                       -1, 0, -1, &qkv_rows) &&
             (m->attn_tp ? !get_tensor(m, nm(LT_WO).c_str(), q_dim, dim, 0, &L.wo, err, err_len, m->d0, m->d1)
                         : !get_tensor(m, nm(LT_WO).c_str(), q_dim, dim, 0, &L.wo, err, err_len));
        if (!ok) break;
        if (in.n_expert) {
            int ne = in.n_expert, fe = in.ffn_exp_dim;
            ok = !get_tensor(m, nm(LT_ROUTER).c_str(), dim, ne, 0, &L.gate_inp, err, err_len) &&
                 !get_proj(m, {nm(LT_GATE_EXPS), nm(LT_UP_EXPS)}, {fe, fe}, dim, ne, &L.gateup, err,
                           err_len, 0, -1, m->e0, m->e1) &&
                 !get_tensor(m, nm(LT_DOWN_EXPS).c_str(), fe, dim, ne, &L.down, err, err_len, 0, -1, m->e0,
                             m->e1);
        } else {
            ok = !get_proj(m, {nm(LT_GATE), nm(LT_UP)}, {in.ffn_dim, in.ffn_dim}, dim, 0,
                           &L.gateup, err, err_len, m->f0, m->f1) &&
                 !get_tensor(m, nm(LT_DOWN).c_str(), in.ffn_dim, dim, 0, &L.down, err, err_len, m->d0,
                             m->d1);
        }
        if (ok && in.qkv_bias)
            ok = !get_vector(m, nm(LT_Q_BIAS).c_str(), q_dim, &L.bq, err, err_len, qkv_rows[0].first,
                             (int)qkv_rows[0].second) &&
                 !get_vector(m, nm(LT_K_BIAS).c_str(), kv_dim, &L.bk, err, err_len, qkv_rows[1].first,
                             (int)qkv_rows[1].second) &&
                 !get_vector(m, nm(LT_V_BIAS).c_str(), kv_dim, &L.bv, err, err_len, qkv_rows[2].first,
                             (int)qkv_rows[2].second);
        if (ok && in.qk_norm)
            ok = !get_vector(m, nm(LT_Q_NORM).c_str(), in.head_dim, &L.q_norm, err, err_len) &&
                 !get_vector(m, nm(LT_K_NORM).c_str(), in.head_dim, &L.k_norm, err, err_len);
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

// Unmaps the peers' exchange buffers and frees this rank's.
void close_peer_exchange(engine_ctx *c) {
    for (int q = 0; q < c->px.world; q++) {
        if (!c->px.base[q]) continue;
        if (q == c->px.rank) cudaFree(c->px.base[q]);
        else cudaIpcCloseMemHandle(c->px.base[q]);
        c->px.base[q] = nullptr;
    }
    c->px_on = false;
}

// Context creation on the ranks of a sharded model, in step on all of them (every rank calls
// engine_ctx_new in the same order, failed or not): this rank's exchange buffer is allocated,
// zeroed and its CUDA IPC handle gathered to every rank (an NCCL all-gather), the peers' buffers
// are mapped, and one all-reduce tells every rank whether all contexts were created and whether
// all ranks can use the peer exchange; otherwise the exchanges stay on NCCL.
// SARDYNE_EXCHANGE=nccl (to be set on every rank alike) keeps them on NCCL.
bool shard_context(engine_ctx *c, bool ok, char *err, size_t err_len) {
    const engine_model *m = c->m;
    const engine_model_info &in = m->info;
    const int world = m->world;
    static const bool want = [] {
        const char *v = getenv("SARDYNE_EXCHANGE");
        return !(v && !strcmp(v, "nccl"));
    }();
    int64_t cap = std::max<int64_t>({(int64_t)in.n_head * in.head_dim, (int64_t)in.dim, (int64_t)in.n_vocab});
    cap = std::max<int64_t>(cap, in.n_expert ? (int64_t)in.n_expert_used * in.dim : (int64_t)in.ffn_dim);
    cap = (int64_t)align_up((size_t)cap, 64);  // the second staging half starts 256-byte aligned
    c->px.cap = cap;
    // how long an exchange waits for the other ranks before it gives up (the ranks' host threads
    // only meet at these exchanges, so one may lag behind another by its own host work)
    static const unsigned long long wait_ns = [] {
        const char *v = getenv("SARDYNE_EXCHANGE_WAIT_MS");
        const long long ms = v ? atoll(v) : 0;
        return (unsigned long long)(ms > 0 ? ms : 4000) * 1000000ull;
    }();
    c->px.wait_ns = wait_ns;
    c->px.rank = m->rank;
    c->px.world = world;
    cudaStream_t s = c->st;
    bool own_stream = false;
    if (!s) own_stream = cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking) == cudaSuccess;
    uint8_t *scratch = nullptr;  // [0, 64): this rank's handle, [64, 64 + 64 * world): all, then 2 floats
    const size_t sbytes = 64 + 64 * (size_t)world + 64;
    bool px_ok = ok && want && world <= PX_MAX_WORLD;
    std::vector<uint8_t> handles(64 * (size_t)world + 64, 0);
    void *own = nullptr;
    if (px_ok) {
        const size_t bytes = peer_exchange_bytes(cap);
        cudaIpcMemHandle_t h{};
        px_ok = cudaMalloc(&own, bytes) == cudaSuccess && cudaMemset(own, 0, bytes) == cudaSuccess &&
                cudaDeviceSynchronize() == cudaSuccess && cudaIpcGetMemHandle(&h, own) == cudaSuccess;
        if (px_ok) memcpy(handles.data(), &h, sizeof h);
    }
    bool net = s && cudaMalloc((void **)&scratch, sbytes) == cudaSuccess;
    const Nccl *nc = nccl();
    if (net && want) {  // the handles, all ranks' to every rank (zeros from a rank that has none)
        net = cudaMemcpy(scratch, handles.data(), 64, cudaMemcpyHostToDevice) == cudaSuccess &&
              nc->all_gather(scratch, scratch + 64, 64, ncclUint8, m->comm, s) == ncclSuccess &&
              cudaMemcpyAsync(handles.data() + 64, scratch + 64, 64 * (size_t)world, cudaMemcpyDeviceToHost, s) ==
                  cudaSuccess &&
              cudaStreamSynchronize(s) == cudaSuccess;
    }
    px_ok = px_ok && net;
    if (px_ok) {
        c->px.base[m->rank] = own;
        own = nullptr;
        for (int q = 0; q < world && px_ok; q++) {
            if (q == m->rank) continue;
            cudaIpcMemHandle_t h;
            memcpy(&h, handles.data() + 64 + 64 * (size_t)q, sizeof h);
            void *peer = nullptr;
            px_ok = cudaIpcOpenMemHandle(&peer, h, cudaIpcMemLazyEnablePeerAccess) == cudaSuccess;
            c->px.base[q] = px_ok ? peer : nullptr;
        }
    }
    float votes[2] = {ok ? 1.f : 0.f, px_ok ? 1.f : 0.f};
    float *dv = (float *)(scratch + 64 + 64 * (size_t)world);
    net = net && cudaMemcpy(dv, votes, sizeof votes, cudaMemcpyHostToDevice) == cudaSuccess &&
          nc->all_reduce(dv, dv, 2, ncclFloat32, ncclSum, m->comm, s) == ncclSuccess &&
          cudaMemcpyAsync(votes, dv, sizeof votes, cudaMemcpyDeviceToHost, s) == cudaSuccess &&
          cudaStreamSynchronize(s) == cudaSuccess;
    if (own) cudaFree(own);
    if (scratch) cudaFree(scratch);
    if (own_stream) cudaStreamDestroy(s);
    cudaGetLastError();  // a refused peer mapping is not an error of the context
    const bool all_ok = net && votes[0] == (float)world;
    c->px_on = all_ok && votes[1] == (float)world;
    if (!c->px_on) close_peer_exchange(c);
    if (ok && !all_ok)
        put_err(err, err_len, net ? "un altro rank non ha potuto creare il contesto"
                                  : "scambio NCCL fallito durante la creazione del contesto");
    return all_ok;
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
    if (getenv("SARDYNE_NO_GRAPH")) c->graph_state = -1;
    const engine_model_info &in = m->info;
    const size_t B = n_batch, S = max_seq, hd = in.head_dim;
    const size_t q_dim = (size_t)in.n_head * hd;
    // this rank's heads (all of them unless attention is split across ranks)
    const size_t q_loc = (size_t)(m->h1 - m->h0) * hd, kv_loc = (size_t)(m->k1 - m->k0) * hd;
    const size_t kv = (size_t)in.n_layer * (m->k1 - m->k0) * S * hd;
    const size_t ffn = in.n_expert ? in.ffn_exp_dim : in.ffn_dim;
    const size_t K = in.n_expert ? in.n_expert_used : 0, slots = B * K;
    c->qkv_ld = (int)(q_loc + 2 * kv_loc);
    c->gu_ld = (int)(2 * (in.n_expert ? ffn : (size_t)(m->f1 - m->f0)));
    const size_t tmp_n = std::max<size_t>((size_t)in.dim, (size_t)in.n_vocab) * B;
    struct Item {
        void **dst;
        size_t bytes;
    };
    std::vector<Item> items = {
        {(void **)&c->k_cache, kv * 4}, {(void **)&c->v_cache, kv * 4},
        {(void **)&c->rope_cos, S * hd / 2 * 4}, {(void **)&c->rope_sin, S * hd / 2 * 4},
        {(void **)&c->x, B * in.dim * 4}, {(void **)&c->xb, B * in.dim * 4},
        {(void **)&c->qkv, B * c->qkv_ld * 4}, {(void **)&c->att, B * q_dim * 4},
        {(void **)&c->hgu, B * c->gu_ld * 4}, {(void **)&c->tmp, tmp_n * 4},
        {(void **)&c->scores, B * in.n_head * S * 4},
        {(void **)&c->logits, (c->logits_all ? B : 1) * in.n_vocab * 4},
        {(void **)&c->tokpos, (B + 1) * 4},
        {(void **)&c->am_v, ARGMAX_CTAS * 4}, {(void **)&c->am_i, ARGMAX_CTAS * 4},
        {(void **)&c->am_count, 4}, {(void **)&c->am_out, 4},
    };
    if (in.n_expert) {
        items.push_back({(void **)&c->moe_probs, B * in.n_expert * 4});
        items.push_back({(void **)&c->moe_count, B * 4});
        items.push_back({(void **)&c->md_sync, 4 * sizeof(unsigned)});
        items.push_back({(void **)&c->grp_off, ((size_t)in.n_expert + 2) * 4});
        items.push_back({(void **)&c->grp_slot, slots * 4});
        items.push_back({(void **)&c->grp_tiles, (slots / GEMM_TILE_TOKENS + in.n_expert) * 4});
        items.push_back({(void **)&c->moe_w, slots * 4});
        items.push_back({(void **)&c->moe_top, slots * 4});
        items.push_back({(void **)&c->moe_gu, slots * 2 * ffn * 4});
        items.push_back({(void **)&c->moe_y, slots * in.dim * 4});
    }
    const size_t logit_rows = c->logits_all ? B : 1;
    if (m->world > 1) {
        if (!in.n_expert) {
            items.push_back({(void **)&c->hsend, B * ffn * 4});
            items.push_back({(void **)&c->hfull, B * ffn * 4});
        }
        if (!in.n_expert || m->attn_tp) items.push_back({(void **)&c->xsend, B * in.dim * 4});
        if (m->attn_tp) {
            items.push_back({(void **)&c->att_loc, B * q_loc * 4});
            items.push_back({(void **)&c->attsend, B * q_dim * 4});
        }
        items.push_back({(void **)&c->lsend, logit_rows * in.n_vocab * 4});
    }
    size_t xq_cap = 0;
    for (int vt : {T_Q8_0, T_Q8_K}) {
        int be = block_elems(vt);
        for (size_t nin : {(size_t)in.dim, q_dim, ffn})
            if (nin % be == 0) xq_cap = std::max(xq_cap, xq_bytes(vt, (int)nin, (int)B));
        if (in.n_expert && ffn % be == 0) xq_cap = std::max(xq_cap, xq_bytes(vt, (int)ffn, (int)slots));
    }
    items.push_back({&c->xq_buf[0], xq_cap});
    items.push_back({&c->xq_buf[1], xq_cap});
    size_t total = 0;
    for (auto &it : items) total += align_up(it.bytes, 256);
    // Failures below do not return at once: the ranks of a sharded model still agree on the
    // outcome together (shard_context), so that none of them waits for a rank that gave up.
    bool ok = SDY_CUDA(cudaMalloc(&c->arena, total));
    if (!ok) put_err(err, err_len, "memoria GPU esaurita (%.1f MB per contesto e KV cache)", total / 1e6);
    if (ok) {
        uint8_t *p = (uint8_t *)c->arena;
        for (auto &it : items) {
            *it.dst = p;
            p += align_up(it.bytes, 256);
        }
        bool zeroed = true;  // all-reduce sources start (and outside this rank's columns stay) zero
        if (c->hsend) zeroed = SDY_CUDA(cudaMemset(c->hsend, 0, B * ffn * 4));
        if (c->xsend) zeroed = zeroed && SDY_CUDA(cudaMemset(c->xsend, 0, B * in.dim * 4));
        if (c->attsend) zeroed = zeroed && SDY_CUDA(cudaMemset(c->attsend, 0, B * q_dim * 4));
        if (c->lsend) zeroed = zeroed && SDY_CUDA(cudaMemset(c->lsend, 0, logit_rows * in.n_vocab * 4));
        if (c->md_sync) zeroed = zeroed && SDY_CUDA(cudaMemset(c->md_sync, 0, 4 * sizeof(unsigned)));
        zeroed = zeroed && SDY_CUDA(cudaMemset(c->am_count, 0, 4));
        ok = zeroed && (!c->moe_count || SDY_CUDA(cudaMemset(c->moe_count, 0, B * 4)));  // router counters start at zero
        if (!ok) put_err(err, err_len, "inizializzazione del contesto fallita: %s", last_error());
    }
    size_t lbytes = (c->logits_all ? B : 1) * in.n_vocab * 4;
    if (ok && (!SDY_CUDA(cudaStreamCreateWithFlags(&c->st, cudaStreamNonBlocking)) ||
               !SDY_CUDA(cudaStreamCreateWithFlags(&c->side, cudaStreamNonBlocking)) ||
               !SDY_CUDA(cudaEventCreateWithFlags(&c->ev_fork, cudaEventDisableTiming)) ||
               !SDY_CUDA(cudaEventCreateWithFlags(&c->ev_join, cudaEventDisableTiming)) ||
               !SDY_CUDA(cudaMallocHost(&c->h_logits, lbytes)) || !SDY_CUDA(cudaMallocHost(&c->h_tokpos, (B + 1) * 4)) ||
               !SDY_CUDA(cudaMallocHost(&c->h_md_status, sizeof(unsigned))) ||
               !SDY_CUDA(cudaMallocHost(&c->h_px_status, sizeof(unsigned))) ||
               !SDY_CUDA(cudaMallocHost(&c->h_am_out, sizeof(int32_t))))) {
        put_err(err, err_len, "inizializzazione del contesto fallita: %s", last_error());
        ok = false;
    }
    if (ok) {
        rope_table(c->rope_cos, c->rope_sin, max_seq, in.head_dim, in.rope_theta, c->st);
        ok = SDY_CUDA(cudaStreamSynchronize(c->st));
        if (!ok) put_err(err, err_len, "inizializzazione del contesto fallita: %s", last_error());
    }
    if (m->world > 1) ok = shard_context(c, ok, err, err_len) && ok;
    if (!ok) {
        engine_ctx_free(c);
        return nullptr;
    }
    return c;
}

int32_t engine_ctx_n_threads(const engine_ctx *c) { return c ? c->n_threads : 0; }

void engine_ctx_free(engine_ctx *c) {
    if (!c) return;
    drop_graphs(c);
    close_peer_exchange(c);
    if (c->h_px_status) cudaFreeHost(c->h_px_status);
    if (c->st) cudaStreamDestroy(c->st);
    if (c->side) cudaStreamDestroy(c->side);
    if (c->ev_fork) cudaEventDestroy(c->ev_fork);
    if (c->ev_join) cudaEventDestroy(c->ev_join);
    if (c->arena) cudaFree(c->arena);
    if (c->h_logits) cudaFreeHost(c->h_logits);
    if (c->h_tokpos) cudaFreeHost(c->h_tokpos);
    if (c->h_md_status) cudaFreeHost(c->h_md_status);
    if (c->h_am_out) cudaFreeHost(c->h_am_out);
    delete c;
}

namespace {
// engine_eval, with the last token's greedy choice made on the device instead of the logits
// copied back when `next` is set.
int eval_tokens(engine_ctx *c, const int32_t *tokens, int32_t n, int32_t *next) {
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
    if (c->px_failed) {
        snprintf(c->err, sizeof c->err, "contesto inutilizzabile: uno scambio tra GPU era scaduto");
        return -1;
    }
    cudaSetDevice(c->m->dev);
    clear_error();
    const int saved = c->n_past;
    int out_rows = 0;
    for (int done = 0; done < n;) {
        int chunk = std::min(n - done, c->n_batch);
        bool last = done + chunk == n;
        out_rows = last ? (c->logits_all ? chunk : 1) : 0;
        step(c, tokens + done, chunk, out_rows);
        if (!last) SDY_CUDA(cudaStreamSynchronize(c->st));  // the staging buffer is reused by the next chunk
        c->n_past += chunk;
        done += chunk;
    }
    const int nv = c->m->info.n_vocab;
    if (next) {
        launch(argmax_kernel, ARGMAX_CTAS, ARGMAX_THREADS, 0, c->st, c->logits + (size_t)(out_rows - 1) * nv, nv,
               c->am_v, c->am_i, c->am_count, c->am_out);
        SDY_LAUNCHED();
        SDY_CUDA(cudaMemcpyAsync(c->h_am_out, c->am_out, 4, cudaMemcpyDeviceToHost, c->st));
    } else {
        SDY_CUDA(cudaMemcpyAsync(c->h_logits, c->logits, (size_t)out_rows * nv * 4, cudaMemcpyDeviceToHost, c->st));
    }
    if (c->md_sync) SDY_CUDA(cudaMemcpyAsync(c->h_md_status, c->md_sync + 3, sizeof(unsigned), cudaMemcpyDeviceToHost, c->st));
    if (c->px_on) SDY_CUDA(cudaMemcpyAsync(c->h_px_status, peer_status(c->px), sizeof(unsigned), cudaMemcpyDeviceToHost, c->st));
    SDY_CUDA(cudaStreamSynchronize(c->st));
    if (c->px_on && *c->h_px_status) {  // a peer exchange gave up waiting for another rank
        set_error("scambio tra GPU: attesa di un altro rank scaduta");
        c->px_failed = true;
    }
    if (c->md_sync && *c->h_md_status) {  // a grid barrier of the fused MoE block gave up
        set_error("blocco MoE: attesa tra i blocchi della griglia scaduta");
        cudaMemsetAsync(c->md_sync, 0, 4 * sizeof(unsigned), c->st);
        cudaStreamSynchronize(c->st);
        *c->h_md_status = 0;
    }
    if (last_error()[0]) {
        c->n_past = saved;
        snprintf(c->err, sizeof c->err, "errore GPU: %s", last_error());
        return -1;
    }
    c->n_logits = next ? 0 : c->logits_all ? n : 1;
    if (next) *next = *c->h_am_out;
    return 0;
}
}  // namespace

int engine_eval(engine_ctx *c, const int32_t *tokens, int32_t n) { return eval_tokens(c, tokens, n, nullptr); }

int sdy_engine_eval_greedy(engine_ctx *c, const int32_t *tokens, int32_t n, int32_t *next) {
    if (c && !next) {
        snprintf(c->err, sizeof c->err, "sdy_engine_eval_greedy: next NULL");
        return -1;
    }
    return eval_tokens(c, tokens, n, next);
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

int sdy_nccl_unique_id(void *out) {
    const Nccl *nc = nccl();
    ncclUniqueId id;
    if (!out || !nc || nc->get_unique_id(&id) != ncclSuccess) {
        set_error("sdy_nccl_unique_id: %s", nc ? "ncclGetUniqueId failed" : "libnccl.so.2 missing");
        return -1;
    }
    memcpy(out, &id, sizeof id);
    return 0;
}

int sdy_engine_set_shard(int32_t rank, int32_t world, const void *nccl_id) {
    if (world < 1 || rank < 0 || rank >= world || (world > 1 && !nccl_id)) {
        set_error("sdy_engine_set_shard: rank %d of %d invalid", rank, world);
        return -1;
    }
    g_shard.rank = rank;
    g_shard.world = world;
    if (world > 1) memcpy(&g_shard.id, nccl_id, sizeof g_shard.id);
    return 0;
}

void sdy_engine_get_shard(int32_t *rank, int32_t *world) {
    if (rank) *rank = g_shard.rank;
    if (world) *world = g_shard.world;
}

int sdy_attention_split(int32_t n_head, int32_t n_kv_head, int32_t head_dim, int32_t world, int32_t rank,
                        int32_t *range) {
    if (n_head < 1 || n_kv_head < 1 || n_head % n_kv_head || head_dim < 1 || world < 1 || rank < 0 || rank >= world ||
        !range)
        return -1;
    engine_model_info in{};
    in.n_head = n_head;
    in.n_kv_head = n_kv_head;
    in.head_dim = head_dim;
    bool tp = false;
    attention_split(in, world, rank, &tp, &range[0], &range[1], &range[2], &range[3]);
    return tp ? 1 : 0;
}

int sdy_engine_exchange(const engine_ctx *c) { return !c || c->m->world < 2 ? -1 : c->px_on ? 1 : 0; }

void sdy_shard_range(int64_t n, int32_t world, int32_t rank, int64_t align, int64_t *begin, int64_t *end) {
    int64_t b = 0, e = n;
    if (world >= 1 && rank >= 0 && rank < world && align >= 1 && n >= 0) shard_range(n, world, rank, align, &b, &e);
    if (begin) *begin = b;
    if (end) *end = e;
}

}  // extern "C"
