// Launchers of the fused per-token kernels (fused.cu). All asynchronous on stream s.
#pragma once
#include "common.cuh"

namespace sdy {

// xb = RMSNorm(x) * w (optional f32 copy) and its quantization into q8k and/or q80 (either may be null).
void rmsnorm_quant(const float *x, int64_t ldx, const float *w, int n, int rows, float eps, float *xb, int64_t ldb,
                   const XQ *q8k, const XQ *q80, cudaStream_t s);
// g = silu(g) * u in place, then quantized into q8k and/or q80.
void silu_quant(float *g, int64_t ldg, const float *u, int64_t ldu, int n, int rows, const XQ *q8k, const XQ *q80,
                cudaStream_t s);

// dst[t*ldd + i] = silu(g) * u for i < n (no quantization): sharded FFN rows.
void silu_scatter(const float *g, int64_t ldg, const float *u, int64_t ldu, int n, int rows, float *dst, int64_t ldd,
                  cudaStream_t s);

struct PostQKV {
    float *q, *k;
    const float *v;
    int64_t ldq, ldk, ldv;          // token strides
    const float *bq, *bk, *bv;      // biases or null
    const float *q_norm, *k_norm;   // qk-norm weights or null
    int n_head, n_kv_head, hd;
    float eps;
    const float *cos, *sin;         // RoPE tables [max_seq][hd/2]
    const int32_t *pos_dev;         // position of token 0 read on the device, or null: pos0
    int pos0, interleaved;
    float *kc, *vc;                 // this layer's cache [n_kv_head][max_seq][hd]
    int max_seq;
};
// Bias, qk-norm, RoPE on q and k, then k and v into the KV cache.
void post_qkv(const PostQKV &p, int n_tok, cudaStream_t s);

// Float router: top [n_tok][k] expert ids and renormalised weights; logits is scratch [n_tok][ne];
// counters: n_tok int32 that start at zero (the kernel leaves them at zero).
// Byte ranges to pull into L2 (hints): upcoming weights.
constexpr int PF_RANGES = 8;
struct L2Ranges {
    const void *p[PF_RANGES];
    size_t bytes[PF_RANGES];
    int n = 0;
    void add(const void *ptr, size_t b) {
        if (ptr && b && n < PF_RANGES) {
            p[n] = ptr;
            bytes[n++] = b;
        }
    }
};
void l2_prefetch(const L2Ranges &r, cudaStream_t s);
// Expert matrices [m] (gate, up, down or gate|up, down): expert e0 + e at base[m] + e * bytes[m],
// e < n_local.
constexpr int PF_EXPERT_MATS = 3;
struct ExpertPrefetch {
    const void *base[PF_EXPERT_MATS] = {};
    size_t bytes[PF_EXPERT_MATS] = {};
    int e0 = 0, n_local = 0;
};
// Pulls the matrices of the experts named by top[0, n_slots) into L2.
void expert_prefetch(const ExpertPrefetch &ep, const int32_t *top, int n_slots, cudaStream_t s);
// Whether router_topk takes this shape (its shared memory holds the CTA's router rows and x).
bool router_topk_supported(int dim, int ne, int k, int n_tok, bool norm);
// norm_w: the router input is RMSNorm(x) * norm_w, computed inside the kernel (x the residual).
void router_topk(const float *x, int64_t ldx, const void *w, int wtype, int dim, int ne, int k, int n_tok,
                 int32_t *top, float *wout, float *logits, int32_t *counters, cudaStream_t s,
                 const float *norm_w = nullptr, float norm_eps = 0.0f);
// Slots grouped by expert e0 + e (e < ne): slots[off[e] .. off[e+1]); tiles[0 .. off[ne+1]) lists
// (e << 16 | token tile) for every `tile` slots of every expert (off: ne + 2 ints).
void moe_group(const int32_t *top, int n_slots, int e0, int ne, int tile, int32_t *off, int32_t *slots,
               int32_t *tiles, cudaStream_t s);
// x[t] += sum over t's k slots in ascending expert id of w * y[slot].
void moe_combine(const float *y, int64_t ldy, const int32_t *top, const float *w, int k, int dim, int n_tok, float *x,
                 int64_t ldx, cudaStream_t s);

// The MoE block of one token in one kernel (moe_decode.cu): x += the k chosen experts' SwiGLU
// FFNs of RMSNorm(x) * norm_w, weighted by the renormalised router probabilities. gu_slabs: the
// fused gate|up matrices of all experts (2 * fe rows each, gpe_gu groups per expert); dn_slabs:
// the down matrices (dim rows each, gpe_dn groups). Scratch: logits [ne], top/wts [k],
// gu [k][2 fe], y [k][dim]; bar: 3 words and status: 1 word, zero before the first launch (a
// nonzero status after a step means a grid barrier gave up; the words must then be cleared).
struct MoeDecode {
    float *x;
    const float *norm_w;
    float eps;
    int dim;
    const void *router;
    int rtype, ne, k;
    const uint8_t *gu_slabs;
    int64_t gpe_gu;
    int fe;
    const uint8_t *dn_slabs;
    int64_t gpe_dn;
    float *logits;
    int32_t *top;
    float *wts, *gu, *y;
    unsigned *bar, *status;
};
bool moe_decode_supported(int tg, int td, int rtype, int dim, int fe, int ne, int k);
// False (nothing launched) when this GPU cannot hold the grid at once.
bool moe_decode(const MoeDecode &a, int tg, int td, cudaStream_t s);

}  // namespace sdy
