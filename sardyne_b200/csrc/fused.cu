// Fused per-token kernels of the decode/prefill forward. Each replaces two to four of the
// reference's sequential steps with one launch while keeping its operation order, so results
// are the same floats as the unfused chain:
//   rmsnorm_quant  op_rmsnorm (ops.c:346-351) + op_quantize_rows (quant.c:98-144)
//   post_qkv       op_add_bias + qk RMSNorm + op_rope + KV-cache store (model_llama.c:781-800)
//   silu_quant     op_silu_mul (ops.c:366-371) + op_quantize_rows
//   router_topk    F32 router matvec + op_softmax + moe_select (model_llama.c:653-684)
//   moe_combine    sum over a token's experts in ascending id + residual add (model_llama.c:734-750, 820)
#include "fused.cuh"
#include "quant_device.cuh"

namespace sdy {
namespace {

__device__ __forceinline__ float exp_cr(float x) { return (float)exp((double)x); }

__device__ double bsum_d(double v, double *part) {
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
    __syncthreads();
    if (lane == 0) part[w] = v;
    __syncthreads();
    v = lane < (int)(blockDim.x >> 5) ? part[lane] : 0.0;
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ float bmax_f(float v, float *part) {
    for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
    __syncthreads();
    if (lane == 0) part[w] = v;
    __syncthreads();
    v = lane < (int)(blockDim.x >> 5) ? part[lane] : -INFINITY;
    for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// Quantize the row in shared memory into the requested activation types (warps take 256-spans).
__device__ void quantize_smem_row(const float *row, int n, int t, const XQ &q8k, const XQ &q80) {
    const int warp = threadIdx.x >> 5, nw = blockDim.x >> 5, spans = (n + 255) / 256;
    for (int sp = warp; sp < spans; sp += nw) {
        if (q8k.qs) quant_q8k_block(row, t, sp, q8k);
        if (q80.qs) quant_q80_span(row, t, sp, n, q80);
    }
}

__global__ void rmsnorm_quant_kernel(const float *x, int64_t ldx, const float *w, int n, float eps, float *xb,
                                     int64_t ldb, XQ q8k, XQ q80) {
    extern __shared__ __align__(16) float row[];
    __shared__ double part[32];
    const int t = blockIdx.x;
    const float *xv = x + (size_t)t * ldx;
    double ss = 0.0;
    for (int i = threadIdx.x; i < n; i += blockDim.x) ss += (double)xv[i] * xv[i];
    ss = bsum_d(ss, part);
    const float scale = (float)(1.0 / sqrt(ss / n + (double)eps));
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        float v = __fmul_rn(__fmul_rn(xv[i], scale), w[i]);
        row[i] = v;
        if (xb) xb[(size_t)t * ldb + i] = v;
    }
    __syncthreads();
    quantize_smem_row(row, n, t, q8k, q80);
}

__global__ void silu_quant_kernel(float *g, int64_t ldg, const float *u, int64_t ldu, int n, XQ q8k, XQ q80) {
    extern __shared__ __align__(16) float row[];
    const int t = blockIdx.x;
    float *gv = g + (size_t)t * ldg;
    const float *uv = u + (size_t)t * ldu;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        float a = gv[i];
        float h = __fmul_rn(__fdiv_rn(a, __fadd_rn(1.0f, exp_cr(-a))), uv[i]);
        row[i] = h;
        gv[i] = h;
    }
    __syncthreads();
    quantize_smem_row(row, n, t, q8k, q80);
}

// One block per (head, token). Heads [0, n_head) are q heads; [n_head, n_head + n_kv_head) are
// k heads, whose block also handles the v head with the same index.
__global__ void post_qkv_kernel(PostQKV p) {
    extern __shared__ __align__(16) float vec[];
    __shared__ double part[32];
    const int t = blockIdx.y, hh = blockIdx.x, hd = p.hd, half = hd / 2;
    const bool is_q = hh < p.n_head;
    const int h = is_q ? hh : hh - p.n_head;
    const int pos = (p.pos_dev ? *p.pos_dev : p.pos0) + t;
    float *gv = is_q ? p.q + (size_t)t * p.ldq + (size_t)h * hd : p.k + (size_t)t * p.ldk + (size_t)h * hd;
    const float *bias = is_q ? p.bq : p.bk;
    const float *norm = is_q ? p.q_norm : p.k_norm;
    for (int i = threadIdx.x; i < hd; i += blockDim.x) {
        float v = gv[i];
        if (bias) v = __fadd_rn(v, bias[(size_t)h * hd + i]);
        vec[i] = v;
    }
    __syncthreads();
    if (norm) {  // per-head RMSNorm (Qwen3 qk-norm), model_llama.c:790-793
        double ss = 0.0;
        for (int i = threadIdx.x; i < hd; i += blockDim.x) ss += (double)vec[i] * vec[i];
        ss = bsum_d(ss, part);
        const float scale = (float)(1.0 / sqrt(ss / hd + (double)p.eps));
        for (int i = threadIdx.x; i < hd; i += blockDim.x) vec[i] = __fmul_rn(__fmul_rn(vec[i], scale), norm[i]);
        __syncthreads();
    }
    const float *c = p.cos + (size_t)pos * half, *sn = p.sin + (size_t)pos * half;
    for (int i = threadIdx.x; i < half; i += blockDim.x) {  // RoPE, ops.c:388-403
        int ia = p.interleaved ? 2 * i : i, ib = p.interleaved ? 2 * i + 1 : i + half;
        float a = vec[ia], b = vec[ib];
        vec[ia] = __fsub_rn(__fmul_rn(a, c[i]), __fmul_rn(b, sn[i]));
        vec[ib] = __fadd_rn(__fmul_rn(a, sn[i]), __fmul_rn(b, c[i]));
    }
    __syncthreads();
    for (int i = threadIdx.x; i < hd; i += blockDim.x) gv[i] = vec[i];
    if (is_q) return;
    const size_t dst = ((size_t)h * p.max_seq + pos) * hd;
    const float *vv = p.v + (size_t)t * p.ldv + (size_t)h * hd;
    for (int i = threadIdx.x; i < hd; i += blockDim.x) {
        p.kc[dst + i] = vec[i];
        float x = vv[i];
        if (p.bv) x = __fadd_rn(x, p.bv[(size_t)h * hd + i]);
        p.vc[dst + i] = x;
    }
}

// Router for float weights, one block per token: logits (the reference's scalar dot order),
// softmax, stable top-k with ties to the lowest index, weights renormalised by their sum.
__global__ void router_topk_kernel(const float *x, int64_t ldx, const void *w, int wtype, int dim, int ne, int k,
                                   int32_t *top, float *wout, float *probs_out) {
    extern __shared__ __align__(16) float prob[];
    __shared__ double dpart[32];
    __shared__ float fpart[32];
    const int t = blockIdx.x;
    const float *xv = x + (size_t)t * ldx;
    for (int e = threadIdx.x; e < ne; e += blockDim.x) {
        size_t base = (size_t)e * dim;
        float s0 = 0.0f, s1 = 0.0f, s2 = 0.0f, s3 = 0.0f;
        auto wv = [&](int i) -> float {
            if (wtype == T_F32) return ((const float *)w)[base + i];
            if (wtype == T_F16) return __half2float(((const __half *)w)[base + i]);
            return __uint_as_float((uint32_t)((const uint16_t *)w)[base + i] << 16);
        };
        int i = 0;
        for (; i + 4 <= dim; i += 4) {
            s0 = __fadd_rn(s0, __fmul_rn(xv[i], wv(i)));
            s1 = __fadd_rn(s1, __fmul_rn(xv[i + 1], wv(i + 1)));
            s2 = __fadd_rn(s2, __fmul_rn(xv[i + 2], wv(i + 2)));
            s3 = __fadd_rn(s3, __fmul_rn(xv[i + 3], wv(i + 3)));
        }
        for (; i < dim; i++) s0 = __fadd_rn(s0, __fmul_rn(xv[i], wv(i)));
        prob[e] = __fadd_rn(__fadd_rn(s0, s1), __fadd_rn(s2, s3));
    }
    __syncthreads();
    float m = -INFINITY;
    for (int e = threadIdx.x; e < ne; e += blockDim.x) m = fmaxf(m, prob[e]);
    m = bmax_f(m, fpart);
    double sum = 0.0;
    for (int e = threadIdx.x; e < ne; e += blockDim.x) {
        float v = exp_cr(__fsub_rn(prob[e], m));
        prob[e] = v;
        sum += v;
    }
    sum = bsum_d(sum, dpart);
    const float inv = (float)(1.0 / sum);
    for (int e = threadIdx.x; e < ne; e += blockDim.x) prob[e] = __fmul_rn(prob[e], inv);
    __syncthreads();
    if (probs_out)
        for (int e = threadIdx.x; e < ne; e += blockDim.x) probs_out[(size_t)t * ne + e] = prob[e];
    if (threadIdx.x != 0) return;
    int32_t *tp = top + (size_t)t * k;
    int n = 0;
    for (int e = 0; e < ne; e++) {
        int pos = n;
        while (pos > 0 && prob[e] > prob[tp[pos - 1]]) pos--;
        if (pos == k) continue;
        for (int j = n < k ? n : k - 1; j > pos; j--) tp[j] = tp[j - 1];
        tp[pos] = e;
        if (n < k) n++;
    }
    float s = 0.0f;
    for (int i = 0; i < k; i++) s = __fadd_rn(s, prob[tp[i]]);
    for (int i = 0; i < k; i++) wout[(size_t)t * k + i] = __fdiv_rn(prob[tp[i]], s);
}

// x[t] += sum over t's k slots, in ascending expert id, of w * y[slot].
__global__ void moe_combine_kernel(const float *y, int64_t ldy, const int32_t *top, const float *w, int k, int dim,
                                   float *x, int64_t ldx) {
    const int t = blockIdx.y;
    int order[64];
    for (int i = 0; i < k; i++) order[i] = i;
    for (int i = 1; i < k; i++) {
        int s = order[i], j = i;
        while (j > 0 && top[(size_t)t * k + order[j - 1]] > top[(size_t)t * k + s]) { order[j] = order[j - 1]; j--; }
        order[j] = s;
    }
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < dim; i += gridDim.x * blockDim.x) {
        float acc = 0.0f;
        for (int j = 0; j < k; j++) {
            int s = order[j];
            acc = __fadd_rn(acc, __fmul_rn(w[(size_t)t * k + s], y[((size_t)t * k + s) * ldy + i]));
        }
        float *xp = x + (size_t)t * ldx + i;
        *xp = __fadd_rn(*xp, acc);
    }
}

int row_threads(int n) { return n >= 1024 ? 512 : n >= 256 ? 256 : 128; }

}  // namespace

void rmsnorm_quant(const float *x, int64_t ldx, const float *w, int n, int rows, float eps, float *xb, int64_t ldb,
                   const XQ *q8k, const XQ *q80, cudaStream_t s) {
    if (rows <= 0) return;
    XQ a = q8k ? *q8k : XQ(), b = q80 ? *q80 : XQ();
    if (!q8k) a.qs = nullptr;
    if (!q80) b.qs = nullptr;
    rmsnorm_quant_kernel<<<rows, row_threads(n), (size_t)n * 4, s>>>(x, ldx, w, n, eps, xb, ldb, a, b);
    SDY_LAUNCHED();
}

void silu_quant(float *g, int64_t ldg, const float *u, int64_t ldu, int n, int rows, const XQ *q8k, const XQ *q80,
                cudaStream_t s) {
    if (rows <= 0) return;
    XQ a = q8k ? *q8k : XQ(), b = q80 ? *q80 : XQ();
    if (!q8k) a.qs = nullptr;
    if (!q80) b.qs = nullptr;
    silu_quant_kernel<<<rows, row_threads(n), (size_t)n * 4, s>>>(g, ldg, u, ldu, n, a, b);
    SDY_LAUNCHED();
}

void post_qkv(const PostQKV &p, int n_tok, cudaStream_t s) {
    if (n_tok <= 0) return;
    post_qkv_kernel<<<dim3(p.n_head + p.n_kv_head, n_tok), 64, (size_t)p.hd * 4, s>>>(p);
    SDY_LAUNCHED();
}

void router_topk(const float *x, int64_t ldx, const void *w, int wtype, int dim, int ne, int k, int n_tok,
                 int32_t *top, float *wout, float *probs_out, cudaStream_t s) {
    if (n_tok <= 0) return;
    router_topk_kernel<<<n_tok, 128, (size_t)ne * 4, s>>>(x, ldx, w, wtype, dim, ne, k, top, wout, probs_out);
    SDY_LAUNCHED();
}

void moe_combine(const float *y, int64_t ldy, const int32_t *top, const float *w, int k, int dim, int n_tok, float *x,
                 int64_t ldx, cudaStream_t s) {
    if (n_tok <= 0) return;
    moe_combine_kernel<<<dim3((dim + 255) / 256, n_tok), 256, 0, s>>>(y, ldy, top, w, k, dim, x, ldx);
    SDY_LAUNCHED();
}

}  // namespace sdy
