// Fused per-token kernels of the decode/prefill forward. Each replaces two to four of the
// reference's sequential steps with one launch while keeping its operation order, so results
// are the same floats as the unfused chain:
//   rmsnorm_quant  op_rmsnorm (ops.c:346-351) + op_quantize_rows (quant.c:98-144)
//   post_qkv       op_add_bias + qk RMSNorm + op_rope + KV-cache store (model_llama.c:781-800)
//   silu_quant     op_silu_mul (ops.c:366-371) + op_quantize_rows
//   router_topk    F32 router matvec + op_softmax + moe_select (model_llama.c:653-684)
//   moe_combine    sum over a token's experts in ascending id + residual add (model_llama.c:734-750, 820)
// In the norm and SiLU kernels lane l of warp w owns elements 256w + 8l .. +7 in registers, so
// each warp quantizes its own 256-element span without staging through shared memory.
#include "fp_device.cuh"

#include <algorithm>
#include "fused.cuh"
#include "quant_device.cuh"

namespace sdy {
namespace {


// Quantize the warp's span (values in registers) into the requested activation types.
__device__ __forceinline__ void quantize_span(const float v[8], int e0, int n, int t, int span, const XQ &q8k,
                                              const XQ &q80) {
    if (q8k.qs) quant_q8k_vals(v, t, span, q8k);  // only requested when n is a multiple of 256
    if (q80.qs) quant_q80_vals(v, e0 < n, t, span, q80);
}

// One block per row, thread i owning elements 8i..8i+7 (blockDim = n/8 rounded up to a warp).
__global__ void rmsnorm_quant_kernel(const float *x, int64_t ldx, const float *w, int n, float eps, float *xb,
                                     int64_t ldb, XQ q8k, XQ q80) {
    pdl_wait();
    pdl_release();
    __shared__ double part[32];
    const int t = blockIdx.x;
    norm_quant_row(x + (size_t)t * ldx, w, n, eps, t, q8k, q80, xb ? xb + (size_t)t * ldb : nullptr, part);
}

// grid (ceil(n/2048), rows), 256 threads: warp w of block b owns span 8b + w.
__global__ void silu_quant_kernel(float *g, int64_t ldg, const float *u, int64_t ldu, int n, XQ q8k, XQ q80) {
    pdl_wait();
    pdl_release();
    const int t = blockIdx.y, span = blockIdx.x * 8 + (threadIdx.x >> 5);
    if (span * 256 >= n) return;  // whole warps leave together
    const int e0 = span * 256 + (threadIdx.x & 31) * 8;
    float *gv = g + (size_t)t * ldg;
    const float *uv = u + (size_t)t * ldu;
    float v[8];
    for (int j = 0; j < 8; j++) {
        v[j] = 0.0f;
        if (e0 + j < n) {
            v[j] = silu_mul(gv[e0 + j], uv[e0 + j]);
            gv[e0 + j] = v[j];
        }
    }
    quantize_span(v, e0, n, t, span, q8k, q80);
}

// One block per (head, token). Heads [0, n_head) are q heads; [n_head, n_head + n_kv_head) are
// k heads, whose block also handles the v head with the same index.
__global__ void post_qkv_kernel(PostQKV p) {
    pdl_wait();
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

// Router logits for float weights: one warp per expert row. The warp copies x and its row into
// shared memory with coalesced loads; lanes 0..3 then run the reference's four accumulator
// chains (ops.c:155-167: s_k over i = 4g + k, the tail into s0) and combine (s0+s1)+(s2+s3).
constexpr int ROUTER_EPC = 8;  // experts per CTA: one warp each
constexpr int ROUTER_THREADS = 32 * ROUTER_EPC;


// Float router, one warp per (expert, token), ROUTER_EPC experts per CTA: logits[t][e] = x[t].w[e]
// with the reference's four-accumulator dot (ops.c:155-167) — the row (a constant weight, staged
// before pdl_wait) and x go through shared memory with 16-byte loads, then lanes 0-3 of the warp
// run one accumulator chain each. The last CTA of a token to finish (a counter per token, left at
// zero again) runs the softmax and top-k. vec: dim % 4 == 0 and 16-byte aligned x rows / weights.
__global__ void __launch_bounds__(ROUTER_THREADS)
    router_topk_kernel(const float *x, int64_t ldx, const void *w, int wtype, int dim, int ne, int k, float *logits,
                       int32_t *counters, int32_t *top, float *wout, int vec, const float *nw, float neps) {
    extern __shared__ __align__(16) float sm[];
    __shared__ double dpart[32];
    __shared__ float fpart[32];
    __shared__ float pv[64];
    __shared__ int last;
    const int dp = (dim + 3) & ~3;
    const int t = blockIdx.y, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int e = blockIdx.x * ROUTER_EPC + warp;
    float *xs = sm, *row = sm + (size_t)(1 + warp) * dp;
    // vec: x and the row are stored de-interleaved, element 4g + a at [a * G + g], so accumulator a's
    // chain reads 4 consecutive terms with one 16-byte load per operand.
    const int G = dim / 4;
    if (e < ne) {
        const size_t base = (size_t)e * dim;
        if (vec) {
            for (int g0 = lane; g0 < G; g0 += 32 * 16) {  // 16 loads in flight per lane before the stores
                float4 v[16];
#pragma unroll
                for (int u = 0; u < 16; u++)
                    if (g0 + 32 * u < G) v[u] = load4_w(w, wtype, base + 4 * (size_t)(g0 + 32 * u));
#pragma unroll
                for (int u = 0; u < 16; u++) {
                    const int g = g0 + 32 * u;
                    if (g < G) {
                        row[g] = v[u].x;
                        row[G + g] = v[u].y;
                        row[2 * G + g] = v[u].z;
                        row[3 * G + g] = v[u].w;
                    }
                }
            }
        } else {
            for (int i = lane; i < dim; i += 32) row[i] = load_w(w, wtype, base + i);
        }
    }
    pdl_wait();
    pdl_release();
    const float *xv = x + (size_t)t * ldx;
    // nw: the router input is RMSNorm(x) * nw, computed here in the shared fixed order (the value
    // the standalone norm kernel would have stored), instead of a normalised copy read from memory.
    float scale = 1.0f;
    if (nw) scale = (float)(1.0 / sqrt(span_sumsq(xv, dim, dpart) / dim + (double)neps));
    auto nrm = [&](float v, int i) { return nw ? __fmul_rn(__fmul_rn(v, scale), nw[i]) : v; };
    if (vec) {
        for (int g0 = tid; g0 < G; g0 += ROUTER_THREADS * 8) {
            float4 v[8];
#pragma unroll
            for (int u = 0; u < 8; u++)
                if (g0 + ROUTER_THREADS * u < G) v[u] = *(const float4 *)(xv + 4 * (g0 + ROUTER_THREADS * u));
#pragma unroll
            for (int u = 0; u < 8; u++) {
                const int g = g0 + ROUTER_THREADS * u;
                if (g < G) {
                    xs[g] = nrm(v[u].x, 4 * g);
                    xs[G + g] = nrm(v[u].y, 4 * g + 1);
                    xs[2 * G + g] = nrm(v[u].z, 4 * g + 2);
                    xs[3 * G + g] = nrm(v[u].w, 4 * g + 3);
                }
            }
        }
    } else {
        for (int i = tid; i < dim; i += ROUTER_THREADS) xs[i] = nrm(xv[i], i);
    }
    __syncthreads();
    if (e < ne) {
        float s = 0.0f;
        if (vec) {
            // The products x_i * w_i by the whole warp (each rounded once, as in the chain), in place
            // in the row; then lane a adds accumulator a's terms in order, one 16-byte load per 4
            // (G % 4 == 0), so the chains wait on the adds alone.
            for (int i = lane * 4; i < dim; i += 128) {
                const float4 a = *(const float4 *)(xs + i);
                float4 b = *(const float4 *)(row + i);
                b.x = __fmul_rn(a.x, b.x);
                b.y = __fmul_rn(a.y, b.y);
                b.z = __fmul_rn(a.z, b.z);
                b.w = __fmul_rn(a.w, b.w);
                *(float4 *)(row + i) = b;
            }
            __syncwarp();
            if (lane < 4) {
                const float4 *ra = (const float4 *)(row + lane * G);
#pragma unroll 8
                for (int q = 0; q < G / 4; q++) {
                    const float4 b = ra[q];
                    s = __fadd_rn(s, b.x);
                    s = __fadd_rn(s, b.y);
                    s = __fadd_rn(s, b.z);
                    s = __fadd_rn(s, b.w);
                }
            }
        } else if (lane < 4) {
            const int groups = dim / 4;
            const float *xa = xs + lane, *ra = row + lane;
            s = ordered_sum<16>(s, groups, [&](int g) { return __fmul_rn(xa[4 * g], ra[4 * g]); });
            if (lane == 0)
                for (int i = groups * 4; i < dim; i++) s = __fadd_rn(s, __fmul_rn(xs[i], row[i]));
        }
        const float s1 = __shfl_sync(0xffffffffu, s, 1), s2 = __shfl_sync(0xffffffffu, s, 2),
                    s3 = __shfl_sync(0xffffffffu, s, 3);
        if (lane == 0) logits[(size_t)t * ne + e] = __fadd_rn(__fadd_rn(s, s1), __fadd_rn(s2, s3));
    }
    __syncthreads();
    if (tid == 0) {
        __threadfence();
        last = atomicAdd(counters + t, 1) == (int)gridDim.x - 1;
    }
    __syncthreads();
    if (!last) return;
    __threadfence();
    if (tid == 0) counters[t] = 0;
    softmax_topk_block(logits + (size_t)t * ne, sm, pv, ne, k, top + (size_t)t * k, wout + (size_t)t * k, dpart,
                       fpart);
}

// One CTA-column of the MoE combine (moe_combine_token in fp_device.cuh) per (element block, token).
__global__ void moe_combine_kernel(const float *y, int64_t ldy, const int32_t *top, const float *w, int k, int dim,
                                   float *x, int64_t ldx) {
    pdl_wait();
    pdl_release();
    moe_combine_token(y, ldy, top, w, k, dim, x, ldx, blockIdx.y, blockIdx.x * blockDim.x, gridDim.x * blockDim.x);
}

// dst[t][i] = silu(g[t][i]) * u[t][i] (ops.c:366-371): the SiLU product of one rank's rows of a
// sharded FFN, written into its columns of the buffer the ranks all-reduce.
__global__ void silu_scatter_kernel(const float *g, int64_t ldg, const float *u, int64_t ldu, int n, float *dst,
                                    int64_t ldd) {
    pdl_wait();
    const int t = blockIdx.y;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
        dst[(size_t)t * ldd + i] = silu_mul(g[(size_t)t * ldg + i], u[(size_t)t * ldu + i]);
    }
}

// Counting sort of the slots by (local) expert: off[e] .. off[e+1] indexes slots[] for expert
// e0 + e; slots of other ranks' experts are left out. One CTA; order within an expert follows the
// atomics (each slot's product does not depend on its position).
// Also the work list of the grouped GEMM: tiles[i] = (e << 16) | token tile, i < off[ne + 1].
__global__ void moe_group_kernel(const int32_t *top, int n_slots, int e0, int ne, int tile, int32_t *off,
                                 int32_t *slots, int32_t *tiles) {
    pdl_wait();
    extern __shared__ int cnt[];  // ne counts, then cursors
    for (int i = threadIdx.x; i < ne; i += blockDim.x) cnt[i] = 0;
    __syncthreads();
    for (int i = threadIdx.x; i < n_slots; i += blockDim.x) {
        const int e = top[i] - e0;
        if (e >= 0 && e < ne) atomicAdd(&cnt[e], 1);
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        int run = 0;
        for (int e = 0; e < ne; e++) {
            const int c = cnt[e];
            cnt[e] = run;
            off[e] = run;
            run += c;
        }
        off[ne] = run;
        int nt = 0;
        for (int e = 0; e < ne; e++) {
            const int c = (e + 1 < ne ? cnt[e + 1] : run) - cnt[e];
            for (int tt = 0; tt * tile < c; tt++) tiles[nt++] = (e << 16) | tt;
        }
        off[ne + 1] = nt;
    }
    __syncthreads();
    for (int i = threadIdx.x; i < n_slots; i += blockDim.x) {
        const int e = top[i] - e0;
        if (e >= 0 && e < ne) slots[atomicAdd(&cnt[e], 1)] = i;
    }
}

// L2 prefetch of byte ranges (cp.async.bulk.prefetch.L2, PF_CHUNK bytes per request): a hint
// that pulls upcoming weights from HBM into L2 while other kernels run. One request per thread
// per pass, spread over many CTAs, since the requests of one SM issue one after another.
constexpr size_t PF_CHUNK = 16384;
__device__ __forceinline__ void prefetch_l2(const char *p, size_t n) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;\n" ::"l"(p), "r"((uint32_t)n) : "memory");
}
__device__ void prefetch_range(const char *p, size_t bytes, size_t thread, size_t n_threads) {
    bytes &= ~(size_t)15;
    for (size_t off = thread * PF_CHUNK; off < bytes; off += n_threads * PF_CHUNK)
        prefetch_l2(p + off, bytes - off < PF_CHUNK ? bytes - off : PF_CHUNK);
}
__global__ void l2_prefetch_kernel(L2Ranges r) {
    const size_t thread = (size_t)blockIdx.x * blockDim.x + threadIdx.x, n = (size_t)gridDim.x * blockDim.x;
    for (int k = 0; k < r.n; k++) prefetch_range((const char *)r.p[k], r.bytes[k], thread, n);
}
// The chosen experts' matrices: blockIdx.y = slot, blockIdx.z = matrix.
__global__ void expert_prefetch_kernel(ExpertPrefetch ep, const int32_t *top) {
    const int m = blockIdx.z, e = top[blockIdx.y] - ep.e0;
    if (!ep.base[m] || e < 0 || e >= ep.n_local) return;
    prefetch_range((const char *)ep.base[m] + (size_t)e * ep.bytes[m], ep.bytes[m],
                   (size_t)blockIdx.x * blockDim.x + threadIdx.x, (size_t)gridDim.x * blockDim.x);
}

XQ pick(const XQ *q) {
    XQ a = q ? *q : XQ();
    if (!q) a.qs = nullptr;
    return a;
}

// Router logits of many tokens (prefill): the same four-accumulator dots as router_topk_kernel,
// with the CTA's RM_EPC router rows held in shared memory while its warps stream the tokens past
// them. Lane l of a warp runs chain a = l % 4 of expert l / 4 for the warp's current token, so a
// warp computes 8 logits at once. Every row and the token's x are stored de-interleaved (element
// 4g + a at plane a, index g) with a plane stride of P = G + pad floats, P = 4 (mod 32), so the
// 16-byte loads of the 32 lanes (32 planes of the rows; 4 planes of x, broadcast) fall into
// distinct banks. Needs dim % 16 == 0 and 16-byte aligned x rows and weights.
constexpr int RM_EPC = 8;
constexpr int RM_WARPS = 8;
constexpr int RM_TPC = 32;  // tokens per CTA

__host__ __device__ inline int rm_plane(int dim) {
    const int G = dim / 4;
    return G + ((4 - G % 32) + 32) % 32;
}

__global__ void __launch_bounds__(RM_WARPS * 32) router_many_kernel(const float *x, int64_t ldx, const void *w,
                                                                    int wtype, int dim, int ne, int n_tok,
                                                                    float *logits) {
    extern __shared__ __align__(16) float sm[];
    const int G = dim / 4, P = rm_plane(dim);
    float *rows = sm;                           // [RM_EPC * 4][P]
    float *xs = sm + (size_t)RM_EPC * 4 * P;    // [RM_WARPS][4][P]
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int e_base = blockIdx.x * RM_EPC;
    for (int i = tid; i < RM_EPC * G; i += blockDim.x) {
        const int el = i / G, g = i - el * G, e = e_base + el;
        const float4 v = e < ne ? load4_w(w, wtype, (size_t)e * dim + 4 * (size_t)g) : make_float4(0.f, 0.f, 0.f, 0.f);
        float *r = rows + (size_t)(4 * el) * P + g;
        r[0] = v.x;
        r[P] = v.y;
        r[2 * P] = v.z;
        r[3 * P] = v.w;
    }
    pdl_wait();
    __syncthreads();
    const int a = lane & 3, el = lane >> 2, e = e_base + el;
    const float *wr = rows + (size_t)lane * P;  // plane 4 * el + a
    float *xw = xs + (size_t)warp * 4 * P;
    const int t_end = min(n_tok, (int)(blockIdx.y + 1) * RM_TPC);
    for (int t = blockIdx.y * RM_TPC + warp; t < t_end; t += RM_WARPS) {
        const float *xv = x + (size_t)t * ldx;
        for (int g = lane; g < G; g += 32) {
            const float4 v = *(const float4 *)(xv + 4 * g);
            xw[g] = v.x;
            xw[P + g] = v.y;
            xw[2 * P + g] = v.z;
            xw[3 * P + g] = v.w;
        }
        __syncwarp();
        const float *xa = xw + (size_t)a * P;
        float s = 0.0f;
#pragma unroll 4
        for (int g = 0; g < G; g += 4) {  // chain a over i = 4g + a, in order (ops.c:155-167)
            const float4 xv4 = *(const float4 *)(xa + g), wv4 = *(const float4 *)(wr + g);
            s = __fadd_rn(s, __fmul_rn(xv4.x, wv4.x));
            s = __fadd_rn(s, __fmul_rn(xv4.y, wv4.y));
            s = __fadd_rn(s, __fmul_rn(xv4.z, wv4.z));
            s = __fadd_rn(s, __fmul_rn(xv4.w, wv4.w));
        }
        const float s1 = __shfl_down_sync(0xffffffffu, s, 1), s2 = __shfl_down_sync(0xffffffffu, s, 2),
                    s3 = __shfl_down_sync(0xffffffffu, s, 3);
        if (a == 0 && e < ne) logits[(size_t)t * ne + e] = __fadd_rn(__fadd_rn(s, s1), __fadd_rn(s2, s3));
        __syncwarp();  // x of the next token overwrites this one
    }
}

// Softmax and top-k of each token's logits (one CTA per token), as the router kernel's last CTA
// runs them.
__global__ void router_select_kernel(const float *logits, int ne, int k, int32_t *top, float *wout) {
    extern __shared__ __align__(16) float prob[];
    __shared__ double dpart[32];
    __shared__ float fpart[32];
    __shared__ float pv[64];
    pdl_wait();
    const int t = blockIdx.x;
    softmax_topk_block(logits + (size_t)t * ne, prob, pv, ne, k, top + (size_t)t * k, wout + (size_t)t * k, dpart,
                       fpart);
}

}  // namespace

void rmsnorm_quant(const float *x, int64_t ldx, const float *w, int n, int rows, float eps, float *xb, int64_t ldb,
                   const XQ *q8k, const XQ *q80, cudaStream_t s) {
    if (rows <= 0) return;
    if (n > 8192) {
        set_error("rmsnorm_quant: rows of %d elements exceed 8192", n);
        return;
    }
    const int threads = ((n + 7) / 8 + 31) / 32 * 32;
    launch(rmsnorm_quant_kernel, rows, threads, 0, s, x, ldx, w, n, eps, xb, ldb, pick(q8k), pick(q80));
    SDY_LAUNCHED();
}

void silu_quant(float *g, int64_t ldg, const float *u, int64_t ldu, int n, int rows, const XQ *q8k, const XQ *q80,
                cudaStream_t s) {
    if (rows <= 0) return;
    launch(silu_quant_kernel, dim3((n + 2047) / 2048, rows), 256, 0, s, g, ldg, u, ldu, n, pick(q8k), pick(q80));
    SDY_LAUNCHED();
}

void post_qkv(const PostQKV &p, int n_tok, cudaStream_t s) {
    if (n_tok <= 0) return;
    launch(post_qkv_kernel, dim3(p.n_head + p.n_kv_head, n_tok), 64, (size_t)p.hd * 4, s, p);
    SDY_LAUNCHED();
}

namespace {
constexpr int ROUTER_MANY_MIN_TOKENS = 8;
size_t router_smem(int dim, int ne) {
    const size_t dp = (size_t)((dim + 3) & ~3);
    return std::max((size_t)(1 + ROUTER_EPC) * dp, (size_t)2 * ne) * 4;
}
}  // namespace

size_t router_many_smem(int dim) { return (size_t)(RM_EPC + RM_WARPS) * 4 * rm_plane(dim) * 4; }

bool router_topk_supported(int dim, int ne, int k, int n_tok, bool norm) {
    return router_smem(dim, ne) <= 200 * 1024 && n_tok <= 65535 && k <= ne && k <= 64 && (!norm || dim <= 8192);
}

void router_topk(const float *x, int64_t ldx, const void *w, int wtype, int dim, int ne, int k, int n_tok,
                 int32_t *top, float *wout, float *logits, int32_t *counters, cudaStream_t s, const float *norm_w,
                 float norm_eps) {
    if (n_tok <= 0) return;
    const size_t smem = router_smem(dim, ne);
    if (!router_topk_supported(dim, ne, k, n_tok, norm_w != nullptr)) {
        set_error("router_topk: hidden size %d / %d tokens / top-%d of %d not supported", dim, n_tok, k, ne);
        return;
    }
    const bool w_aligned = wtype == T_F32 ? ((uintptr_t)w & 15) == 0 : ((uintptr_t)w & 7) == 0;
    const int vec = dim % 16 == 0 && ldx % 4 == 0 && ((uintptr_t)x & 15) == 0 && w_aligned;
    if (n_tok >= ROUTER_MANY_MIN_TOKENS && vec && !norm_w && router_many_smem(dim) <= 200 * 1024 && k <= 64) {
        // many tokens: logits with the router rows resident per CTA, then one CTA per token selects
        static std::atomic<uint64_t> configured_many{0};
        smem_limit_once(router_many_kernel, 200 * 1024, configured_many);
        launch(router_many_kernel, dim3((ne + RM_EPC - 1) / RM_EPC, (n_tok + RM_TPC - 1) / RM_TPC), RM_WARPS * 32,
               router_many_smem(dim), s, x, ldx, w, wtype, dim, ne, n_tok, logits);
        SDY_LAUNCHED();
        launch(router_select_kernel, dim3(n_tok), 256, (size_t)ne * 4, s, logits, ne, k, top, wout);
        SDY_LAUNCHED();
        return;
    }
    static std::atomic<uint64_t> configured{0};
    smem_limit_once(router_topk_kernel, 200 * 1024, configured);
    launch(router_topk_kernel, dim3((ne + ROUTER_EPC - 1) / ROUTER_EPC, n_tok), ROUTER_THREADS, smem, s, x, ldx, w,
           wtype, dim, ne, k, logits, counters, top, wout, vec, norm_w, norm_eps);
    SDY_LAUNCHED();
}

void moe_combine(const float *y, int64_t ldy, const int32_t *top, const float *w, int k, int dim, int n_tok, float *x,
                 int64_t ldx, cudaStream_t s) {
    if (n_tok <= 0) return;
    launch(moe_combine_kernel, dim3((dim + 255) / 256, n_tok), 256, 0, s, y, ldy, top, w, k, dim, x, ldx);
    SDY_LAUNCHED();
}

void silu_scatter(const float *g, int64_t ldg, const float *u, int64_t ldu, int n, int rows, float *dst, int64_t ldd,
                  cudaStream_t s) {
    if (rows <= 0 || n <= 0) return;
    launch(silu_scatter_kernel, dim3((n + 255) / 256, rows), 256, 0, s, g, ldg, u, ldu, n, dst, ldd);
    SDY_LAUNCHED();
}

void moe_group(const int32_t *top, int n_slots, int e0, int ne, int tile, int32_t *off, int32_t *slots,
               int32_t *tiles, cudaStream_t s) {
    if (ne <= 0) return;
    if (ne >= (1 << 15) || n_slots / tile >= (1 << 16)) {
        set_error("moe_group: %d experts / %d slots not supported", ne, n_slots);
        return;
    }
    launch(moe_group_kernel, 1, 1024, (size_t)ne * 4, s, top, n_slots, e0, ne, tile, off, slots, tiles);
    SDY_LAUNCHED();
}

void l2_prefetch(const L2Ranges &r, cudaStream_t s) {
    size_t chunks = 0;
    for (int k = 0; k < r.n; k++) chunks += (r.bytes[k] + PF_CHUNK - 1) / PF_CHUNK;
    if (!chunks) return;
    l2_prefetch_kernel<<<(unsigned)std::min<size_t>((chunks + 31) / 32, 296), 32, 0, s>>>(r);
    SDY_LAUNCHED();
}

void expert_prefetch(const ExpertPrefetch &ep, const int32_t *top, int n_slots, cudaStream_t s) {
    size_t most = 0;
    for (int m = 0; m < PF_EXPERT_MATS; m++) most = std::max(most, ep.base[m] ? ep.bytes[m] : 0);
    if (!most || n_slots <= 0) return;
    const unsigned per = (unsigned)std::min<size_t>(((most + PF_CHUNK - 1) / PF_CHUNK + 31) / 32, 16);
    expert_prefetch_kernel<<<dim3(per, n_slots, PF_EXPERT_MATS), 32, 0, s>>>(ep, top);
    SDY_LAUNCHED();
}

}  // namespace sdy
