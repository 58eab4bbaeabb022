// Causal attention over the KV cache (reference csrc/ops.c:405-423, called per token from
// model_llama.c:803-806): for each query head, scores = q.k_j * (1/sqrt(hd)) over the n_kv
// cached positions, softmax, then out[i] = sum over j IN KEY ORDER of p_j * v_j[i].
//
// The reference's result is a sequential rounding chain per output element (axpy into out, one
// key at a time, no fused multiply-add), so the only parallelism that keeps it exact is across
// heads and elements, never across keys of one element. The main kernel is built around that:
//
//   one cluster of AC = 8 CTAs per (KV head, token), serving the n_rep query heads that share
//   the KV head (GQA), so each K/V row is read from HBM once for all of them;
//   phase A  CTA c scores keys [c*L, (c+1)*L): K tiles staged with cp.async, one key per thread,
//            dot products in the reference's four-accumulator order (ops.c:155-167), scores kept
//            in the CTA's shared memory;
//   phase B  max and double sum of exp(s - max) per head reduced across the cluster through
//            distributed shared memory (two cluster barriers);
//   phase C  CTA c owns elements [c*S, (c+1)*S) of every head: n_rep*S exact chains, fed by the
//            probabilities (each CTA pushes its keys' exponentials into every CTA's shared memory
//            during phase B when all keys fit; otherwise chunks are read from their owners) and
//            double-buffered cp.async chunks of the V columns it needs (the first chunk requested
//            in phase A).
//
// A per-head kernel (one CTA per (head, token)) covers the shapes the cluster kernel does not
// (head_dim not a multiple of 32, more than 32 query heads per KV head, unaligned buffers, a
// context too long for the scores to stay in shared memory).
#include "fp_device.cuh"
#include "fp_ops.cuh"
#include "fused.cuh"

#include <cooperative_groups.h>

namespace sdy {
namespace cg = cooperative_groups;
namespace {

__device__ __forceinline__ void cp_async16(void *dst, const void *src) {
    unsigned d = (unsigned)__cvta_generic_to_shared(dst);
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(d), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory");
}
__device__ __forceinline__ void cluster_arrive() { asm volatile("barrier.cluster.arrive.release.aligned;\n" ::: "memory"); }
__device__ __forceinline__ void cluster_wait() { asm volatile("barrier.cluster.wait.acquire.aligned;\n" ::: "memory"); }

constexpr int AC = 8;             // CTAs per cluster
constexpr int AC_THREADS = 256;
constexpr int AC_KT = 64;         // keys per K tile (phase A)
constexpr int AC_HG = AC_THREADS / AC_KT;  // head groups in phase A
constexpr int AC_KC = 256;        // keys per chunk (phase C)
constexpr int AC_PLD = AC_KC + 4; // probability row stride in shared memory (rows on distinct banks)
constexpr int AC_MAX_REP = 32;    // query heads per KV head
constexpr int AC_MAX_GROUP = AC * AC_THREADS;  // n_rep * hd: one chain per thread in phase C
constexpr int AC_SMEM_LIMIT = 200 * 1024;

// Scores row length per head: this CTA's share of the keys, at most ceil(stride / AC).
__host__ __device__ inline int ac_lmax(int stride) { return ((stride + AC - 1) / AC + 3) & ~3; }
struct AcSmem {
    int qs, kv, scl, vb, work, total;  // float offsets
};
// Probability row stride when every CTA holds all keys' exponentials (push mode).
__host__ __device__ inline int ac_ldp(int stride) { return ((stride + 3) & ~3) + 4; }
// push: the work area also holds n_rep rows of ac_ldp(stride) exponentials (all keys) for phase C.
__host__ __device__ inline AcSmem ac_smem(int n_rep, int hd, int stride, bool push) {
    AcSmem m;
    const int S = hd / AC;
    m.qs = 0;
    m.kv = n_rep * hd;            // the new token's K and V rows (fused post-QKV)
    m.scl = m.kv + 2 * hd;
    m.vb = m.scl + n_rep * ac_lmax(stride);
    m.work = m.vb + 2 * AC_KC * S;
    const int a = 2 * AC_KT * (hd + 4), c = push ? n_rep * ac_ldp(stride) : 2 * n_rep * AC_PLD;
    m.total = m.work + (a > c ? a : c);
    return m;
}

// One head of the reference's post-projection steps (model_llama.c:781-800) by one warp: bias,
// per-head RMSNorm (qk-norm: double sum of squares, lane-strided then a shuffle tree), RoPE
// (ops.c:388-403) at table row `pos`; result in dst (shared, hd floats; hd % 32 == 0, hd <= 256).
// Split in three so that a kernel can load the operands that do not depend on the projection
// (head_consts, rope_consts) before pdl_wait, and the rows of all of a warp's heads at once.
struct HeadConsts {
    float b[8], n[8];  // bias and norm weight, element lane + 32u
};
struct RopeConsts {
    float c[4], s[4];  // cos / sin of pair lane + 32u
};
__device__ __forceinline__ void head_consts(const float *bias, const float *norm, int hd, HeadConsts &h) {
    const int lane = threadIdx.x & 31, nu = hd / 32;
#pragma unroll
    for (int u = 0; u < 8; u++)
        if (u < nu) {
            h.b[u] = bias ? bias[lane + 32 * u] : 0.0f;
            h.n[u] = norm ? norm[lane + 32 * u] : 0.0f;
        }
}
__device__ __forceinline__ void rope_consts(const float *cs, const float *sn, int hd, RopeConsts &r) {
    const int lane = threadIdx.x & 31, half = hd / 2;
#pragma unroll
    for (int u = 0; u < 4; u++)
        if (lane + 32 * u < half) {
            r.c[u] = cs[lane + 32 * u];
            r.s[u] = sn[lane + 32 * u];
        }
}
__device__ __forceinline__ void head_load(const float *src, int hd, float v[8]) {
    const int lane = threadIdx.x & 31, nu = hd / 32;
#pragma unroll
    for (int u = 0; u < 8; u++)
        if (u < nu) v[u] = src[lane + 32 * u];
}
__device__ __forceinline__ void head_finish(float v[8], const HeadConsts &h, bool bias, bool norm, float eps,
                                            bool rope, const RopeConsts &rc, int interleaved, int hd, float *dst) {
    const int lane = threadIdx.x & 31, nu = hd / 32, half = hd / 2;
    double ss = 0.0;
#pragma unroll
    for (int u = 0; u < 8; u++)
        if (u < nu) {
            if (bias) v[u] = __fadd_rn(v[u], h.b[u]);
            ss += (double)v[u] * v[u];
        }
    if (norm) {
        for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        const float scale = (float)(1.0 / sqrt(ss / hd + (double)eps));
#pragma unroll
        for (int u = 0; u < 8; u++)
            if (u < nu) v[u] = __fmul_rn(__fmul_rn(v[u], scale), h.n[u]);
    }
#pragma unroll
    for (int u = 0; u < 8; u++)
        if (u < nu) dst[lane + 32 * u] = v[u];
    __syncwarp();
    if (rope)
#pragma unroll
        for (int u = 0; u < 4; u++) {
            const int i = lane + 32 * u;
            if (i < half) {
                const int ia = interleaved ? 2 * i : i, ib = interleaved ? 2 * i + 1 : i + half;
                const float a = dst[ia], b = dst[ib];
                dst[ia] = __fsub_rn(__fmul_rn(a, rc.c[u]), __fmul_rn(b, rc.s[u]));
                dst[ib] = __fadd_rn(__fmul_rn(a, rc.s[u]), __fmul_rn(b, rc.c[u]));
            }
        }
    __syncwarp();
}

// Head r of a KV group's post step: r < n_rep the query heads h0 + r, then the K head, then V.
struct HeadOp {
    const float *src, *bias, *norm;
    bool rope;
    float *dst;
};
__device__ __forceinline__ HeadOp head_op(const PostQKV &pp, int r, int n_rep, int h0, int g, int t, int hd,
                                          float *qs, float *knew, float *vnew) {
    if (r < n_rep) {
        const int h = h0 + r;
        return {pp.q + (size_t)t * pp.ldq + (size_t)h * hd, pp.bq ? pp.bq + (size_t)h * hd : nullptr, pp.q_norm,
                true, qs + r * hd};
    }
    if (r == n_rep)
        return {pp.k + (size_t)t * pp.ldk + (size_t)g * hd, pp.bk ? pp.bk + (size_t)g * hd : nullptr, pp.k_norm,
                true, knew};
    return {pp.v + (size_t)t * pp.ldv + (size_t)g * hd, pp.bv ? pp.bv + (size_t)g * hd : nullptr, nullptr, false,
            vnew};
}

// q: token t at q + t*ldq, heads of hd; k/v cache [n_kv_head][stride][hd]; the first token's
// position is *pos_dev when given, else pos0; fixed_nkv > 0 overrides the causal count.
// hd % (4*AC) == 0, stride % 4 == 0, n_rep <= 32, n_rep*hd <= AC*AC_THREADS.
//
// Shared memory: q of the n_rep heads; this CTA's scores (then exponentials) per head, which the
// other CTAs of the cluster read in phase C through distributed shared memory; two V chunks of
// this CTA's column slice (the first one requested together with the first K tile); and a work
// area holding the K tiles in phase A and the probability chunks in phase C.
__global__ void __cluster_dims__(AC, 1, 1) __launch_bounds__(AC_THREADS, 1)
    attention_cluster_kernel(float *__restrict__ out, const float *__restrict__ q, int64_t ldq,
                             const float *__restrict__ kc, const float *__restrict__ vc, int n_head, int n_kv_head,
                             int hd, int pos0, const int32_t *pos_dev, int stride, int fixed_nkv, int push,
                             PostQKV pp) {
    extern __shared__ __align__(16) float sm[];
    __shared__ float cmax[AC_MAX_REP], gmax[AC_MAX_REP], ginv[AC_MAX_REP];
    __shared__ double csum[AC][AC_MAX_REP];  // [rank][head]: every CTA's partial sums, pushed to all
    cg::cluster_group cl = cg::this_cluster();
    const int c = (int)cl.block_rank();
    const int g = blockIdx.y, t = blockIdx.z, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int n_kv = fixed_nkv > 0 ? fixed_nkv : (pos_dev ? *pos_dev : pos0) + t + 1;
    const int n_rep = n_head / n_kv_head, h0 = g * n_rep;
    const float *kh = kc + (size_t)g * stride * hd, *vh = vc + (size_t)g * stride * hd;
    const AcSmem lay = ac_smem(n_rep, hd, stride, push);
    const int ldp = ac_ldp(stride);
    const int lmax = ac_lmax(stride);
    float *qs = sm + lay.qs, *scl = sm + lay.scl, *vb = sm + lay.vb, *work = sm + lay.work;
    float *knew = sm + lay.kv, *vnew = knew + hd;
    const bool post = pp.kc != nullptr;  // fused post-QKV (single token): the new row is key n_kv - 1
    const float scale = __fdiv_rn(1.0f, sqrtf((float)hd));
    const int L = (n_kv + AC - 1) / AC;
    const int jb = min(n_kv, c * L), je = min(n_kv, jb + L);
    const int S = hd / AC, S4 = S / 4, e0 = c * S;
    // The positions are host-written before the step's first kernel, so n_kv is known here. While
    // the previous kernel (which stores the newest K/V rows) finishes, pull this CTA's K rows and
    // the same V rows into L2: a cache hint only, the reads below still follow pdl_wait.
    if (tid == 0 && je > jb) {
        const uint32_t bytes = (uint32_t)((size_t)(je - jb) * hd * 4);
        asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;\n" ::"l"(kh + (size_t)jb * hd), "r"(bytes) : "memory");
        asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;\n" ::"l"(vh + (size_t)jb * hd), "r"(bytes) : "memory");
    }
    // Fused post-QKV: warp w handles heads w and w + 8 of the group (n_rep + 2 <= 16). Their
    // biases, norm weights and the RoPE row do not depend on the projection: loaded here.
    constexpr int NWARP = AC_THREADS / 32;
    const int n_post = n_rep + 2;
    const bool post_regs = post && n_post <= 2 * NWARP;
    HeadConsts hc[2];
    RopeConsts rc;
    if (post_regs) {
        const int pos = n_kv - 1, half = hd / 2;
        rope_consts(pp.cos + (size_t)pos * half, pp.sin + (size_t)pos * half, hd, rc);
#pragma unroll
        for (int i = 0; i < 2; i++)
            if (warp + NWARP * i < n_post) {
                const HeadOp op = head_op(pp, warp + NWARP * i, n_rep, h0, g, t, hd, qs, knew, vnew);
                head_consts(op.bias, op.norm, hd, hc[i]);
            }
    }
    pdl_wait();
    pdl_release();

    // ---- phase A: scores of this CTA's keys into scl
    const int ldk = hd + 4, hd4 = hd / 4;  // padded rows: a quarter-warp's 16-byte reads hit all banks once
    const int kk = tid % AC_KT, hg = tid / AC_KT;
    const int ntile = (je - jb + AC_KT - 1) / AC_KT;
    auto load_k = [&](int it) {
        const int j0 = jb + it * AC_KT, nk = min(AC_KT, je - j0);
        float *dst = work + (it & 1) * AC_KT * ldk;
        for (int idx = tid; idx < nk * hd4; idx += AC_THREADS) {
            const int j = idx / hd4, i = (idx - j * hd4) * 4;
            cp_async16(dst + j * ldk + i, kh + (size_t)(j0 + j) * hd + i);
        }
    };
    auto load_v = [&](int ic) {  // V columns [e0, e0+S) of chunk ic's keys into vb[ic & 1]
        const int j0 = ic * AC_KC, nk = min(AC_KC, n_kv - j0);
        float *dst = vb + (ic & 1) * AC_KC * S;
        for (int idx = tid; idx < nk * S4; idx += AC_THREADS) {
            const int j = idx / S4, i = (idx - j * S4) * 4;
            cp_async16(dst + j * S + i, vh + (size_t)(j0 + j) * hd + e0 + i);
        }
    };
    // The projection rows of the warp's post heads are requested first (before the K/V tiles
    // below, which would otherwise sit ahead of them in the memory pipeline).
    float v[2][8];
    if (post_regs)
#pragma unroll
        for (int i = 0; i < 2; i++)
            if (warp + NWARP * i < n_post)
                head_load(head_op(pp, warp + NWARP * i, n_rep, h0, g, t, hd, qs, knew, vnew).src, hd, v[i]);
    if (ntile > 0) load_k(0);
    load_v(0);  // phase C's first chunk travels with the first K tile
    cp_async_commit();
    if (post) {
        // Each CTA transforms its query heads and the new K and V rows itself; rank 0 stores the
        // rows in the cache for later steps, and every CTA patches them into its staged tiles
        // below (its own copies of the cache rows may predate rank 0's store).
        if (post_regs) {
#pragma unroll
            for (int i = 0; i < 2; i++)
                if (warp + NWARP * i < n_post) {
                    const HeadOp op = head_op(pp, warp + NWARP * i, n_rep, h0, g, t, hd, qs, knew, vnew);
                    head_finish(v[i], hc[i], op.bias != nullptr, op.norm != nullptr, pp.eps, op.rope, rc,
                                pp.interleaved, hd, op.dst);
                }
        } else {
            const int pos = n_kv - 1, half = hd / 2;
            RopeConsts r1;
            rope_consts(pp.cos + (size_t)pos * half, pp.sin + (size_t)pos * half, hd, r1);
            for (int r = warp; r < n_post; r += NWARP) {
                const HeadOp op = head_op(pp, r, n_rep, h0, g, t, hd, qs, knew, vnew);
                HeadConsts h1;
                float v[8];
                head_consts(op.bias, op.norm, hd, h1);
                head_load(op.src, hd, v);
                head_finish(v, h1, op.bias != nullptr, op.norm != nullptr, pp.eps, op.rope, r1, pp.interleaved, hd,
                            op.dst);
            }
        }
        __syncthreads();
        const int pos = n_kv - 1;
        if (c == 0)
            for (int i = tid; i < hd; i += AC_THREADS) {
                pp.kc[((size_t)g * pp.max_seq + pos) * hd + i] = knew[i];
                pp.vc[((size_t)g * pp.max_seq + pos) * hd + i] = vnew[i];
            }
    } else {  // the n_rep query heads: n_rep*hd/4 16-byte loads, all issued before any store
        const float4 *q4 = (const float4 *)(q + (size_t)t * ldq + (size_t)h0 * hd);
        const int n4 = n_rep * hd / 4;
        for (int i0 = 0; i0 < n4; i0 += 4 * AC_THREADS) {
            float4 v[4];
#pragma unroll
            for (int u = 0; u < 4; u++) {
                const int i = i0 + u * AC_THREADS + tid;
                if (i < n4) v[u] = q4[i];
            }
#pragma unroll
            for (int u = 0; u < 4; u++) {
                const int i = i0 + u * AC_THREADS + tid;
                if (i < n4) ((float4 *)qs)[i] = v[u];
            }
        }
    }
    for (int it = 0; it < ntile; it++) {
        if (it + 1 < ntile) {
            load_k(it + 1);
            cp_async_commit();
            cp_async_wait<1>();
        } else {
            cp_async_wait<0>();
        }
        __syncthreads();
        if (post) {  // the tile holding the new key: its row from knew
            const int j0 = jb + it * AC_KT, jn = n_kv - 1 - j0;
            if (jn >= 0 && jn < AC_KT && j0 + jn < je) {
                for (int i = tid; i < hd; i += AC_THREADS) work[(it & 1) * AC_KT * ldk + jn * ldk + i] = knew[i];
                __syncthreads();
            }
        }
        const int jl = it * AC_KT + kk;  // index within this CTA's keys
        if (jb + jl < je) {
            const float *row = work + (it & 1) * AC_KT * ldk + kk * ldk;
            for (int r0 = hg; r0 < n_rep; r0 += 2 * AC_HG) {
                const int r1 = r0 + AC_HG;
                const bool two = r1 < n_rep;
                const float *x0 = qs + r0 * hd, *x1 = qs + (two ? r1 : r0) * hd;
                float a0 = 0.0f, a1 = 0.0f, a2 = 0.0f, a3 = 0.0f, b0 = 0.0f, b1 = 0.0f, b2 = 0.0f, b3 = 0.0f;
                for (int i0 = 0; i0 < hd; i0 += 16) {  // loads of 16 elements issued ahead of their adds
                    float4 k4[4], u[4], w[4];
#pragma unroll
                    for (int v = 0; v < 4; v++) {
                        k4[v] = *(const float4 *)(row + i0 + 4 * v);
                        u[v] = *(const float4 *)(x0 + i0 + 4 * v);
                        w[v] = *(const float4 *)(x1 + i0 + 4 * v);
                    }
#pragma unroll
                    for (int v = 0; v < 4; v++) {
                        a0 = __fadd_rn(a0, __fmul_rn(u[v].x, k4[v].x));
                        a1 = __fadd_rn(a1, __fmul_rn(u[v].y, k4[v].y));
                        a2 = __fadd_rn(a2, __fmul_rn(u[v].z, k4[v].z));
                        a3 = __fadd_rn(a3, __fmul_rn(u[v].w, k4[v].w));
                        b0 = __fadd_rn(b0, __fmul_rn(w[v].x, k4[v].x));
                        b1 = __fadd_rn(b1, __fmul_rn(w[v].y, k4[v].y));
                        b2 = __fadd_rn(b2, __fmul_rn(w[v].z, k4[v].z));
                        b3 = __fadd_rn(b3, __fmul_rn(w[v].w, k4[v].w));
                    }
                }
                scl[r0 * lmax + jl] = __fmul_rn(__fadd_rn(__fadd_rn(a0, a1), __fadd_rn(a2, a3)), scale);
                if (two) scl[r1 * lmax + jl] = __fmul_rn(__fadd_rn(__fadd_rn(b0, b1), __fadd_rn(b2, b3)), scale);
            }
        }
        __syncthreads();
    }
    if (ntile == 0) {
        cp_async_wait<0>();
        __syncthreads();
    }

    // ---- phase B: cluster-wide max and sum of exponentials per head
    const int nl = je - jb;
    for (int r = warp; r < n_rep; r += AC_THREADS / 32) {
        float m = -INFINITY;
        for (int j = lane; j < nl; j += 32) m = fmaxf(m, scl[r * lmax + j]);
        for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        if (lane == 0) cmax[r] = m;
    }
    cl.sync();
    if (tid < n_rep) {
        float m = -INFINITY;
        for (int p = 0; p < AC; p++) m = fmaxf(m, *cl.map_shared_rank(cmax + tid, p));
        gmax[tid] = m;
    }
    __syncthreads();
    // After the first cluster barrier every CTA is past phase A, so the work areas (K tiles until
    // then) can receive the exponentials: in push mode each CTA stores its keys' values into the
    // probability rows of all 8 CTAs (remote stores, made visible by the next cluster barrier).
    for (int r = warp; r < n_rep; r += AC_THREADS / 32) {
        const float m = gmax[r];
        double sacc = 0.0;
        for (int j = lane; j < nl; j += 32) {
            const float e = expf_ref(__fsub_rn(scl[r * lmax + j], m));
            scl[r * lmax + j] = e;
            sacc += e;
            if (push)
#pragma unroll
                for (int p = 0; p < AC; p++) *cl.map_shared_rank(work + r * ldp + jb + j, p) = e;
        }
        for (int o = 16; o; o >>= 1) sacc += __shfl_xor_sync(0xffffffffu, sacc, o);
        if (lane < AC) *cl.map_shared_rank(&csum[c][r], lane) = sacc;
    }
    cl.sync();  // publishes every CTA's partial sums and (push mode) exponentials
    // From here on a CTA reads another's shared memory only in pull mode (load_p), which then
    // ends with a cluster barrier before any CTA exits.
    if (tid < n_rep) {
        double sacc = 0.0;
        for (int p = 0; p < AC; p++) sacc += csum[p][tid];
        ginv[tid] = (float)(1.0 / sacc);
    }
    __syncthreads();

    // ---- phase C: out[e] = sum_j (e_j * inv) * v_j[e] in key order, e in this CTA's slice
    const int ch_r = tid / S, ch_e = tid - ch_r * S;
    const bool chain = tid < n_rep * S;
    const int nchunk = (n_kv + AC_KC - 1) / AC_KC;
    // Probabilities p_j = e_j * inv (ops.c:363) of chunk ic's keys: the exponentials read from their
    // owners' shared memory, 8 remote loads in flight per thread before the stores.
    auto load_p = [&](int ic) {
        const int j0 = ic * AC_KC, nk = min(AC_KC, n_kv - j0), tot = n_rep * nk;
        float *pb = work + (ic & 1) * n_rep * AC_PLD;
        for (int i0 = 0; i0 < tot; i0 += 8 * AC_THREADS) {
            float v[8];
#pragma unroll
            for (int u = 0; u < 8; u++) {
                const int idx = i0 + u * AC_THREADS + tid;
                if (idx < tot) {
                    const int r = idx / nk, j = j0 + idx - r * nk, owner = j / L;
                    v[u] = *cl.map_shared_rank(scl + r * lmax + (j - owner * L), owner);
                }
            }
#pragma unroll
            for (int u = 0; u < 8; u++) {
                const int idx = i0 + u * AC_THREADS + tid;
                if (idx < tot) {
                    const int r = idx / nk, jj = idx - r * nk;
                    pb[r * AC_PLD + jj] = v[u];
                }
            }
        }
    };
    float acc = 0.0f;
    if (!push) load_p(0);
    const float inv = chain ? ginv[ch_r] : 0.0f;
    for (int ic = 0; ic < nchunk; ic++) {
        if (ic + 1 < nchunk) {
            load_v(ic + 1);
            cp_async_commit();
        }
        __syncthreads();
        if (post && ic == nchunk - 1) {  // the chunk holding the new key: its V columns from vnew
            const int jn = n_kv - 1 - ic * AC_KC;
            for (int i = tid; i < S; i += AC_THREADS) vb[(ic & 1) * AC_KC * S + jn * S + i] = vnew[e0 + i];
            __syncthreads();
        }
        if (chain) {
            const float *pr = push ? work + ch_r * ldp + ic * AC_KC
                                   : work + (ic & 1) * n_rep * AC_PLD + ch_r * AC_PLD;
            const float *vr = vb + (ic & 1) * AC_KC * S + ch_e;
            const int nk = min(AC_KC, n_kv - ic * AC_KC);
            // p_j = e_j * inv (ops.c:363), then acc += p_j * v_j[e]: the FADD chain is the
            // critical path, so the next 8 keys' operands are loaded while the current 8 are added.
            const float4 *e4 = (const float4 *)pr;  // 4 keys' exponentials per 16-byte load
            const int n8 = nk >> 3;
            float4 ea0, ea1, eb0, eb1;
            float va[8], vbb[8];
            auto fetch = [&](int q, float4 &x0, float4 &x1, float *vv) {
                x0 = e4[2 * q];
                x1 = e4[2 * q + 1];
#pragma unroll
                for (int k = 0; k < 8; k++) vv[k] = vr[(8 * q + k) * S];
            };
            auto add8 = [&](const float4 &x0, const float4 &x1, const float *vv) {
                const float ev[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
#pragma unroll
                for (int k = 0; k < 8; k++) acc = __fadd_rn(acc, __fmul_rn(__fmul_rn(ev[k], inv), vv[k]));
            };
            if (n8 > 0) fetch(0, ea0, ea1, va);
            int q = 0;
            for (; q + 2 <= n8; q += 2) {
                fetch(q + 1, eb0, eb1, vbb);
                add8(ea0, ea1, va);
                if (q + 2 < n8) fetch(q + 2, ea0, ea1, va);
                add8(eb0, eb1, vbb);
            }
            if (q < n8) add8(ea0, ea1, va);
            for (int j = n8 * 8; j < nk; j++) acc = __fadd_rn(acc, __fmul_rn(__fmul_rn(pr[j], inv), vr[j * S]));
        }
        if (!push && ic + 1 < nchunk) load_p(ic + 1);
        cp_async_wait<0>();
        __syncthreads();
    }
    if (!push) cluster_arrive();  // done reading the other CTAs' shared memory; the wait is below
    if (chain) out[((size_t)t * n_head + h0 + ch_r) * hd + e0 + ch_e] = acc;
    if (!push) cluster_wait();
}

// General per-(head, token) kernel, one CTA of ATT_THREADS each: K and V staged through shared
// memory in coalesced tiles (K rows padded to hd+1 floats), scores in the scratch rows, block
// softmax, then thread i adds p_j * v_j[i] for the keys in order. hd a multiple of 4, at most
// 2*ATT_THREADS.
constexpr int ATT_THREADS = 128;
__host__ __device__ inline int att_smem_floats(int hd) { return hd + ATT_THREADS * (hd + 1) + 2 * ATT_THREADS + 8; }

__global__ void attention_head_kernel(float *out, const float *q, int64_t ldq, const float *kc, const float *vc,
                                      int n_head, int n_kv_head, int hd, int pos0, const int32_t *pos_dev, int stride,
                                      float *scratch, int fixed_nkv) {
    pdl_wait();
    extern __shared__ __align__(16) float sm[];
    const int t = blockIdx.y, h = blockIdx.x, tid = threadIdx.x;
    const int n_kv = fixed_nkv > 0 ? fixed_nkv : (pos_dev ? *pos_dev : pos0) + t + 1;
    const int n_rep = n_head / n_kv_head, ldt = hd + 1, hd4 = hd / 4;
    const float *qv = q + (size_t)t * ldq + (size_t)h * hd;
    const float *kh = kc + (size_t)(h / n_rep) * stride * hd;
    const float *vh = vc + (size_t)(h / n_rep) * stride * hd;
    float *sc = scratch + ((size_t)t * n_head + h) * stride;
    float *qs = sm, *tile = sm + ((hd + 3) & ~3), *ps = tile + ATT_THREADS * ldt;
    const float scale = __fdiv_rn(1.0f, sqrtf((float)hd));
    for (int i = tid; i < hd; i += ATT_THREADS) qs[i] = qv[i];
    for (int j0 = 0; j0 < n_kv; j0 += ATT_THREADS) {
        const int nk = min(ATT_THREADS, n_kv - j0);
        __syncthreads();
        for (int idx = tid; idx < nk * hd4; idx += ATT_THREADS) {
            const int j = idx / hd4, i = (idx - j * hd4) * 4;
            const float4 v = *(const float4 *)(kh + (size_t)(j0 + j) * hd + i);
            float *d = tile + j * ldt + i;
            d[0] = v.x;
            d[1] = v.y;
            d[2] = v.z;
            d[3] = v.w;
        }
        __syncthreads();
        if (tid < nk) {
            const float *row = tile + tid * ldt;
            sc[j0 + tid] = __fmul_rn(dot4(qs, [&](int i) { return row[i]; }, hd), scale);
        }
    }
    __syncthreads();
    softmax_block(sc, n_kv);
    __syncthreads();
    const int tv = (ATT_THREADS * ldt) / hd;  // keys per V tile
    float acc0 = 0.0f, acc1 = 0.0f;
    const int i0 = tid, i1 = tid + ATT_THREADS;
    for (int j0 = 0; j0 < n_kv; j0 += tv) {
        const int nv = min(tv, n_kv - j0);
        __syncthreads();
        for (int idx = tid; idx < nv * hd4; idx += ATT_THREADS)
            *(float4 *)(tile + idx * 4) = *(const float4 *)(vh + (size_t)j0 * hd + idx * 4);
        for (int j = tid; j < nv; j += ATT_THREADS) ps[j] = sc[j0 + j];
        __syncthreads();
        for (int j = 0; j < nv; j++) {
            const float p = ps[j];
            if (i0 < hd) acc0 = __fadd_rn(acc0, __fmul_rn(p, tile[j * hd + i0]));
            if (i1 < hd) acc1 = __fadd_rn(acc1, __fmul_rn(p, tile[j * hd + i1]));
        }
    }
    float *ov = out + ((size_t)t * n_head + h) * hd;
    if (i0 < hd) ov[i0] = acc0;
    if (i1 < hd) ov[i1] = acc1;
}

// Prefill: one CTA per (head, PQ consecutive query tokens), PF_THREADS threads. The reference's
// per-query work in the same operation order, with K and V tiles shared by the PQ queries:
//   scores  s[q][j] = dot4(q_q, k_j) * scale for j < n_kv(q) = pos(q) + 1, into the scratch rows;
//   softmax one warp per query (exp in double rounded once, double sum, p = e * (float)(1/sum));
//   output  thread (element e, query half) runs PQ/2 chains acc_q += p[q][j] * v_j[e] in key order
//           (probabilities of masked keys are 0, and adding +0 leaves a chain unchanged).
constexpr int PQ = 16;
constexpr int PF_THREADS = 256;
constexpr int PF_KT = 64;  // keys per K/V tile
__host__ __device__ inline int pf_smem_floats(int hd) {
    return PQ * hd + PF_KT * (hd + 4) + PF_KT * hd + PF_KT * PQ;
}

__global__ void __launch_bounds__(PF_THREADS)
    attention_prefill_kernel(float *__restrict__ out, const float *__restrict__ q, int64_t ldq,
                             const float *__restrict__ kc, const float *__restrict__ vc, int n_tok, int n_head,
                             int n_kv_head, int hd, int pos0, const int32_t *pos_dev, int stride, float *scratch) {
    pdl_wait();
    extern __shared__ __align__(16) float sm[];
    const int h = blockIdx.x, t0 = blockIdx.y * PQ, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int nq = min(PQ, n_tok - t0);
    const int p0 = (pos_dev ? *pos_dev : pos0) + t0;  // position of query 0; query i sees p0 + i + 1 keys
    const int kv_max = p0 + nq;
    const int n_rep = n_head / n_kv_head;
    const float *kh = kc + (size_t)(h / n_rep) * stride * hd, *vh = vc + (size_t)(h / n_rep) * stride * hd;
    float *qs = sm, *kt = qs + PQ * hd, *vt = kt + PF_KT * (hd + 4), *pt = vt + PF_KT * hd;
    const int ldk = hd + 4, hd4 = hd / 4;
    const float scale = __fdiv_rn(1.0f, sqrtf((float)hd));
    auto srow = [&](int i) { return scratch + ((size_t)(t0 + i) * n_head + h) * stride; };
    for (int idx = tid; idx < PQ * hd4; idx += PF_THREADS) {
        const int i = idx / hd4, c = idx - i * hd4;
        const float4 v = i < nq ? *(const float4 *)(q + (size_t)(t0 + i) * ldq + (size_t)h * hd + 4 * c)
                                : make_float4(0.f, 0.f, 0.f, 0.f);
        *(float4 *)(qs + i * hd + 4 * c) = v;
    }
    // ---- scores
    for (int j0 = 0; j0 < kv_max; j0 += PF_KT) {
        const int nk = min(PF_KT, kv_max - j0);
        __syncthreads();
        for (int idx = tid; idx < nk * hd4; idx += PF_THREADS) {
            const int j = idx / hd4, c = idx - j * hd4;
            *(float4 *)(kt + j * ldk + 4 * c) = *(const float4 *)(kh + (size_t)(j0 + j) * hd + 4 * c);
        }
        __syncthreads();
        for (int pr = tid; pr < PQ * PF_KT; pr += PF_THREADS) {  // (query, key) pairs, key fastest
            const int i = pr / PF_KT, j = pr - i * PF_KT;
            if (i >= nq || j >= nk || j0 + j >= p0 + i + 1) continue;
            const float *x = qs + i * hd, *k = kt + j * ldk;
            float a0 = 0.0f, a1 = 0.0f, a2 = 0.0f, a3 = 0.0f;
            for (int c = 0; c < hd; c += 4) {
                const float4 u = *(const float4 *)(x + c), w = *(const float4 *)(k + c);
                a0 = __fadd_rn(a0, __fmul_rn(u.x, w.x));
                a1 = __fadd_rn(a1, __fmul_rn(u.y, w.y));
                a2 = __fadd_rn(a2, __fmul_rn(u.z, w.z));
                a3 = __fadd_rn(a3, __fmul_rn(u.w, w.w));
            }
            srow(i)[j0 + j] = __fmul_rn(__fadd_rn(__fadd_rn(a0, a1), __fadd_rn(a2, a3)), scale);
        }
    }
    __syncthreads();
    // ---- softmax, one warp per query
    for (int i = warp; i < nq; i += PF_THREADS / 32) {
        float *r = srow(i);
        const int nk = p0 + i + 1;
        float m = -INFINITY;
        for (int j = lane; j < nk; j += 32) m = fmaxf(m, r[j]);
        for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        double sacc = 0.0;
        for (int j = lane; j < nk; j += 32) {
            const float e = expf_ref(__fsub_rn(r[j], m));
            r[j] = e;
            sacc += e;
        }
        for (int o = 16; o; o >>= 1) sacc += __shfl_xor_sync(0xffffffffu, sacc, o);
        const float inv = (float)(1.0 / sacc);
        for (int j = lane; j < nk; j += 32) r[j] = __fmul_rn(r[j], inv);
    }
    __syncthreads();
    // ---- weighted sums: thread (e, half) keeps the chains of queries half*PQ/2 .. +PQ/2-1
    constexpr int QH = PQ / 2;
    const int e = tid % hd, half = tid / hd;  // hd <= 128: 2*hd <= 256 threads
    const bool active = tid < 2 * hd;
    float acc[QH];
#pragma unroll
    for (int c = 0; c < QH; c++) acc[c] = 0.0f;
    for (int j0 = 0; j0 < kv_max; j0 += PF_KT) {
        const int nk = min(PF_KT, kv_max - j0);
        __syncthreads();
        for (int idx = tid; idx < nk * hd4; idx += PF_THREADS)
            *(float4 *)(vt + idx * 4) = *(const float4 *)(vh + (size_t)j0 * hd + idx * 4);
        for (int idx = tid; idx < PF_KT * PQ; idx += PF_THREADS) {  // pt[j][i]: 0 where masked
            const int j = idx / PQ, i = idx - j * PQ;
            pt[idx] = (i < nq && j < nk && j0 + j < p0 + i + 1) ? srow(i)[j0 + j] : 0.0f;
        }
        __syncthreads();
        if (active) {
            const float *pq = pt + half * QH;
            for (int j = 0; j < nk; j++) {
                const float v = vt[j * hd + e];
                const float4 pa = *(const float4 *)(pq + j * PQ), pb = *(const float4 *)(pq + j * PQ + 4);
                acc[0] = __fadd_rn(acc[0], __fmul_rn(pa.x, v));
                acc[1] = __fadd_rn(acc[1], __fmul_rn(pa.y, v));
                acc[2] = __fadd_rn(acc[2], __fmul_rn(pa.z, v));
                acc[3] = __fadd_rn(acc[3], __fmul_rn(pa.w, v));
                acc[4] = __fadd_rn(acc[4], __fmul_rn(pb.x, v));
                acc[5] = __fadd_rn(acc[5], __fmul_rn(pb.y, v));
                acc[6] = __fadd_rn(acc[6], __fmul_rn(pb.z, v));
                acc[7] = __fadd_rn(acc[7], __fmul_rn(pb.w, v));
            }
        }
    }
    if (active)
#pragma unroll
        for (int c = 0; c < QH; c++) {
            const int i = half * QH + c;
            if (i < nq) out[((size_t)(t0 + i) * n_head + h) * hd + e] = acc[c];
        }
}

bool aligned16(const void *p) { return ((uintptr_t)p & 15) == 0; }

}  // namespace

void attention(float *out, const float *q, int64_t ldq, const float *kc, const float *vc, int n_tok, int n_head,
               int n_kv_head, int hd, int pos0, const int32_t *pos_dev, int stride, float *scratch, int fixed_nkv,
               cudaStream_t s, const PostQKV *post) {
    if (n_tok <= 0) return;
    if (hd % 4 || n_kv_head <= 0 || n_head % n_kv_head) {
        set_error("attention: head_dim %d / heads %d/%d not supported", hd, n_head, n_kv_head);
        return;
    }
    // The post-projection steps are fused into the single-token cluster kernel; otherwise they run first.
    PostQKV pp{};
    if (post && n_tok != 1) {
        post_qkv(*post, n_tok, s);
        post = nullptr;
    }
    // Many queries (prefill): the query-tile kernel (causal counts only; fixed_nkv is op_attention's
    // single query).
    if (n_tok >= PQ && fixed_nkv <= 0 && hd <= 128 && aligned16(q) && ldq % 4 == 0 && aligned16(kc) &&
        aligned16(vc) && n_tok <= 65535 * PQ) {
        const size_t smem = (size_t)pf_smem_floats(hd) * 4;
        static std::atomic<uint64_t> configured{0};
        smem_limit_once(attention_prefill_kernel, pf_smem_floats(128) * 4, configured);
        launch(attention_prefill_kernel, dim3(n_head, (n_tok + PQ - 1) / PQ), PF_THREADS, smem, s, out, q, ldq, kc, vc,
               n_tok, n_head, n_kv_head, hd, pos0, pos_dev, stride, scratch);
        SDY_LAUNCHED();
        return;
    }
    const int n_rep = n_head / n_kv_head;
    const int push = (size_t)ac_smem(n_rep, hd, stride, true).total * 4 <= AC_SMEM_LIMIT;
    const bool cluster = hd % (4 * AC) == 0 && stride % 4 == 0 && n_rep <= AC_MAX_REP &&
                         n_rep * hd <= AC_MAX_GROUP && aligned16(kc) && aligned16(vc) && aligned16(q) &&
                         ldq % 4 == 0 &&
                         (size_t)ac_smem(n_rep, hd, stride, push).total * 4 <= AC_SMEM_LIMIT && n_kv_head <= 65535 &&
                         n_tok <= 65535;
    if (post && !(cluster && hd <= 256 && fixed_nkv <= 0)) {
        post_qkv(*post, n_tok, s);
        post = nullptr;
    }
    if (post) pp = *post;
    if (cluster) {
        const size_t smem = (size_t)ac_smem(n_rep, hd, stride, push).total * 4;
        static std::atomic<uint64_t> configured{0};
        smem_limit_once(attention_cluster_kernel, AC_SMEM_LIMIT, configured);
        launch(attention_cluster_kernel, dim3(AC, n_kv_head, n_tok), AC_THREADS, smem, s, out, q, ldq, kc, vc, n_head,
               n_kv_head, hd, pos0, pos_dev, stride, fixed_nkv, push, pp);
        SDY_LAUNCHED();
        return;
    }
    if (hd > 2 * ATT_THREADS) {
        set_error("attention: head_dim %d not supported (multiple of 4, at most %d)", hd, 2 * ATT_THREADS);
        return;
    }
    const size_t smem = (size_t)att_smem_floats(hd) * 4;
    static std::atomic<uint64_t> configured{0};
    smem_limit_once(attention_head_kernel, att_smem_floats(2 * ATT_THREADS) * 4, configured);
    launch(attention_head_kernel, dim3(n_head, n_tok), ATT_THREADS, smem, s, out, q, ldq, kc, vc, n_head, n_kv_head, hd,
                                                                         pos0, pos_dev, stride, scratch, fixed_nkv);
    SDY_LAUNCHED();
}

}  // namespace sdy
