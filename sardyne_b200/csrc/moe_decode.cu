// The MoE block of a single-token step as ONE kernel (reference csrc/model_llama.c:653-751 and the
// residual add at :820): RMSNorm of the residual, the float router's logits, softmax and top-k,
// the chosen experts' gate|up products, their SwiGLU gate, the down products and the weighted sum
// into the residual. It replaces the decode step's norm, router, gate|up, down and combine
// launches (five dependent kernels) with one.
//
// Shape. A persistent grid of P CTAs, one per SM (all resident at once), so all are
// resident together, runs the phases with two grid barriers between them:
//   0  every CTA: RMSNorm of x, kept as floats (router input) and as Q8_K (gate|up input) in
//      shared memory (norm_quant_row, the same floats as the standalone norm kernel);
//   1  CTAs e < ne (and e + P, ...): router logit e, the reference's four-accumulator dot
//      (ops.c:155-167) over the row staged before the dependency wait;       -- grid barrier --
//   2  every CTA: softmax and top-k of the ne logits (the same code as router_topk_kernel, so
//      every CTA holds the same choice); L2 prefetch of the down rows it will read;
//   3  gate|up: the k slots' (slot, 8-row group) units split evenly over the CTAs, each pair of
//      (row, superblock) in registers, per-row ordered sums (qmv_device.cuh);  -- grid barrier --
//   4  down: the same over the down matrices, the CTA's slots' SwiGLU rows quantized in shared
//      memory first (act_quant_row, the same floats as the fused down kernel);
//   5  the last CTA to finish (a counter) adds the k expert rows, in ascending expert id, to x.
// Every value equals the one the separate kernels produce (same device functions, same order).
//
// Waits. The barriers spin on a generation word with a poll limit; a CTA that gives up sets the
// status word and returns, the others then give up too, and the host reports the error and
// clears the barrier words. Nothing waits without a limit. CTAs of the previous kernel that still
// occupy SMs (dependent launch) retire on their own, so every CTA of this grid gets placed.
#include "common.cuh"
#include "fp_device.cuh"
#include "fused.cuh"
#include "qmv_device.cuh"
#include "quant_device.cuh"

#include <algorithm>

namespace sdy {
namespace {

constexpr int MD_THREADS = 512;
constexpr int MD_CTAS_PER_SM = 1;
constexpr int MD_MAX_K = 64;
constexpr long long MD_SPIN_LIMIT = 1ll << 22;  // polls of ~32 ns sleep: well under a second

__device__ __forceinline__ unsigned ld_acquire(const unsigned *p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];\n" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_release(unsigned *p, unsigned v) {
    asm volatile("st.release.gpu.global.u32 [%0], %1;\n" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned atom_add_acq_rel(unsigned *p, unsigned v) {
    unsigned old;
    asm volatile("atom.add.acq_rel.gpu.global.u32 %0, [%1], %2;\n" : "=r"(old) : "l"(p), "r"(v) : "memory");
    return old;
}

// Grid barrier over n CTAs: bar[0] counts arrivals, bar[1] is the generation the last arrival
// advances. False (and *status set) when the wait gave up.
__device__ bool grid_barrier(unsigned *bar, unsigned n, unsigned *status) {
    __shared__ int ok;
    __syncthreads();
    if (threadIdx.x == 0) {
        int good = 1;
        const unsigned gen = ld_acquire(bar + 1);
        __threadfence();
        if (atom_add_acq_rel(bar, 1) == n - 1) {
            bar[0] = 0;
            st_release(bar + 1, gen + 1);
        } else {
            for (long long it = 0; ld_acquire(bar + 1) == gen; it++) {
                if (it > MD_SPIN_LIMIT || ld_acquire(status)) {
                    atomicOr(status, 1u);
                    good = 0;
                    break;
                }
                if (it > 4096) __nanosleep(64);  // tight polling first: most waits are short
            }
        }
        __threadfence();
        ok = good;
    }
    __syncthreads();
    return ok;
}

__device__ __forceinline__ void prefetch_l2(const void *p, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;\n" ::"l"(p), "r"(bytes) : "memory");
}

// Units [u0, u1) of the experts' products: unit u is (slot u / gpe, 8-row group u % gpe) of
// expert top[slot]. Each thread takes pairs (row, superblock); the block terms go to `terms`
// and one thread per row adds them in block order into out[slot * ldo + row]. The activations
// of local slot ls (slot - slot0) are the XQ at sq + ls * qrow, sd + ls * nb, ss + ls * nb * 8
// (xq_per_slot false: one XQ for every slot).
template <int TYPE>
__device__ void expert_units(const uint8_t *slabs, int64_t gpe, int nb, const int *top, int64_t u0, int64_t u1,
                             int slot0, bool xq_per_slot, const uint8_t *sq, int qrow, const float *sd,
                             const int32_t *ss, int64_t rows_per_expert, float *out, int64_t ldo, float *terms) {
    constexpr int SB = slab_bytes(TYPE);
    const int rows = (int)(u1 - u0) * GROUP_ROWS;
    const int ppu = GROUP_ROWS * nb;  // pairs per unit
    const int npairs = (int)(u1 - u0) * ppu;
    for (int p = threadIdx.x; p < npairs; p += MD_THREADS) {
        const int ul = p / ppu, rem = p - ul * ppu;
        const int u = rem >> 3, r = rem & 7;
        const int64_t unit = u0 + ul;
        const int slot = (int)(unit / gpe);
        const int64_t g = unit - (int64_t)slot * gpe;
        const int ls = xq_per_slot ? slot - slot0 : 0;
        Raw<TYPE> w;
        load_pair(w, slabs + ((size_t)top[slot] * gpe + g) * nb * SB, u, r, nb);
        pair_compute<TYPE, 1>(w, u, sq + (size_t)ls * qrow, qrow, sd + (size_t)ls * nb, ss + (size_t)ls * nb * 8, nb,
                              terms, rows, ul * GROUP_ROWS + r);
    }
    __syncthreads();
    for (int i = threadIdx.x; i < rows; i += MD_THREADS) {
        const int64_t unit = u0 + i / GROUP_ROWS;
        const int slot = (int)(unit / gpe);
        const int64_t row = (unit - (int64_t)slot * gpe) * GROUP_ROWS + (i % GROUP_ROWS);
        if (row >= rows_per_expert) continue;
        const float *tp = terms + i;
        out[(size_t)slot * ldo + row] = ordered_sum<8>(0.0f, nb, [&](int b) { return tp[(size_t)b * rows]; });
    }
    __syncthreads();
}

// Shared-memory carve-up, identical on host and device.
struct MdSmem {
    int xs, prod, xq_gu, xq_dn, gs, terms, prob, total;
    int dn_slots;
};
__host__ __device__ inline MdSmem md_plan(int dim, int fe, int ne, int64_t units3_cta, int64_t units4_cta,
                                          int64_t gpe_dn) {
    MdSmem m;
    const int nb_gu = dim / 256, nb_dn = fe / 256;
    m.dn_slots = (int)((units4_cta + gpe_dn - 1) / gpe_dn) + 1;
    int o = 0;
    m.xs = o;
    o += dim * 4;
    m.prod = o;
    o += dim * 4;
    m.xq_gu = o;
    o += (xq_qrow(dim) + nb_gu * 4 + nb_gu * 32 + 15) & ~15;
    m.xq_dn = o;
    o += m.dn_slots * ((xq_qrow(fe) + nb_dn * 4 + nb_dn * 32 + 15) & ~15);
    m.gs = o;
    o += m.dn_slots * 2 * fe * 4;
    m.terms = o;
    const int64_t t3 = units3_cta * GROUP_ROWS * nb_gu, t4 = units4_cta * GROUP_ROWS * nb_dn;
    o += (int)((t3 > t4 ? t3 : t4) * 4);
    m.prob = o;
    o += ((ne + MD_MAX_K) * 4 + 15) & ~15;  // probabilities, then the k chosen ones
    m.total = o;
    return m;
}

template <int TG, int TD>
__global__ void __launch_bounds__(MD_THREADS) moe_decode_kernel(MoeDecode a) {
    extern __shared__ __align__(16) uint8_t smem[];
    __shared__ double dpart[32];
    __shared__ float fpart[32];
    __shared__ int top_s[MD_MAX_K];
    __shared__ float w_s[MD_MAX_K];
    __shared__ int last;
    const unsigned P = gridDim.x, cta = blockIdx.x;
    const int tid = threadIdx.x, dim = a.dim, fe = a.fe, ne = a.ne, k = a.k;
    const int G = dim / 4;
    const int64_t U3 = (int64_t)k * a.gpe_gu, U4 = (int64_t)k * a.gpe_dn;
    const int64_t u3a = U3 * cta / P, u3b = U3 * (cta + 1) / P;
    const int64_t u4a = U4 * cta / P, u4b = U4 * (cta + 1) / P;
    const MdSmem plan = md_plan(dim, fe, ne, (U3 + P - 1) / P, (U4 + P - 1) / P, a.gpe_dn);
    float *xs = (float *)(smem + plan.xs), *prod = (float *)(smem + plan.prod);
    float *terms = (float *)(smem + plan.terms), *prob = (float *)(smem + plan.prob);

    // The CTA's first router row (a weight: read before the dependency wait): float4 column
    // f = tid + j * MD_THREADS of the row (dim <= 8192).
    const int nf = dim / 4;
    float4 wrow[4];
    int e_router = (int)cta;
    if (e_router < ne) {
#pragma unroll
        for (int j = 0; j < 4; j++)
            if (tid + j * MD_THREADS < nf)
                wrow[j] = load4_w(a.router, a.rtype, (size_t)e_router * dim + 4 * (size_t)(tid + j * MD_THREADS));
    }
    pdl_wait();

    // 0: RMSNorm of the residual: floats (router) and Q8_K (gate|up), every CTA.
    XQ qg;
    qg.vtype = T_Q8_K;
    qg.n_in = dim;
    qg.n_tok = 1;
    qg.qrow = xq_qrow(dim);
    qg.nbx = dim / 256;
    qg.qs = (int8_t *)(smem + plan.xq_gu);
    qg.d = (float *)(smem + plan.xq_gu + qg.qrow);
    qg.sums = smem + plan.xq_gu + qg.qrow + qg.nbx * 4;
    XQ none;
    none.qs = nullptr;
    norm_quant_row(a.x, a.norm_w, dim, a.eps, 0, qg, none, xs, dpart);
    __syncthreads();

    // 1: router logits; the products x_i * w_i (each rounded, as in the chain) are stored
    // de-interleaved (element 4g + c at [c * G + g]) so each chain reads 4 terms per load.
    for (; e_router < ne; e_router += P) {
        if (e_router != (int)cta) {
#pragma unroll
            for (int j = 0; j < 4; j++)
                if (tid + j * MD_THREADS < nf)
                    wrow[j] = load4_w(a.router, a.rtype, (size_t)e_router * dim + 4 * (size_t)(tid + j * MD_THREADS));
        }
#pragma unroll
        for (int j = 0; j < 4; j++) {
            const int g = tid + j * MD_THREADS;
            if (g >= nf) break;
            const int i = 4 * g;
            prod[g] = __fmul_rn(xs[i], wrow[j].x);
            prod[G + g] = __fmul_rn(xs[i + 1], wrow[j].y);
            prod[2 * G + g] = __fmul_rn(xs[i + 2], wrow[j].z);
            prod[3 * G + g] = __fmul_rn(xs[i + 3], wrow[j].w);
        }
        __syncthreads();
        if (tid < 32) {
            float s = 0.0f;
            if (tid < 4) {
                const float4 *ra = (const float4 *)(prod + tid * G);
#pragma unroll 8
                for (int q = 0; q < G / 4; q++) {
                    const float4 b = ra[q];
                    s = __fadd_rn(s, b.x);
                    s = __fadd_rn(s, b.y);
                    s = __fadd_rn(s, b.z);
                    s = __fadd_rn(s, b.w);
                }
            }
            const float s1 = __shfl_sync(0xffffffffu, s, 1), s2 = __shfl_sync(0xffffffffu, s, 2),
                        s3 = __shfl_sync(0xffffffffu, s, 3);
            if (tid == 0) a.logits[e_router] = __fadd_rn(__fadd_rn(s, s1), __fadd_rn(s2, s3));
        }
        __syncthreads();
    }
    if (!grid_barrier(a.bar, P, a.status)) return;

    // 2: softmax and top-k (every CTA the same), weights renormalised. The slots start at expert
    // 0, so that no expert id outside [0, ne) can reach the weight addressing below.
    if (tid < k) top_s[tid] = 0;
    softmax_topk_block(a.logits, prob, prob + ne, ne, k, top_s, w_s, dpart, fpart);
    __syncthreads();
    if (cta == 0 && tid < k) {
        a.top[tid] = top_s[tid];
        a.wts[tid] = w_s[tid];
    }
    if (tid == 0 && u4b > u4a) {  // this CTA's down rows into L2 (one contiguous range per slot)
        for (int64_t u = u4a; u < u4b;) {
            const int slot = (int)(u / a.gpe_dn);
            const int64_t g = u - (int64_t)slot * a.gpe_dn, end = std::min<int64_t>(u4b, (int64_t)(slot + 1) * a.gpe_dn);
            const size_t gb = (size_t)(fe / 256) * slab_bytes(TD);
            prefetch_l2(a.dn_slabs + ((size_t)top_s[slot] * a.gpe_dn + g) * gb, (uint32_t)((end - u) * gb));
            u = end;
        }
    }

    // 3: gate|up of the chosen experts.
    if (u3b > u3a)
        expert_units<TG>(a.gu_slabs, a.gpe_gu, dim / 256, top_s, u3a, u3b, 0, false, (const uint8_t *)qg.qs, qg.qrow,
                         qg.d, (const int32_t *)qg.sums, 2 * fe, a.gu, 2 * fe, terms);
    if (!grid_barrier(a.bar, P, a.status)) return;

    // 4: down: the SwiGLU rows of this CTA's slots, quantized, then the products.
    if (u4b > u4a) {
        const int s0 = (int)(u4a / a.gpe_dn), s1 = (int)((u4b - 1) / a.gpe_dn), ns = s1 - s0 + 1;
        float *gs = (float *)(smem + plan.gs);
        {  // the slots' gate|up rows, float4 loads all issued before the stores
            const float4 *src = (const float4 *)(a.gu + (size_t)s0 * 2 * fe);
            const int n4 = ns * 2 * fe / 4;
            for (int i0 = tid; i0 < n4; i0 += 4 * MD_THREADS) {
                float4 v[4];
#pragma unroll
                for (int u = 0; u < 4; u++)
                    if (i0 + u * MD_THREADS < n4) v[u] = __ldcg(src + i0 + u * MD_THREADS);
#pragma unroll
                for (int u = 0; u < 4; u++)
                    if (i0 + u * MD_THREADS < n4) ((float4 *)gs)[i0 + u * MD_THREADS] = v[u];
            }
        }
        __syncthreads();
        XQ qd;
        qd.vtype = T_Q8_K;
        qd.n_in = fe;
        qd.n_tok = ns;
        qd.qrow = xq_qrow(fe);
        qd.nbx = fe / 256;
        qd.qs = (int8_t *)(smem + plan.xq_dn);
        qd.d = (float *)(smem + plan.xq_dn + plan.dn_slots * qd.qrow);
        qd.sums = smem + plan.xq_dn + plan.dn_slots * (qd.qrow + qd.nbx * 4);
        ActIn gate;
        gate.x = gs;
        gate.ldx = 2 * fe;
        gate.u = gs + fe;
        gate.ldu = 2 * fe;
        for (int t = 0; t < ns; t++) act_quant_row(gate, fe, t, qd, none, dpart);
        __syncthreads();
        expert_units<TD>(a.dn_slabs, a.gpe_dn, fe / 256, top_s, u4a, u4b, s0, true, (const uint8_t *)qd.qs, qd.qrow,
                         qd.d, (const int32_t *)qd.sums, dim, a.y, dim, terms);
    }

    // 5: the last CTA adds the experts' rows to the residual, in ascending expert id.
    if (tid == 0) {
        __threadfence();
        last = atom_add_acq_rel(a.bar + 2, 1) == P - 1;
    }
    __syncthreads();
    if (!last) return;
    __threadfence();
    if (tid == 0) a.bar[2] = 0;
    __shared__ int order[MD_MAX_K];
    __shared__ float ws[MD_MAX_K];
    if (tid < k) {
        int rank = 0;
        for (int j = 0; j < k; j++) rank += top_s[j] < top_s[tid] || (top_s[j] == top_s[tid] && j < tid);
        order[rank] = tid;
    }
    __syncthreads();
    if (tid < k) ws[tid] = w_s[order[tid]];
    __syncthreads();
    // four elements a thread, the k rows' loads issued 8 at a time ahead of their ordered adds
    for (int f = tid; f < nf; f += MD_THREADS) {
        float4 acc = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        for (int j0 = 0; j0 < k; j0 += 8) {
            float4 yv[8];
#pragma unroll
            for (int u = 0; u < 8; u++)
                if (j0 + u < k) yv[u] = __ldcg((const float4 *)(a.y + (size_t)order[j0 + u] * dim) + f);
#pragma unroll
            for (int u = 0; u < 8; u++)
                if (j0 + u < k) {
                    const float w = ws[j0 + u];
                    acc.x = __fadd_rn(acc.x, __fmul_rn(w, yv[u].x));
                    acc.y = __fadd_rn(acc.y, __fmul_rn(w, yv[u].y));
                    acc.z = __fadd_rn(acc.z, __fmul_rn(w, yv[u].z));
                    acc.w = __fadd_rn(acc.w, __fmul_rn(w, yv[u].w));
                }
        }
        float4 xv = ((float4 *)a.x)[f];
        xv.x = __fadd_rn(xv.x, acc.x);
        xv.y = __fadd_rn(xv.y, acc.y);
        xv.z = __fadd_rn(xv.z, acc.z);
        xv.w = __fadd_rn(xv.w, acc.w);
        ((float4 *)a.x)[f] = xv;
    }
}

template <int TG, int TD>
int grid_for(int smem) {
    static std::atomic<uint64_t> configured{0};
    smem_limit_once(moe_decode_kernel<TG, TD>, 200 * 1024, configured);
    int n = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, moe_decode_kernel<TG, TD>, MD_THREADS, smem) !=
        cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    int dev = 0, sms = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    return std::min(n, MD_CTAS_PER_SM) * sms;
}

template <int TG, int TD>
void launch_md(const MoeDecode &a, int grid, int smem, cudaStream_t s) {
    launch(moe_decode_kernel<TG, TD>, dim3(grid), dim3(MD_THREADS), smem, s, a);
}

int plan_grid(int tg, int td, const MoeDecode &a, int *smem) {
    // the shared memory depends on the grid (units per CTA): plan for MD_CTAS_PER_SM CTAs per SM,
    // then check that the SMs hold that many
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const int64_t P = (int64_t)MD_CTAS_PER_SM * sms;
    const int64_t U3 = (int64_t)a.k * a.gpe_gu, U4 = (int64_t)a.k * a.gpe_dn;
    *smem = md_plan(a.dim, a.fe, a.ne, (U3 + P - 1) / P, (U4 + P - 1) / P, a.gpe_dn).total;
    int grid = 0;
    if (tg == T_Q4_K && td == T_Q4_K) grid = grid_for<T_Q4_K, T_Q4_K>(*smem);
    else if (tg == T_Q4_K && td == T_Q6_K) grid = grid_for<T_Q4_K, T_Q6_K>(*smem);
    else if (tg == T_Q6_K && td == T_Q4_K) grid = grid_for<T_Q6_K, T_Q4_K>(*smem);
    else if (tg == T_Q6_K && td == T_Q6_K) grid = grid_for<T_Q6_K, T_Q6_K>(*smem);
    return grid >= P ? (int)P : 0;  // fewer resident CTAs than planned: not taken
}

}  // namespace

bool moe_decode_supported(int tg, int td, int rtype, int dim, int fe, int ne, int k) {
    const bool kq = (tg == T_Q4_K || tg == T_Q6_K) && (td == T_Q4_K || td == T_Q6_K);
    const bool ft = rtype == T_F32 || rtype == T_F16 || rtype == T_BF16;
    return kq && ft && dim % 256 == 0 && dim >= 1024 && dim <= 4 * 4 * MD_THREADS &&
           fe % 256 == 0 && fe <= 4096 && k >= 1 && k <= MD_MAX_K && k <= ne && ne <= 4096;
}

bool moe_decode(const MoeDecode &a, int tg, int td, cudaStream_t s) {
    int smem = 0;
    const int grid = plan_grid(tg, td, a, &smem);
    if (grid <= 0 || smem > 200 * 1024) return false;
    if (tg == T_Q4_K && td == T_Q4_K) launch_md<T_Q4_K, T_Q4_K>(a, grid, smem, s);
    else if (tg == T_Q4_K && td == T_Q6_K) launch_md<T_Q4_K, T_Q6_K>(a, grid, smem, s);
    else if (tg == T_Q6_K && td == T_Q4_K) launch_md<T_Q6_K, T_Q4_K>(a, grid, smem, s);
    else launch_md<T_Q6_K, T_Q6_K>(a, grid, smem, s);
    SDY_LAUNCHED();
    return true;
}

}  // namespace sdy
