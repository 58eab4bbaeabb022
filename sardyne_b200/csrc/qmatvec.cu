// Decode / small-batch quantized matvec: y[t][r] = W[r] . x[t] for 1..8 tokens.
//
// Replaces the reference's per-row dot products (reference csrc/quant.c:148-235,
// csrc/quant_avx2.c:106-385) and their row dispatch (csrc/ops.c:293-309).
//
// Mapping. A CTA owns a contiguous range of 8-row groups and sweeps it in batches. Every lane
// owns one (row, superblock) pair — for the 32-element formats one (row, run of 8 blocks) — and
// computes that pair's integer sums entirely in registers with dp4a, so no cross-lane reduction
// happens per block. Lanes r = 0..7 of a pair column read the same 16-byte chunk of 8 rows: one
// 128-byte segment of the slab layout per 8 lanes, 4 segments per warp instruction. The token
// activations (int8 + scales + sums) sit in shared memory and are read as broadcasts.
//
// Exactness. Each pair produces the reference's per-block fp32 term (q4k_combine / q6k_combine /
// (float)s*(dw*dx), quant.h:84-91, quant.c:160) with explicit round-to-nearest intrinsics; the
// terms go to shared memory and one thread per (token, row) adds them in block order. The
// result is bit-identical to the reference's scalar kernels (and, for Q4_K/Q6_K, to its AVX2
// kernels, which share the same combine).
#include "common.cuh"
#include "qmv_device.cuh"
#include "quant_device.cuh"

#include <algorithm>
#include <cstdlib>
#include <atomic>

namespace sdy {

namespace {

constexpr int THREADS = 256;
constexpr int CTAS_PER_SM = 4;
constexpr int SMEM_BUDGET = 48 * 1024;  // keeps up to CTAS_PER_SM resident for one token
constexpr int SMEM_LIMIT = 200 * 1024;

struct Args {
    const uint8_t *slabs;
    int nb;             // blocks per row (of the weight type)
    int64_t g_begin;    // first group of the whole launch
    int64_t n_groups;   // groups in the launch
    int G;              // groups per batch
    const int8_t *xqs;  // XQ of the first token of this chunk
    const float *xd;
    const void *xsums;
    int qrow;           // XQ row stride (bytes)
    int nbx;            // XQ blocks per token
    float *out;
    int64_t ldo, row0, row1, out_row0;
    const float *residual;  // when set: out = residual + product (same indexing as out)
    // Gathered experts (MoE): grid.y = slot; slot s multiplies expert slot_expert[s], whose
    // groups start at expert * gpe, with the activations of token s / tok_div, into out + s*ldo_slot.
    const int32_t *slot_expert;
    int64_t gpe, ldo_slot;
    // When act.x is set, the activations are not read from the XQ: each CTA prepares its tokens'
    // rows (RMSNorm, SwiGLU gate or as is) and quantizes them into shared memory itself.
    ActIn act;
    int tok_div, n_expert, expert0;  // slot_expert ids are global; this matrix holds experts expert0..
};

// Shared-memory carve-up, identical on host and device.
struct Smem {
    int q_off, d_off, s_off, t_off, total;
};
__host__ __device__ inline Smem smem_plan(int type, int NT, int qrow, int nb, int G) {
    Smem m;
    const bool kq = (type == T_Q4_K || type == T_Q6_K);
    m.q_off = 0;
    m.d_off = (NT * qrow + 15) & ~15;
    m.s_off = m.d_off + ((NT * nb * 4 + 15) & ~15);
    m.t_off = m.s_off + ((NT * nb * (kq ? 32 : 4) + 15) & ~15);
    m.total = m.t_off + NT * nb * G * GROUP_ROWS * 4;
    return m;
}

// ---------------------------------------------------------------------------- the kernel

// The CTA's work: CTA `cta` of the n_cta that share the launch's groups.
template <int TYPE, int NT>
__device__ __forceinline__ void qmv_body(const Args &a, int cta, int n_cta, uint8_t *smem,
                                         const PeerGatherTail *pg = nullptr) {
    constexpr bool KQ = (TYPE == T_Q4_K || TYPE == T_Q6_K);
    constexpr int SB = slab_bytes(TYPE);
    const Smem plan = smem_plan(TYPE, NT, a.qrow, a.nb, a.G);
    uint8_t *sq = smem + plan.q_off;
    float *sd = (float *)(smem + plan.d_off);
    int32_t *ss = (int32_t *)(smem + plan.s_off);
    float *terms = (float *)(smem + plan.t_off);
    const int tid = threadIdx.x;
    const int nb = a.nb;
    const uint8_t *slabs = a.slabs;
    const int8_t *xqs = a.xqs;
    const float *xd = a.xd;
    const int32_t *xsums = (const int32_t *)a.xsums;
    float *out = a.out;
    // This CTA's contiguous share of the launch's groups, swept in batches of a.G groups.
    const int64_t gA = a.g_begin + a.n_groups * cta / n_cta;
    const int64_t gB = a.g_begin + a.n_groups * (cta + 1) / n_cta;
    const int units = KQ ? nb : (nb + 7) / 8;  // pair columns per row
    const int ppg = GROUP_ROWS * units;        // pairs per group
    // The thread's first pair (pair tid of the first batch): loaded before waiting on the
    // activations' producer. For gathered experts the expert id is itself produced upstream.
    Raw<TYPE> w;
    const int G0 = (int)((gB - gA) < a.G ? (gB - gA) : a.G);
    const bool pre = !a.slot_expert && tid < G0 * ppg;
    if (pre) {
        const int gl = tid / ppg, rem = tid - gl * ppg;
        load_pair(w, slabs + (size_t)(gA + gl) * nb * SB, rem >> 3, rem & 7, nb);
    }
    pdl_wait();
    ActIn act = a.act;
    if (a.slot_expert) {
        const int slot = blockIdx.y, e = a.slot_expert[slot] - a.expert0;
        if (e < 0 || e >= a.n_expert) return;  // another rank's expert (or an invalid id)
        const int tok = slot / a.tok_div;
        slabs += (size_t)e * a.gpe * nb * SB;
        xqs += (size_t)tok * a.qrow;
        xd += (size_t)tok * a.nbx;
        xsums += (size_t)tok * a.nbx * (KQ ? 8 : 1);
        if (act.x) act.x += (size_t)tok * act.ldx;
        if (act.u) act.u += (size_t)tok * act.ldu;
        out += (size_t)slot * a.ldo_slot;
    }

    if (act.x) {  // prepare and quantize the NT rows into the shared-memory XQ
        __shared__ double part[32];
        XQ v;
        v.vtype = KQ ? T_Q8_K : T_Q8_0;
        v.n_in = nb * block_elems(TYPE);
        v.n_tok = NT;
        v.qrow = a.qrow;
        v.nbx = nb;
        v.qs = (int8_t *)sq;
        v.d = sd;
        v.sums = ss;
        XQ none;
        none.qs = nullptr;
        for (int t = 0; t < NT; t++) act_quant_row(act, v.n_in, t, KQ ? v : none, KQ ? none : v, part);
    } else {  // stage the activations of NT tokens (broadcast operands for every pair)
        const int qv = NT * a.qrow / 16;
        for (int i = tid; i < qv; i += THREADS) {
            int t = i / (a.qrow / 16), k = i % (a.qrow / 16);
            ((uint4 *)sq)[i] = __ldg((const uint4 *)(xqs + (size_t)t * a.qrow) + k);
        }
        for (int i = tid; i < NT * nb; i += THREADS) {
            int t = i / nb, b = i % nb;
            sd[i] = xd[(size_t)t * a.nbx + b];
        }
        const int per = KQ ? 8 : 1;  // int32 words per block: 8 bsum pairs, or one block sum
        for (int i = tid; i < NT * nb * per; i += THREADS) {
            int t = i / (nb * per), k = i % (nb * per);
            ss[i] = xsums[(size_t)t * a.nbx * per + k];
        }
    }
    __syncthreads();

    for (int64_t gb = gA; gb < gB; gb += a.G) {
        const int G = (int)((gB - gb) < a.G ? (gB - gb) : a.G);
        const int rows = G * GROUP_ROWS;
        const int npairs = rows * units;
        for (int p = tid; p < npairs; p += THREADS) {
            const int gl = p / ppg;
            const int rem = p - gl * ppg;
            const int u = rem >> 3, r = rem & 7;
            if (!(pre && gb == gA && p == tid)) load_pair(w, slabs + (size_t)(gb + gl) * nb * SB, u, r, nb);
            pair_compute<TYPE, NT>(w, u, sq, a.qrow, sd, ss, nb, terms, rows, gl * GROUP_ROWS + r);
        }
        __syncthreads();
        // Ordered combine: the reference adds block terms left to right (acc = acc + term).
        for (int i = tid; i < NT * rows; i += THREADS) {
            const int t = i / rows, rl = i % rows;
            const int64_t row = gb * GROUP_ROWS + rl;
            if (row < a.row0 || row >= a.row1) continue;
            const float *tp = terms + (size_t)t * nb * rows + rl;
            const float acc = ordered_sum<8>(0.0f, nb, [&](int b) { return tp[(size_t)b * rows]; });
            const size_t o = (size_t)t * a.ldo + (row - a.out_row0);
            // residual stream: x = x + W.a, the reference's `x[i] += xb[i]` (model_llama.c:804,820)
            const float v = a.residual ? __fadd_rn(a.residual[o], acc) : acc;
            out[o] = v;
            if (pg)  // the same value into every peer's copy of the buffer
                for (int q = 0; q < pg->n_peer; q++) *(float *)((char *)(out + o) + pg->delta[q]) = v;
        }
        __syncthreads();
    }
}

template <int TYPE, int NT>
__global__ void __launch_bounds__(THREADS) qmv_kernel(Args a) {
    extern __shared__ __align__(16) uint8_t smem[];
    qmv_body<TYPE, NT>(a, blockIdx.x, gridDim.x, smem);
}

// Two matrices that share one single-token input (the parts of a projection whose weight types
// differ, e.g. Q/K in Q4_K and V in Q6_K) in one launch: CTAs [0, na) multiply the first, the
// rest the second.
template <int TA, int TB>
__global__ void __launch_bounds__(THREADS) qmv2_kernel(Args a, Args b, int na) {
    extern __shared__ __align__(16) uint8_t smem[];
    if ((int)blockIdx.x < na) qmv_body<TA, 1>(a, blockIdx.x, na, smem);
    else qmv_body<TB, 1>(b, blockIdx.x - na, gridDim.x - na, smem);
}


// Independent single-token products in one launch (a grouped matvec): CTAs [cta0[i], cta0[i+1])
// sweep matrix i, of type TA or TB. One launch latency for all of them, and their bytes stream
// from HBM together.
constexpr int BATCH_MAX = 8;
struct BatchArgs {
    Args a[BATCH_MAX];
    int type[BATCH_MAX];
    int cta0[BATCH_MAX + 1];
    int n;
    int gather;  // 1: pg holds a fused all-gather
    PeerGatherTail pg;
};

__device__ unsigned g_qmvb_status;
// flag store after one system fence (see p2p.cu: a st.release.sys per flag costs a fence each)
__device__ __forceinline__ void st_relaxed_sys(unsigned *p, unsigned v) {
    asm volatile("st.relaxed.sys.global.u32 [%0], %1;\n" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned *p) {
    unsigned v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];\n" : "=r"(v) : "l"(p) : "memory");
    return v;
}

template <int TA, int TB, bool GATHER>
__global__ void __launch_bounds__(THREADS) qmvb_kernel(const __grid_constant__ BatchArgs b) {
    extern __shared__ __align__(16) uint8_t smem[];
    int i = 0;
    while (i + 1 < b.n && (int)blockIdx.x >= b.cta0[i + 1]) i++;
    const int c = blockIdx.x - b.cta0[i], nc = b.cta0[i + 1] - b.cta0[i];
    const PeerGatherTail *pg = GATHER ? &b.pg : nullptr;
    if (b.type[i] == TA) qmv_body<TA, 1>(b.a[i], c, nc, smem, pg);
    else qmv_body<TB, 1>(b.a[i], c, nc, smem, pg);
    if constexpr (!GATHER) return;
    // fused all-gather: the CTA's peer stores ordered before its arrival (one system fence by
    // thread 0 after the barrier, cumulative); the last CTA publishes the round and waits
    __shared__ int last;
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence_system();
        last = atomicAdd(b.pg.done, 1u) == gridDim.x - 1;
    }
    __syncthreads();
    if (!last || threadIdx.x != 0) return;
    *b.pg.done = 0;
    const unsigned r = *(volatile unsigned *)b.pg.round + 1;
    *b.pg.round = r;
    __threadfence_system();  // every CTA's stores (each fenced before arriving) before the flags
    for (int q = 0; q < b.pg.world; q++) st_relaxed_sys(b.pg.flags[q] + b.pg.rank, r);
    const unsigned *mine = b.pg.flags[b.pg.rank];
    unsigned long long t0;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t0));
    for (int q = 0; q < b.pg.world; q++) {
        for (long long it = 0; (int)(ld_acquire_sys(mine + q) - r) < 0; it++) {
            if (it > 256) {
                unsigned long long t;
                asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
                if (t - t0 > 1000000000ull) {  // one second
                    atomicOr(&g_qmvb_status, 1u);
                    return;
                }
                __nanosleep(128);
            }
        }
    }
}

// Raises the instantiation's dynamic shared memory limit to SMEM_LIMIT on the current device
// (once): without it a launch or occupancy query above 48 KB minus the static shared memory fails.
template <int TYPE, int NT>
void configure_one() {
    static std::atomic<uint64_t> configured{0};
    smem_limit_once(qmv_kernel<TYPE, NT>, SMEM_LIMIT, configured);
}

template <int TYPE, int NT>
void launch_one(const Args &a, int smem, dim3 grid, cudaStream_t s) {
    configure_one<TYPE, NT>();
    launch(qmv_kernel<TYPE, NT>, grid, THREADS, smem, s, a);
}

template <int TYPE>
void launch_nt(int nt, const Args &a, int smem, dim3 grid, cudaStream_t s) {
    switch (nt) {
    case 1: launch_one<TYPE, 1>(a, smem, grid, s); break;
    case 2: launch_one<TYPE, 2>(a, smem, grid, s); break;
    case 3: launch_one<TYPE, 3>(a, smem, grid, s); break;
    case 4: launch_one<TYPE, 4>(a, smem, grid, s); break;
    default: launch_one<TYPE, 8>(a, smem, grid, s); break;
    }
}

int sm_count() {
    static int n = 0;
    if (!n) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        if (n <= 0) n = 148;
    }
    return n;
}

// Resident CTAs per SM of one instantiation at the shared-memory budget (register use differs
// by format and token count), at most CTAS_PER_SM; cached per (type, nt).
template <int TYPE, int NT>
int occupancy_one() {
    static const int cap = [] {  // SARDYNE_QMV_CTAS_PER_SM: a lower cap, for tuning
        const char *e = getenv("SARDYNE_QMV_CTAS_PER_SM");
        return e && atoi(e) > 0 ? std::min(atoi(e), CTAS_PER_SM) : CTAS_PER_SM;
    }();
    configure_one<TYPE, NT>();
    int n = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, qmv_kernel<TYPE, NT>, THREADS, SMEM_BUDGET) != cudaSuccess) {
        cudaGetLastError();  // not sticky: fall back to one CTA per SM
        n = 1;
    }
    return std::max(1, std::min(n, cap));
}
template <int TYPE>
int occupancy_nt(int nt) {
    switch (nt) {
    case 1: return occupancy_one<TYPE, 1>();
    case 2: return occupancy_one<TYPE, 2>();
    case 3: return occupancy_one<TYPE, 3>();
    case 4: return occupancy_one<TYPE, 4>();
    default: return occupancy_one<TYPE, 8>();
    }
}
int ctas_per_sm(int type, int nt) {
    static std::atomic<int> cache[5][9];  // 0 = not yet queried
    const int ti = type == T_Q4_K ? 0 : type == T_Q6_K ? 1 : type == T_Q8_0 ? 2 : type == T_Q4_0 ? 3 : 4;
    const int ni = nt >= 8 ? 8 : nt;
    int v = cache[ti][ni].load();
    if (v) return v;
    switch (type) {
    case T_Q4_K: v = occupancy_nt<T_Q4_K>(nt); break;
    case T_Q6_K: v = occupancy_nt<T_Q6_K>(nt); break;
    case T_Q8_0: v = occupancy_nt<T_Q8_0>(nt); break;
    case T_Q4_0: v = occupancy_nt<T_Q4_0>(nt); break;
    default: v = occupancy_nt<T_Q5_0>(nt); break;
    }
    cache[ti][ni].store(v);
    return v;
}

void dispatch(int type, int nt, const Args &a, int smem, dim3 grid, cudaStream_t s) {
    switch (type) {
    case T_Q4_K: launch_nt<T_Q4_K>(nt, a, smem, grid, s); break;
    case T_Q6_K: launch_nt<T_Q6_K>(nt, a, smem, grid, s); break;
    case T_Q8_0: launch_nt<T_Q8_0>(nt, a, smem, grid, s); break;
    case T_Q4_0: launch_nt<T_Q4_0>(nt, a, smem, grid, s); break;
    case T_Q5_0: launch_nt<T_Q5_0>(nt, a, smem, grid, s); break;
    default: set_error("qmatvec: unsupported weight type %d", type); return;
    }
    SDY_LAUNCHED();
}

// Launch shape: at most CTAS_PER_SM CTAs per SM and at least THREADS pairs per CTA where the
// matrix has them, each CTA sweeping its contiguous share of groups in batches of G groups; G is
// the whole share when its block terms fit the shared-memory budget (one ordered combine per
// CTA), else as many as fit.

struct Plan {
    int grid = 0, G = 0, nt = 0, smem = 0;
};

bool plan_launch(int type, int nb, int qrow, int64_t ng, int64_t cta_cap, int nt_want, Plan *p) {
    // Enough groups per CTA that every thread has a pair: small matrices then take about one CTA
    // per SM, which leaves room on the SMs for the next kernel's CTAs to be placed early.
    const int units = (type == T_Q4_K || type == T_Q6_K) ? nb : (nb + 7) / 8;
    const int64_t gmin = std::max(1, THREADS / (GROUP_ROWS * units));
    p->grid = (int)std::max<int64_t>(1, std::min<int64_t>((ng + gmin - 1) / gmin, cta_cap));
    const int64_t per_cta = (ng + p->grid - 1) / p->grid;
    int nt = nt_want;
    for (;;) {
        int G = (int)std::min<int64_t>(per_cta, 1 << 20);
        while (G > 1 && smem_plan(type, nt, qrow, nb, G).total > SMEM_BUDGET) G = (G + 1) / 2;
        int total = smem_plan(type, nt, qrow, nb, G).total;
        if (total <= SMEM_LIMIT) {
            p->G = G;
            p->nt = nt;
            p->smem = total;
            return true;
        }
        if (nt == 1) return false;
        nt = nt >= 8 ? 4 : nt == 4 ? 3 : nt - 1;
    }
}

}  // namespace

// Token count from which a product goes to the tensor-core GEMM (SARDYNE_GEMM_MIN_TOKENS; 0 = never).
int gemm_min_tokens() {
    static const int v = [] {
        const char *e = getenv("SARDYNE_GEMM_MIN_TOKENS");
        return e ? atoi(e) : 32;
    }();
    return v;
}

void qmatvec(const QMat &w, const XQ &xq, float *out, int64_t ldo, int64_t row0, int64_t row1, int64_t out_row0,
             cudaStream_t s, const float *residual, const ActIn *act, bool split_ok) {
    if (row1 <= row0 || xq.n_tok <= 0) return;
    const int gmin = gemm_min_tokens();
    if (!act && gmin > 0 && xq.n_tok >= gmin && qgemm_supported(w.type, w.n_in) && xq.vtype == vec_dot_type(w.type) &&
        xq.n_in == w.n_in) {
        qgemm(w, xq, out, ldo, row0, row1, out_row0, s, residual, split_ok);
        return;
    }
    if (xq.vtype != vec_dot_type(w.type) || xq.n_in != w.n_in) {
        set_error("qmatvec: activation type/size does not match the weights");
        return;
    }
    const bool kq = (w.type == T_Q4_K || w.type == T_Q6_K);
    const int64_t g0 = row0 / GROUP_ROWS, g1 = (row1 + GROUP_ROWS - 1) / GROUP_ROWS;
    const int64_t ng = g1 - g0;
    for (int t0 = 0; t0 < xq.n_tok;) {
        int rem = xq.n_tok - t0;
        Plan plan;
        const int nt_want = rem >= 8 ? 8 : rem >= 4 ? 4 : rem;
        if (!plan_launch(w.type, w.nb, xq.qrow, ng, (int64_t)sm_count() * ctas_per_sm(w.type, nt_want), nt_want,
                         &plan)) {
            set_error("qmatvec: row of %d elements too long for one CTA", w.n_in);
            return;
        }
        const int nt = plan.nt;
        Args a{};
        a.slabs = w.slabs;
        a.nb = w.nb;
        a.g_begin = g0;
        a.n_groups = ng;
        a.G = plan.G;
        a.xqs = xq.qs + (size_t)t0 * xq.qrow;
        a.xd = xq.d + (size_t)t0 * xq.nbx;
        a.xsums = (const uint8_t *)xq.sums + (size_t)t0 * xq.nbx * (kq ? 32 : 4);
        a.qrow = xq.qrow;
        a.nbx = xq.nbx;
        a.out = out + (size_t)t0 * ldo;
        a.residual = residual ? residual + (size_t)t0 * ldo : nullptr;
        if (act) {
            a.act = *act;
            a.act.x += (size_t)t0 * act->ldx;
            if (act->u) a.act.u += (size_t)t0 * act->ldu;
        }
        a.ldo = ldo;
        a.row0 = row0;
        a.row1 = row1;
        a.out_row0 = out_row0;
        dispatch(w.type, nt, a, plan.smem, dim3(plan.grid), s);
        t0 += nt;
    }
}

}  // namespace sdy

namespace sdy {

void qmatvec_gather(const QMat &experts, int64_t gpe, int n_expert, const XQ &xq, int tok_div, const int32_t *slot_expert,
                    int n_slots, int64_t rows_per_expert, float *out, int64_t ldo_slot, cudaStream_t s, int expert0,
                    const ActIn *act) {
    if (n_slots <= 0) return;
    if (xq.vtype != vec_dot_type(experts.type) || xq.n_in != experts.n_in) {
        set_error("qmatvec_gather: activation type/size does not match the weights");
        return;
    }
    const int64_t cap =
        std::max<int64_t>(1, ((int64_t)sm_count() * ctas_per_sm(experts.type, 1) + n_slots - 1) / n_slots);
    Plan plan;
    if (!plan_launch(experts.type, experts.nb, xq.qrow, gpe, cap, 1, &plan)) {
        set_error("qmatvec_gather: row of %d elements too long for one CTA", experts.n_in);
        return;
    }
    Args a{};
    a.slabs = experts.slabs;
    a.nb = experts.nb;
    a.g_begin = 0;
    a.n_groups = gpe;
    a.G = plan.G;
    a.xqs = xq.qs;
    a.xd = xq.d;
    a.xsums = xq.sums;
    a.qrow = xq.qrow;
    a.nbx = xq.nbx;
    a.out = out;
    a.ldo = 0;
    a.row0 = 0;
    a.row1 = rows_per_expert;
    a.out_row0 = 0;
    a.slot_expert = slot_expert;
    a.gpe = gpe;
    a.ldo_slot = ldo_slot;
    a.tok_div = tok_div;
    a.n_expert = n_expert;
    a.expert0 = expert0;
    if (act) a.act = *act;
    dispatch(experts.type, 1, a, plan.smem, dim3(plan.grid, n_slots), s);
}

namespace {

template <int TA, int TB>
void launch_pair(const Args &a, const Args &b, int na, int grid, int smem, cudaStream_t s) {
    static std::atomic<uint64_t> configured{0};
    smem_limit_once(qmv2_kernel<TA, TB>, SMEM_LIMIT, configured);
    launch(qmv2_kernel<TA, TB>, dim3(grid), THREADS, smem, s, a, b, na);
    SDY_LAUNCHED();
}

Args pair_args(const QMat &w, const Plan &plan, const XQ &xq, float *out, const ActIn *act) {
    Args a{};
    a.slabs = w.slabs;
    a.nb = w.nb;
    a.g_begin = 0;
    a.n_groups = w.n_groups();
    a.G = plan.G;
    a.xqs = xq.qs;
    a.xd = xq.d;
    a.xsums = xq.sums;
    a.qrow = xq.qrow;
    a.nbx = xq.nbx;
    a.out = out;
    a.row0 = 0;
    a.row1 = w.n_rows;
    if (act) a.act = *act;
    return a;
}

}  // namespace

bool qmatvec2_supported(int ta, int tb) {
    return (ta == T_Q4_K && tb == T_Q6_K) || (ta == T_Q6_K && tb == T_Q4_K);
}

void qmatvec2(const QMat &wa, float *outa, const QMat &wb, float *outb, const XQ &xq, cudaStream_t s,
              const ActIn *act) {
    if (!qmatvec2_supported(wa.type, wb.type) || xq.n_tok != 1 || wa.n_in != wb.n_in ||
        xq.vtype != vec_dot_type(wa.type) || xq.vtype != vec_dot_type(wb.type) || xq.n_in != wa.n_in) {
        set_error("qmatvec2: unsupported pair of matrices");
        return;
    }
    // The SMs' CTA slots split in proportion to the bytes of each matrix.
    const int64_t cap = (int64_t)sm_count() * std::min(ctas_per_sm(wa.type, 1), ctas_per_sm(wb.type, 1));
    const double fa = (double)wa.bytes() / (double)(wa.bytes() + wb.bytes());
    const int64_t cap_a = std::max<int64_t>(1, std::min<int64_t>(cap - 1, (int64_t)(cap * fa + 0.5)));
    Plan pa, pb;
    if (!plan_launch(wa.type, wa.nb, xq.qrow, wa.n_groups(), cap_a, 1, &pa) ||
        !plan_launch(wb.type, wb.nb, xq.qrow, wb.n_groups(), std::max<int64_t>(1, cap - cap_a), 1, &pb)) {
        set_error("qmatvec2: row of %d elements too long for one CTA", wa.n_in);
        return;
    }
    const Args a = pair_args(wa, pa, xq, outa, act), b = pair_args(wb, pb, xq, outb, act);
    const int smem = std::max(pa.smem, pb.smem), grid = pa.grid + pb.grid;
    if (wa.type == T_Q4_K) launch_pair<T_Q4_K, T_Q6_K>(a, b, pa.grid, grid, smem, s);
    else launch_pair<T_Q6_K, T_Q4_K>(a, b, pa.grid, grid, smem, s);
}


bool qmatvec_batch_supported(int n, const QMat *const *w) {
    if (n < 1 || n > BATCH_MAX) return false;
    for (int i = 0; i < n; i++)
        if (!w[i] || (w[i]->type != T_Q4_K && w[i]->type != T_Q6_K)) return false;
    return true;
}

unsigned qmatvec_status() {
    unsigned v = 0;
    if (cudaMemcpyFromSymbol(&v, g_qmvb_status, sizeof v) != cudaSuccess) return ~0u;
    return v;
}

void qmatvec_clear_status() {
    const unsigned z = 0;
    SDY_CUDA(cudaMemcpyToSymbol(g_qmvb_status, &z, sizeof z));
}

void qmatvec_batch(int n, const QMat *const *w, const XQ *const *xq, float *const *out, cudaStream_t s,
                   const ActIn *acts, const PeerGatherTail *tail) {
    if (!qmatvec_batch_supported(n, w)) {
        set_error("qmatvec_batch: 1..%d matrices of Q4_K / Q6_K", BATCH_MAX);
        return;
    }
    for (int i = 0; i < n; i++)
        if (xq[i]->n_tok != 1 || xq[i]->vtype != T_Q8_K || xq[i]->n_in != w[i]->n_in) {
            set_error("qmatvec_batch: product %d: activations are not one Q8_K row of %d", i, w[i]->n_in);
            return;
        }
    // the SMs' CTA slots split in proportion to each matrix's bytes (at least one CTA each)
    const int64_t cap = (int64_t)sm_count() * std::min(ctas_per_sm(T_Q4_K, 1), ctas_per_sm(T_Q6_K, 1));
    double total = 0;
    for (int i = 0; i < n; i++) total += (double)w[i]->bytes();
    BatchArgs b{};
    b.n = n;
    int grid = 0, smem = 0;
    for (int i = 0; i < n; i++) {
        const int64_t ci = std::max<int64_t>(1, (int64_t)(cap * (double)w[i]->bytes() / total));
        Plan p;
        if (!plan_launch(w[i]->type, w[i]->nb, xq[i]->qrow, w[i]->n_groups(), ci, 1, &p)) {
            set_error("qmatvec_batch: row of %d elements too long for one CTA", w[i]->n_in);
            return;
        }
        b.a[i] = pair_args(*w[i], p, *xq[i], out[i], acts ? &acts[i] : nullptr);
        b.type[i] = w[i]->type;
        b.cta0[i] = grid;
        grid += p.grid;
        smem = std::max(smem, p.smem);
    }
    b.cta0[n] = grid;
    if (tail) {
        b.gather = 1;
        b.pg = *tail;
    }
    if (b.gather) {
        static std::atomic<uint64_t> configured{0};
        smem_limit_once(qmvb_kernel<T_Q4_K, T_Q6_K, true>, SMEM_LIMIT, configured);
        launch(qmvb_kernel<T_Q4_K, T_Q6_K, true>, dim3(grid), THREADS, smem, s, b);
    } else {
        static std::atomic<uint64_t> configured{0};
        smem_limit_once(qmvb_kernel<T_Q4_K, T_Q6_K, false>, SMEM_LIMIT, configured);
        launch(qmvb_kernel<T_Q4_K, T_Q6_K, false>, dim3(grid), THREADS, smem, s, b);
    }
    SDY_LAUNCHED();
}

}  // namespace sdy
