// Shared definitions for the B200 quantized-weight path: ggml type ids, block geometry, the
// device weight layout ("slabs"), the device activation layout ("XQ"), and error plumbing.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <stdio.h>

#include <atomic>
#include <string>
#include <utility>

namespace sdy {

// ggml type ids as stored in GGUF (reference csrc/ops.h:21-22).
enum : int { T_F32 = 0, T_F16 = 1, T_Q4_0 = 2, T_Q5_0 = 6, T_Q8_0 = 8, T_Q4_K = 12, T_Q6_K = 14,
             T_Q8_K = 15, T_BF16 = 30 };

__host__ __device__ constexpr int block_elems(int t) {
    return (t == T_Q4_K || t == T_Q6_K || t == T_Q8_K) ? 256
         : (t == T_Q8_0 || t == T_Q4_0 || t == T_Q5_0) ? 32 : 1;
}
__host__ __device__ constexpr int block_bytes(int t) {
    return t == T_Q8_0 ? 34 : t == T_Q4_0 ? 18 : t == T_Q5_0 ? 22 : t == T_Q4_K ? 144 : t == T_Q6_K ? 210
         : t == T_Q8_K ? 292 : t == T_F32 ? 4 : (t == T_F16 || t == T_BF16) ? 2 : 0;
}
inline bool is_quant_weight(int t) {
    return t == T_Q8_0 || t == T_Q4_0 || t == T_Q5_0 || t == T_Q4_K || t == T_Q6_K;
}
inline bool is_float_weight(int t) { return t == T_F32 || t == T_F16 || t == T_BF16; }
// Activation type paired with a weight type (reference csrc/ops.c:249-255).
inline int vec_dot_type(int t) {
    return (t == T_Q4_K || t == T_Q6_K) ? T_Q8_K : (t == T_Q8_0 || t == T_Q4_0 || t == T_Q5_0) ? T_Q8_0 : T_F32;
}
inline size_t row_bytes(int t, int64_t n) {
    int be = block_elems(t);
    return be ? (size_t)(n / be) * block_bytes(t) : 0;
}

// ------------------------------------------------------------------------------------------
// Device weight layout ("slabs").
//
// Rows are taken 8 at a time (a row group, padded with zero rows at the end). For row group g
// and block b the 8 rows' bytes of block b form one slab of 8 * block_bytes bytes, stored at
// (g * nb + b) * SLAB. Inside a slab every field of the block is a "plane": a 16-byte-wide
// field is cut into 16-byte chunks and chunk c of row r sits at plane + c*128 + r*16, so the 8
// lanes that read chunk c of 8 rows touch one contiguous 128-byte segment; narrow fields
// (2-byte d, 4-byte qh) sit at plane + r*width. Byte totals equal the raw GGUF bytes (no
// padding inside a slab), every plane starts 16-byte aligned, and the values are the raw
// bytes rearranged, so dequantization stays bit-exact.
//
//   Q4_K (1152 B): hdr [d, dmin, scales[12]] 16 B/row @0 | qs 8 chunks @128
//   Q6_K (1680 B): ql 8 chunks @0 | qh 4 chunks @1024 | scales 16 B/row @1536 | d 2 B/row @1664
//   Q8_0 ( 272 B): qs 2 chunks @0 | d @256
//   Q4_0 ( 144 B): qs 1 chunk  @0 | d @128
//   Q5_0 ( 176 B): qs 1 chunk  @0 | qh 4 B/row @128 | d @160
// ------------------------------------------------------------------------------------------
constexpr int GROUP_ROWS = 8;
__host__ __device__ constexpr int slab_bytes(int t) { return GROUP_ROWS * block_bytes(t); }

// Device activation layout ("XQ"), for T tokens of n_in elements quantized to Q8_0 or Q8_K:
//   qs    int8  [T][qrow], element e at (e/256)*272 + e%256 (16 zero bytes after every 256, so
//         lanes reading different 256-element spans from shared memory hit different banks)
//   d     f32   [T][nbx]   per-block scale (Q8_0: the f16-rounded scale, exactly as the dot uses it)
//   bsum  int16 [T][nbx][16] (Q8_K: sums of each 16 quants)  |  int32 [T][nbx] (Q8_0: block sums)
constexpr int XQ_SPAN = 272;
__host__ __device__ inline int xq_qrow(int n_in) { return ((n_in + 255) / 256) * XQ_SPAN; }
__host__ __device__ inline int xq_pos(int e) { return (e >> 8) * XQ_SPAN + (e & 255); }

struct XQ {
    int vtype = T_Q8_K;
    int n_in = 0, n_tok = 0, qrow = 0, nbx = 0;
    int8_t *qs = nullptr;
    float *d = nullptr;
    void *sums = nullptr;  // int16 [T][nbx][16] (Q8_K) or int32 [T][nbx] (Q8_0)
};
inline size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }
// Bytes needed for an XQ of n_tok rows, and carving it out of a buffer.
inline size_t xq_bytes(int vtype, int n_in, int n_tok) {
    int nbx = n_in / block_elems(vtype);
    size_t s = align_up((size_t)n_tok * xq_qrow(n_in), 256);
    s += align_up((size_t)n_tok * nbx * 4, 256);
    s += align_up((size_t)n_tok * nbx * (vtype == T_Q8_K ? 32 : 4), 256);
    return s;
}
inline XQ xq_carve(void *base, int vtype, int n_in, int n_tok) {
    XQ x;
    x.vtype = vtype; x.n_in = n_in; x.n_tok = n_tok; x.qrow = xq_qrow(n_in); x.nbx = n_in / block_elems(vtype);
    uint8_t *p = (uint8_t *)base;
    x.qs = (int8_t *)p;
    p += align_up((size_t)n_tok * x.qrow, 256);
    x.d = (float *)p;
    p += align_up((size_t)n_tok * x.nbx * 4, 256);
    x.sums = p;
    return x;
}

// A quantized weight matrix resident on the device in the slab layout.
struct QMat {
    const uint8_t *slabs = nullptr;
    int type = 0;
    int n_in = 0;
    int nb = 0;            // blocks per row
    int64_t n_rows = 0;    // logical rows (the layout holds ceil(n_rows/8) groups)
    int64_t n_groups() const { return (n_rows + GROUP_ROWS - 1) / GROUP_ROWS; }
    size_t bytes() const { return (size_t)n_groups() * nb * slab_bytes(type); }
};

// The matrix behind a handle returned by sdy_qmat_upload (nullptr for a null handle).
const QMat *qmat_of(const void *handle);

// ------------------------------------------------------------------------------------------ errors
void set_error(const char *fmt, ...);
const char *last_error();
void clear_error();
bool cuda_check(cudaError_t e, const char *what, const char *file, int line);
#define SDY_CUDA(call) ::sdy::cuda_check((call), #call, __FILE__, __LINE__)
// After every kernel launch: count it and surface launch errors.
void note_launch();
// Raises `kernel`'s dynamic shared memory limit to `bytes` on the current device the first time
// it is called there: the attribute is per device, so `done` keeps one bit per device ordinal.
template <class Kernel>
inline void smem_limit_once(Kernel kernel, int bytes, std::atomic<uint64_t> &done) {
    int dev = 0;
    cudaGetDevice(&dev);
    const uint64_t bit = 1ull << (dev & 63);
    if (done.load() & bit) return;
    if (SDY_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes))) done.fetch_or(bit);
}

#define SDY_LAUNCHED()                                   \
    do {                                                 \
        ::sdy::note_launch();                            \
        SDY_CUDA(cudaGetLastError());                    \
    } while (0)

// ------------------------------------------------------------------------------ dependent launch
// Kernels are launched with programmatic dependent launch: a kernel's CTAs are set up while the
// previous kernel's last CTAs retire and block in pdl_wait() until it has completed and its writes
// are visible, which takes launch latency off the critical path. Only kernels of few CTAs signal
// their dependents early (pdl_release, griddepcontrol.launch_dependents): after a kernel that
// fills the SMs the next kernel's CTAs would be placed while it still occupies them, packed onto
// the few with room (measured slower than launching without PDL), while after a small kernel they
// find most SMs free and load their weights during it (+3-5% per decode step). Every kernel reads
// or writes no activation before pdl_wait(); only weights may be read before it (the matvec loads
// its first weight pair there). Kernels that write weights (repacking, format conversion) neither
// signal early nor run inside a step. Launched without the attribute (SARDYNE_NO_PDL set),
// pdl_wait() and pdl_release() are no-ops.
#ifdef __CUDACC__
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;\n" ::: "memory"); }
// The early signal, for kernels of few CTAs only: called after pdl_wait(), it lets the next
// kernel's CTAs start and load their weights while this kernel runs.
__device__ __forceinline__ void pdl_release() {
#ifndef SDY_NO_EARLY_RELEASE
    asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory");
#endif
}

// acc + term(0) + term(1) + ... + term(n-1), added left to right with every sum rounded (the
// reference's sequential loops). Software-pipelined: the terms of batch k+1 (their loads) are
// requested before batch k's dependent adds run.
template <int B, class Term>
__device__ __forceinline__ float ordered_sum(float acc, int n, Term term) {
    const int full = n / B;
    if (full > 0) {
        float cur[B];
#pragma unroll
        for (int u = 0; u < B; u++) cur[u] = term(u);
        for (int k = 1; k < full; k++) {
            float nxt[B];
#pragma unroll
            for (int u = 0; u < B; u++) nxt[u] = term(k * B + u);
#pragma unroll
            for (int u = 0; u < B; u++) acc = __fadd_rn(acc, cur[u]);
#pragma unroll
            for (int u = 0; u < B; u++) cur[u] = nxt[u];
        }
#pragma unroll
        for (int u = 0; u < B; u++) acc = __fadd_rn(acc, cur[u]);
    }
    for (int j = full * B; j < n; j++) acc = __fadd_rn(acc, term(j));
    return acc;
}
#endif
bool pdl_enabled();
template <typename... KArgs, typename... Args>
void launch(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s, Args &&...args) {
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cfg.attrs = attr;
    cfg.numAttrs = pdl_enabled() ? 1 : 0;
    SDY_CUDA(cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...));
}

// ------------------------------------------------------------------------------------------ kernels
// Launchers (sardyne_b200/csrc/*.cu). All are asynchronous on `s` and record errors with set_error.
void repack_to_slabs(const uint8_t *raw, int type, int64_t n_rows, int n_in, uint8_t *slabs, cudaStream_t s);
void dequant_rows(const QMat &w, const int32_t *row_ids, int n_ids, int64_t first_row, float *out, int64_t ldo,
                  cudaStream_t s);
void quantize_rows(int vtype, const float *x, int64_t ldx, int n_tok, int n_in, const XQ &xq, cudaStream_t s);
void xq_import(int vtype, const uint8_t *raw, int n_tok, int n_in, const XQ &xq, cudaStream_t s);
void xq_export(const XQ &xq, uint8_t *raw, cudaStream_t s);
// out[t*ldo + (r - out_row0)] = W[r] . x[t] for rows r in [row0, row1) and tokens t < xq.n_tok.
// With `residual`, out = residual + product (same indexing; residual may alias out).
// The input rows a product kernel prepares and quantizes itself, instead of reading quantized
// activations, so that the decode step's elementwise producers fuse into their consumers:
//   w set:  RMSNorm(x[t]) * w, epsilon eps (ops.c:346-351);
//   u set:  silu(x[t]) * u[t], the SwiGLU gate (ops.c:366-371);
//   else:   x[t] as is.
struct ActIn {
    const float *x = nullptr;
    int64_t ldx = 0;
    const float *w = nullptr;
    float eps = 0.0f;
    const float *u = nullptr;
    int64_t ldu = 0;
};

// Token count from which products go to the tensor-core GEMM (0 = never).
int gemm_min_tokens();
// Many-token product on the tensor cores (qgemm.cu), same contract as qmatvec. With split_ok, a
// product whose tiles leave SMs idle is split along K: the CTAs store their blocks' terms in a
// scratch buffer taken from a stream-ordered pool (outside stream capture), and a second kernel
// adds every output's terms in block order.
bool qgemm_supported(int type, int n_in);
void qgemm(const QMat &w, const XQ &xq, float *out, int64_t ldo, int64_t row0, int64_t row1, int64_t out_row0,
           cudaStream_t s, const float *residual = nullptr, bool split_ok = true);
unsigned qgemm_status();  // nonzero when a qgemm completion wait timed out
void qgemm_clear_status();
// Grouped experts on the tensor cores (MoE prefill): for local expert e, the slots
// grp_slot[grp_off[e] .. grp_off[e+1]) (device arrays from moe_group with tile GEMM_TILE_TOKENS;
// at most max_slots in all) multiply expert e with activation row slot / xdiv into
// out + slot * ldo_slot; rows_per_expert rows each.
constexpr int GEMM_TILE_TOKENS = 128;
void qgemm_grouped(const QMat &experts, int64_t gpe, int n_expert, const XQ &xq, int xdiv, const int32_t *grp_off,
                   const int32_t *grp_slot, const int32_t *grp_tiles, int max_slots, int64_t rows_per_expert,
                   float *out, int64_t ldo_slot, cudaStream_t s);
// act: the input rows are prepared and quantized inside the kernel (xq then only gives the
// activation geometry). split_ok: the tensor-core route may take scratch memory (qgemm).
void qmatvec(const QMat &w, const XQ &xq, float *out, int64_t ldo, int64_t row0, int64_t row1, int64_t out_row0,
             cudaStream_t s, const float *residual = nullptr, const ActIn *act = nullptr, bool split_ok = true);
// Two matrices with one single-token input in one launch: outa[r] = A[r] . x, outb[r] = B[r] . x
// over all rows (the parts of a projection whose weight types differ).
bool qmatvec2_supported(int ta, int tb);
void qmatvec2(const QMat &wa, float *outa, const QMat &wb, float *outb, const XQ &xq, cudaStream_t s,
              const ActIn *act = nullptr);
// Independent single-token products in one launch: out[i][r] = W_i[r] . x_i for every row of
// each of the n (<= 8) Q4_K / Q6_K matrices, x_i the Q8_K row xq[i].
bool qmatvec_batch_supported(int n, const QMat *const *w);
// acts set: product i's input row is act[i] (f32, prepared as ActIn says) and every CTA quantizes
// it itself; xq[i] then gives the activation geometry only.
// tail set (processes that drive one GPU each): every output value is also stored at byte offset
// delta[q] from its local address, in the peers' buffers (an all-gather over NVLink fused into the
// launch); the last CTA then, after one system fence, stores the next round into flags[q][rank] of every rank and
// waits (acquire, at most one second) until its own flags show it from every rank. The buffer
// layout and round protocol are those of sdy_allgather_p2p (p2p.cu).
struct PeerGatherTail {
    int64_t delta[8] = {};
    int n_peer = 0;
    unsigned *flags[8] = {};
    unsigned *done = nullptr, *round = nullptr;
    int rank = 0, world = 1;
};
void qmatvec_batch(int n, const QMat *const *w, const XQ *const *xq, float *const *out, cudaStream_t s,
                   const ActIn *acts = nullptr, const PeerGatherTail *tail = nullptr);
unsigned qmatvec_status();  // nonzero when a fused gather's wait gave up
void qmatvec_clear_status();
// MoE: for each slot s < n_slots, out[s*ldo_slot + r] = E[slot_expert[s]][r] . x[s / tok_div] for
// r < rows_per_expert. `experts` holds n_expert matrices (global experts expert0 .. expert0 +
// n_expert - 1), each padded to gpe groups; slots naming other experts are left untouched. The
// expert ids are read on the device, so no host round trip sits between the router and the experts.
void qmatvec_gather(const QMat &experts, int64_t gpe, int n_expert, const XQ &xq, int tok_div, const int32_t *slot_expert,
                    int n_slots, int64_t rows_per_expert, float *out, int64_t ldo_slot, cudaStream_t s,
                    int expert0 = 0, const ActIn *act = nullptr);

// Exchange of the sharded engine over NVLink peer memory (p2p.cu). Every rank owns one buffer of
// peer_exchange_bytes(cap) bytes, zeroed before it is shared, and maps every peer's (CUDA IPC).
// peer_gather assembles in `recv` the rows x ld floats of which each rank computed a disjoint part
// in its own `send`: columns [lo, hi) of every row, and with `top` set only the rows j with
// e0 <= top[j] < e1 (MoE slots of this rank's experts; the parts of all ranks must cover every
// element). Each rank stores its part into every rank's staging area; the last CTA then, after
// one system fence, stores the round number into every rank's flag for this rank, and every CTA waits (at
// most px.wait_ns, acquire loads) for all ranks' flags before copying the staging area to
// `recv`. Two staging halves alternate by round, so a rank can run one exchange ahead of another.
// All ranks make the same sequence of calls (eager or replayed from a graph; the round counter
// lives on the device). A wait that runs out sets the status word (peer_status) and returns.
constexpr int PX_MAX_WORLD = 8;
struct PeerExchange {
    void *base[PX_MAX_WORLD] = {};  // every rank's buffer as mapped in this process
    int rank = 0, world = 1;
    int64_t cap = 0;  // floats per staging half, a multiple of 64
    unsigned long long wait_ns = 1000000000ull;  // a wait for the other ranks gives up after this
};
size_t peer_exchange_bytes(int64_t cap);
unsigned *peer_status(const PeerExchange &px);  // this rank's status word (device)
void peer_gather(const PeerExchange &px, const float *send, float *recv, int rows, int64_t ld, int64_t lo,
                 int64_t hi, const int32_t *top, int e0, int e1, cudaStream_t s);

}  // namespace sdy
