// All-gather over NVLink peer memory between processes that drive one GPU each (a B200 extension;
// the reference runs on one host). Rank r's `count` floats land at offset r * count of every rank's
// receive buffer, written directly into the peers' memory by the GPU (stores over NVLink /
// NVSwitch), so the exchange costs one kernel and a flag round trip instead of a library
// collective. It closes the row-sharded products (each GPU computes its rows of y, and every GPU
// needs all of y).
//
// Buffers. Each rank allocates one buffer with sdy_p2p_alloc(sdy_allgather_p2p_bytes(count, world))
// and shares it through a CUDA IPC handle (sdy_p2p_handle / sdy_p2p_open); layout: world * count
// floats, then at offset F = align256(world * count * 4) the flag words flags[0..world) (flag q:
// the last round rank q delivered), the CTA counter (F + 128) and the round counter (F + 132).
// sdy_p2p_alloc zeroes the buffer; every rank must make the same sequence of sdy_allgather_p2p
// calls (eagerly or replayed from a CUDA graph).
//
// Ordering. Each CTA's peer stores are fenced system-wide (thread 0, after a barrier) before the
// CTA counts itself done; the last CTA then advances the round counter and, after one more system
// fence, stores it into flag `rank` of every peer, and waits (acquire loads, at most one second)
// until every peer's flag in its own buffer shows the round. When
// the kernel ends, the local buffer holds every rank's slice of this round. A wait that runs out
// sets the status word (sdy_p2p_status) and returns.
#include "common.cuh"
#include "sardyne_b200.h"

#include <string.h>

#include <algorithm>

namespace sdy {
namespace {

constexpr int P2P_MAX_WORLD = 8;
constexpr int P2P_THREADS = 512;
constexpr unsigned long long P2P_WAIT_NS = 1000000000ull;  // a wait gives up after one second

__device__ unsigned g_p2p_status;

struct Gather {
    const float *send;
    int64_t count;
    float *recv[P2P_MAX_WORLD];      // every rank's receive buffer, as mapped in this process
    unsigned *flags[P2P_MAX_WORLD];  // every rank's flag words
    unsigned *done, *round;          // this rank's CTA counter and round counter
    int rank, world;
};

size_t flags_offset(int64_t count, int world) { return align_up((size_t)world * count * 4, 256); }

// A flag store after one system fence (fence + relaxed store is a release): a st.release.sys per
// peer flag costs about a whole system fence each, measured ~3 us apiece over NVLink.
__device__ __forceinline__ void st_relaxed_sys(unsigned *p, unsigned v) {
    asm volatile("st.relaxed.sys.global.u32 [%0], %1;\n" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned *p) {
    unsigned v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];\n" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__global__ void __launch_bounds__(P2P_THREADS) allgather_kernel(Gather g) {
    pdl_wait();
    __shared__ int last;
    const int64_t tid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x, nth = (int64_t)gridDim.x * blockDim.x;
    const bool vec = ((uintptr_t)g.send & 15) == 0 && (g.count & 3) == 0;
    for (int q = 0; q < g.world; q++) {
        float *dst = g.recv[q] + (size_t)g.rank * g.count;
        if (vec) {
            const float4 *s4 = (const float4 *)g.send;
            float4 *d4 = (float4 *)dst;
            for (int64_t i = tid; i < g.count / 4; i += nth) d4[i] = s4[i];
        } else {
            for (int64_t i = tid; i < g.count; i += nth) dst[i] = g.send[i];
        }
    }
    // the CTA's stores ordered before its arrival: one system fence by thread 0 after the barrier
    // (the barrier makes them observed by thread 0, whose fence is cumulative)
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence_system();
        last = atomicAdd(g.done, 1u) == gridDim.x - 1;
    }
    __syncthreads();
    if (!last || threadIdx.x != 0) return;
    *g.done = 0;
    const unsigned r = *g.round + 1;
    *g.round = r;
    __threadfence_system();  // every CTA's stores (each fenced before arriving) before the flags
    for (int q = 0; q < g.world; q++) st_relaxed_sys(g.flags[q] + g.rank, r);
    const unsigned *mine = g.flags[g.rank];
    unsigned long long t0;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t0));
    for (int q = 0; q < g.world; q++) {
        for (long long it = 0; (int)(ld_acquire_sys(mine + q) - r) < 0; it++) {
            if (it > 256) {
                unsigned long long t;
                asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
                if (t - t0 > P2P_WAIT_NS) {
                    atomicOr(&g_p2p_status, 1u);
                    return;
                }
                __nanosleep(128);
            }
        }
    }
}

// ---------------------------------------------------------------- the sharded engine's exchange
// Buffer: staging halves [2][cap] floats, then at X = align256(2 * cap * 4) the flag words
// flags[0..8) (flag q: the last round rank q delivered here), the CTA counter (X + 64), the round
// counter (X + 68) and the status word (X + 72).
constexpr int PX_THREADS = 512;
constexpr int PX_MAX_CTAS = 74;

size_t px_flags_offset(int64_t cap) { return align_up((size_t)cap * 8, 256); }

struct PxArgs {
    const float *send;
    float *recv;
    int64_t ld, lo, hi;
    int rows;
    const int32_t *top;
    int e0, e1;
    float *stage[PX_MAX_WORLD];
    unsigned *flags[PX_MAX_WORLD];
    unsigned *done, *round, *status;
    int64_t cap;
    unsigned long long wait_ns;
    int rank, world;
};

__device__ __forceinline__ bool px_owned(const PxArgs &a, int64_t row) {
    if (!a.top) return true;
    const int e = a.top[row];
    return e >= a.e0 && e < a.e1;
}

__global__ void __launch_bounds__(PX_THREADS) peer_gather_kernel(PxArgs a) {
    pdl_wait();
    pdl_release();  // the consumer's CTAs start and load their weights while the ranks meet here
    __shared__ int last;
    const unsigned r = *(volatile unsigned *)a.round + 1;
    const int64_t half = (int64_t)(r & 1) * a.cap;
    const int64_t tid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x, nth = (int64_t)gridDim.x * blockDim.x;
    const int64_t w = a.hi - a.lo, count = (int64_t)a.rows * a.ld;
    const bool vec = ((a.ld | a.lo | w | a.cap) & 3) == 0 && ((uintptr_t)a.send & 15) == 0 &&
                     ((uintptr_t)a.recv & 15) == 0;
    // this rank's part into every rank's staging half
    if (vec) {
        const int64_t w4 = w / 4;
        for (int64_t i = tid; i < a.rows * w4; i += nth) {
            const int64_t row = i / w4, off = row * a.ld + a.lo + (i - row * w4) * 4;
            if (!px_owned(a, row)) continue;
            const float4 v = *(const float4 *)(a.send + off);
            for (int q = 0; q < a.world; q++) *(float4 *)(a.stage[q] + half + off) = v;
        }
    } else {
        for (int64_t i = tid; i < a.rows * w; i += nth) {
            const int64_t row = i / w, off = row * a.ld + a.lo + (i - row * w);
            if (!px_owned(a, row)) continue;
            const float v = a.send[off];
            for (int q = 0; q < a.world; q++) a.stage[q][half + off] = v;
        }
    }
    // the CTA's stores, ordered before its arrival by one system-scope fence after the barrier
    // (the barrier makes them observed by thread 0, whose fence is cumulative)
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence_system();
        last = atomicAdd(a.done, 1u) == gridDim.x - 1;
    }
    __syncthreads();
    if (last && threadIdx.x == 0) {
        *a.done = 0;
        *a.round = r;
        __threadfence_system();  // every CTA's stores (each fenced before arriving) before the flags
        for (int q = 0; q < a.world; q++) st_relaxed_sys(a.flags[q] + a.rank, r);
    }
    // every rank's part of this round has arrived once all flags show it
    if (threadIdx.x < a.world) {
        const unsigned *f = a.flags[a.rank] + threadIdx.x;
        unsigned long long t0 = 0;
        for (long long it = 0; (int)(ld_acquire_sys(f) - r) < 0; it++) {
            if (it == 256) asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t0));
            if (it > 256) {
                unsigned long long t;
                asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
                if (t - t0 > a.wait_ns) {
                    atomicOr(a.status, 1u);
                    break;
                }
                __nanosleep(128);
            }
        }
    }
    __syncthreads();
    const float *src = a.stage[a.rank] + half;
    if (vec) {
        for (int64_t i = tid; i < count / 4; i += nth) ((float4 *)a.recv)[i] = __ldcg((const float4 *)src + i);
    } else {
        for (int64_t i = tid; i < count; i += nth) a.recv[i] = __ldcg(src + i);
    }
}

}  // namespace

size_t peer_exchange_bytes(int64_t cap) { return px_flags_offset(cap) + 256; }

unsigned *peer_status(const PeerExchange &px) {
    return (unsigned *)((uint8_t *)px.base[px.rank] + px_flags_offset(px.cap) + 72);
}

void peer_gather(const PeerExchange &px, const float *send, float *recv, int rows, int64_t ld, int64_t lo,
                 int64_t hi, const int32_t *top, int e0, int e1, cudaStream_t s) {
    if (rows < 1 || ld < 1 || lo < 0 || hi > ld || lo > hi || (int64_t)rows * ld > px.cap || px.world < 1 ||
        px.world > PX_MAX_WORLD) {
        set_error("peer_gather: bad arguments (rows %d, ld %lld, [%lld, %lld), cap %lld)", rows, (long long)ld,
                  (long long)lo, (long long)hi, (long long)px.cap);
        return;
    }
    PxArgs a{};
    a.send = send;
    a.recv = recv;
    a.ld = ld;
    a.lo = lo;
    a.hi = hi;
    a.rows = rows;
    a.top = top;
    a.e0 = e0;
    a.e1 = e1;
    const size_t X = px_flags_offset(px.cap);
    for (int q = 0; q < px.world; q++) {
        a.stage[q] = (float *)px.base[q];
        a.flags[q] = (unsigned *)((uint8_t *)px.base[q] + X);
    }
    uint8_t *own = (uint8_t *)px.base[px.rank];
    a.done = (unsigned *)(own + X + 64);
    a.round = (unsigned *)(own + X + 68);
    a.status = (unsigned *)(own + X + 72);
    a.cap = px.cap;
    a.wait_ns = px.wait_ns;
    a.rank = px.rank;
    a.world = px.world;
    const int64_t work = std::max<int64_t>((int64_t)rows * (hi - lo) * px.world, (int64_t)rows * ld) / 4;
    const int grid = (int)std::max<int64_t>(1, std::min<int64_t>(PX_MAX_CTAS, (work + PX_THREADS - 1) / PX_THREADS));
    launch(peer_gather_kernel, dim3(grid), dim3(PX_THREADS), 0, s, a);
    SDY_LAUNCHED();
}

}  // namespace sdy

using namespace sdy;

extern "C" {

size_t sdy_allgather_p2p_bytes(int64_t count, int32_t world) {
    if (count < 0 || world < 1 || world > P2P_MAX_WORLD) return 0;
    return flags_offset(count, world) + 256;
}

void *sdy_p2p_alloc(size_t bytes) {
    clear_error();
    void *p = nullptr;
    if (!SDY_CUDA(cudaMalloc(&p, bytes ? bytes : 256))) return nullptr;
    if (!SDY_CUDA(cudaMemset(p, 0, bytes ? bytes : 256)) || !SDY_CUDA(cudaDeviceSynchronize())) {
        cudaFree(p);
        return nullptr;
    }
    return p;
}

void sdy_p2p_free(void *p) {
    if (p) cudaFree(p);
}

int sdy_p2p_handle(const void *d_ptr, void *handle_out) {
    clear_error();
    cudaIpcMemHandle_t h;
    if (!d_ptr || !handle_out || !SDY_CUDA(cudaIpcGetMemHandle(&h, (void *)d_ptr))) return -1;
    memcpy(handle_out, &h, sizeof h);
    return 0;
}

void *sdy_p2p_open(const void *handle) {
    clear_error();
    if (!handle) {
        set_error("sdy_p2p_open: null handle");
        return nullptr;
    }
    cudaIpcMemHandle_t h;
    memcpy(&h, handle, sizeof h);
    void *p = nullptr;
    if (!SDY_CUDA(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess))) return nullptr;
    return p;
}

int sdy_p2p_close(void *d_peer) {
    clear_error();
    return d_peer && SDY_CUDA(cudaIpcCloseMemHandle(d_peer)) ? 0 : -1;
}

int sdy_allgather_p2p(const float *d_send, int64_t count, void *const *bases, int32_t rank, int32_t world,
                      void *stream) {
    clear_error();
    if (!d_send || count <= 0 || !bases || world < 1 || world > P2P_MAX_WORLD || rank < 0 || rank >= world) {
        set_error("sdy_allgather_p2p: bad arguments (1 <= world <= %d)", P2P_MAX_WORLD);
        return -1;
    }
    Gather g{};
    g.send = d_send;
    g.count = count;
    g.rank = rank;
    g.world = world;
    const size_t F = flags_offset(count, world);
    for (int q = 0; q < world; q++) {
        if (!bases[q]) {
            set_error("sdy_allgather_p2p: buffer of rank %d missing", q);
            return -1;
        }
        g.recv[q] = (float *)bases[q];
        g.flags[q] = (unsigned *)((uint8_t *)bases[q] + F);
    }
    g.done = (unsigned *)((uint8_t *)bases[rank] + F + 128);
    g.round = (unsigned *)((uint8_t *)bases[rank] + F + 132);
    const int64_t work = (count + 3) / 4 * world;
    const int grid = (int)std::max<int64_t>(1, std::min<int64_t>(128, (work + P2P_THREADS - 1) / P2P_THREADS));
    launch(allgather_kernel, dim3(grid), dim3(P2P_THREADS), 0, (cudaStream_t)stream, g);
    SDY_LAUNCHED();
    return last_error()[0] ? -1 : 0;
}

int sdy_p2p_read(void *host_dst, const void *d_src, size_t bytes) {
    clear_error();
    return host_dst && d_src && SDY_CUDA(cudaMemcpy(host_dst, d_src, bytes, cudaMemcpyDeviceToHost)) ? 0 : -1;
}

uint32_t sdy_p2p_status(void) {
    unsigned v = 0;
    if (cudaMemcpyFromSymbol(&v, g_p2p_status, sizeof v) != cudaSuccess) return ~0u;
    return v;
}

void sdy_p2p_clear_status(void) {
    const unsigned z = 0;
    cudaMemcpyToSymbol(g_p2p_status, &z, sizeof z);
}

}  // extern "C"
