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
// Ordering. Every thread fences its peer stores system-wide before its CTA counts itself done; the
// last CTA then advances the round counter, release-stores it into flag `rank` of every peer and
// waits (acquire loads, at most one second) until every peer's flag in its own buffer shows the
// round. When
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

__device__ __forceinline__ void st_release_sys(unsigned *p, unsigned v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;\n" ::"l"(p), "r"(v) : "memory");
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
    __threadfence_system();
    __syncthreads();
    if (threadIdx.x == 0) last = atomicAdd(g.done, 1u) == gridDim.x - 1;
    __syncthreads();
    if (!last || threadIdx.x != 0) return;
    *g.done = 0;
    const unsigned r = *g.round + 1;
    *g.round = r;
    __threadfence_system();
    for (int q = 0; q < g.world; q++) st_release_sys(g.flags[q] + g.rank, r);
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

}  // namespace
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
