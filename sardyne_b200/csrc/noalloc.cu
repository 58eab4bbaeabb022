// An entry point for callers that cannot allocate device memory.
//
// sdy_qmatvec_f32_noalloc quantizes f32 activations and runs the quantized matvec, like
// sdy_quantize_rows_dev followed by sdy_qmatvec_dev, but it takes no scratch buffer from the
// caller and allocates none: the quantized activations live in g_noalloc_scratch, a fixed
// file-scope device array that every GPU loading this library holds until the process exits.
// It serves callers that must not call cudaMalloc/cudaFree or a framework allocator where they
// call it: a host framework that accounts for every byte of device memory through its own pool
// (a library allocation behind its back breaks that accounting), and serving loops that keep
// allocation out of their steady state (cudaFree waits for the whole device, and a fresh
// cudaMalloc can stall the step that makes it). The caller still provides the weights (an
// sdy_qmat_upload handle), the activations and the output, all in device memory.
//
// Rules of use (also stated in include/sardyne_b200.h):
//   * at most NOALLOC_SCRATCH_BYTES of quantized activations per call (sdy_xq_bytes; for
//     16384-element rows that is 26 tokens); larger requests fail with -1 and a message in
//     sdy_last_error, before anything is launched;
//   * the first call on a device looks up the array's device address (cudaGetSymbolAddress)
//     with that device current and keeps it for the process: do not reset the device
//     (cudaDeviceReset) afterwards, since the kept address would then be stale;
//   * every call on a device shares the one array, so calls whose GPU work overlaps in time
//     (different streams, no ordering between them) race on it and must not be issued;
//   * the array keeps whatever the last call left there. Nothing needs clearing: each call
//     writes every scratch byte its matvec reads before reading it.
#include "common.cuh"

#include <mutex>

namespace sdy {
namespace {

constexpr size_t NOALLOC_SCRATCH_BYTES = 512 * 1024;
constexpr int MAX_DEVICES = 64;

__device__ __align__(256) uint8_t g_noalloc_scratch[NOALLOC_SCRATCH_BYTES];

std::mutex g_mu;
void *g_addr[MAX_DEVICES] = {};

// Device address of g_noalloc_scratch on the current device. In host code the symbol is only a
// host-side stand-in; the kernels must be given the address the runtime reports.
void *scratch_address() {
    int dev = 0;
    if (!SDY_CUDA(cudaGetDevice(&dev))) return nullptr;
    if (dev < 0 || dev >= MAX_DEVICES) {
        set_error("sdy_qmatvec_f32_noalloc: device %d out of range", dev);
        return nullptr;
    }
    std::lock_guard<std::mutex> lk(g_mu);
    if (!g_addr[dev]) {
        void *p = nullptr;
        if (!SDY_CUDA(cudaGetSymbolAddress(&p, g_noalloc_scratch))) return nullptr;
        g_addr[dev] = p;
    }
    return g_addr[dev];
}

}  // namespace
}  // namespace sdy

using namespace sdy;

extern "C" int sdy_qmatvec_f32_noalloc(const void *w, const float *d_x, int n_tok, float *d_out, int64_t ldo,
                                       int64_t row0, int64_t row1, void *stream) {
    clear_error();
    const QMat *m = qmat_of(w);
    if (!m || !d_x || !d_out || n_tok <= 0 || row0 < 0 || row1 > m->n_rows || row1 < row0) {
        set_error("sdy_qmatvec_f32_noalloc: bad arguments");
        return -1;
    }
    const int vt = vec_dot_type(m->type);
    const size_t need = xq_bytes(vt, m->n_in, n_tok);
    if (need > NOALLOC_SCRATCH_BYTES) {
        set_error("sdy_qmatvec_f32_noalloc: %d tokens of %d elements need %zu bytes of scratch, more than the %zu "
                  "this entry point owns; use sdy_quantize_rows_dev + sdy_qmatvec_dev with a caller buffer",
                  n_tok, m->n_in, need, NOALLOC_SCRATCH_BYTES);
        return -1;
    }
    void *scratch = scratch_address();
    if (!scratch) return -1;
    XQ q = xq_carve(scratch, vt, m->n_in, n_tok);
    quantize_rows(vt, d_x, m->n_in, n_tok, m->n_in, q, (cudaStream_t)stream);
    qmatvec(*m, q, d_out, ldo, row0, row1, row0, (cudaStream_t)stream, nullptr, nullptr, /*split_ok=*/false);
    return last_error()[0] ? -1 : 0;
}
