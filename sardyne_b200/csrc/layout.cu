// Layout kernels: raw GGUF blocks -> device slabs, slab dequantization (bit-exact), and the
// activation (XQ) quantizers/importers. Formulas follow the reference's scalar kernels
// (reference csrc/quant.c:13-144); every fp32 step uses an explicit round-to-nearest intrinsic
// so nothing is contracted into an FMA (the reference builds with -ffp-contract=off).
#include "common.cuh"
#include "quant_device.cuh"

namespace sdy {

// Offset inside a slab of byte k of row r's raw block (the inverse of the slab layout).
__device__ __forceinline__ int slab_off(int type, int r, int k) {
    switch (type) {
    case T_Q4_K:  // [d dmin scales] 16 B, then qs[128]
        return k < 16 ? r * 16 + k : 128 + ((k - 16) >> 4) * 128 + r * 16 + ((k - 16) & 15);
    case T_Q6_K:  // ql[128] qh[64] scales[16] d[2]
        if (k < 128) return (k >> 4) * 128 + r * 16 + (k & 15);
        if (k < 192) return 1024 + ((k - 128) >> 4) * 128 + r * 16 + ((k - 128) & 15);
        if (k < 208) return 1536 + r * 16 + (k - 192);
        return 1664 + r * 2 + (k - 208);
    case T_Q8_0:  // d[2] qs[32]
        return k < 2 ? 256 + r * 2 + k : ((k - 2) >> 4) * 128 + r * 16 + ((k - 2) & 15);
    case T_Q4_0:  // d[2] qs[16]
        return k < 2 ? 128 + r * 2 + k : r * 16 + (k - 2);
    case T_Q5_0:  // d[2] qh[4] qs[16]
        return k < 2 ? 160 + r * 2 + k : k < 6 ? 128 + r * 4 + (k - 2) : r * 16 + (k - 6);
    default: return 0;
    }
}

__global__ void repack_kernel(const uint8_t *__restrict__ raw, int type, int64_t n_rows, int nb,
                              uint8_t *__restrict__ slabs) {
    pdl_wait();
    const int bb = block_bytes(type), sb = slab_bytes(type);
    int64_t n_groups = (n_rows + GROUP_ROWS - 1) / GROUP_ROWS;
    int64_t total = n_groups * GROUP_ROWS * nb;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        int64_t row = i / nb;
        int b = (int)(i - row * nb);
        int64_t g = row / GROUP_ROWS;
        int r = (int)(row % GROUP_ROWS);
        uint8_t *slab = slabs + ((size_t)g * nb + b) * sb;
        const uint8_t *src = raw + ((size_t)row * nb + b) * bb;
        bool live = row < n_rows;
        for (int k = 0; k < bb; k++) slab[slab_off(type, r, k)] = live ? src[k] : 0;
    }
}

void repack_to_slabs(const uint8_t *raw, int type, int64_t n_rows, int n_in, uint8_t *slabs, cudaStream_t s) {
    int nb = n_in / block_elems(type);
    int64_t total = ((n_rows + 7) / 8) * 8 * nb;
    int blocks = (int)std::min<int64_t>((total + 255) / 256, 148 * 32);
    launch(repack_kernel, blocks, 256, 0, s, raw, type, n_rows, nb, slabs);
    SDY_LAUNCHED();
}

// ------------------------------------------------------------------------------ dequantization

__device__ __forceinline__ float h2f(uint16_t h) { return __half2float(__ushort_as_half(h)); }

// Element e of logical row `row` of w, as the reference's dequant would write it.
__device__ float dequant_elem(const QMat &w, int64_t row, int e) {
    const int type = w.type, QB = block_elems(type);
    const int b = e / QB, j = e % QB, r = (int)(row % GROUP_ROWS);
    const uint8_t *slab = w.slabs + ((size_t)(row / GROUP_ROWS) * w.nb + b) * slab_bytes(type);
    auto byte = [&](int k) -> int { return slab[slab_off(type, r, k)]; };
    auto half_at = [&](int k) -> float { return h2f((uint16_t)(byte(k) | (byte(k + 1) << 8))); };
    switch (type) {
    case T_Q8_0: return __fmul_rn((float)(int8_t)byte(2 + j), half_at(0));
    case T_Q4_0: {
        int v = (j < 16 ? (byte(2 + j) & 15) : (byte(2 + j - 16) >> 4)) - 8;
        return __fmul_rn((float)v, half_at(0));
    }
    case T_Q5_0: {
        uint32_t qh = byte(2) | (byte(3) << 8) | (byte(4) << 16) | ((uint32_t)byte(5) << 24);
        int nib = j < 16 ? (byte(6 + j) & 15) : (byte(6 + j - 16) >> 4);
        int v = (nib | (int)(((qh >> j) & 1) << 4)) - 16;
        return __fmul_rn((float)v, half_at(0));
    }
    case T_Q4_K: {  // y = (d*sc)*q - dmin*m   (quant.c:41-48)
        int sub = j >> 5, sc, mn;
        if (sub < 4) { sc = byte(4 + sub) & 63; mn = byte(8 + sub) & 63; }
        else {
            sc = (byte(8 + sub) & 15) | ((byte(sub) >> 6) << 4);
            mn = (byte(8 + sub) >> 4) | ((byte(4 + sub) >> 6) << 4);
        }
        int qb = byte(16 + 32 * (sub >> 1) + (j & 31));
        int q = (sub & 1) ? (qb >> 4) : (qb & 15);
        float d1 = __fmul_rn(half_at(0), (float)sc), m1 = __fmul_rn(half_at(2), (float)mn);
        return __fsub_rn(__fmul_rn(d1, (float)q), m1);
    }
    case T_Q6_K: {  // (d*sc)*(q-32)   (quant.c:62-81)
        int half = j >> 7, w7 = j & 127, quarter = w7 >> 5, l = w7 & 31;
        int lo = byte(64 * half + l + ((quarter & 1) ? 32 : 0));
        lo = (quarter >> 1) ? (lo >> 4) : (lo & 15);
        int q = lo | (((byte(128 + 32 * half + l) >> (2 * quarter)) & 3) << 4);
        float dsc = __fmul_rn(half_at(208), (float)(int8_t)byte(192 + j / 16));
        return __fmul_rn(dsc, (float)(q - 32));
    }
    }
    return 0.0f;
}

__global__ void dequant_kernel(QMat w, const int32_t *__restrict__ ids, int64_t first_row, float *__restrict__ out,
                               int64_t ldo) {
    pdl_wait();
    int64_t row = ids ? (int64_t)ids[blockIdx.x] : first_row + blockIdx.x;
    float *o = out + (int64_t)blockIdx.x * ldo;
    for (int e = threadIdx.x; e < w.n_in; e += blockDim.x) o[e] = dequant_elem(w, row, e);
}

void dequant_rows(const QMat &w, const int32_t *row_ids, int n_ids, int64_t first_row, float *out, int64_t ldo,
                  cudaStream_t s) {
    if (n_ids <= 0) return;
    launch(dequant_kernel, n_ids, 256, 0, s, w, row_ids, first_row, out, ldo);
    SDY_LAUNCHED();
}

// ------------------------------------------------------------------------------ activation quantization

__global__ void quantize_kernel(int vtype, const float *__restrict__ x, int64_t ldx, int n_in, XQ xq) {
    pdl_wait();
    pdl_release();
    const int t = blockIdx.y;
    const int span = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (span * 256 >= n_in) return;
    const float *xt = x + (size_t)t * ldx;
    if (vtype == T_Q8_K) quant_q8k_block(xt, t, span, xq);
    else quant_q80_span(xt, t, span, n_in, xq);
}

void quantize_rows(int vtype, const float *x, int64_t ldx, int n_tok, int n_in, const XQ &xq, cudaStream_t s) {
    if (n_tok <= 0) return;
    int spans = (n_in + 255) / 256;
    dim3 grid((spans + 7) / 8, n_tok);
    launch(quantize_kernel, grid, 256, 0, s, vtype, x, ldx, n_in, xq);
    SDY_LAUNCHED();
}

// Reference-format activation bytes (Q8_K 292 B / Q8_0 34 B blocks) <-> XQ.
__global__ void xq_import_kernel(int vtype, const uint8_t *__restrict__ raw, int n_tok, XQ xq) {
    pdl_wait();
    const int QB = block_elems(vtype), BB = block_bytes(vtype);
    int64_t total = (int64_t)n_tok * xq.nbx;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        int t = (int)(i / xq.nbx), b = (int)(i % xq.nbx);
        const uint8_t *src = raw + (size_t)i * BB;
        int8_t *qs = xq.qs + (size_t)t * xq.qrow;
        if (vtype == T_Q8_K) {
            float d;
            memcpy(&d, src, 4);
            xq.d[i] = d;
            for (int k = 0; k < 256; k++) qs[xq_pos(b * 256 + k)] = (int8_t)src[4 + k];
            int16_t *bs = (int16_t *)xq.sums + (size_t)i * 16;
            for (int g = 0; g < 16; g++) bs[g] = (int16_t)(src[260 + 2 * g] | (src[261 + 2 * g] << 8));
        } else {
            xq.d[i] = h2f((uint16_t)(src[0] | (src[1] << 8)));
            int sum = 0;
            for (int k = 0; k < QB; k++) {
                int8_t q = (int8_t)src[2 + k];
                qs[xq_pos(b * QB + k)] = q;
                sum += q;
            }
            ((int32_t *)xq.sums)[i] = sum;
        }
    }
}

__global__ void xq_export_kernel(XQ xq, uint8_t *__restrict__ raw) {
    pdl_wait();
    const int vtype = xq.vtype, QB = block_elems(vtype), BB = block_bytes(vtype);
    int64_t total = (int64_t)xq.n_tok * xq.nbx;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        int t = (int)(i / xq.nbx), b = (int)(i % xq.nbx);
        uint8_t *dst = raw + (size_t)i * BB;
        const int8_t *qs = xq.qs + (size_t)t * xq.qrow;
        if (vtype == T_Q8_K) {
            memcpy(dst, &xq.d[i], 4);
            for (int k = 0; k < 256; k++) dst[4 + k] = (uint8_t)qs[xq_pos(b * 256 + k)];
            const int16_t *bs = (const int16_t *)xq.sums + (size_t)i * 16;
            for (int g = 0; g < 16; g++) { dst[260 + 2 * g] = (uint8_t)bs[g]; dst[261 + 2 * g] = (uint8_t)((uint16_t)bs[g] >> 8); }
        } else {
            // 34-byte blocks keep dst 2-byte aligned: one 16-bit store of the f16 pattern.
            *(uint16_t *)dst = __half_as_ushort(__float2half_rn(xq.d[i]));
            for (int k = 0; k < QB; k++) dst[2 + k] = (uint8_t)qs[xq_pos(b * QB + k)];
        }
    }
}

void xq_import(int vtype, const uint8_t *raw, int n_tok, int n_in, const XQ &xq, cudaStream_t s) {
    (void)n_in;
    int64_t total = (int64_t)n_tok * xq.nbx;
    if (total <= 0) return;
    launch(xq_import_kernel, (int)std::min<int64_t>((total + 127) / 128, 4096), 128, 0, s, vtype, raw, n_tok, xq);
    SDY_LAUNCHED();
}

void xq_export(const XQ &xq, uint8_t *raw, cudaStream_t s) {
    int64_t total = (int64_t)xq.n_tok * xq.nbx;
    if (total <= 0) return;
    launch(xq_export_kernel, (int)std::min<int64_t>((total + 127) / 128, 4096), 128, 0, s, xq, raw);
    SDY_LAUNCHED();
}

}  // namespace sdy
