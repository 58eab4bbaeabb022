// Warp-level activation quantizers shared by the standalone quantize kernel and the fused
// norm/activation kernels: byte-exact Q8_K and Q8_0 (reference csrc/quant.c:98-144).
//
// Every function is warp-collective: lane l holds elements span*256 + 8l .. +7 of token t.
#pragma once
#include "common.cuh"
#include "fp_device.cuh"

namespace sdy {

// The reference's integer conversions as its x86 host computes them, including the rows whose
// largest magnitude is so small (below ~3.7e-37) that the inverse scale overflows to infinity.
// nearest_int (quant.c:111-116): the integer left in the mantissa bits by adding 1.5 * 2^23,
// i.e. round half to even for |p| < 2^22; +-inf leave 0 mantissa bits (-2^22), and the NaN of
// inf * 0 is the x86 default NaN, whose mantissa bits give 0.
__device__ __forceinline__ int nearest_int_ref(float p) {
    if (isnan(p)) return 0;
    return (__float_as_int(__fadd_rn(p, 12582912.0f)) & 0x007FFFFF) - 0x00400000;
}
// (int8_t)roundf(p) (quant.c:106): the x86 conversion of a value outside the int range, or NaN,
// gives INT_MIN, whose low byte is 0.
__device__ __forceinline__ int8_t round_to_int8_ref(float p) {
    const float r = roundf(p);
    return r >= -2147483648.0f && r < 2147483648.0f ? (int8_t)(int)r : (int8_t)0;
}

// Q8_K (quant.c:118-144) of one 256-element block whose 8 values per lane are in v. The scale
// comes from the FIRST element of largest magnitude, with its sign.
__device__ __forceinline__ void quant_q8k_vals(const float v[8], int t, int blk, const XQ &xq) {
    const int lane = threadIdx.x & 31;
    float amax = 0.0f;
    int idx = 0x7FFFFFFF;
    for (int i = 0; i < 8; i++)
        if (fabsf(v[i]) > amax) { amax = fabsf(v[i]); idx = lane * 8 + i; }
    for (int o = 16; o; o >>= 1) {
        float a2 = __shfl_xor_sync(0xffffffffu, amax, o);
        int i2 = __shfl_xor_sync(0xffffffffu, idx, o);
        if (a2 > amax || (a2 == amax && i2 < idx)) { amax = a2; idx = i2; }
    }
    int8_t *qs = xq.qs + (size_t)t * xq.qrow + blk * XQ_SPAN + lane * 8;
    int16_t *bs = (int16_t *)xq.sums + ((size_t)t * xq.nbx + blk) * 16;
    float *dd = xq.d + (size_t)t * xq.nbx + blk;
    if (amax == 0.0f) {
        *(uint2 *)qs = make_uint2(0, 0);
        if ((lane & 1) == 0) bs[lane >> 1] = 0;
        if (lane == 0) *dd = 0.0f;
        return;
    }
    float mine = 0.0f;
    for (int i = 0; i < 8; i++)
        if (i == (idx & 7)) mine = v[i];
    const float vmax = __shfl_sync(0xffffffffu, mine, (idx >> 3) & 31);
    const float iscale = __fdiv_rn(-127.0f, vmax);
    int q[8], sum = 0;
    for (int i = 0; i < 8; i++) {
        const int r = nearest_int_ref(__fmul_rn(iscale, v[i]));
        q[i] = (int8_t)(r < 127 ? r : 127);  // the stored byte; the sums add the stored values
        sum += q[i];
    }
    uint32_t lo = (q[0] & 255) | ((q[1] & 255) << 8) | ((q[2] & 255) << 16) | ((uint32_t)(q[3] & 255) << 24);
    uint32_t hi = (q[4] & 255) | ((q[5] & 255) << 8) | ((q[6] & 255) << 16) | ((uint32_t)(q[7] & 255) << 24);
    *(uint2 *)qs = make_uint2(lo, hi);
    sum += __shfl_xor_sync(0xffffffffu, sum, 1);  // 16 elements = 2 lanes
    if ((lane & 1) == 0) bs[lane >> 1] = (int16_t)sum;
    if (lane == 0) *dd = __fdiv_rn(1.0f, iscale);
}

// Q8_0 (quant.c:98-108) of span `span`: 4 lanes per 32-element block. Lanes whose elements lie
// past the row (live = false; n_in is a multiple of 32, so a 4-lane group is all live or dead)
// take part in the shuffles and write nothing.
__device__ __forceinline__ void quant_q80_vals(const float v[8], bool live, int t, int span, const XQ &xq) {
    const int lane = threadIdx.x & 31;
    const int e0 = span * 256 + lane * 8;
    float amax = 0.0f;
    for (int i = 0; i < 8; i++) amax = fmaxf(amax, fabsf(live ? v[i] : 0.0f));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
    float d = __fdiv_rn(amax, 127.0f);
    float id = d != 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
    int q[8], sum = 0;
    for (int i = 0; i < 8; i++) { q[i] = live ? round_to_int8_ref(__fmul_rn(v[i], id)) : 0; sum += q[i]; }
    sum += __shfl_xor_sync(0xffffffffu, sum, 1);
    sum += __shfl_xor_sync(0xffffffffu, sum, 2);
    if (!live) return;
    uint32_t lo = (q[0] & 255) | ((q[1] & 255) << 8) | ((q[2] & 255) << 16) | ((uint32_t)(q[3] & 255) << 24);
    uint32_t hi = (q[4] & 255) | ((q[5] & 255) << 8) | ((q[6] & 255) << 16) | ((uint32_t)(q[7] & 255) << 24);
    *(uint2 *)(xq.qs + (size_t)t * xq.qrow + span * XQ_SPAN + lane * 8) = make_uint2(lo, hi);
    if ((lane & 3) == 0) {
        int blk = e0 >> 5;
        xq.d[(size_t)t * xq.nbx + blk] = __half2float(__float2half_rn(d));
        ((int32_t *)xq.sums)[(size_t)t * xq.nbx + blk] = sum;
    }
}

// The same, reading the lane's 8 values from x (row of token t).
__device__ __forceinline__ void load8(const float *x, int e0, bool live, float v[8]) {
    if (live) {
        float4 a = *(const float4 *)(x + e0), c = *(const float4 *)(x + e0 + 4);
        v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = c.x; v[5] = c.y; v[6] = c.z; v[7] = c.w;
    } else {
        for (int i = 0; i < 8; i++) v[i] = 0.0f;
    }
}

__device__ __forceinline__ void quant_q8k_block(const float *x, int t, int blk, const XQ &xq) {
    float v[8];
    load8(x, blk * 256 + (threadIdx.x & 31) * 8, true, v);
    quant_q8k_vals(v, t, blk, xq);
}

__device__ __forceinline__ void quant_q80_span(const float *x, int t, int span, int n_in, const XQ &xq) {
    const int e0 = span * 256 + (threadIdx.x & 31) * 8;
    float v[8];
    load8(x, e0, e0 < n_in, v);
    quant_q80_vals(v, e0 < n_in, t, span, xq);
}

// ------------------------------------------------------------------------------ RMSNorm rows
// The reference's RMSNorm (ops.c:346-351) of one row, shared by the standalone norm kernel and
// the kernels that normalise their own input in a prologue, so that all of them produce the same
// floats: the double sum of squares is taken in one fixed order that does not depend on the block
// size (8 consecutive elements per lane in order, a 256-element span by a warp's shuffle tree, the
// span partials by a second shuffle tree over part[0 .. ceil(n/256))). n <= 8192.

// Every thread of the block calls it and gets the total; part: 32 shared doubles.
__device__ inline double span_sumsq(const float *x, int n, double *part) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5, ns = (n + 255) / 256;
    for (int s = warp; s < ns; s += nw) {
        const int e0 = s * 256 + lane * 8;
        double ss = 0.0;
        for (int j = 0; j < 8; j++) {
            const float v = e0 + j < n ? x[e0 + j] : 0.0f;
            ss += (double)v * v;
        }
        for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        if (lane == 0) part[s] = ss;
    }
    __syncthreads();
    double v = lane < ns ? part[lane] : 0.0;
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    __syncthreads();  // part may be reused
    return v;
}

// v = x * (float)(1/sqrt(ss/n + eps)) * w for token t, quantized into q8k and/or q80 (XQ views of
// global or shared memory; a null qs skips that type; q8k needs n % 256 == 0) and optionally
// stored to xb. Whole block. When every warp has at most one span the row stays in registers
// between the sum of squares and the scaling (same order and values as span_sumsq).
__device__ inline void norm_quant_row(const float *x, const float *w, int n, float eps, int t, const XQ &q8k,
                                      const XQ &q80, float *xb, double *part) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5, ns = (n + 255) / 256;
    double ss;
    float r[8], wr[8];
    const bool one = ns <= nw;
    if (one) {
        const int e0 = warp * 256 + lane * 8;
        for (int j = 0; j < 8; j++) {  // x and the norm weights requested together
            const bool in = warp < ns && e0 + j < n;
            r[j] = in ? x[e0 + j] : 0.0f;
            wr[j] = in ? w[e0 + j] : 0.0f;
        }
        double p = 0.0;
        for (int j = 0; j < 8; j++) p += (double)r[j] * r[j];
        for (int o = 16; o; o >>= 1) p += __shfl_xor_sync(0xffffffffu, p, o);
        if (lane == 0 && warp < ns) part[warp] = p;
        __syncthreads();
        ss = lane < ns ? part[lane] : 0.0;
        for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        __syncthreads();
    } else {
        ss = span_sumsq(x, n, part);
    }
    const float scale = (float)(1.0 / sqrt(ss / n + (double)eps));
    for (int s = warp; s < ns; s += nw) {
        const int e0 = s * 256 + lane * 8;
        float v[8];
        for (int j = 0; j < 8; j++) {
            const float xv = one ? r[j] : (e0 + j < n ? x[e0 + j] : 0.0f);
            const float wv = one ? wr[j] : (e0 + j < n ? w[e0 + j] : 0.0f);
            v[j] = e0 + j < n ? __fmul_rn(__fmul_rn(xv, scale), wv) : 0.0f;
            if (xb && e0 + j < n) xb[e0 + j] = v[j];
        }
        if (q8k.qs) quant_q8k_vals(v, t, s, q8k);
        if (q80.qs) quant_q80_vals(v, e0 < n, t, s, q80);
    }
}

// The SwiGLU gate of one element, silu(g) * u, in the reference's operation order (ops.c:369).
__device__ __forceinline__ float silu_mul(float g, float u) {
    return __fmul_rn(__fdiv_rn(g, __fadd_rn(1.0f, expf_ref(-g))), u);
}

// Token t's input row as ActIn describes it (RMSNorm, SwiGLU gate or x as is), quantized into
// q8k and/or q80 by the whole block; the values equal those of the standalone kernels
// (rmsnorm_quant, silu_quant, quantize), warp w quantizing spans w, w + warps, ...
__device__ inline void act_quant_row(const ActIn &in, int n, int t, const XQ &q8k, const XQ &q80, double *part) {
    const float *x = in.x + (size_t)t * in.ldx;
    if (in.w) {
        norm_quant_row(x, in.w, n, in.eps, t, q8k, q80, nullptr, part);
        return;
    }
    const float *u = in.u ? in.u + (size_t)t * in.ldu : nullptr;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5, ns = (n + 255) / 256;
    for (int s = warp; s < ns; s += nw) {
        const int e0 = s * 256 + lane * 8;
        float r[8], ur[8], v[8];
        for (int j = 0; j < 8; j++) {  // every load of the span issued before the arithmetic
            const bool live = e0 + j < n;
            r[j] = live ? x[e0 + j] : 0.0f;
            ur[j] = live && u ? u[e0 + j] : 0.0f;
        }
        for (int j = 0; j < 8; j++) v[j] = e0 + j < n ? (u ? silu_mul(r[j], ur[j]) : r[j]) : 0.0f;
        if (q8k.qs) quant_q8k_vals(v, t, s, q8k);
        if (q80.qs) quant_q80_vals(v, e0 < n, t, s, q80);
    }
}

}  // namespace sdy
