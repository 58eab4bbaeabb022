// Per-pair device code of the quantized products, shared by the matvec (qmatvec.cu) and the
// fused MoE decode block (moe_decode.cu).
//
// A pair is one row and one superblock (Q4_K/Q6_K) or one row and a run of 8 blocks (Q8_0, Q4_0,
// Q5_0). load_pair reads the pair's bytes from the slab layout (common.cuh) into registers;
// pair_compute combines them with activations staged in shared memory in XQ layout (qs at
// sq + t*qrow, block scales sd[t*nb + b], block sums) into the reference's per-block fp32 term
// (q4k_combine / q6k_combine, reference csrc/quant.h:84-91; (float)s * (dw*dx) for the
// 32-element formats, csrc/quant.c:160), every product and sum rounded as the reference rounds it.
#pragma once
#include "common.cuh"

namespace sdy {

__device__ __forceinline__ uint4 ldg16(const uint8_t *p) { return __ldg((const uint4 *)p); }
__device__ __forceinline__ uint32_t word(const uint4 &v, int k) {
    return k == 0 ? v.x : k == 1 ? v.y : k == 2 ? v.z : v.w;
}
__device__ __forceinline__ float h2f(uint32_t h) { return __half2float(__ushort_as_half((uint16_t)h)); }
// 4 bits -> bit 4 of each of 4 bytes (Q5_0's fifth bits).
__device__ __forceinline__ uint32_t spread4(uint32_t x) { return ((x * 0x00204081u) & 0x01010101u) << 4; }

// ---------------------------------------------------------------------------- per-pair work
// A pair's weight bytes are first loaded into registers (Raw), then combined with the staged
// activations. Splitting the two lets each thread load its first pair before pdl_wait, so the
// DRAM latency of the weights overlaps the kernel that produces the activations.

template <int TYPE> struct Raw;
template <> struct Raw<T_Q4_K> { uint4 hdr, q[8]; };
template <> struct Raw<T_Q6_K> { uint4 ql[8], qh[4], sc; uint32_t d; };
template <> struct Raw<T_Q8_0> { uint4 qa[8], qb[8]; uint32_t d[8]; };
template <> struct Raw<T_Q4_0> { uint4 qa[8]; uint32_t d[8]; };
template <> struct Raw<T_Q5_0> { uint4 qa[8]; uint32_t qh[8], d[8]; };

__device__ __forceinline__ uint32_t ldg_u16(const uint8_t *p) { return __ldg((const unsigned short *)p); }

// gslabs: the group's first slab; u: pair column (superblock, or run of 8 blocks); r: row.
__device__ __forceinline__ void load_pair(Raw<T_Q4_K> &w, const uint8_t *gslabs, int u, int r, int) {
    const uint8_t *slab = gslabs + (size_t)u * slab_bytes(T_Q4_K);
    w.hdr = ldg16(slab + r * 16);
#pragma unroll
    for (int c = 0; c < 8; c++) w.q[c] = ldg16(slab + 128 + c * 128 + r * 16);
}
__device__ __forceinline__ void load_pair(Raw<T_Q6_K> &w, const uint8_t *gslabs, int u, int r, int) {
    const uint8_t *slab = gslabs + (size_t)u * slab_bytes(T_Q6_K);
#pragma unroll
    for (int c = 0; c < 8; c++) w.ql[c] = ldg16(slab + c * 128 + r * 16);
#pragma unroll
    for (int c = 0; c < 4; c++) w.qh[c] = ldg16(slab + 1024 + c * 128 + r * 16);
    w.sc = ldg16(slab + 1536 + r * 16);
    w.d = ldg_u16(slab + 1664 + r * 2);
}
__device__ __forceinline__ void load_pair(Raw<T_Q8_0> &w, const uint8_t *gslabs, int u, int r, int nb) {
    const int nblk = min(8, nb - u * 8);
#pragma unroll
    for (int i = 0; i < 8; i++)
        if (i < nblk) {
            const uint8_t *slab = gslabs + (size_t)(u * 8 + i) * slab_bytes(T_Q8_0);
            w.qa[i] = ldg16(slab + r * 16);
            w.qb[i] = ldg16(slab + 128 + r * 16);
            w.d[i] = ldg_u16(slab + 256 + r * 2);
        }
}
__device__ __forceinline__ void load_pair(Raw<T_Q4_0> &w, const uint8_t *gslabs, int u, int r, int nb) {
    const int nblk = min(8, nb - u * 8);
#pragma unroll
    for (int i = 0; i < 8; i++)
        if (i < nblk) {
            const uint8_t *slab = gslabs + (size_t)(u * 8 + i) * slab_bytes(T_Q4_0);
            w.qa[i] = ldg16(slab + r * 16);
            w.d[i] = ldg_u16(slab + 128 + r * 2);
        }
}
__device__ __forceinline__ void load_pair(Raw<T_Q5_0> &w, const uint8_t *gslabs, int u, int r, int nb) {
    const int nblk = min(8, nb - u * 8);
#pragma unroll
    for (int i = 0; i < 8; i++)
        if (i < nblk) {
            const uint8_t *slab = gslabs + (size_t)(u * 8 + i) * slab_bytes(T_Q5_0);
            w.qa[i] = ldg16(slab + r * 16);
            w.qh[i] = __ldg((const uint32_t *)(slab + 128 + r * 4));
            w.d[i] = ldg_u16(slab + 160 + r * 2);
        }
}

// Each writes the block term of token t to terms[(t * nb + b) * rows + rl].
template <int NT>
__device__ __forceinline__ void pair_terms(const Raw<T_Q4_K> &w, int b, const uint8_t *sq, int qrow,
                                           const float *sd, const int32_t *sbs, int nb, float *terms, int rows,
                                           int rl) {
    const uint4 hdr = w.hdr;
    const float d = h2f(hdr.x & 0xFFFF), dmin = h2f(hdr.x >> 16);
    // 6-bit scales and mins (quant.h:72-80), four per word.
    const uint32_t sc0 = hdr.y & 0x3F3F3F3F, m0 = hdr.z & 0x3F3F3F3F;
    const uint32_t sc1 = (hdr.w & 0x0F0F0F0F) | ((hdr.y >> 2) & 0x30303030);
    const uint32_t m1 = ((hdr.w >> 4) & 0x0F0F0F0F) | ((hdr.z >> 2) & 0x30303030);
#pragma unroll
    for (int t = 0; t < NT; t++) {
        const int *y = (const int *)(sq + t * qrow + b * XQ_SPAN);
        int isum = 0;
#pragma unroll
        for (int j = 0; j < 4; j++) {  // 64 elements: low nibbles -> sub-block 2j, high -> 2j+1
            int slo = 0, shi = 0;
#pragma unroll
            for (int k = 0; k < 8; k++) {
                uint32_t qw = word(w.q[2 * j + (k >> 2)], k & 3);
                slo = __dp4a((int)(qw & 0x0F0F0F0F), y[16 * j + k], slo);
                shi = __dp4a((int)((qw >> 4) & 0x0F0F0F0F), y[16 * j + 8 + k], shi);
            }
            const uint32_t scw = j < 2 ? sc0 : sc1;
            const int s_lo = (scw >> (16 * (j & 1))) & 0xFF, s_hi = (scw >> (16 * (j & 1) + 8)) & 0xFF;
            isum += s_lo * slo + s_hi * shi;
        }
        // Mins: msum = sum_j m_j * (bsum[2j] + bsum[2j+1]); one bsum pair per int32 word.
        const int32_t *bw = sbs + (t * nb + b) * 8;
        int msum = 0;
#pragma unroll
        for (int j = 0; j < 8; j++) {
            const uint32_t mw = j < 4 ? m0 : m1;
            msum = __dp2a_lo(bw[j], (int)__byte_perm(mw, 0, (j & 3) * 0x11), msum);
        }
        const float yd = sd[t * nb + b];
        const float dall = __fmul_rn(yd, d), dmn = __fmul_rn(yd, dmin);
        terms[(t * nb + b) * rows + rl] =
            __fsub_rn(__fmul_rn(dall, __int2float_rn(isum)), __fmul_rn(dmn, __int2float_rn(msum)));
    }
}

template <int NT>
__device__ __forceinline__ void pair_terms(const Raw<T_Q6_K> &w, int b, const uint8_t *sq, int qrow,
                                           const float *sd, const int32_t *sbs, int nb, float *terms, int rows,
                                           int rl) {
    const float d = h2f(w.d);
#pragma unroll
    for (int t = 0; t < NT; t++) {
        const int *y = (const int *)(sq + t * qrow + b * XQ_SPAN);
        int s[16];
#pragma unroll
        for (int g = 0; g < 16; g++) s[g] = 0;
#pragma unroll
        for (int h = 0; h < 2; h++) {
#pragma unroll
            for (int k = 0; k < 8; k++) {
                const uint32_t QL0 = word(w.ql[4 * h + (k >> 2)], k & 3);
                const uint32_t QL1 = word(w.ql[4 * h + 2 + (k >> 2)], k & 3);
                const uint32_t QH = word(w.qh[2 * h + (k >> 2)], k & 3);
                // unsigned 6-bit values of elements 128h + 32k + 4w .. +3 (quant.c:62-74)
                const uint32_t v0 = (QL0 & 0x0F0F0F0F) | ((QH << 4) & 0x30303030);
                const uint32_t v1 = (QL1 & 0x0F0F0F0F) | ((QH << 2) & 0x30303030);
                const uint32_t v2 = ((QL0 >> 4) & 0x0F0F0F0F) | (QH & 0x30303030);
                const uint32_t v3 = ((QL1 >> 4) & 0x0F0F0F0F) | ((QH >> 2) & 0x30303030);
                const int gw = k >> 2;
                s[8 * h + 0 + gw] = __dp4a((int)v0, y[32 * h + 0 + k], s[8 * h + 0 + gw]);
                s[8 * h + 2 + gw] = __dp4a((int)v1, y[32 * h + 8 + k], s[8 * h + 2 + gw]);
                s[8 * h + 4 + gw] = __dp4a((int)v2, y[32 * h + 16 + k], s[8 * h + 4 + gw]);
                s[8 * h + 6 + gw] = __dp4a((int)v3, y[32 * h + 24 + k], s[8 * h + 6 + gw]);
            }
        }
        // isum = sum_g sc_g * (sum q*y - 32 * bsum_g): exact, as the reference's AVX2 path.
        int isum = 0;
#pragma unroll
        for (int g = 0; g < 16; g++) isum += (int)(int8_t)(word(w.sc, g >> 2) >> (8 * (g & 3))) * s[g];
        const int32_t *bw = sbs + (t * nb + b) * 8;
        int corr = 0;
#pragma unroll
        for (int i = 0; i < 8; i++)
            corr = (i & 1) ? __dp2a_hi(bw[i], (int)word(w.sc, i >> 1), corr)
                           : __dp2a_lo(bw[i], (int)word(w.sc, i >> 1), corr);
        isum -= 32 * corr;
        const float yd = sd[t * nb + b];
        terms[(t * nb + b) * rows + rl] = __fmul_rn(__fmul_rn(yd, d), __int2float_rn(isum));
    }
}

// 32-element formats: the pair is blocks 8u .. 8u+7 (clipped to nb) of one row.
template <int TYPE, int NT, class R>
__device__ __forceinline__ void pair_terms_q0(const R &w, int u, const uint8_t *sq, int qrow, const float *sd,
                                              const int32_t *ssum, int nb, float *terms, int rows, int rl) {
    const int nblk = min(8, nb - u * 8);
#pragma unroll
    for (int i = 0; i < 8; i++) {
        if (i >= nblk) break;
        const int b = u * 8 + i;
        const float dw = h2f(w.d[i]);
#pragma unroll
        for (int t = 0; t < NT; t++) {
            const int *y = (const int *)(sq + t * qrow + xq_pos(32 * b));
            int s = 0;
            if constexpr (TYPE == T_Q8_0) {
#pragma unroll
                for (int k = 0; k < 4; k++) s = __dp4a((int)word(w.qa[i], k), y[k], s);
#pragma unroll
                for (int k = 0; k < 4; k++) s = __dp4a((int)word(w.qb[i], k), y[4 + k], s);
            } else {
#pragma unroll
                for (int k = 0; k < 4; k++) {
                    uint32_t lo = word(w.qa[i], k) & 0x0F0F0F0F, hi = (word(w.qa[i], k) >> 4) & 0x0F0F0F0F;
                    if constexpr (TYPE == T_Q5_0) {
                        lo |= spread4((w.qh[i] >> (4 * k)) & 15);
                        hi |= spread4((w.qh[i] >> (16 + 4 * k)) & 15);
                    }
                    s = __dp4a((int)lo, y[k], s);
                    s = __dp4a((int)hi, y[4 + k], s);
                }
                s -= (TYPE == T_Q4_0 ? 8 : 16) * ssum[t * nb + b];  // sum (u - bias) y
            }
            // (float)s * (dw * dx), quant.c:160
            terms[(t * nb + b) * rows + rl] = __fmul_rn(__int2float_rn(s), __fmul_rn(dw, sd[t * nb + b]));
        }
    }
}

template <int TYPE, int NT>
__device__ __forceinline__ void pair_compute(const Raw<TYPE> &w, int u, const uint8_t *sq, int qrow, const float *sd,
                                             const int32_t *ss, int nb, float *terms, int rows, int rl) {
    if constexpr (TYPE == T_Q4_K || TYPE == T_Q6_K)
        pair_terms<NT>(w, u, sq, qrow, sd, ss, nb, terms, rows, rl);
    else
        pair_terms_q0<TYPE, NT>(w, u, sq, qrow, sd, ss, nb, terms, rows, rl);
}

}  // namespace sdy
