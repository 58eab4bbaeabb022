// Device helpers shared by the fp32 kernels (fp_ops.cu, attention.cu, fused.cu): the
// reference's scalar dot product, the reference host's expf (expf_ref.h), and block reductions.
#pragma once
#include "common.cuh"
#include "expf_ref.h"

#include <cuda_bf16.h>

namespace sdy {

__device__ __forceinline__ float load_w(const void *w, int type, size_t i) {
    if (type == T_F32) return ((const float *)w)[i];
    if (type == T_F16) return __half2float(((const __half *)w)[i]);
    return __bfloat162float(((const __nv_bfloat16 *)w)[i]);
}

// The reference's scalar dot (ops.c:155-167): four accumulators, tail into the first.
template <class Load>
__device__ __forceinline__ float dot4(const float *x, Load w, int n) {
    float s0 = 0.0f, s1 = 0.0f, s2 = 0.0f, s3 = 0.0f;
    int i = 0;
    for (; i + 4 <= n; i += 4) {
        s0 = __fadd_rn(s0, __fmul_rn(x[i], w(i)));
        s1 = __fadd_rn(s1, __fmul_rn(x[i + 1], w(i + 1)));
        s2 = __fadd_rn(s2, __fmul_rn(x[i + 2], w(i + 2)));
        s3 = __fadd_rn(s3, __fmul_rn(x[i + 3], w(i + 3)));
    }
    for (; i < n; i++) s0 = __fadd_rn(s0, __fmul_rn(x[i], w(i)));
    return __fadd_rn(__fadd_rn(s0, s1), __fadd_rn(s2, s3));
}

// Block-wide sum of doubles (blockDim.x a multiple of 32, at most 1024).
__device__ inline double block_sum_d(double v) {
    __shared__ double part[32];
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
    __syncthreads();
    if (lane == 0) part[w] = v;
    __syncthreads();
    int nw = blockDim.x >> 5;
    v = lane < nw ? part[lane] : 0.0;
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ inline float block_max_f(float v) {
    __shared__ float part[32];
    for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
    __syncthreads();
    if (lane == 0) part[w] = v;
    __syncthreads();
    int nw = blockDim.x >> 5;
    v = lane < nw ? part[lane] : -INFINITY;
    for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// Softmax in place by the whole block (ops.c:353-364): exp(x - max), double sum, scaled by
// (float)(1/sum). The double sum is taken in a different order than the reference's sequential
// one; the two agree to ~1e-16 relative before the final rounding to float.
__device__ inline void softmax_block(float *v, int n) {
    float m = -INFINITY;
    for (int i = threadIdx.x; i < n; i += blockDim.x) m = fmaxf(m, v[i]);
    m = block_max_f(m);
    double sum = 0.0;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        float e = expf_ref(__fsub_rn(v[i], m));
        v[i] = e;
        sum += e;
    }
    sum = block_sum_d(sum);
    float inv = (float)(1.0 / sum);
    __syncthreads();
    for (int i = threadIdx.x; i < n; i += blockDim.x) v[i] = __fmul_rn(v[i], inv);
}

// x[t] += sum over t's k slots, in ascending expert id, of w * y[slot] (model_llama.c:723-750),
// elements i0, i0 + step, ... of the row by the calling CTA (k <= 64). The slots are ranked in
// shared memory (ties keep slot order); each element then adds its k terms in that order with the
// loads issued ahead of the adds.
__device__ inline void moe_combine_token(const float *y, int64_t ldy, const int32_t *top, const float *w, int k,
                                         int dim, float *x, int64_t ldx, int t, int i0, int step) {
    __shared__ int order[64];
    __shared__ float ws[64];
    const int32_t *tt = top + (size_t)t * k;
    if ((int)threadIdx.x < k) {
        const int i = threadIdx.x, ei = tt[i];
        int rank = 0;
        for (int j = 0; j < k; j++) {
            const int ej = tt[j];
            rank += (ej < ei || (ej == ei && j < i));
        }
        order[rank] = i;
    }
    __syncthreads();
    if ((int)threadIdx.x < k) ws[threadIdx.x] = w[(size_t)t * k + order[threadIdx.x]];
    __syncthreads();
    for (int i = i0 + threadIdx.x; i < dim; i += step) {
        const float acc = ordered_sum<8>(0.0f, k, [&](int j) {
            return __fmul_rn(ws[j], y[((size_t)t * k + order[j]) * ldy + i]);
        });
        float *xp = x + (size_t)t * ldx + i;
        *xp = __fadd_rn(*xp, acc);
    }
}

__device__ inline double bsum_d(double v, double *part) {
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
    __syncthreads();
    if (lane == 0) part[w] = v;
    __syncthreads();
    v = lane < (int)(blockDim.x >> 5) ? part[lane] : 0.0;
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ inline float bmax_f(float v, float *part) {
    for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
    __syncthreads();
    if (lane == 0) part[w] = v;
    __syncthreads();
    v = lane < (int)(blockDim.x >> 5) ? part[lane] : -INFINITY;
    for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}


__device__ __forceinline__ float4 load4_w(const void *w, int wtype, size_t i) {  // i a multiple of 4
    if (wtype == T_F32) return *(const float4 *)((const float *)w + i);
    const uint2 u = *(const uint2 *)((const uint16_t *)w + i);
    if (wtype == T_F16) {
        const float2 a = __half22float2(*(const __half2 *)&u.x), b = __half22float2(*(const __half2 *)&u.y);
        return make_float4(a.x, a.y, b.x, b.y);
    }
    return make_float4(__uint_as_float(u.x << 16), __uint_as_float(u.x & 0xFFFF0000u), __uint_as_float(u.y << 16),
                       __uint_as_float(u.y & 0xFFFF0000u));
}

// Softmax (ops.c:353-364) and top-k (model_llama.c:653-666) of one token's ne logits by the whole
// block; prob: shared array of ne floats, pv: k floats. The reference's insertion keeps the k
// largest probabilities in descending order, equal values in ascending expert id: expert e is at
// position rank(e) = #{j : p_j > p_e} + #{j < e : p_j == p_e}, computed for every expert in
// parallel. Weights are renormalised by their float sum taken in that order. The caller syncs the
// block before reading tp / wout.
__device__ inline void softmax_topk_block(const float *logits, float *prob, float *pv, int ne, int k, int32_t *tp,
                                          float *wout, double *dpart, float *fpart) {
    constexpr int PER = 8;  // logits per lane when one warp takes the softmax (ne <= 256)
    if (ne <= 32 * PER) {
        // Softmax by warp 0 alone, its logits in registers (lane l: e = l + 32 i): no block barrier
        // until the probabilities are in shared memory.
        if (threadIdx.x < 32) {
            const int lane = threadIdx.x;
            float v[PER];
            float m = -INFINITY;
#pragma unroll
            for (int i = 0; i < PER; i++) {
                const int e = lane + 32 * i;
                v[i] = e < ne ? __ldcg(logits + e) : -INFINITY;
            }
#pragma unroll
            for (int i = 0; i < PER; i++) m = fmaxf(m, v[i]);
            for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
            double sum = 0.0;
#pragma unroll
            for (int i = 0; i < PER; i++)
                if (lane + 32 * i < ne) {
                    v[i] = expf_ref(__fsub_rn(v[i], m));
                    sum += v[i];
                }
            for (int o = 16; o; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
            const float inv = (float)(1.0 / sum);
#pragma unroll
            for (int i = 0; i < PER; i++)
                if (lane + 32 * i < ne) prob[lane + 32 * i] = __fmul_rn(v[i], inv);
        }
    } else {
        for (int e = threadIdx.x; e < ne; e += blockDim.x) prob[e] = __ldcg(logits + e);
        __syncthreads();
        float m = -INFINITY;
        for (int e = threadIdx.x; e < ne; e += blockDim.x) m = fmaxf(m, prob[e]);
        m = bmax_f(m, fpart);
        double sum = 0.0;
        for (int e = threadIdx.x; e < ne; e += blockDim.x) {
            const float v = expf_ref(__fsub_rn(prob[e], m));
            prob[e] = v;
            sum += v;
        }
        sum = bsum_d(sum, dpart);
        const float inv = (float)(1.0 / sum);
        for (int e = threadIdx.x; e < ne; e += blockDim.x) prob[e] = __fmul_rn(prob[e], inv);
    }
    __syncthreads();
    for (int e = threadIdx.x; e < ne; e += blockDim.x) {
        const float pe = prob[e];
        int rank = 0;
        for (int j = 0; j < ne; j++) {
            const float pj = prob[j];
            rank += (pj > pe) | ((pj == pe) & (j < e));
        }
        if (rank < k) {
            tp[rank] = e;
            pv[rank] = pe;
        }
    }
    __syncthreads();
    if (threadIdx.x < 32) {  // the float sum of the k weights in order, then the renormalisation
        float sm = 0.0f;
        if (threadIdx.x == 0)
            for (int i = 0; i < k; i++) sm = __fadd_rn(sm, pv[i]);
        sm = __shfl_sync(0xffffffffu, sm, 0);
        for (int i = threadIdx.x; i < k; i += 32) wout[i] = __fdiv_rn(pv[i], sm);
    }
}

}  // namespace sdy
