// fp32 kernels around the quantized products: float-weight matmul (F32/F16/BF16, e.g. the MoE
// router), RMSNorm, softmax, SiLU*up, RoPE, attention, and small vector ops (reference
// csrc/ops.c:277-423).
//
// They follow the reference's scalar kernels operation for operation, so that the activations
// fed to the next int8 quantization are the same floats and the forward stays bit-comparable:
//   * dot products use the reference's four interleaved accumulators and (s0+s1)+(s2+s3)
//     (ops.c:155-167), every product and sum rounded separately (the reference builds with
//     -ffp-contract=off);
//   * attention adds p_j * v_j in key order (ops.c:405-413); softmax and RMSNorm sum in double;
//   * exp is evaluated as exp() in double rounded once to float, i.e. the correctly rounded
//     expf, which is what the reference's libm returns (its documented error is < 0.51 ulp).
#include "common.cuh"
#include "fp_ops.cuh"

#include <cuda_bf16.h>

namespace sdy {

__device__ __forceinline__ float exp_cr(float x) { return (float)exp((double)x); }

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

// out[t*ldo + (j-out_row0)] = x[t] . w[j]: one thread per (row, token).
__global__ void fmatmul_kernel(const float *__restrict__ x, int64_t ldx, const void *__restrict__ w, int type,
                               int n_tok, int n_in, int64_t row0, int64_t row1, float *__restrict__ out,
                               int64_t ldo, int64_t out_row0) {
    int64_t k = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    int64_t rows = row1 - row0;
    if (k >= rows * n_tok) return;
    int64_t j = row0 + k % rows;
    int t = (int)(k / rows);
    size_t base = (size_t)j * n_in;
    float r = dot4(x + (size_t)t * ldx, [&](int i) { return load_w(w, type, base + i); }, n_in);
    out[(size_t)t * ldo + (j - out_row0)] = r;
}

void fmatmul(const float *x, int64_t ldx, const void *w, int type, int n_tok, int n_in, int64_t row0, int64_t row1,
             float *out, int64_t ldo, int64_t out_row0, cudaStream_t s) {
    int64_t n = (row1 - row0) * n_tok;
    if (n <= 0) return;
    fmatmul_kernel<<<(unsigned)((n + 127) / 128), 128, 0, s>>>(x, ldx, w, type, n_tok, n_in, row0, row1, out, ldo,
                                                                out_row0);
    SDY_LAUNCHED();
}

// Block-wide sum of doubles (blockDim.x a multiple of 32, at most 1024).
__device__ double block_sum_d(double v) {
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
__device__ float block_max_f(float v) {
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

// RMSNorm of `rows` vectors of n (ops.c:346-351): out = x * (float)(1/sqrt(mean(x^2)+eps)) * w.
__global__ void rmsnorm_kernel(float *out, int64_t ldo, const float *x, int64_t ldx, const float *w, int n, float eps) {
    const float *xv = x + blockIdx.x * ldx;
    float *ov = out + blockIdx.x * ldo;
    double ss = 0.0;
    for (int i = threadIdx.x; i < n; i += blockDim.x) ss += (double)xv[i] * xv[i];
    ss = block_sum_d(ss);
    float scale = (float)(1.0 / sqrt(ss / n + (double)eps));
    for (int i = threadIdx.x; i < n; i += blockDim.x) ov[i] = __fmul_rn(__fmul_rn(xv[i], scale), w[i]);
}

void rmsnorm(float *out, int64_t ldo, const float *x, int64_t ldx, const float *w, int n, int rows, float eps,
             cudaStream_t s) {
    if (rows <= 0) return;
    rmsnorm_kernel<<<rows, n >= 1024 ? 1024 : ((n + 31) / 32) * 32, 0, s>>>(out, ldo, x, ldx, w, n, eps);
    SDY_LAUNCHED();
}

// Softmax in place (ops.c:353-364): exp(x - max), double sum, scaled by (float)(1/sum).
__device__ void softmax_block(float *v, int n) {
    float m = -INFINITY;
    for (int i = threadIdx.x; i < n; i += blockDim.x) m = fmaxf(m, v[i]);
    m = block_max_f(m);
    double sum = 0.0;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        float e = exp_cr(__fsub_rn(v[i], m));
        v[i] = e;
        sum += e;
    }
    sum = block_sum_d(sum);
    float inv = (float)(1.0 / sum);
    __syncthreads();
    for (int i = threadIdx.x; i < n; i += blockDim.x) v[i] = __fmul_rn(v[i], inv);
}

__global__ void softmax_kernel(float *x, int64_t ldx, int n) { softmax_block(x + blockIdx.x * ldx, n); }

void softmax(float *x, int64_t ldx, int n, int rows, cudaStream_t s) {
    if (rows <= 0) return;
    softmax_kernel<<<rows, 256, 0, s>>>(x, ldx, n);
    SDY_LAUNCHED();
}

// gate = gate / (1 + exp(-gate)) * up  (ops.c:366-371)
__global__ void silu_mul_kernel(float *gate, const float *up, int64_t n) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        float g = gate[i];
        gate[i] = __fmul_rn(__fdiv_rn(g, __fadd_rn(1.0f, exp_cr(-g))), up[i]);
    }
}

void silu_mul(float *gate, const float *up, int64_t n, cudaStream_t s) {
    if (n <= 0) return;
    silu_mul_kernel<<<(unsigned)std::min<int64_t>((n + 255) / 256, 148 * 16), 256, 0, s>>>(gate, up, n);
    SDY_LAUNCHED();
}

// cos/sin tables in double (ops.c:375-386): angle = pos * theta^(-2i/head_dim).
__global__ void rope_table_kernel(float *c, float *sn, int n_pos, int head_dim, float theta) {
    int half = head_dim / 2;
    int64_t total = (int64_t)n_pos * half;
    for (int64_t k = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; k < total; k += (int64_t)gridDim.x * blockDim.x) {
        int p = (int)(k / half), i = (int)(k % half);
        double inv_freq = 1.0 / pow((double)theta, (double)(2 * i) / head_dim);
        double ang = (double)p * inv_freq;
        c[k] = (float)cos(ang);
        sn[k] = (float)sin(ang);
    }
}

void rope_table(float *c, float *sn, int n_pos, int head_dim, float theta, cudaStream_t s) {
    int64_t total = (int64_t)n_pos * (head_dim / 2);
    if (total <= 0) return;
    rope_table_kernel<<<(unsigned)std::min<int64_t>((total + 255) / 256, 4096), 256, 0, s>>>(c, sn, n_pos, head_dim,
                                                                                             theta);
    SDY_LAUNCHED();
}

// Pair (a, b) rotated by angle i: (a cos - b sin, a sin + b cos) (ops.c:388-403).
__device__ __forceinline__ void rope_one(float *v, int head_dim, const float *c, const float *sn, int interleaved,
                                         int i) {
    int half = head_dim / 2;
    int ia = interleaved ? 2 * i : i, ib = interleaved ? 2 * i + 1 : i + half;
    float a = v[ia], b = v[ib];
    v[ia] = __fsub_rn(__fmul_rn(a, c[i]), __fmul_rn(b, sn[i]));
    v[ib] = __fadd_rn(__fmul_rn(a, sn[i]), __fmul_rn(b, c[i]));
}

// x: [n_tok][ldx] with n_heads vectors of head_dim each; token t uses table row pos[t] (or pos0+t).
__global__ void rope_kernel(float *x, int64_t ldx, int n_heads, int head_dim, const float *c, const float *sn,
                            int pos0, const int32_t *pos, int interleaved) {
    int t = blockIdx.y, h = blockIdx.x;
    int p = pos ? pos[t] : pos0 + t;
    int half = head_dim / 2;
    float *v = x + (size_t)t * ldx + (size_t)h * head_dim;
    for (int i = threadIdx.x; i < half; i += blockDim.x)
        rope_one(v, head_dim, c + (size_t)p * half, sn + (size_t)p * half, interleaved, i);
}

void rope(float *x, int64_t ldx, int n_tok, int n_heads, int head_dim, const float *c, const float *sn, int pos0,
          const int32_t *pos, int interleaved, cudaStream_t s) {
    if (n_tok <= 0 || n_heads <= 0) return;
    rope_kernel<<<dim3(n_heads, n_tok), 64, 0, s>>>(x, ldx, n_heads, head_dim, c, sn, pos0, pos, interleaved);
    SDY_LAUNCHED();
}

// One (head, token) per block of ATT_THREADS (ops.c:405-423): scores over n_kv = pos0 + t + 1
// positions (the causal mask); softmax; then out[i] = sum_j p_j v_j[i] in key order.
// K and V are staged through shared memory in tiles read with coalesced 16-byte loads: a K tile
// holds one key per thread (rows padded to hd+1 floats, so the threads' dot products, each over
// its own row, hit distinct banks); a V tile holds as many keys as fit the same space, and thread
// i adds p_j * v_j[i] for the tile's keys in order. q: token t at q + t*ldq, heads of hd (a
// multiple of 4, at most 2*ATT_THREADS); k/v cache [n_kv_head][stride][hd]; the first token's
// position is *pos_dev when given, else pos0; scratch: n_tok*n_head*stride floats (scores).
constexpr int ATT_THREADS = 128;
__host__ __device__ inline int att_smem_floats(int hd) { return hd + ATT_THREADS * (hd + 1) + 2 * ATT_THREADS + 8; }

__global__ void attention_kernel(float *out, const float *q, int64_t ldq, const float *kc, const float *vc, int n_head,
                                 int n_kv_head, int hd, int pos0, const int32_t *pos_dev, int stride, float *scratch,
                                 int fixed_nkv) {
    extern __shared__ __align__(16) float sm[];
    const int t = blockIdx.y, h = blockIdx.x, tid = threadIdx.x;
    const int n_kv = fixed_nkv > 0 ? fixed_nkv : (pos_dev ? *pos_dev : pos0) + t + 1;
    const int n_rep = n_head / n_kv_head, ldt = hd + 1, hd4 = hd / 4;
    const float *qv = q + (size_t)t * ldq + (size_t)h * hd;
    const float *kh = kc + (size_t)(h / n_rep) * stride * hd;
    const float *vh = vc + (size_t)(h / n_rep) * stride * hd;
    float *sc = scratch + ((size_t)t * n_head + h) * stride;
    float *qs = sm, *tile = sm + ((hd + 3) & ~3), *ps = tile + ATT_THREADS * ldt;
    const float scale = __fdiv_rn(1.0f, sqrtf((float)hd));
    for (int i = tid; i < hd; i += ATT_THREADS) qs[i] = qv[i];
    for (int j0 = 0; j0 < n_kv; j0 += ATT_THREADS) {
        const int nk = min(ATT_THREADS, n_kv - j0);
        __syncthreads();
        for (int idx = tid; idx < nk * hd4; idx += ATT_THREADS) {
            const int j = idx / hd4, i = (idx - j * hd4) * 4;
            const float4 v = *(const float4 *)(kh + (size_t)(j0 + j) * hd + i);
            float *d = tile + j * ldt + i;
            d[0] = v.x; d[1] = v.y; d[2] = v.z; d[3] = v.w;
        }
        __syncthreads();
        if (tid < nk) {
            const float *row = tile + tid * ldt;
            sc[j0 + tid] = __fmul_rn(dot4(qs, [&](int i) { return row[i]; }, hd), scale);
        }
    }
    __syncthreads();
    softmax_block(sc, n_kv);
    __syncthreads();
    const int tv = (ATT_THREADS * ldt) / hd;  // keys per V tile
    float acc0 = 0.0f, acc1 = 0.0f;
    const int i0 = tid, i1 = tid + ATT_THREADS;
    for (int j0 = 0; j0 < n_kv; j0 += tv) {
        const int nv = min(tv, n_kv - j0);
        __syncthreads();
        for (int idx = tid; idx < nv * hd4; idx += ATT_THREADS)
            *(float4 *)(tile + idx * 4) = *(const float4 *)(vh + (size_t)j0 * hd + idx * 4);
        for (int j = tid; j < nv; j += ATT_THREADS) ps[j] = sc[j0 + j];
        __syncthreads();
        for (int j = 0; j < nv; j++) {
            const float p = ps[j];
            if (i0 < hd) acc0 = __fadd_rn(acc0, __fmul_rn(p, tile[j * hd + i0]));
            if (i1 < hd) acc1 = __fadd_rn(acc1, __fmul_rn(p, tile[j * hd + i1]));
        }
    }
    float *ov = out + ((size_t)t * n_head + h) * hd;
    if (i0 < hd) ov[i0] = acc0;
    if (i1 < hd) ov[i1] = acc1;
}

void attention(float *out, const float *q, int64_t ldq, const float *kc, const float *vc, int n_tok, int n_head,
               int n_kv_head, int hd, int pos0, const int32_t *pos_dev, int stride, float *scratch, int fixed_nkv,
               cudaStream_t s) {
    if (n_tok <= 0) return;
    if (hd % 4 || hd > 2 * ATT_THREADS) {
        set_error("attention: head_dim %d not supported (multiple of 4, at most %d)", hd, 2 * ATT_THREADS);
        return;
    }
    const size_t smem = (size_t)att_smem_floats(hd) * 4;
    static bool configured = false;
    if (!configured) {
        SDY_CUDA(cudaFuncSetAttribute(attention_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      att_smem_floats(2 * ATT_THREADS) * 4));
        configured = true;
    }
    attention_kernel<<<dim3(n_head, n_tok), ATT_THREADS, smem, s>>>(out, q, ldq, kc, vc, n_head, n_kv_head, hd, pos0,
                                                                    pos_dev, stride, scratch, fixed_nkv);
    SDY_LAUNCHED();
}

__global__ void axpy_kernel(float *y, float a, const float *x, int64_t n) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        y[i] = __fadd_rn(y[i], __fmul_rn(a, x[i]));
}
void axpy(float *y, float a, const float *x, int64_t n, cudaStream_t s) {
    if (n <= 0) return;
    axpy_kernel<<<(unsigned)std::min<int64_t>((n + 255) / 256, 4096), 256, 0, s>>>(y, a, x, n);
    SDY_LAUNCHED();
}

__global__ void add_kernel(float *out, const float *a, const float *b, int64_t n) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        out[i] = __fadd_rn(a[i], b[i]);
}
void add(float *out, const float *a, const float *b, int64_t n, cudaStream_t s) {
    if (n <= 0) return;
    add_kernel<<<(unsigned)std::min<int64_t>((n + 255) / 256, 4096), 256, 0, s>>>(out, a, b, n);
    SDY_LAUNCHED();
}

// x[t][i] += b[i]
__global__ void add_bias_kernel(float *x, int64_t ldx, const float *b, int n, int n_tok) {
    int64_t total = (int64_t)n * n_tok;
    for (int64_t k = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; k < total; k += (int64_t)gridDim.x * blockDim.x) {
        int t = (int)(k / n), i = (int)(k % n);
        x[(size_t)t * ldx + i] = __fadd_rn(x[(size_t)t * ldx + i], b[i]);
    }
}
void add_bias(float *x, int64_t ldx, const float *b, int n, int n_tok, cudaStream_t s) {
    int64_t total = (int64_t)n * n_tok;
    if (total <= 0) return;
    add_bias_kernel<<<(unsigned)std::min<int64_t>((total + 255) / 256, 4096), 256, 0, s>>>(x, ldx, b, n, n_tok);
    SDY_LAUNCHED();
}

// The reference's scalar dot on one thread (op_dot_f32 is a test hook, not a hot path).
__global__ void dot_kernel(const float *a, const float *b, int n, float *out) {
    if (threadIdx.x == 0 && blockIdx.x == 0) *out = dot4(a, [&](int i) { return b[i]; }, n);
}
void dot(const float *a, const float *b, int n, float *out, cudaStream_t s) {
    dot_kernel<<<1, 32, 0, s>>>(a, b, n, out);
    SDY_LAUNCHED();
}

// Element conversion of F32/F16/BF16 rows to f32.
__global__ void convert_kernel(const void *src, int type, float *dst, int64_t n) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        dst[i] = load_w(src, type, (size_t)i);
}
void convert_to_f32(const void *src, int type, float *dst, int64_t n, cudaStream_t s) {
    if (n <= 0) return;
    convert_kernel<<<(unsigned)std::min<int64_t>((n + 255) / 256, 4096), 256, 0, s>>>(src, type, dst, n);
    SDY_LAUNCHED();
}

__global__ void f32_to_f16_kernel(const float *src, uint16_t *dst, int64_t n) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        dst[i] = __half_as_ushort(__float2half_rn(src[i]));
}
void f32_to_f16(const float *src, uint16_t *dst, int64_t n, cudaStream_t s) {
    if (n <= 0) return;
    f32_to_f16_kernel<<<(unsigned)std::min<int64_t>((n + 255) / 256, 4096), 256, 0, s>>>(src, dst, n);
    SDY_LAUNCHED();
}

}  // namespace sdy
