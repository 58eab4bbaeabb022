// fp32 kernels around the quantized products: float-weight matmul (F32/F16/BF16, e.g. the MoE
// router), RMSNorm, softmax, SiLU*up, RoPE and small vector ops (reference
// csrc/ops.c:277-423).
//
// They follow the reference's scalar kernels operation for operation, so that the activations
// fed to the next int8 quantization are the same floats and the forward stays bit-comparable:
//   * dot products use the reference's four interleaved accumulators and (s0+s1)+(s2+s3)
//     (ops.c:155-167), every product and sum rounded separately (the reference builds with
//     -ffp-contract=off);
//   * softmax and RMSNorm sum in double;
//   * exp is evaluated as exp() in double rounded once to float, i.e. the correctly rounded
//     expf; glibc's expf, which the reference calls, differs from it in the last bit on ~0.06%
//     of inputs.
#include "common.cuh"
#include "fp_device.cuh"
#include "fp_ops.cuh"

namespace sdy {

// out[t*ldo + (j-out_row0)] = x[t] . w[j]: one thread per (row, token).
__global__ void fmatmul_kernel(const float *__restrict__ x, int64_t ldx, const void *__restrict__ w, int type,
                               int n_tok, int n_in, int64_t row0, int64_t row1, float *__restrict__ out,
                               int64_t ldo, int64_t out_row0) {
    pdl_wait();
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
    launch(fmatmul_kernel, (unsigned)((n + 127) / 128), 128, 0, s, x, ldx, w, type, n_tok, n_in, row0, row1, out, ldo,
                                                                out_row0);
    SDY_LAUNCHED();
}

// RMSNorm of `rows` vectors of n (ops.c:346-351): out = x * (float)(1/sqrt(mean(x^2)+eps)) * w.
__global__ void rmsnorm_kernel(float *out, int64_t ldo, const float *x, int64_t ldx, const float *w, int n, float eps) {
    pdl_wait();
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
    launch(rmsnorm_kernel, rows, n >= 1024 ? 1024 : ((n + 31) / 32) * 32, 0, s, out, ldo, x, ldx, w, n, eps);
    SDY_LAUNCHED();
}

__global__ void softmax_kernel(float *x, int64_t ldx, int n) { pdl_wait(); softmax_block(x + blockIdx.x * ldx, n); }

void softmax(float *x, int64_t ldx, int n, int rows, cudaStream_t s) {
    if (rows <= 0) return;
    launch(softmax_kernel, rows, 256, 0, s, x, ldx, n);
    SDY_LAUNCHED();
}

// gate = gate / (1 + exp(-gate)) * up  (ops.c:366-371)
__global__ void silu_mul_kernel(float *gate, const float *up, int64_t n) {
    pdl_wait();
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        float g = gate[i];
        gate[i] = __fmul_rn(__fdiv_rn(g, __fadd_rn(1.0f, expf_ref(-g))), up[i]);
    }
}

void silu_mul(float *gate, const float *up, int64_t n, cudaStream_t s) {
    if (n <= 0) return;
    launch(silu_mul_kernel, (unsigned)std::min<int64_t>((n + 255) / 256, 148 * 16), 256, 0, s, gate, up, n);
    SDY_LAUNCHED();
}

// cos/sin tables in double (ops.c:375-386): angle = pos * theta^(-2i/head_dim).
__global__ void rope_table_kernel(float *c, float *sn, int n_pos, int head_dim, float theta) {
    pdl_wait();
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
    launch(rope_table_kernel, (unsigned)std::min<int64_t>((total + 255) / 256, 4096), 256, 0, s, c, sn, n_pos, head_dim,
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
    pdl_wait();
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
    launch(rope_kernel, dim3(n_heads, n_tok), 64, 0, s, x, ldx, n_heads, head_dim, c, sn, pos0, pos, interleaved);
    SDY_LAUNCHED();
}

__global__ void axpy_kernel(float *y, float a, const float *x, int64_t n) {
    pdl_wait();
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        y[i] = __fadd_rn(y[i], __fmul_rn(a, x[i]));
}
void axpy(float *y, float a, const float *x, int64_t n, cudaStream_t s) {
    if (n <= 0) return;
    launch(axpy_kernel, (unsigned)std::min<int64_t>((n + 255) / 256, 4096), 256, 0, s, y, a, x, n);
    SDY_LAUNCHED();
}

__global__ void add_kernel(float *out, const float *a, const float *b, int64_t n) {
    pdl_wait();
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        out[i] = __fadd_rn(a[i], b[i]);
}
void add(float *out, const float *a, const float *b, int64_t n, cudaStream_t s) {
    if (n <= 0) return;
    launch(add_kernel, (unsigned)std::min<int64_t>((n + 255) / 256, 4096), 256, 0, s, out, a, b, n);
    SDY_LAUNCHED();
}

// x[t][i] += b[i]
__global__ void add_bias_kernel(float *x, int64_t ldx, const float *b, int n, int n_tok) {
    pdl_wait();
    int64_t total = (int64_t)n * n_tok;
    for (int64_t k = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; k < total; k += (int64_t)gridDim.x * blockDim.x) {
        int t = (int)(k / n), i = (int)(k % n);
        x[(size_t)t * ldx + i] = __fadd_rn(x[(size_t)t * ldx + i], b[i]);
    }
}
void add_bias(float *x, int64_t ldx, const float *b, int n, int n_tok, cudaStream_t s) {
    int64_t total = (int64_t)n * n_tok;
    if (total <= 0) return;
    launch(add_bias_kernel, (unsigned)std::min<int64_t>((total + 255) / 256, 4096), 256, 0, s, x, ldx, b, n, n_tok);
    SDY_LAUNCHED();
}

// The reference's scalar dot on one thread (op_dot_f32 is a test hook, not a hot path).
__global__ void dot_kernel(const float *a, const float *b, int n, float *out) {
    pdl_wait();
    if (threadIdx.x == 0 && blockIdx.x == 0) *out = dot4(a, [&](int i) { return b[i]; }, n);
}
void dot(const float *a, const float *b, int n, float *out, cudaStream_t s) {
    launch(dot_kernel, 1, 32, 0, s, a, b, n, out);
    SDY_LAUNCHED();
}

// Element conversion of F32/F16/BF16 rows to f32.
__global__ void convert_kernel(const void *src, int type, float *dst, int64_t n) {
    pdl_wait();
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        dst[i] = load_w(src, type, (size_t)i);
}
void convert_to_f32(const void *src, int type, float *dst, int64_t n, cudaStream_t s) {
    if (n <= 0) return;
    launch(convert_kernel, (unsigned)std::min<int64_t>((n + 255) / 256, 4096), 256, 0, s, src, type, dst, n);
    SDY_LAUNCHED();
}

__global__ void f32_to_f16_kernel(const float *src, uint16_t *dst, int64_t n) {
    pdl_wait();
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        dst[i] = __half_as_ushort(__float2half_rn(src[i]));
}
void f32_to_f16(const float *src, uint16_t *dst, int64_t n, cudaStream_t s) {
    if (n <= 0) return;
    launch(f32_to_f16_kernel, (unsigned)std::min<int64_t>((n + 255) / 256, 4096), 256, 0, s, src, dst, n);
    SDY_LAUNCHED();
}

}  // namespace sdy
