// Launchers for the fp32 kernels in fp_ops.cu (all asynchronous on stream s).
#pragma once
#include "common.cuh"

namespace sdy {

void fmatmul(const float *x, int64_t ldx, const void *w, int type, int n_tok, int n_in, int64_t row0, int64_t row1,
             float *out, int64_t ldo, int64_t out_row0, cudaStream_t s);
void rmsnorm(float *out, int64_t ldo, const float *x, int64_t ldx, const float *w, int n, int rows, float eps,
             cudaStream_t s);
void softmax(float *x, int64_t ldx, int n, int rows, cudaStream_t s);
void silu_mul(float *gate, const float *up, int64_t n, cudaStream_t s);
void rope_table(float *c, float *sn, int n_pos, int head_dim, float theta, cudaStream_t s);
void rope(float *x, int64_t ldx, int n_tok, int n_heads, int head_dim, const float *c, const float *sn, int pos0,
          const int32_t *pos, int interleaved, cudaStream_t s);
struct PostQKV;
// post: the bias / qk-norm / RoPE / KV-store step of the same tokens, fused into the kernel for a
// single token and run before it otherwise.
void attention(float *out, const float *q, int64_t ldq, const float *kc, const float *vc, int n_tok, int n_head,
               int n_kv_head, int hd, int pos0, const int32_t *pos_dev, int stride, float *scratch, int fixed_nkv,
               cudaStream_t s, const PostQKV *post = nullptr);
void axpy(float *y, float a, const float *x, int64_t n, cudaStream_t s);
void add(float *out, const float *a, const float *b, int64_t n, cudaStream_t s);
void add_bias(float *x, int64_t ldx, const float *b, int n, int n_tok, cudaStream_t s);
void dot(const float *a, const float *b, int n, float *out, cudaStream_t s);
void convert_to_f32(const void *src, int type, float *dst, int64_t n, cudaStream_t s);
void f32_to_f16(const float *src, uint16_t *dst, int64_t n, cudaStream_t s);

}  // namespace sdy
