/* sardyne_b200 — C-ABI of the B200 drop-in for Sardyne's libsardyne.so.
 *
 * Every function below has the name, argument list, argument meaning and error behaviour of the
 * reference symbol it replaces, so the reference's ctypes layer (sardyne/capi.py:33-102, which
 * binds all of them by name at load) and everything above it run unchanged with
 * SARDYNE_LIB=<path to this library>. Pointers are HOST pointers, exactly as in the reference;
 * the library moves data to and from the GPU itself. Only the last block ("B200 extensions") is
 * new, and nothing in the reference calls it.
 *
 * Types are ggml ids: F32 0, F16 1, Q4_0 2, Q5_0 6, Q8_0 8, Q4_K 12, Q6_K 14, Q8_K 15, BF16 30
 * (reference csrc/ops.h:21-22).
 */
#ifndef SARDYNE_B200_H
#define SARDYNE_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ------------------------------------------------------------------ engine (reference csrc/engine.h) */

typedef struct engine_model engine_model;
typedef struct engine_ctx engine_ctx;

/* Same field order and types as reference csrc/engine.h:24-40. */
typedef struct {
    int32_t n_vocab, dim, n_layer, n_head, n_kv_head, head_dim, ffn_dim, max_pos;
    float norm_eps, rope_theta;
    int32_t rope_interleaved, qkv_bias, tied_embeddings, qk_norm;
    int32_t n_expert, n_expert_used, ffn_exp_dim;
} engine_model_info;

const char *engine_version(void);                                                  /* engine.h:43 */
void engine_add_f32(const float *a, const float *b, float *out, size_t n);        /* engine.h:44 */
/* Loads a GGUF (llama, qwen2, qwen3, qwen3moe) and uploads every weight to the GPU(s) in the
 * device layout. NULL plus a message in err on failure.                              engine.h:48 */
engine_model *engine_model_load(const char *path, char *err, size_t err_len);
void engine_model_free(engine_model *m);                                           /* engine.h:49 */
void engine_model_get_info(const engine_model *m, engine_model_info *out);         /* engine.h:50 */
/* Limits as the reference: max_seq 1..min(1<<20, context_length), n_batch 1..4096,
 * n_threads 0..256 (accepted and echoed; the GPU path does not use host threads). engine.h:56 */
engine_ctx *engine_ctx_new(const engine_model *m, int32_t max_seq, int32_t n_batch, int32_t logits_all,
                           int32_t n_threads, char *err, size_t err_len);
int32_t engine_ctx_n_threads(const engine_ctx *c);                                 /* engine.h:58 */
void engine_ctx_free(engine_ctx *c);                                               /* engine.h:59 */
/* 0 on success; -1 with the reason in engine_last_error and the context unchanged. engine.h:64 */
int engine_eval(engine_ctx *c, const int32_t *tokens, int32_t n);
const float *engine_logits(const engine_ctx *c); /* host [n_logits][n_vocab]     engine.h:66 */
int32_t engine_n_logits(const engine_ctx *c);                                      /* engine.h:67 */
int32_t engine_n_past(const engine_ctx *c);                                        /* engine.h:68 */
void engine_reset(engine_ctx *c);                                                  /* engine.h:69 */
int engine_truncate(engine_ctx *c, int32_t n);                                     /* engine.h:71 */
const char *engine_last_error(const engine_ctx *c);                                /* engine.h:72 */

/* ------------------------------------------------------------------ kernels (reference csrc/ops.h) */

int op_simd(void);                       /* ops.h:25 — 1 when the fast kernels are selected */
int op_set_simd(int enable);             /* ops.h:26 — both modes run the same bit-exact GPU kernels */
void op_f16_to_f32_n(const uint16_t *x, float *out, size_t n);                      /* ops.h:36 */
uint16_t op_f32_to_f16(float f);                                                    /* ops.h:35 */
void op_row_to_f32(const void *row, int type, float *out, size_t n);               /* ops.h:37 */
size_t op_row_size(int type, int n);                                                /* ops.h:30 */
/* out[t][j] = x[t] . w[j] for row0 <= j < row1 (float weights).                      ops.h:42 */
void op_matmul_rows(float *out, const float *x, const void *w, int wtype, int n_tok, int n_in, int n_out,
                    int row0, int row1);
void op_matmul(float *out, const float *x, const void *w, int wtype, int n_tok, int n_in, int n_out); /* ops.h:45 */
/* Activation quantization of token rows t0..t1 into Q8_0 / Q8_K blocks (byte-exact).  ops.h:49 */
void op_quantize_rows(int vtype, const float *x, void *xq, int n_in, int t0, int t1);
/* Quantized product on pre-quantized activations, rows row0..row1 (bit-exact to the reference's
 * scalar kernels; K-quants also to its AVX2 kernels).                                  ops.h:50 */
void op_matmul_q_rows(float *out, const void *xq, const void *w, int wtype, int n_tok, int n_in, int n_out,
                      int row0, int row1);
float op_vec_dot_q(int wtype, const void *w, const void *xq, int n);                 /* ops.h:52 */
float op_dot_f32(const float *a, const float *b, int n);                            /* ops.h:55 */
void op_axpy(float *y, float a, const float *x, int n);                             /* ops.h:56 */
void op_rmsnorm(float *out, const float *x, const float *w, int n, float eps);      /* ops.h:58 */
void op_softmax(float *x, int n);                                                   /* ops.h:59 */
void op_silu_mul(float *gate, const float *up, int n);                              /* ops.h:60 */
void op_rope_table(float *cos_out, float *sin_out, int n_pos, int head_dim, float theta); /* ops.h:63 */
void op_rope(float *x, int n_heads, int head_dim, const float *cos, const float *sin, int interleaved); /* ops.h:66 */
void op_attention(float *out, const float *q, const float *k_cache, const float *v_cache, int n_head,
                  int n_kv_head, int head_dim, int n_kv, int stride, float *scores);  /* ops.h:73 */

/* ------------------------------------------------------------------ GGUF (reference csrc/gguf.h) */

typedef struct {             /* gguf.h:40-48 */
    const char *name;
    uint32_t n_dims, type;
    uint64_t ne[4];
    uint64_t offset, nbytes;
    const void *data;
} gguf_tensor;
typedef struct {             /* gguf.h:50-57 */
    const char *key;
    uint32_t type, arr_type;
    uint64_t n;
    const uint8_t *ptr;
    uint64_t *str_pos;
} gguf_kv;
typedef struct gguf_file gguf_file;

gguf_file *gguf_open(const char *path, char *err, size_t err_len);                  /* gguf.h:62 */
void gguf_close(gguf_file *f);                                                      /* gguf.h:63 */
uint32_t gguf_version(const gguf_file *f);                                          /* gguf.h:67 */
uint32_t gguf_alignment(const gguf_file *f);                                        /* gguf.h:68 */
uint64_t gguf_data_offset(const gguf_file *f);                                      /* gguf.h:69 */
uint64_t gguf_n_kv(const gguf_file *f);                                             /* gguf.h:70 */
uint64_t gguf_n_tensors(const gguf_file *f);                                        /* gguf.h:71 */
const gguf_kv *gguf_get_kv(const gguf_file *f, uint64_t i);                         /* gguf.h:73 */
int64_t gguf_find_kv(const gguf_file *f, const char *key);                          /* gguf.h:74 */
const gguf_tensor *gguf_get_tensor(const gguf_file *f, uint64_t i);                 /* gguf.h:75 */
int64_t gguf_find_tensor(const gguf_file *f, const char *name);                     /* gguf.h:76 */
int gguf_kv_get_u64(const gguf_file *f, int64_t i, uint64_t *out);                  /* gguf.h:79 */
int gguf_kv_get_f64(const gguf_file *f, int64_t i, double *out);                    /* gguf.h:80 */
const char *gguf_kv_get_str(const gguf_file *f, int64_t i, uint64_t *len);          /* gguf.h:81 */
const char *gguf_kv_get_arr_str(const gguf_file *f, int64_t i, uint64_t j, uint64_t *len); /* gguf.h:82 */
const char *gguf_type_name(uint32_t ggml_type);                                     /* gguf.h:84 */

/* ------------------------------------------------------------------ B200 extensions (no reference counterpart) */

/* Make a host weight matrix resident on the current GPU in the device layout. Afterwards every
 * op_matmul_q_rows / op_matmul / op_vec_dot_q / op_row_to_f32 call whose `w` points at a row of
 * this range reads the resident copy instead of copying the rows over PCIe; the caller promises
 * the host bytes no longer change (as the reference assumes of its read-only mmap, gguf.h:13-16).
 * n_rows rows of n_in elements of a quantized type. 0 on success, -1 (see sdy_last_error). */
int sdy_weights_register(const void *host, int wtype, int64_t n_rows, int32_t n_in);
int sdy_weights_unregister(const void *host);
/* Message of the last failed call on this host thread ("" when none); reset by sdy_clear_error. */
const char *sdy_last_error(void);
void sdy_clear_error(void);
/* Number of GPU kernels this process has launched through the library (for launch counting). */
uint64_t sdy_kernel_launches(void);
/* Nonzero when a kernel's bounded wait ran out: a tensor-core completion barrier (the kernel then
 * skipped its output and freed its tensor memory) or a fused gather's wait for the other ranks
 * (sdy_qmatvec_batch_f32_gather_dev). Stays set until sdy_kernel_clear_status; synchronises the
 * device. */
uint32_t sdy_kernel_status(void);
void sdy_kernel_clear_status(void);

/* Sharding across processes, one GPU each (no counterpart in the reference, which runs on one
 * host). sdy_nccl_unique_id writes the 128-byte NCCL id rank 0 creates and shares with the other
 * ranks; sdy_engine_set_shard(rank, world, id) configures the next engine_model_load of this
 * process: world 1 (the default) is the unsharded engine. A sharded model keeps attention and
 * the router on every rank and splits the FFN rows, the experts and the vocabulary; logits are
 * gathered on every rank and equal the one-GPU logits bit for bit. */
int sdy_nccl_unique_id(void *out);
int sdy_engine_set_shard(int32_t rank, int32_t world, const void *nccl_id);
/* No counterpart in the reference, whose greedy loop takes numpy.argmax of the host logits
 * (sardyne/runtime.py:115-140). engine_eval of `tokens`, then the id of the largest logit of the
 * last token chosen on the device (the first on ties, the first NaN if any, as numpy.argmax) into
 * *next; no logits are copied to the host (engine_logits returns NULL until the next engine_eval).
 * Same errors as engine_eval. 0 or -1. */
int sdy_engine_eval_greedy(engine_ctx *c, const int32_t *tokens, int32_t n, int32_t *next);
void sdy_engine_get_shard(int32_t *rank, int32_t *world);
/* The attention heads rank `rank` of `world` holds when the model is sharded: range = {first query
 * head, end, first KV head, end}. 1: attention split by heads (query heads with their KV heads; a
 * KV head shared by several ranks when world > n_kv_head); 0: attention replicated (range covers
 * every head); -1: bad arguments. */
int sdy_attention_split(int32_t n_head, int32_t n_kv_head, int32_t head_dim, int32_t world, int32_t rank,
                        int32_t *range);
/* How the context's cross-rank exchanges travel: 1 over NVLink peer memory for the single-token
 * sizes (NCCL for larger ones), 0 all over NCCL (SARDYNE_EXCHANGE=nccl, or a rank could not map
 * its peers), -1 not sharded or no context. No counterpart in the reference (one host). */
int sdy_engine_exchange(const engine_ctx *c);
/* Rows [*begin, *end) of n that `rank` of `world` holds, in whole units of `align` rows. */
void sdy_shard_range(int64_t n, int32_t world, int32_t rank, int64_t align, int64_t *begin, int64_t *end);

/* Device-pointer API (current device; `stream` is a cudaStream_t, NULL = legacy default stream).
 * A quantized matrix uploaded once in the device layout, activations quantized on the device,
 * and the matvec on device buffers, for callers that keep everything in HBM. */
void *sdy_qmat_upload(const void *host, int wtype, int64_t n_rows, int32_t n_in); /* NULL on error */
void sdy_qmat_free(void *w);
size_t sdy_qmat_bytes(const void *w);          /* device bytes of the uploaded matrix */
size_t sdy_xq_bytes(int vtype, int n_in, int n_tok); /* device bytes of quantized activations */
/* d_x f32 [n_tok][n_in] -> d_xq (sdy_xq_bytes bytes). 0 or -1. */
int sdy_quantize_rows_dev(int vtype, const float *d_x, int n_tok, int n_in, void *d_xq, void *stream);
/* d_out[t*ldo + (r - row0)] = w[r] . x[t] for row0 <= r < row1. 0 or -1. */
int sdy_qmatvec_dev(const void *w, const void *d_xq, int n_tok, float *d_out, int64_t ldo, int64_t row0,
                    int64_t row1, void *stream);

/* No counterpart in the reference (its products run one after another, csrc/model_llama.c:554-611).
 * n independent single-token products in one launch (a grouped matvec): d_out[i][r] = w_i[r] . x_i
 * for every row of each matrix, x_i the Q8_K row at d_xq[i] (sdy_xq_bytes(15, n_in_i, 1) bytes,
 * from sdy_quantize_rows_dev). 1 <= n <= 8, Q4_K / Q6_K weights; each result equals
 * sdy_qmatvec_dev's bit for bit. 0 or -1. */
int sdy_qmatvec_batch_dev(int n, const void *const *w, const void *const *d_xq, float *const *d_out, void *stream);
/* No counterpart in the reference. The same grouped products with f32 input rows d_x[i] (n_in_i
 * floats, 16-byte aligned, n_in_i a multiple of 256): every CTA quantizes its product's row to
 * Q8_K itself (the reference's quant_q8_K, byte-exact) while its first weights load, so no
 * quantization launch precedes the products; results equal sdy_quantize_rows_dev followed by
 * sdy_qmatvec_batch_dev bit for bit. 0 or -1. */
int sdy_qmatvec_batch_f32_dev(int n, const void *const *w, const float *const *d_x, float *const *d_out,
                              void *stream);
/* No counterpart in the reference (one host). sdy_qmatvec_batch_f32_dev with the all-gather of
 * sdy_allgather_p2p fused into the launch, for processes that drive one GPU each: product i's rows
 * go to offset rank * count + out_off[i] of every rank's gather buffer (bases: every rank's buffer
 * from sdy_p2p_alloc(sdy_allgather_p2p_bytes(count, world)), as mapped here; this rank's rows of
 * each matrix, out_off[i] + rows <= count). Each output value is stored into the peers' buffers
 * over NVLink as it is produced; the launch's last CTA then exchanges round flags with the other
 * ranks (bounded one-second wait; sdy_kernel_status nonzero if it gave up). Every rank makes the
 * same sequence of calls; the buffers' flags are shared with sdy_allgather_p2p. 0 or -1. */
int sdy_qmatvec_batch_f32_gather_dev(int n, const void *const *w, const float *const *d_x, const int64_t *out_off,
                                     int64_t count, void *const *bases, int32_t rank, int32_t world, void *stream);

/* No counterpart in the reference (it runs on one host). All-gather over NVLink peer memory for
 * processes that drive one GPU each: rank r's count floats (d_send) are stored by the GPU into
 * offset r * count of every rank's buffer. bases[q]: rank q's buffer as mapped in this process
 * (bases[rank] its own, from sdy_p2p_alloc(sdy_allgather_p2p_bytes(count, world)); the others from
 * sdy_p2p_open of their sdy_p2p_handle). Every rank makes the same sequence of calls; when this
 * call's work ends on `stream`, the own buffer holds every rank's slice. A rank may begin writing
 * the next call's slices as soon as every rank has finished this call, so a caller that reads the
 * buffer between calls alternates two buffers. world <= 8. 0 or -1; a peer that never arrives
 * makes the wait give up after one second and sets sdy_p2p_status. */
size_t sdy_allgather_p2p_bytes(int64_t count, int32_t world);
void *sdy_p2p_alloc(size_t bytes); /* zeroed device memory that can be shared; NULL on error */
void sdy_p2p_free(void *d_ptr);
int sdy_p2p_handle(const void *d_ptr, void *handle_out); /* 64-byte IPC handle of an sdy_p2p_alloc buffer */
void *sdy_p2p_open(const void *handle);                  /* a peer's buffer mapped here; NULL on error */
int sdy_p2p_close(void *d_peer);
int sdy_allgather_p2p(const float *d_send, int64_t count, void *const *bases, int32_t rank, int32_t world,
                      void *stream);
int sdy_p2p_read(void *host_dst, const void *d_src, size_t bytes); /* device -> host copy, synchronous */
uint32_t sdy_p2p_status(void); /* nonzero: an sdy_allgather_p2p wait gave up */
void sdy_p2p_clear_status(void);

/* No counterpart in the reference. For callers that cannot allocate device memory where they
 * call: a host framework that accounts for all device memory through its own pool, or a serving
 * loop that keeps cudaMalloc/cudaFree (which can stall or synchronise the device) out of its
 * steady state. f32 activations d_x [n_tok][n_in] are quantized and multiplied by w
 * (d_out[t*ldo + (r - row0)] = w[r] . x[t], as sdy_quantize_rows_dev + sdy_qmatvec_dev) with no
 * scratch argument and no allocation. The quantized activations live in a fixed 512 KiB device
 * array inside the library (held by every GPU that loads it until exit): requests that need
 * more (sdy_xq_bytes(vtype, n_in, n_tok) > 512 KiB; for 16384-element rows, more than 26 tokens)
 * return -1 with a message and launch nothing. The first call on a device looks up the array's
 * address with that device current and keeps it: do not reset the device afterwards. All calls on a device share the array: calls whose GPU work may
 * overlap (unordered streams) race. 0 or -1 (sdy_last_error). */
int sdy_qmatvec_f32_noalloc(const void *w, const float *d_x, int n_tok, float *d_out, int64_t ldo, int64_t row0,
                            int64_t row1, void *stream);

#ifdef __cplusplus
}
#endif

#endif
