/* zynfer oracle: CPU restatement of the Zynfer reference's f32 Qwen3 path.
 *
 * TEST INFRASTRUCTURE ONLY. This library is the checker for the CUDA backend:
 * only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may load
 * it. The product library (zynfer_b200/libzynfer_cuda.so) never links or calls
 * it, and has no CPU fallback.
 *
 * Every function restates a reference function in its loop order (cited as
 * file:line within the reference project). Compiled with -O2
 * -ffp-contract=off and no fast-math, so each f32 operation rounds like the
 * reference's scalar Zig loops. Threads only split independent outputs; no
 * summation order changes.
 *
 * Extensions (not reference behaviour, labelled where defined): the int8
 * weight-only model (linears and the tied LM head via matvecQ8, embedding rows
 * dequantised as f32(q)*scale), bf16 rounding of K/V on cache append, and the
 * greedy decode loop.
 */
#ifndef ZYNFER_ORACLE_H
#define ZYNFER_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- ops (src/backends/cpu/ops.zig) ---- */
void zo_add(float *z, const float *x, const float *y, size_t n);
float zo_silu_scalar(float x);
void zo_silu_mul(float *o, const float *g, const float *u, size_t n);
void zo_rms_norm(float *y, const float *x, const float *w, size_t rows, size_t cols, float eps);
void zo_softmax(float *y, const float *x, size_t rows, size_t cols);
void zo_matmul_f32(float *c, const float *a, const float *b, size_t m, size_t n, size_t k, int threads);
void zo_matvec_f32(float *y, const float *a, const float *x, size_t m, size_t k);
int zo_pack_row_q8(const float *w, size_t m, size_t k, int8_t *q, float *scale);
int zo_pack_tensor_q8(const float *w, size_t m, size_t k, int8_t *q, float *scale);
/* per_tensor: 0 = per-row scale[m], 1 = single scale[0] */
void zo_matvec_q8(float *y, const int8_t *q, const float *scale, const float *x, size_t m, size_t k,
                  int per_tensor, int threads);
void zo_matmul_q8(float *c, const int8_t *q, const float *scale, const float *b, size_t m, size_t n,
                  size_t k, int per_tensor);
void zo_rope(float *x, size_t tokens, size_t n_heads, size_t head_dim, size_t pos0, float theta);
int zo_attention_into(float *out, const float *q, const float *k, const float *v, size_t n_q,
                      size_t q_len, size_t d, size_t n_kv, size_t kv_len, size_t kv_stride,
                      float *scores, int threads);
void zo_tokens_heads_to_heads_tokens(float *out, const float *in, size_t tokens, size_t n_heads,
                                     size_t d);
void zo_heads_tokens_to_tokens_heads(float *out, const float *in, size_t n_heads, size_t tokens,
                                     size_t d);
int zo_embedding_gather(float *dst, const float *table, size_t vocab, size_t hidden,
                        const uint32_t *ids, size_t n);

/* ---- runtime helpers ---- */
float zo_bf16_to_f32(uint16_t w);          /* src/runtime/bf16.zig:6-9 */
uint16_t zo_f32_to_bf16_rne(float x);      /* extension: round to nearest even */
typedef struct {
    float max_abs, max_rel, rms;
    size_t failing_index;
    float expected, actual;
} ZoDiff;
void zo_diff_f32(const float *expected, const float *actual, size_t n, ZoDiff *out);
int zo_expect_close(const float *expected, const float *actual, size_t n, float atol, float rtol);
void zo_top_k(const float *logits, size_t n, size_t k, uint32_t *ids, float *vals);

/* Extension: temperature / top-k / top-p sampling of one row of logits (see
 * zynfer_oracle.c for the exact rule and the draws). */
int zo_sample_row(const float *logits, size_t V, float inv_t, uint32_t top_k, float top_p, uint64_t seed,
                  uint32_t slot, uint32_t pos, uint32_t *out);

/* ---- synthetic data (same generator as the CUDA library) ---- */
void zo_synth_normal(float *out, size_t n, uint64_t seed, uint64_t stream, float std_dev);
void zo_synth_tokens(uint32_t *out, size_t n, uint64_t seed, uint64_t stream, uint32_t vocab);

/* ---- model (src/model/qwen3.zig, qwen_block.zig, qwen_forward.zig) ---- */
typedef struct {
    uint32_t vocab, hidden, inter, layers, n_q, n_kv, head_dim, max_pos;
    float eps, theta;
} ZoArch;

enum { ZO_W_F32 = 0, ZO_W_BF16 = 1, ZO_W_Q8 = 2 };

typedef struct ZoModel ZoModel;
typedef struct ZoSession ZoSession;

/* Empty model; tensors are set by zo_model_set_tensor (HF names, HF [out,in]
 * layout, f32 values as loaded; BF16 weights already widened). */
ZoModel *zo_model_create(const ZoArch *arch, int wkind, int kv_bf16, int threads);
/* Synthetic weights: linears and embedding ~ normal(0, w_std); norm weights
 * 1 + normal(0, norm_std) (exactly 1 when norm_std == 0). wkind BF16 rounds
 * every weight to bf16 (RNE) first, the way a bf16 checkpoint stores it. */
ZoModel *zo_model_create_synthetic(const ZoArch *arch, int wkind, int kv_bf16, uint64_t seed,
                                   float w_std, float norm_std, int threads);
void zo_model_destroy(ZoModel *m);
int zo_model_set_tensor(ZoModel *m, const char *name, const float *data, size_t rows, size_t cols);
/* Packed int8 tensor (wkind == ZO_W_Q8): q [rows*cols], scale [rows]. */
int zo_model_get_q8(const ZoModel *m, const char *name, int8_t *q, float *scale, size_t rows,
                    size_t cols);
void zo_model_set_threads(ZoModel *m, int threads);

ZoSession *zo_session_create(ZoModel *m, size_t max_seq);
void zo_session_destroy(ZoSession *s);
void zo_session_reset(ZoSession *s);
size_t zo_session_used(const ZoSession *s);
/* Forward t tokens at pos0 = used (qwen_block.zig:161-235 for each layer),
 * then final norm + LM head on the last row. logits may be NULL. dump_layers
 * (nullable) receives the last row after each layer [layers][hidden];
 * dump_normed (nullable) the final-normed last row [hidden]. */
int zo_session_forward(ZoSession *s, const uint32_t *ids, size_t t, float *logits,
                       float *dump_layers, float *dump_normed);
/* qwen_block.zig:161-235 on one layer only: x [t][hidden] -> out [t][hidden]
 * at pos0 = used, then used += t (single-block sessions). */
int zo_session_block(ZoSession *s, uint32_t layer, const float *x, size_t t, float *out);
/* qwen_forward.zig:89-160: reset, then forward. */
int zo_prefill_last_logits(ZoSession *s, const uint32_t *ids, size_t t, float *logits);
/* Extension: greedy decode. Feeds `first` then each argmax for n_steps;
 * out_ids[i] = argmax after step i (lowest index on ties, as topK). If
 * teacher (nullable) is given, step i+1 feeds teacher[i] instead of the
 * argmax. logits_out (nullable) [n_steps][vocab]. */
int zo_greedy_decode(ZoSession *s, uint32_t first, size_t n_steps, const uint32_t *teacher,
                     uint32_t *out_ids, float *logits_out);
/* Timing helper: fill every layer's cache with n seeded normal(0, 1) K/V rows
 * (bf16-rounded when kv_bf16) and set used = n, standing in for a prefill. */
int zo_session_fill_kv(ZoSession *s, size_t n, uint64_t seed);
/* Copy K or V of one layer, positions [0, used): out [n_kv][used][d]. */
int zo_session_kv(const ZoSession *s, uint32_t layer, int which_v, float *out);

#ifdef __cplusplus
}
#endif

#endif
