/* zynfer oracle: CPU restatement of the Zynfer reference's f32 Qwen3 path.
 *
 * TEST INFRASTRUCTURE ONLY (the checker, never the product): see
 * zynfer_oracle.h. Citations are file:line within the reference project.
 */
#include "zynfer_oracle.h"

#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "../zynfer_b200/csrc/synth_rng.h"

#ifdef _OPENMP
#include <omp.h>
#endif

#define ZO_OK 0
#define ZO_SHAPE 1
#define ZO_INVALID 2
#define ZO_OOM 3

/* ------------------------------------------------------------------ ops */

/* ops.zig:13-19 */
void zo_add(float *z, const float *x, const float *y, size_t n) {
    for (size_t i = 0; i < n; i++) z[i] = x[i] + y[i];
}

/* ops.zig:44-46: x * (1 / (1 + exp(-x))) */
float zo_silu_scalar(float x) { return x * (1.0f / (1.0f + expf(-x))); }

/* ops.zig:36-42 */
void zo_silu_mul(float *o, const float *g, const float *u, size_t n) {
    for (size_t i = 0; i < n; i++) o[i] = zo_silu_scalar(g[i]) * u[i];
}

/* ops.zig:49-67: sequential sum of squares, inv = 1/sqrt(mean + eps),
 * y = (w * v) * inv. Safe in place (the row sum is taken first). */
void zo_rms_norm(float *y, const float *x, const float *w, size_t rows, size_t cols, float eps) {
    for (size_t r = 0; r < rows; r++) {
        const float *row = x + r * cols;
        float *out = y + r * cols;
        float acc = 0.0f;
        for (size_t c = 0; c < cols; c++) acc += row[c] * row[c];
        const float inv = 1.0f / sqrtf(acc / (float)cols + eps);
        for (size_t c = 0; c < cols; c++) out[c] = w[c] * row[c] * inv;
    }
}

/* ops.zig:70-91 */
void zo_softmax(float *y, const float *x, size_t rows, size_t cols) {
    for (size_t r = 0; r < rows; r++) {
        const float *row = x + r * cols;
        float *out = y + r * cols;
        float max_v = row[0];
        for (size_t c = 1; c < cols; c++) max_v = fmaxf(max_v, row[c]);
        float sum = 0.0f;
        for (size_t c = 0; c < cols; c++) {
            out[c] = expf(row[c] - max_v);
            sum += out[c];
        }
        const float inv = 1.0f / sum;
        for (size_t c = 0; c < cols; c++) out[c] *= inv;
    }
}

/* ops.zig:118-131: C = A[m,k] * B[k,n], i-p-j order, C zeroed first. Threads
 * split (i, j-range) blocks; each element still accumulates over p in order. */
void zo_matmul_f32(float *c, const float *a, const float *b, size_t m, size_t n, size_t k,
                   int threads) {
    const size_t jb = 256;
    const size_t nj = (n + jb - 1) / jb;
    const long total = (long)(m * nj);
#pragma omp parallel for schedule(static) num_threads(threads > 0 ? threads : 1)
    for (long blk = 0; blk < total; blk++) {
        const size_t i = (size_t)blk / nj;
        const size_t j0 = ((size_t)blk % nj) * jb;
        const size_t j1 = j0 + jb < n ? j0 + jb : n;
        float *crow = c + i * n;
        for (size_t j = j0; j < j1; j++) crow[j] = 0.0f;
        for (size_t p = 0; p < k; p++) {
            const float av = a[i * k + p];
            const float *brow = b + p * n;
            for (size_t j = j0; j < j1; j++) crow[j] += av * brow[j];
        }
    }
}

/* ops.zig:133-141 */
void zo_matvec_f32(float *y, const float *a, const float *x, size_t m, size_t k) {
    for (size_t i = 0; i < m; i++) {
        float acc = 0.0f;
        for (size_t p = 0; p < k; p++) acc += a[i * k + p] * x[p];
        y[i] = acc;
    }
}

/* ops.zig:145-162: scale = max|w| / 127 (1 when the row is all zero),
 * inv = 1 / scale, q = clamp(round(w * inv), -127, 127); @round rounds half
 * away from zero, as C roundf does. */
int zo_pack_row_q8(const float *w, size_t m, size_t k, int8_t *q, float *scale) {
    for (size_t r = 0; r < m; r++) {
        const float *row = w + r * k;
        float max_abs = 0.0f;
        for (size_t c = 0; c < k; c++) max_abs = fmaxf(max_abs, fabsf(row[c]));
        const float s = max_abs == 0.0f ? 1.0f : max_abs / 127.0f;
        scale[r] = s;
        const float inv = 1.0f / s;
        for (size_t c = 0; c < k; c++) {
            const float qv = roundf(row[c] * inv);
            const float cl = fmaxf(-127.0f, fminf(127.0f, qv));
            q[r * k + c] = (int8_t)cl;
        }
    }
    return ZO_OK;
}

/* ops.zig:165-176 */
int zo_pack_tensor_q8(const float *w, size_t m, size_t k, int8_t *q, float *scale) {
    float max_abs = 0.0f;
    for (size_t i = 0; i < m * k; i++) max_abs = fmaxf(max_abs, fabsf(w[i]));
    const float s = max_abs == 0.0f ? 1.0f : max_abs / 127.0f;
    *scale = s;
    const float inv = 1.0f / s;
    for (size_t i = 0; i < m * k; i++) {
        const float r = roundf(w[i] * inv);
        q[i] = (int8_t)fmaxf(-127.0f, fminf(127.0f, r));
    }
    return ZO_OK;
}

/* ops.zig:181-197: y[r] = (sum_c f32(q[r,c]) * x[c]) * scale[r]. Four rows
 * are interleaved so their independent sequential sums overlap in the CPU
 * pipeline; each row's sum keeps the reference's order. */
void zo_matvec_q8(float *y, const int8_t *q, const float *scale, const float *x, size_t m, size_t k,
                  int per_tensor, int threads) {
    const long groups = (long)((m + 3) / 4);
#pragma omp parallel for schedule(static) num_threads(threads > 0 ? threads : 1)
    for (long g = 0; g < groups; g++) {
        const size_t r0 = (size_t)g * 4;
        if (r0 + 4 <= m) {
            const int8_t *q0 = q + r0 * k, *q1 = q0 + k, *q2 = q1 + k, *q3 = q2 + k;
            float a0 = 0.0f, a1 = 0.0f, a2 = 0.0f, a3 = 0.0f;
            for (size_t c = 0; c < k; c++) {
                const float xv = x[c];
                a0 += (float)q0[c] * xv;
                a1 += (float)q1[c] * xv;
                a2 += (float)q2[c] * xv;
                a3 += (float)q3[c] * xv;
            }
            y[r0 + 0] = a0 * (per_tensor ? scale[0] : scale[r0 + 0]);
            y[r0 + 1] = a1 * (per_tensor ? scale[0] : scale[r0 + 1]);
            y[r0 + 2] = a2 * (per_tensor ? scale[0] : scale[r0 + 2]);
            y[r0 + 3] = a3 * (per_tensor ? scale[0] : scale[r0 + 3]);
        } else {
            for (size_t r = r0; r < m; r++) {
                float acc = 0.0f;
                for (size_t c = 0; c < k; c++) acc += (float)q[r * k + c] * x[c];
                y[r] = acc * (per_tensor ? scale[0] : scale[r]);
            }
        }
    }
}

/* ops.zig:200-228: C[i,j] = sum_p (f32(q[i,p]) * s_i) * B[p,j] (the scale is
 * applied inside the sum here, unlike matvecQ8). */
void zo_matmul_q8(float *c, const int8_t *q, const float *scale, const float *b, size_t m, size_t n,
                  size_t k, int per_tensor) {
    memset(c, 0, m * n * sizeof(float));
    for (size_t i = 0; i < m; i++) {
        const float s = per_tensor ? scale[0] : scale[i];
        for (size_t p = 0; p < k; p++) {
            const float qv = (float)q[i * k + p] * s;
            for (size_t j = 0; j < n; j++) c[i * n + j] += qv * b[p * n + j];
        }
    }
}

/* ops.zig:233-261: split-half rotation, freq = 1 / theta^(i/half),
 * angle = pos * freq. x is [tokens, n_heads, head_dim]. */
void zo_rope(float *x, size_t tokens, size_t n_heads, size_t head_dim, size_t pos0, float theta) {
    const size_t half = head_dim / 2;
    for (size_t t = 0; t < tokens; t++) {
        const size_t pos = pos0 + t;
        for (size_t h = 0; h < n_heads; h++) {
            const size_t base = (t * n_heads + h) * head_dim;
            for (size_t i = 0; i < half; i++) {
                const float freq = 1.0f / powf(theta, (float)i / (float)half);
                const float angle = (float)pos * freq;
                const float c = cosf(angle);
                const float s = sinf(angle);
                const float a = x[base + i];
                const float b = x[base + i + half];
                x[base + i] = a * c - b * s;
                x[base + i + half] = a * s + b * c;
            }
        }
    }
}

/* ops.zig:285-354: causal GQA. q [n_q, q_len, d]; k, v [n_kv, kv_stride, d]
 * with kv_len valid rows; out [n_q, q_len, d]. Query tq sees key tk when
 * (kv_len - q_len + tq) >= tk. Threads split (head, query) rows; `scores`
 * must hold threads * kv_len floats. */
int zo_attention_into(float *out, const float *q, const float *k, const float *v, size_t n_q,
                      size_t q_len, size_t d, size_t n_kv, size_t kv_len, size_t kv_stride,
                      float *scores, int threads) {
    if (n_q % n_kv != 0) return ZO_INVALID;
    if (kv_len > kv_stride || q_len > kv_len) return ZO_INVALID;
    const size_t group = n_q / n_kv;
    const float scale = 1.0f / sqrtf((float)d);
    const long rows = (long)(n_q * q_len);
#pragma omp parallel for schedule(dynamic, 1) num_threads(threads > 0 ? threads : 1)
    for (long row = 0; row < rows; row++) {
        int tid = 0;
#ifdef _OPENMP
        tid = omp_get_thread_num();
#endif
        float *sc = scores + (size_t)tid * kv_len;
        const size_t h = (size_t)row / q_len;
        const size_t tq = (size_t)row % q_len;
        const size_t kv_h = h / group;
        const float *qrow = q + (h * q_len + tq) * d;
        float max_s = -INFINITY;
        for (size_t tk = 0; tk < kv_len; tk++) {
            const int causal_ok = (kv_len - q_len + tq) >= tk;
            if (!causal_ok) {
                sc[tk] = -INFINITY;
                continue;
            }
            const float *krow = k + (kv_h * kv_stride + tk) * d;
            float dot = 0.0f;
            for (size_t i = 0; i < d; i++) dot += qrow[i] * krow[i];
            sc[tk] = dot * scale;
            max_s = fmaxf(max_s, sc[tk]);
        }
        float sum = 0.0f;
        for (size_t tk = 0; tk < kv_len; tk++) {
            if (isinf(sc[tk])) {
                sc[tk] = 0.0f;
            } else {
                sc[tk] = expf(sc[tk] - max_s);
                sum += sc[tk];
            }
        }
        const float inv = sum == 0.0f ? 0.0f : 1.0f / sum;
        float *orow = out + (h * q_len + tq) * d;
        for (size_t i = 0; i < d; i++) orow[i] = 0.0f;
        for (size_t tk = 0; tk < kv_len; tk++) {
            const float w = sc[tk] * inv;
            if (w == 0.0f) continue;
            const float *vrow = v + (kv_h * kv_stride + tk) * d;
            for (size_t i = 0; i < d; i++) orow[i] += w * vrow[i];
        }
    }
    return ZO_OK;
}

/* ops.zig:357-374 */
void zo_tokens_heads_to_heads_tokens(float *out, const float *in, size_t tokens, size_t n_heads,
                                     size_t d) {
    for (size_t t = 0; t < tokens; t++)
        for (size_t h = 0; h < n_heads; h++)
            memcpy(out + (h * tokens + t) * d, in + (t * n_heads + h) * d, d * sizeof(float));
}

/* ops.zig:377-394 */
void zo_heads_tokens_to_tokens_heads(float *out, const float *in, size_t n_heads, size_t tokens,
                                     size_t d) {
    for (size_t h = 0; h < n_heads; h++)
        for (size_t t = 0; t < tokens; t++)
            memcpy(out + (t * n_heads + h) * d, in + (h * tokens + t) * d, d * sizeof(float));
}

/* ops.zig:397-411 */
int zo_embedding_gather(float *dst, const float *table, size_t vocab, size_t hidden,
                        const uint32_t *ids, size_t n) {
    for (size_t t = 0; t < n; t++) {
        if (ids[t] >= vocab) return ZO_INVALID;
        memcpy(dst + t * hidden, table + (size_t)ids[t] * hidden, hidden * sizeof(float));
    }
    return ZO_OK;
}

/* ------------------------------------------------------------ runtime */

/* bf16.zig:6-9: widen by shifting into the high half. */
float zo_bf16_to_f32(uint16_t w) {
    uint32_t bits = (uint32_t)w << 16;
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

/* Extension: f32 -> bf16, round to nearest even (NaN kept quiet). */
uint16_t zo_f32_to_bf16_rne(float x) {
    uint32_t u;
    memcpy(&u, &x, 4);
    if ((u & 0x7FFFFFFFu) > 0x7F800000u) return (uint16_t)((u >> 16) | 0x40u);
    const uint32_t lsb = (u >> 16) & 1u;
    u += 0x7FFFu + lsb;
    return (uint16_t)(u >> 16);
}

static float bf16_round(float x) { return zo_bf16_to_f32(zo_f32_to_bf16_rne(x)); }

/* compare.zig:14-41: the last index with the largest |a - e| wins (>=). */
void zo_diff_f32(const float *expected, const float *actual, size_t n, ZoDiff *out) {
    memset(out, 0, sizeof(*out));
    if (n == 0) return;
    double sum_sq = 0.0;
    for (size_t i = 0; i < n; i++) {
        const float e = expected[i], a = actual[i];
        const float abs_d = fabsf(a - e);
        const float denom = fmaxf(fabsf(e), 1e-8f);
        const float rel = abs_d / denom;
        sum_sq += (double)abs_d * (double)abs_d;
        if (abs_d >= out->max_abs) {
            out->max_abs = abs_d;
            out->max_rel = rel;
            out->failing_index = i;
            out->expected = e;
            out->actual = a;
        }
    }
    out->rms = (float)sqrt(sum_sq / (double)n);
}

/* compare.zig:49-59: max_abs <= atol + rtol * |expected at argmax|. */
int zo_expect_close(const float *expected, const float *actual, size_t n, float atol, float rtol) {
    ZoDiff d;
    zo_diff_f32(expected, actual, n, &d);
    return d.max_abs <= atol + rtol * fabsf(d.expected);
}

/* qwen_forward.zig:177-193: insertion top-k with strict '>' (lowest index
 * wins ties). */
void zo_top_k(const float *logits, size_t n, size_t k, uint32_t *ids, float *vals) {
    for (size_t i = 0; i < k; i++) {
        ids[i] = 0;
        vals[i] = -INFINITY;
    }
    for (size_t id = 0; id < n; id++) {
        const float logit = logits[id];
        for (size_t i = 0; i < k; i++) {
            if (logit > vals[i]) {
                for (size_t j = k - 1; j > i; j--) {
                    ids[j] = ids[j - 1];
                    vals[j] = vals[j - 1];
                }
                ids[i] = (uint32_t)id;
                vals[i] = logit;
                break;
            }
        }
    }
}

/* Extension (sampling: the reference has greedy topK only; its roadmap
 * Stage 12, docs/roadmap.md:29, is not started). One row of logits:
 * - temperature only (top_k == 0, top_p >= 1): the Gumbel-max draw
 *   argmax_v (l_v * inv_t + g_v), g_v = -log(-log(u_v)), first maximum on ties
 *   (topK's rule, qwen_forward.zig:177-193);
 * - otherwise the K = top_k (64 when 0, at most 64) largest logits in topK's
 *   order, p_i = exp((l_i - l_0) * inv_t) summed in that order, the shortest
 *   prefix m whose sum reaches top_p times the total (all K when top_p >= 1),
 *   and the first i < m whose running sum exceeds u times the prefix sum
 *   (m - 1 if rounding leaves none).
 * Draws: zs_uniform01 of ZS_SAMPLE_STREAM(slot) at pos * (vocab + 1) + v, and
 * + vocab for the row's draw. Every f32 step is a single rounded operation. */
int zo_sample_row(const float *logits, size_t V, float inv_t, uint32_t top_k, float top_p, uint64_t seed,
                  uint32_t slot, uint32_t pos, uint32_t *out) {
    const uint64_t key = zs_key(seed, ZS_SAMPLE_STREAM(slot));
    const uint64_t base = (uint64_t)pos * (V + 1);
    if (top_k == 0 && !(top_p < 1.0f)) {
        uint32_t best = 0;
        float best_s = -INFINITY;
        for (size_t v = 0; v < V; v++) {
            const float u = zs_uniform01(key, base + v);
            const float g = -logf(-logf(u));
            const float sv = logits[v] * inv_t + g;
            if (sv > best_s) {
                best_s = sv;
                best = (uint32_t)v;
            }
        }
        *out = best;
        return ZO_OK;
    }
    const size_t K = top_k == 0 || top_k > 64 ? 64 : top_k;
    uint32_t ids[64];
    float vals[64], p[64];
    zo_top_k(logits, V, K, ids, vals);
    size_t n = 0;
    while (n < K && vals[n] != -INFINITY) n++;
    if (n == 0) {
        *out = 0;
        return ZO_OK;
    }
    float z = 0.0f;
    for (size_t i = 0; i < n; i++) {
        p[i] = expf((vals[i] - vals[0]) * inv_t);
        z += p[i];
    }
    size_t m = n;
    if (top_p < 1.0f) {
        const float target = top_p * z;
        float c = 0.0f;
        for (m = 0; m < n;) {
            c += p[m++];
            if (c >= target) break;
        }
    }
    float zm = 0.0f;
    for (size_t i = 0; i < m; i++) zm += p[i];
    const float r = zs_uniform01(key, base + V) * zm;
    float c = 0.0f;
    size_t pick = m - 1;
    for (size_t i = 0; i < m; i++) {
        c += p[i];
        if (c > r) {
            pick = i;
            break;
        }
    }
    *out = ids[pick];
    return ZO_OK;
}

void zo_synth_normal(float *out, size_t n, uint64_t seed, uint64_t stream, float std_dev) {
    const uint64_t key = zs_key(seed, stream);
    const float k = (float)((double)std_dev / ZS_IH4_SIGMA);
    for (size_t i = 0; i < n; i++) out[i] = zs_normal(key, i, k);
}

void zo_synth_tokens(uint32_t *out, size_t n, uint64_t seed, uint64_t stream, uint32_t vocab) {
    const uint64_t key = zs_key(seed, stream);
    for (size_t i = 0; i < n; i++) out[i] = zs_uniform_u32(key, i, vocab);
}

/* -------------------------------------------------------------- model */

typedef struct {
    /* ZO_W_F32 / ZO_W_BF16: transposed [in, out] f32, as qwen_weights.zig:209-218 */
    float *wq, *wk, *wv, *wo, *wg, *wu, *wd;
    /* ZO_W_Q8: HF [out, in] int8 + per-row scale (packRowQ8) */
    int8_t *qq, *qk, *qv, *qo, *qg, *qu, *qd;
    float *sq, *sk, *sv, *so, *sg, *su, *sd;
    float *input_ln, *q_norm, *k_norm, *post_ln;
} ZoLayer;

struct ZoModel {
    ZoArch a;
    int wkind, kv_bf16, threads;
    float *embed; /* [V, H] f32 (F32/BF16) */
    int8_t *embed_q;
    float *embed_s; /* [V, H] int8 + [V] (Q8) */
    float *final_norm;
    ZoLayer *layers;
};

struct ZoSession {
    ZoModel *m;
    size_t max_seq, used;
    float **kc, **vc; /* per layer [n_kv, max_seq, d] (kv_cache.zig:14-47) */
    /* scratch sized max_seq (qwen_block.zig:13-64) */
    float *xa, *xb, *xn, *q_lin, *k_lin, *v_lin, *q_htd, *k_htd, *v_htd, *attn_htd, *attn_lin, *ao,
        *x1, *mlp_n, *gate, *up, *hact, *down, *scores, *normed, *logits;
};

static void *zalloc(size_t bytes) { return calloc(1, bytes ? bytes : 1); }

ZoModel *zo_model_create(const ZoArch *arch, int wkind, int kv_bf16, int threads) {
    ZoModel *m = (ZoModel *)zalloc(sizeof(ZoModel));
    if (!m) return NULL;
    m->a = *arch;
    m->wkind = wkind;
    m->kv_bf16 = kv_bf16;
    m->threads = threads > 0 ? threads : 1;
    const size_t H = arch->hidden, V = arch->vocab, I = arch->inter;
    const size_t qd = (size_t)arch->n_q * arch->head_dim, kvd = (size_t)arch->n_kv * arch->head_dim;
    m->final_norm = (float *)zalloc(H * 4);
    if (wkind == ZO_W_Q8) {
        m->embed_q = (int8_t *)zalloc(V * H);
        m->embed_s = (float *)zalloc(V * 4);
    } else {
        m->embed = (float *)zalloc(V * H * 4);
    }
    m->layers = (ZoLayer *)zalloc(sizeof(ZoLayer) * arch->layers);
    for (uint32_t l = 0; l < arch->layers; l++) {
        ZoLayer *L = &m->layers[l];
        L->input_ln = (float *)zalloc(H * 4);
        L->post_ln = (float *)zalloc(H * 4);
        L->q_norm = (float *)zalloc(arch->head_dim * 4);
        L->k_norm = (float *)zalloc(arch->head_dim * 4);
        if (wkind == ZO_W_Q8) {
            L->qq = (int8_t *)zalloc(qd * H); L->sq = (float *)zalloc(qd * 4);
            L->qk = (int8_t *)zalloc(kvd * H); L->sk = (float *)zalloc(kvd * 4);
            L->qv = (int8_t *)zalloc(kvd * H); L->sv = (float *)zalloc(kvd * 4);
            L->qo = (int8_t *)zalloc(H * qd); L->so = (float *)zalloc(H * 4);
            L->qg = (int8_t *)zalloc(I * H); L->sg = (float *)zalloc(I * 4);
            L->qu = (int8_t *)zalloc(I * H); L->su = (float *)zalloc(I * 4);
            L->qd = (int8_t *)zalloc(H * I); L->sd = (float *)zalloc(H * 4);
        } else {
            L->wq = (float *)zalloc(H * qd * 4);
            L->wk = (float *)zalloc(H * kvd * 4);
            L->wv = (float *)zalloc(H * kvd * 4);
            L->wo = (float *)zalloc(qd * H * 4);
            L->wg = (float *)zalloc(H * I * 4);
            L->wu = (float *)zalloc(H * I * 4);
            L->wd = (float *)zalloc(I * H * 4);
        }
    }
    return m;
}

void zo_model_destroy(ZoModel *m) {
    if (!m) return;
    for (uint32_t l = 0; l < m->a.layers; l++) {
        ZoLayer *L = &m->layers[l];
        free(L->wq); free(L->wk); free(L->wv); free(L->wo); free(L->wg); free(L->wu); free(L->wd);
        free(L->qq); free(L->qk); free(L->qv); free(L->qo); free(L->qg); free(L->qu); free(L->qd);
        free(L->sq); free(L->sk); free(L->sv); free(L->so); free(L->sg); free(L->su); free(L->sd);
        free(L->input_ln); free(L->q_norm); free(L->k_norm); free(L->post_ln);
    }
    free(m->layers);
    free(m->embed); free(m->embed_q); free(m->embed_s); free(m->final_norm);
    free(m);
}

void zo_model_set_threads(ZoModel *m, int threads) { m->threads = threads > 0 ? threads : 1; }

/* Resolve an HF tensor name (qwen3.zig:86-132) to its slots. */
typedef struct {
    float **vec;         /* norm vector */
    float **wt;          /* transposed f32 matrix */
    int8_t **q;
    float **s;
    size_t rows, cols;   /* HF shape */
} Slot;

static int find_slot(ZoModel *m, const char *name, Slot *out) {
    memset(out, 0, sizeof(*out));
    const ZoArch *a = &m->a;
    const size_t H = a->hidden, I = a->inter;
    const size_t qd = (size_t)a->n_q * a->head_dim, kvd = (size_t)a->n_kv * a->head_dim;
    if (strcmp(name, "model.embed_tokens.weight") == 0 || strcmp(name, "lm_head.weight") == 0) {
        out->rows = a->vocab; out->cols = H;
        out->wt = &m->embed; /* not transposed: gather and lmHeadTied read rows */
        out->q = &m->embed_q; out->s = &m->embed_s;
        return 0;
    }
    if (strcmp(name, "model.norm.weight") == 0) {
        out->vec = &m->final_norm; out->rows = H; out->cols = 1;
        return 0;
    }
    unsigned layer = 0;
    char rest[128];
    if (sscanf(name, "model.layers.%u.%127s", &layer, rest) != 2 || layer >= a->layers) return -1;
    ZoLayer *L = &m->layers[layer];
#define VEC(nm, field, n) if (strcmp(rest, nm) == 0) { out->vec = &L->field; out->rows = n; out->cols = 1; return 0; }
#define MAT(nm, wf, qf, sf, r, c) if (strcmp(rest, nm) == 0) { out->wt = &L->wf; out->q = &L->qf; out->s = &L->sf; out->rows = r; out->cols = c; return 0; }
    VEC("input_layernorm.weight", input_ln, H)
    VEC("post_attention_layernorm.weight", post_ln, H)
    VEC("self_attn.q_norm.weight", q_norm, a->head_dim)
    VEC("self_attn.k_norm.weight", k_norm, a->head_dim)
    MAT("self_attn.q_proj.weight", wq, qq, sq, qd, H)
    MAT("self_attn.k_proj.weight", wk, qk, sk, kvd, H)
    MAT("self_attn.v_proj.weight", wv, qv, sv, kvd, H)
    MAT("self_attn.o_proj.weight", wo, qo, so, H, qd)
    MAT("mlp.gate_proj.weight", wg, qg, sg, I, H)
    MAT("mlp.up_proj.weight", wu, qu, su, I, H)
    MAT("mlp.down_proj.weight", wd, qd, sd, H, I)
#undef VEC
#undef MAT
    return -1;
}

int zo_model_set_tensor(ZoModel *m, const char *name, const float *data, size_t rows, size_t cols) {
    Slot s;
    if (find_slot(m, name, &s) != 0) return ZO_INVALID;
    if (s.vec) {
        if (rows * cols != s.rows) return ZO_SHAPE;
        memcpy(*s.vec, data, s.rows * 4);
        return ZO_OK;
    }
    if (rows != s.rows || cols != s.cols) return ZO_SHAPE;
    const int is_embed = (s.wt == &m->embed);
    if (m->wkind == ZO_W_Q8) return zo_pack_row_q8(data, rows, cols, *s.q, *s.s);
    if (is_embed) {
        memcpy(*s.wt, data, rows * cols * 4);
    } else {
        /* qwen_weights.zig:235-243: HF [out,in] -> [in,out] */
        float *dst = *s.wt;
        for (size_t r = 0; r < rows; r++)
            for (size_t c = 0; c < cols; c++) dst[c * rows + r] = data[r * cols + c];
    }
    return ZO_OK;
}

int zo_model_get_q8(const ZoModel *m, const char *name, int8_t *q, float *scale, size_t rows,
                    size_t cols) {
    Slot s;
    if (m->wkind != ZO_W_Q8) return ZO_INVALID;
    if (find_slot((ZoModel *)m, name, &s) != 0 || !s.q) return ZO_INVALID;
    if (rows != s.rows || cols != s.cols) return ZO_SHAPE;
    memcpy(q, *s.q, rows * cols);
    memcpy(scale, *s.s, rows * 4);
    return ZO_OK;
}

static const char *const kLayerNames[11] = {
    "input_layernorm.weight", "self_attn.q_norm.weight", "self_attn.k_norm.weight",
    "self_attn.q_proj.weight", "self_attn.k_proj.weight", "self_attn.v_proj.weight",
    "self_attn.o_proj.weight", "post_attention_layernorm.weight", "mlp.gate_proj.weight",
    "mlp.up_proj.weight", "mlp.down_proj.weight"};
static const int kLayerCodes[11] = {ZS_INPUT_LN, ZS_Q_NORM, ZS_K_NORM, ZS_WQ, ZS_WK, ZS_WV,
                                    ZS_WO, ZS_POST_LN, ZS_WG, ZS_WU, ZS_WD};

static void synth_tensor(float *buf, size_t n, uint64_t seed, uint64_t stream, int is_norm,
                         float w_std, float norm_std, int wkind) {
    if (is_norm) {
        if (norm_std == 0.0f) {
            for (size_t i = 0; i < n; i++) buf[i] = 1.0f;
        } else {
            zo_synth_normal(buf, n, seed, stream, norm_std);
            for (size_t i = 0; i < n; i++) buf[i] = 1.0f + buf[i];
        }
    } else {
        zo_synth_normal(buf, n, seed, stream, w_std);
    }
    if (wkind == ZO_W_BF16)
        for (size_t i = 0; i < n; i++) buf[i] = bf16_round(buf[i]);
}

ZoModel *zo_model_create_synthetic(const ZoArch *arch, int wkind, int kv_bf16, uint64_t seed,
                                   float w_std, float norm_std, int threads) {
    ZoModel *m = zo_model_create(arch, wkind, kv_bf16, threads);
    if (!m) return NULL;
    const size_t big = (size_t)arch->vocab * arch->hidden;
    float *buf = (float *)malloc(big * 4);
    if (!buf) { zo_model_destroy(m); return NULL; }
    synth_tensor(buf, big, seed, ZS_EMBED, 0, w_std, norm_std, wkind);
    zo_model_set_tensor(m, "model.embed_tokens.weight", buf, arch->vocab, arch->hidden);
    synth_tensor(buf, arch->hidden, seed, ZS_FINAL_NORM, 1, w_std, norm_std, wkind);
    zo_model_set_tensor(m, "model.norm.weight", buf, arch->hidden, 1);
    char name[160];
    for (uint32_t l = 0; l < arch->layers; l++) {
        for (int t = 0; t < 11; t++) {
            snprintf(name, sizeof(name), "model.layers.%u.%s", l, kLayerNames[t]);
            Slot s;
            find_slot(m, name, &s);
            const int is_norm = s.vec != NULL;
            const size_t n = s.rows * s.cols;
            synth_tensor(buf, n, seed, zs_layer_stream(l, (uint32_t)kLayerCodes[t]), is_norm, w_std,
                         norm_std, wkind);
            zo_model_set_tensor(m, name, buf, s.rows, s.cols);
        }
    }
    free(buf);
    return m;
}

ZoSession *zo_session_create(ZoModel *m, size_t max_seq) {
    const ZoArch *a = &m->a;
    if (max_seq == 0 || max_seq > a->max_pos) return NULL;
    ZoSession *s = (ZoSession *)zalloc(sizeof(ZoSession));
    s->m = m;
    s->max_seq = max_seq;
    const size_t H = a->hidden, I = a->inter, d = a->head_dim;
    const size_t qd = (size_t)a->n_q * d, kvd = (size_t)a->n_kv * d;
    s->kc = (float **)zalloc(sizeof(float *) * a->layers);
    s->vc = (float **)zalloc(sizeof(float *) * a->layers);
    for (uint32_t l = 0; l < a->layers; l++) {
        s->kc[l] = (float *)zalloc((size_t)a->n_kv * max_seq * d * 4);
        s->vc[l] = (float *)zalloc((size_t)a->n_kv * max_seq * d * 4);
    }
    s->xa = (float *)zalloc(max_seq * H * 4);
    s->xb = (float *)zalloc(max_seq * H * 4);
    s->xn = (float *)zalloc(max_seq * H * 4);
    s->q_lin = (float *)zalloc(max_seq * qd * 4);
    s->k_lin = (float *)zalloc(max_seq * kvd * 4);
    s->v_lin = (float *)zalloc(max_seq * kvd * 4);
    s->q_htd = (float *)zalloc(max_seq * qd * 4);
    s->k_htd = (float *)zalloc(max_seq * kvd * 4);
    s->v_htd = (float *)zalloc(max_seq * kvd * 4);
    s->attn_htd = (float *)zalloc(max_seq * qd * 4);
    s->attn_lin = (float *)zalloc(max_seq * qd * 4);
    s->ao = (float *)zalloc(max_seq * H * 4);
    s->x1 = (float *)zalloc(max_seq * H * 4);
    s->mlp_n = (float *)zalloc(max_seq * H * 4);
    s->gate = (float *)zalloc(max_seq * I * 4);
    s->up = (float *)zalloc(max_seq * I * 4);
    s->hact = (float *)zalloc(max_seq * I * 4);
    s->down = (float *)zalloc(max_seq * H * 4);
    s->scores = (float *)zalloc((size_t)m->threads * max_seq * 4 + 64 * max_seq * 4);
    s->normed = (float *)zalloc(H * 4);
    s->logits = (float *)zalloc((size_t)a->vocab * 4);
    return s;
}

void zo_session_destroy(ZoSession *s) {
    if (!s) return;
    for (uint32_t l = 0; l < s->m->a.layers; l++) { free(s->kc[l]); free(s->vc[l]); }
    free(s->kc); free(s->vc);
    free(s->xa); free(s->xb); free(s->xn); free(s->q_lin); free(s->k_lin); free(s->v_lin);
    free(s->q_htd); free(s->k_htd); free(s->v_htd); free(s->attn_htd); free(s->attn_lin);
    free(s->ao); free(s->x1); free(s->mlp_n); free(s->gate); free(s->up); free(s->hact);
    free(s->down); free(s->scores); free(s->normed); free(s->logits);
    free(s);
}

void zo_session_reset(ZoSession *s) { s->used = 0; } /* kv_cache.zig:41-43 */
size_t zo_session_used(const ZoSession *s) { return s->used; }

/* A linear layer y[t, out] = x[t, in] * W. F32/BF16: matmulF32 on the
 * transposed weight (qwen_block.zig:184). Q8 (extension): matvecQ8 per token
 * row on the HF-layout int8 weight (ops.zig:181-197). */
static void linear(const ZoModel *m, float *y, const float *x, size_t t, size_t in, size_t out,
                   const float *wt, const int8_t *q, const float *sc) {
    if (m->wkind == ZO_W_Q8) {
        for (size_t i = 0; i < t; i++) zo_matvec_q8(y + i * out, q, sc, x + i * in, out, in, 0, m->threads);
    } else {
        zo_matmul_f32(y, x, wt, t, out, in, m->threads);
    }
}

/* kv_cache.zig:49-73: append [n_kv, t, d] at `used`. With kv_bf16 (extension)
 * each value is rounded to bf16 first, the way a bf16 paged cache stores it. */
static void kv_append(ZoSession *s, uint32_t layer, const float *k_new, const float *v_new, size_t t) {
    const ZoArch *a = &s->m->a;
    const size_t d = a->head_dim;
    for (size_t h = 0; h < a->n_kv; h++) {
        for (size_t i = 0; i < t; i++) {
            float *kd = s->kc[layer] + (h * s->max_seq + s->used + i) * d;
            float *vd = s->vc[layer] + (h * s->max_seq + s->used + i) * d;
            const float *ks = k_new + (h * t + i) * d;
            const float *vs = v_new + (h * t + i) * d;
            if (s->m->kv_bf16) {
                for (size_t j = 0; j < d; j++) { kd[j] = bf16_round(ks[j]); vd[j] = bf16_round(vs[j]); }
            } else {
                memcpy(kd, ks, d * 4);
                memcpy(vd, vs, d * 4);
            }
        }
    }
}

/* qwen_block.zig:161-235 for one layer; `used` is advanced by the caller
 * after all layers (each layer's cache holds the same positions). */
static int block_forward(ZoSession *s, uint32_t layer, const float *x, size_t t, float *out) {
    const ZoModel *m = s->m;
    const ZoArch *a = &m->a;
    const ZoLayer *L = &m->layers[layer];
    const size_t H = a->hidden, I = a->inter, d = a->head_dim;
    const size_t n_q = a->n_q, n_kv = a->n_kv, qd = n_q * d, kvd = n_kv * d;
    const size_t pos0 = s->used;

    zo_rms_norm(s->xn, x, L->input_ln, t, H, a->eps);                      /* :179 */
    linear(m, s->q_lin, s->xn, t, H, qd, L->wq, L->qq, L->sq);              /* :184 */
    linear(m, s->k_lin, s->xn, t, H, kvd, L->wk, L->qk, L->sk);             /* :185 */
    linear(m, s->v_lin, s->xn, t, H, kvd, L->wv, L->qv, L->sv);             /* :186 */
    zo_rms_norm(s->q_lin, s->q_lin, L->q_norm, t * n_q, d, a->eps);         /* :191 */
    zo_rms_norm(s->k_lin, s->k_lin, L->k_norm, t * n_kv, d, a->eps);        /* :192 */
    zo_rope(s->q_lin, t, n_q, d, pos0, a->theta);                           /* :193 */
    zo_rope(s->k_lin, t, n_kv, d, pos0, a->theta);                          /* :194 */
    zo_tokens_heads_to_heads_tokens(s->q_htd, s->q_lin, t, n_q, d);         /* :199 */
    zo_tokens_heads_to_heads_tokens(s->k_htd, s->k_lin, t, n_kv, d);        /* :200 */
    zo_tokens_heads_to_heads_tokens(s->v_htd, s->v_lin, t, n_kv, d);        /* :201 */
    kv_append(s, layer, s->k_htd, s->v_htd, t);                             /* :203 */
    int rc = zo_attention_into(s->attn_htd, s->q_htd, s->kc[layer], s->vc[layer], n_q, t, d, n_kv,
                               pos0 + t, s->max_seq, s->scores, m->threads); /* :206-214 */
    if (rc) return rc;
    zo_heads_tokens_to_tokens_heads(s->attn_lin, s->attn_htd, n_q, t, d);   /* :217 */
    linear(m, s->ao, s->attn_lin, t, qd, H, L->wo, L->qo, L->so);           /* :221 */
    zo_add(s->x1, x, s->ao, t * H);                                         /* :223 */
    zo_rms_norm(s->mlp_n, s->x1, L->post_ln, t, H, a->eps);                 /* :226 */
    linear(m, s->gate, s->mlp_n, t, H, I, L->wg, L->qg, L->sg);             /* :231 */
    linear(m, s->up, s->mlp_n, t, H, I, L->wu, L->qu, L->su);               /* :232 */
    zo_silu_mul(s->hact, s->gate, s->up, t * I);                            /* :233 */
    linear(m, s->down, s->hact, t, I, H, L->wd, L->qd, L->sd);              /* :234 */
    zo_add(out, s->x1, s->down, t * H);                                     /* :235 */
    return ZO_OK;
}

/* qwen_forward.zig:163-175 (f32 tied head); Q8 extension: matvecQ8 over the
 * packed embedding. */
static void lm_head(const ZoModel *m, float *logits, const float *h) {
    const ZoArch *a = &m->a;
    const size_t V = a->vocab, H = a->hidden;
    if (m->wkind == ZO_W_Q8) {
        zo_matvec_q8(logits, m->embed_q, m->embed_s, h, V, H, 0, m->threads);
        return;
    }
    const long groups = (long)((V + 3) / 4);
#pragma omp parallel for schedule(static) num_threads(m->threads)
    for (long g = 0; g < groups; g++) {
        const size_t v0 = (size_t)g * 4;
        for (size_t v = v0; v < v0 + 4 && v < V; v++) {
            const float *row = m->embed + v * H;
            float dot = 0.0f;
            for (size_t i = 0; i < H; i++) dot += h[i] * row[i];
            logits[v] = dot;
        }
    }
}

int zo_session_forward(ZoSession *s, const uint32_t *ids, size_t t, float *logits,
                       float *dump_layers, float *dump_normed) {
    const ZoModel *m = s->m;
    const ZoArch *a = &m->a;
    const size_t H = a->hidden;
    if (t == 0 || t > s->max_seq - s->used) return ZO_INVALID; /* qwen_block.zig:175-176 */
    for (size_t i = 0; i < t; i++)
        if (ids[i] >= a->vocab) return ZO_INVALID;
    /* ops.zig:397-411 (Q8 extension: dequantised int8 row) */
    if (m->wkind == ZO_W_Q8) {
        for (size_t i = 0; i < t; i++) {
            const int8_t *qr = m->embed_q + (size_t)ids[i] * H;
            const float sc = m->embed_s[ids[i]];
            for (size_t c = 0; c < H; c++) s->xa[i * H + c] = (float)qr[c] * sc;
        }
    } else {
        zo_embedding_gather(s->xa, m->embed, a->vocab, H, ids, t);
    }
    float *in = s->xa, *out = s->xb;
    for (uint32_t l = 0; l < a->layers; l++) { /* qwen_forward.zig:121-143 */
        int rc = block_forward(s, l, in, t, out);
        if (rc) return rc;
        if (dump_layers) memcpy(dump_layers + (size_t)l * H, out + (t - 1) * H, H * 4);
        float *tmp = in; in = out; out = tmp;
    }
    s->used += t;
    zo_rms_norm(s->normed, in + (t - 1) * H, m->final_norm, 1, H, a->eps); /* :145-148 */
    if (dump_normed) memcpy(dump_normed, s->normed, H * 4);
    if (logits) lm_head(m, logits, s->normed);
    return ZO_OK;
}

int zo_session_block(ZoSession *s, uint32_t layer, const float *x, size_t t, float *out) {
    const ZoArch *a = &s->m->a;
    if (layer >= a->layers) return ZO_INVALID;
    if (t == 0 || t > s->max_seq - s->used) return ZO_INVALID; /* qwen_block.zig:175-176 */
    int rc = block_forward(s, layer, x, t, out);
    if (rc) return rc;
    s->used += t;
    return ZO_OK;
}

int zo_prefill_last_logits(ZoSession *s, const uint32_t *ids, size_t t, float *logits) {
    zo_session_reset(s);
    return zo_session_forward(s, ids, t, logits, NULL, NULL);
}

int zo_greedy_decode(ZoSession *s, uint32_t first, size_t n_steps, const uint32_t *teacher,
                     uint32_t *out_ids, float *logits_out) {
    const size_t V = s->m->a.vocab;
    uint32_t tok = first;
    for (size_t i = 0; i < n_steps; i++) {
        int rc = zo_session_forward(s, &tok, 1, s->logits, NULL, NULL);
        if (rc) return rc;
        if (logits_out) memcpy(logits_out + i * V, s->logits, V * 4);
        uint32_t id;
        float val;
        zo_top_k(s->logits, V, 1, &id, &val);
        out_ids[i] = id;
        tok = teacher ? teacher[i] : id;
    }
    return ZO_OK;
}

int zo_session_fill_kv(ZoSession *s, size_t n, uint64_t seed) {
    const ZoArch *a = &s->m->a;
    if (n > s->max_seq) return ZO_INVALID;
    const size_t d = a->head_dim;
    /* every (layer, K|V) plane is independent: threads split them, values unchanged */
#pragma omp parallel for schedule(dynamic, 1) num_threads(s->m->threads)
    for (int lw = 0; lw < (int)(2 * a->layers); lw++) {
        const uint32_t l = (uint32_t)lw / 2;
        const int which = lw % 2;
        {
            const uint64_t key = zs_key(seed, zs_layer_stream(l, (uint32_t)(100 + which)));
            const float k = (float)(1.0 / ZS_IH4_SIGMA);
            float *dst = which ? s->vc[l] : s->kc[l];
            for (size_t h = 0; h < a->n_kv; h++)
                for (size_t p = 0; p < n; p++)
                    for (size_t j = 0; j < d; j++) {
                        const float v = zs_normal(key, (h * n + p) * d + j, k);
                        dst[(h * s->max_seq + p) * d + j] = s->m->kv_bf16 ? bf16_round(v) : v;
                    }
        }
    }
    s->used = n;
    return ZO_OK;
}

int zo_session_kv(const ZoSession *s, uint32_t layer, int which_v, float *out) {
    const ZoArch *a = &s->m->a;
    if (layer >= a->layers) return ZO_INVALID;
    const size_t d = a->head_dim;
    const float *src = which_v ? s->vc[layer] : s->kc[layer];
    for (size_t h = 0; h < a->n_kv; h++)
        memcpy(out + h * s->used * d, src + h * s->max_seq * d, s->used * d * 4);
    return ZO_OK;
}
