/* zynfer_cuda.h: C ABI of the Zynfer `cuda` backend (libzynfer_cuda.so, sm_100a).
 *
 * Pure C99 so that Zig's @cImport, ctypes, cgo and JNI can bind it. It plays
 * the role the Apple bridge plays for the `apple` backend
 * (src/backends/apple/bridge.h:11-99 in the reference): opaque handles, an int
 * status with 0 = OK, a per-handle last-error string, and one single-owner
 * context per device per thread.
 *
 * Citations name the reference function each entry point replaces
 * (file:line within the Zynfer reference project).
 *
 * Ownership: the context owns all device memory (weights, paged KV pool,
 * scratch, graphs). Host pointers passed in are borrowed for the duration of
 * the call; output arrays are caller-allocated. zynfer_cu_decode_step and
 * zynfer_cu_generate allocate no memory (device or host) after
 * zynfer_cu_model_init.
 *
 * Threading: a context is not internally synchronised; use one per owner
 * thread (bridge.h:37-43). Several contexts may run on different devices
 * (one per GPU, one process or thread each) without any collective.
 *
 * Errors: every function returns a status; no exception, abort, assert or
 * device trap crosses the ABI. Device-side failures (a bounded wait that ran
 * out, an out-of-range index) raise a device error word that the next
 * synchronising call turns into a status.
 *
 * Fault injection (host side, for tests of the error paths): the environment
 * variable ZYNFER_CUDA_FAIL_AT, or zynfer_cu_set_fail_at, takes
 * "alloc:N" (the N-th device allocation after the call fails with OOM),
 * "upload" (the next weight upload fails with INTERNAL), "launch" (the next
 * call that would launch kernels fails with LAUNCH before launching any) or
 * "wait" (the next "persistent" decode step of a model with two or more
 * layers polls one input with a tag that nothing writes: its bounded device
 * wait runs out after a few seconds, every CTA stops, and the call returns
 * TIMEOUT with the context still usable). zynfer_cu_set_fail_at(NULL, "wait")
 * arms the same for the next zynfer_cu_linear_q8_static call, which has no
 * context: none of its CTAs loads the first K stage, its bounded waits run
 * out, and zynfer_cu_linear_q8_static_status reports TIMEOUT.
 */
#ifndef ZYNFER_CUDA_H
#define ZYNFER_CUDA_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define ZYNFER_CU_API __attribute__((visibility("default")))
#else
#define ZYNFER_CU_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef struct ZynferCuCtx ZynferCuCtx;

/* Status codes (bridge.h:14-23 pattern). */
enum {
    ZYNFER_CU_OK = 0,
    ZYNFER_CU_NO_DEVICE = 1,
    ZYNFER_CU_OOM = 2,
    ZYNFER_CU_INVALID = 3,
    ZYNFER_CU_UNSUPPORTED = 4,
    ZYNFER_CU_LAUNCH = 5,
    ZYNFER_CU_TIMEOUT = 6,
    ZYNFER_CU_INTERNAL = 7
};

/* Weight storage of a model. */
enum {
    ZYNFER_CU_W_Q8 = 0,   /* int8 per-output-row + f32 scale (packRowQ8, src/backends/cpu/ops.zig:145-162) */
    ZYNFER_CU_W_BF16 = 1  /* bf16 as stored in a checkpoint (src/runtime/bf16.zig:6-19) */
};

/* Stable capability record (bridge.h:25-35, hip_probe.h:10-35 pattern). */
typedef struct ZynferCuCaps {
    char device_name[256];
    int sm_major, sm_minor;
    int sm_count;
    uint64_t hbm_bytes;
    uint64_t l2_bytes;
    uint32_t max_smem_per_block;
    int bulk_copy;       /* cp.async.bulk + mbarrier path usable (sm_90+) */
    int tcgen05;         /* sm_100a tensor-core (tcgen05/TMEM) path usable */
} ZynferCuCaps;

/* Architecture and runtime sizing. Architecture fields follow Arch
 * (src/model/qwen3.zig:36-59). */
typedef struct ZynferCuModelDesc {
    uint32_t vocab, hidden, inter, layers, n_q, n_kv, head_dim, max_pos;
    float eps, theta;
    uint32_t weights;         /* ZYNFER_CU_W_Q8 or ZYNFER_CU_W_BF16 */
    uint32_t max_batch;       /* sequences per decode step */
    uint32_t max_seqs;        /* sequence slots (ids 0 .. max_seqs-1) */
    uint32_t max_seq_len;     /* positions per sequence (KvCache max_seq, kv_cache.zig:14-33) */
    uint32_t kv_blocks;       /* paged pool size in 16-token blocks; 0 = enough for every slot */
    uint32_t max_prefill;     /* tokens per zynfer_cu_prefill call */
    uint32_t prefill_kv_f32;  /* 1: prefill attention reads unrounded f32 K/V (the f32
                                 reference path); 0: the bf16 values the cache stores */
} ZynferCuModelDesc;

/* ---- context (bridge.h:44-48) ---- */
ZYNFER_CU_API int zynfer_cu_create(int device, ZynferCuCtx **out);
ZYNFER_CU_API void zynfer_cu_destroy(ZynferCuCtx *ctx);
ZYNFER_CU_API int zynfer_cu_caps(const ZynferCuCtx *ctx, ZynferCuCaps *out);
ZYNFER_CU_API const char *zynfer_cu_last_error(const ZynferCuCtx *ctx);
ZYNFER_CU_API int zynfer_cu_sync(ZynferCuCtx *ctx);
ZYNFER_CU_API int zynfer_cu_set_fail_at(ZynferCuCtx *ctx, const char *spec);
/* Label of the last executed path, e.g. "decode:gemv:graph" (block.zig:20-25 counters). */
ZYNFER_CU_API const char *zynfer_cu_last_path(const ZynferCuCtx *ctx);
/* Library build identity (sm target, version). */
ZYNFER_CU_API const char *zynfer_cu_build_info(void);

/* ---- model and weights (qwen_forward.Session.init, qwen_forward.zig:32-71;
 *      Weights.load, qwen_weights.zig:61-175) ---- */
ZYNFER_CU_API int zynfer_cu_model_init(ZynferCuCtx *ctx, const ZynferCuModelDesc *desc);
/* Upload one tensor by its HF name (qwen3.zig:86-132) in HF layout [out, in].
 * f32 data is packed on the device (int8 models, bit-exact packRowQ8) or
 * rounded to bf16 (bf16 models). */
ZYNFER_CU_API int zynfer_cu_upload_f32(ZynferCuCtx *ctx, const char *name, const float *data, uint64_t rows,
                         uint64_t cols);
ZYNFER_CU_API int zynfer_cu_upload_bf16(ZynferCuCtx *ctx, const char *name, const uint16_t *data, uint64_t rows,
                          uint64_t cols);
ZYNFER_CU_API int zynfer_cu_upload_q8(ZynferCuCtx *ctx, const char *name, const int8_t *q, const float *scale,
                        uint64_t rows, uint64_t cols);
/* Generate every tensor on the device from the seeded synthetic generator:
 * linears and embedding ~ normal(0, w_std), norm weights 1 + normal(0, norm_std). */
ZYNFER_CU_API int zynfer_cu_fill_synthetic(ZynferCuCtx *ctx, uint64_t seed, float w_std, float norm_std);
/* Read back a packed int8 tensor (int8 models) in HF layout. */
ZYNFER_CU_API int zynfer_cu_download_q8(ZynferCuCtx *ctx, const char *name, int8_t *q, float *scale, uint64_t rows,
                          uint64_t cols);

/* ---- .zynfer artifacts (src/model/artifact.zig) ----
 * The reference's file format (artifact.zig:42-66: 88-byte header, 116-byte
 * model record, 120-byte tensor entries, 64-byte-aligned payload, SHA-256 of
 * the file) with one addition in format version 2: dtype 3 = int8, whose
 * packRowQ8 row scales are the f32 tensor "<name>.scale" [rows]. Version-1
 * files (f32 / f16 / bf16) load unchanged. */
typedef struct ZynferCuArtifact ZynferCuArtifact;
enum { ZYNFER_CU_DT_F32 = 0, ZYNFER_CU_DT_F16 = 1, ZYNFER_CU_DT_BF16 = 2, ZYNFER_CU_DT_I8 = 3 };
typedef struct ZynferCuArtifactMeta {   /* Meta (artifact.zig:68-99) */
    char model_id[64];
    uint32_t format_version;
    uint32_t vocab, hidden, inter, layers, n_q, n_kv, head_dim, max_pos, bos, eos;
    float rope_theta, rms_norm_eps;
    uint32_t tie_word_embeddings;
    uint32_t tensor_count;
    uint64_t file_bytes;
} ZynferCuArtifactMeta;
typedef struct ZynferCuTensorInfo {     /* TensorEntry (artifact.zig:124-150) */
    char name[64];
    uint32_t tensor_id, dtype, rank;
    uint32_t shape[8];
    uint64_t nbytes;
    const void *data;                   /* inside the mapped file, valid until close */
} ZynferCuTensorInfo;
/* Artifact.loadFile (artifact.zig:394-433) + validate (artifact.zig:487-532):
 * maps the file read-only and checks it in the reference's order. *out is set
 * even on failure, to a handle whose zynfer_cu_artifact_error names the
 * reference's error (InvalidMagic, UnsupportedVersion, BadEndian, BadHeader,
 * BadAlignment, Truncated, ChecksumMismatch, InvalidRank, InvalidDtype,
 * InvalidName, DuplicateTensorId, Overflow for files over 4 GiB); close it
 * either way. Needs no GPU. */
ZYNFER_CU_API int zynfer_cu_artifact_open(const char *path, ZynferCuArtifact **out);
ZYNFER_CU_API void zynfer_cu_artifact_close(ZynferCuArtifact *art);
ZYNFER_CU_API const char *zynfer_cu_artifact_error(const ZynferCuArtifact *art);
ZYNFER_CU_API int zynfer_cu_artifact_meta(const ZynferCuArtifact *art, ZynferCuArtifactMeta *out);
/* Directory entry `index` (0 .. tensor_count - 1). */
ZYNFER_CU_API int zynfer_cu_artifact_tensor(const ZynferCuArtifact *art, uint32_t index, ZynferCuTensorInfo *out);
/* Artifact.findById (artifact.zig:449-458) and findByName (:466-471). */
ZYNFER_CU_API int zynfer_cu_artifact_find_id(const ZynferCuArtifact *art, uint32_t tensor_id, ZynferCuTensorInfo *out);
ZYNFER_CU_API int zynfer_cu_artifact_find_name(const ZynferCuArtifact *art, const char *name, ZynferCuTensorInfo *out);
/* Meta.toArch (artifact.zig:101-121): the architecture fields of a model
 * descriptor (vocab .. theta); the runtime sizing fields are left as they are. */
ZYNFER_CU_API int zynfer_cu_model_desc_from_artifact(const ZynferCuArtifact *art, ZynferCuModelDesc *desc);
/* Weights.load (qwen_weights.zig:61-175) onto the device: every tensor of an
 * initialised model of the artifact's architecture, by HF name, from the
 * mapping (f32 and bf16 through zynfer_cu_upload_f32 / _bf16, int8 with its
 * scales through zynfer_cu_upload_q8). A missing tensor is INVALID
 * ("TensorNotFound: <name>"), f16 INVALID ("InvalidDtype"), an untied LM head
 * UNSUPPORTED. */
ZYNFER_CU_API int zynfer_cu_load_artifact(ZynferCuCtx *ctx, const ZynferCuArtifact *art);

/* ---- sequences (KvCache.reset/used, kv_cache.zig:41-47) ---- */
ZYNFER_CU_API int zynfer_cu_seq_reset(ZynferCuCtx *ctx, uint32_t seq);
ZYNFER_CU_API int zynfer_cu_seq_len(const ZynferCuCtx *ctx, uint32_t seq, uint32_t *len);
/* K or V of one layer for positions [0, len): out [n_kv][len][head_dim] f32. */
ZYNFER_CU_API int zynfer_cu_kv_read(ZynferCuCtx *ctx, uint32_t seq, uint32_t layer, int which_v, float *out);
/* Seeded stand-in for a prefill, for test and benchmark workloads at long
 * contexts: resets `seq` and fills its cache, every layer, positions [0, n),
 * then sets its length to n. K (code 100) and V (code 101) of layer l use
 * the generator of synth_rng.h with key(seed, ((l + 1) << 8) | code); the
 * element (kv head h, position p, dim j) is bf16(normal(key, (h n + p) d + j,
 * std 1)). A CPU restatement that fills a dense KvCache (kv_cache.zig:14-33)
 * the same way holds bit-identical K/V. */
ZYNFER_CU_API int zynfer_cu_kv_fill_synthetic(ZynferCuCtx *ctx, uint32_t seq, uint32_t n, uint64_t seed);

/* Prefix reuse over the paged pool (no counterpart in the reference; its
 * roadmap's Stage 22, docs/roadmap.md:39, names it): `dst` (reset first)
 * becomes a sequence of the first n positions of `src`. Whole 16-token
 * blocks are shared, counted per block and returned to the pool when the last
 * sequence holding them is reset; only a partly filled last block is copied,
 * because it is the one `dst` appends into next. Appends only ever write
 * positions at or past a sequence's length, so no shared block is written
 * again. n <= the length of src. */
ZYNFER_CU_API int zynfer_cu_seq_fork(ZynferCuCtx *ctx, uint32_t dst, uint32_t src, uint32_t n);
/* Append n tokens to `seq` (decode steps of one row, from position = its
 * length): what follows a shared prefix. last_logits [vocab] (of the last
 * token) and argmax may be NULL. */
ZYNFER_CU_API int zynfer_cu_extend(ZynferCuCtx *ctx, uint32_t seq, const uint32_t *tokens, uint32_t n,
                                   float *last_logits, uint32_t *argmax);
/* Free pool blocks and blocks held by more than one sequence. */
ZYNFER_CU_API int zynfer_cu_pool_stats(const ZynferCuCtx *ctx, uint32_t *free_blocks, uint32_t *shared_blocks);

/* ---- forward ---- */
/* Session.prefillLastLogits (qwen_forward.zig:89-160): resets `seq`, runs the
 * n prompt tokens through all layers, then the final norm and tied LM head on
 * the last row. last_logits [vocab] and argmax may be NULL. */
ZYNFER_CU_API int zynfer_cu_prefill(ZynferCuCtx *ctx, uint32_t seq, const uint32_t *tokens, uint32_t n,
                      float *last_logits, uint32_t *argmax);
/* One greedy decode step for `batch` sequences (block-level decode,
 * qwen_block.zig:161-235 with t = 1 at pos0 = used, for every layer): feeds
 * tokens[i] to seqs[i], appends its K/V, and returns the argmax of the new
 * logits (lowest index on ties, topK qwen_forward.zig:177-193). logits
 * [batch][vocab] may be NULL. Host buffers; copies are part of the call. */
ZYNFER_CU_API int zynfer_cu_decode_step(ZynferCuCtx *ctx, const uint32_t *seqs, const uint32_t *tokens,
                          uint32_t batch, uint32_t *argmax, float *logits);
/* `steps` greedy steps kept on the device (each step's argmax is the next
 * step's input). out_ids [steps][batch]; device_ms (nullable) receives the
 * CUDA-event time of the steps on the context stream. */
ZYNFER_CU_API int zynfer_cu_generate(ZynferCuCtx *ctx, const uint32_t *seqs, const uint32_t *first,
                       uint32_t batch, uint32_t steps, uint32_t *out_ids, float *device_ms);
/* Next-token rule of zynfer_cu_decode_step, zynfer_cu_generate and the token
 * zynfer_cu_prefill returns (no counterpart in the reference, which decodes
 * greedily with topK, qwen_forward.zig:177-193; its roadmap's Stage 12,
 * docs/roadmap.md:29, names sampling without specifying it).
 * temperature 0 (the default): greedy, the argmax. temperature > 0: temperature
 * only (top_k 0, top_p 1) draws from softmax(logits / temperature) exactly
 * (Gumbel-max); otherwise the top_k (1..64; 0 = 64) largest logits, their
 * softmax at that temperature summed in descending order, cut to the shortest
 * prefix whose sum reaches top_p (0 < top_p <= 1) of the total, and one draw
 * from that prefix. Draws come from the counter generator of synth_rng.h keyed
 * by (seed, sequence slot) at the position of the step's input token, so a
 * sequence's tokens do not depend on its batch neighbours. Logits are
 * written to device memory whenever sampling is on; the persistent schedule
 * is not used while it is. Rebuilds the decode graphs on the next step. */
ZYNFER_CU_API int zynfer_cu_set_sampling(ZynferCuCtx *ctx, float temperature, uint32_t top_k, float top_p,
                                         uint64_t seed);
/* The same rule on caller-owned device logits [rows][vocab] (rows <= the
 * model's max_batch): slots[i] and positions[i] (host) key row i's draws;
 * out_ids (host) receives one id per row. temperature > 0. Synchronises. */
ZYNFER_CU_API int zynfer_cu_sample(ZynferCuCtx *ctx, const float *logits, uint32_t rows, uint32_t vocab,
                                   const uint32_t *slots, const uint32_t *positions, float temperature,
                                   uint32_t top_k, float top_p, uint64_t seed, uint32_t *out_ids);
/* One transformer block (qwen_block.forward, qwen_block.zig:161-235) of layer
 * `layer` on host hidden states x [t][hidden] at pos0 = the sequence's length;
 * out [t][hidden]. Appends to the sequence's cache for that layer. */
ZYNFER_CU_API int zynfer_cu_block_forward(ZynferCuCtx *ctx, uint32_t layer, uint32_t seq, const float *x,
                            uint32_t t, float *out);

/* ---- op level (device pointers; run on the context stream) ---- */
/* matvecQ8 / matmul over `batch` rows (ops.zig:181-197): y[b][m] = (W[m,:] . x[b,:]) * scale[m].
 * w and x must be 16-byte aligned and y 8-byte aligned. */
ZYNFER_CU_API int zynfer_cu_linear(ZynferCuCtx *ctx, int wkind, const void *w, const float *scale,
                     const float *x, uint32_t batch, uint32_t m, uint32_t k, float *y);
/* Kernel family for linear layers: "auto" (model schedules and zynfer_cu_linear:
 * the CUDA-core GEMV for one activation row, the few-row integer-MMA kernel for
 * 2..6 int8 rows (2..8 when k <= 1024), each up to 16384 outputs; tcgen05
 * tensor cores otherwise),
 * "gemv", "mma" (int8, 2..8 rows of k <= 3072 or 9..16 rows of k <= 1024; its
 * results equal the tcgen05 path's bit for bit), "tcgen05", or "simt" (the CUDA-core tiled GEMM, kept for
 * comparisons). A family that cannot take a call falls back to tcgen05.
 * Applies to later calls of this context. */
ZYNFER_CU_API int zynfer_cu_set_linear_path(ZynferCuCtx *ctx, const char *path);
/* Decode schedule for zynfer_cu_decode_step / zynfer_cu_generate: "kernels"
 * (one kernel per op, captured in a CUDA graph per batch size), "persistent"
 * (the whole step as one cooperative dataflow kernel: weights and KV blocks
 * streamed into shared memory ahead of the layer chain, tagged activations
 * instead of grid barriers; int8 models of hidden 1024, intermediate 3072,
 * 16 x 128 query and 8 x 128 kv dims, at most 62 layers, batch <= 8;
 * ZYNFER_CU_UNSUPPORTED otherwise), or "auto" (= "kernels", measured faster
 * at every batch size). Both follow qwen_block.forward (qwen_block.zig:161-235) per layer
 * and qwen_forward's tied LM head + topK(1) (qwen_forward.zig:163-193). */
ZYNFER_CU_API int zynfer_cu_set_decode_schedule(ZynferCuCtx *ctx, const char *schedule);
/* Allocation-free int8 linear (no counterpart in the reference; an addition
 * of this backend). Same result as zynfer_cu_linear with ZYNFER_CU_W_Q8:
 * y[b][i] = (W[i,:] . x[b,:]) * scale[i], computed on the tcgen05 path, for
 * callers that cannot call cudaMalloc: an embedding application that owns
 * every device allocation, a custom allocator that must not be bypassed, or
 * code running where allocation is forbidden. It takes no context and calls
 * no cudaMalloc, cudaFree or allocating library routine; all pointers are
 * caller-owned device memory and `stream` is a cudaStream_t (NULL = the
 * default stream). Its only scratch (the activations' int8 digit planes and
 * row scales, 768 KiB) is a file-scope device array that every GPU loading
 * the library holds until the process exits.
 * Limits: batch <= ZYNFER_CU_STATIC_MAX_ROWS, k <= ZYNFER_CU_STATIC_MAX_K,
 * k and m multiples of 128, m < 2^31, x 16-byte aligned, y and scale 4-byte
 * aligned; otherwise ZYNFER_CU_INVALID.
 * The first call on a device resolves the array's device address and sets
 * kernel attributes on that device; make it before any stream capture. All
 * calls share the array, so calls that overlap on the GPU (other streams,
 * other threads) race: serialise them. The return value covers the launch
 * only: the kernel's bounded device waits report through a device error word
 * that is also a file-scope array, read by zynfer_cu_linear_q8_static_status
 * after the caller has synchronised its stream. */
#define ZYNFER_CU_STATIC_MAX_ROWS 64
#define ZYNFER_CU_STATIC_MAX_K 4096
ZYNFER_CU_API int zynfer_cu_linear_q8_static(const int8_t *w, const float *scale, const float *x,
                                             uint32_t batch, uint32_t m, uint32_t k, float *y, void *stream);
/* Device error word of zynfer_cu_linear_q8_static on the current device
 * (no counterpart in the reference): ZYNFER_CU_OK when every call since the
 * last clear finished its waits, ZYNFER_CU_TIMEOUT when one ran out (that
 * call's y is not valid). clear != 0 resets the word. Synchronous (plain
 * cudaMemcpy of 4 bytes, nothing allocated); call it after synchronising the
 * stream of the calls it covers. */
ZYNFER_CU_API int zynfer_cu_linear_q8_static_status(int clear);
/* attentionInto (ops.zig:285-354) for one decode token per sequence, the
 * kernel the decode step runs for layer `layer`: qkv [batch][(n_q + 2 n_kv)
 * head_dim] holds each row's raw q, k, v projections (device); the kernel
 * applies the layer's per-head RMSNorm to q and k and split-half RoPE at
 * position p = the sequence's length (qwen_block.zig:190-194, ops.zig:233-261),
 * writes this token's K/V (bf16) into the sequence's paged cache of that layer
 * at p, and attends over the p + 1 cached positions with a log-sum-exp merge of
 * its KV splits. out [batch][n_q][head_dim] (device). The sequence's length is
 * not advanced (the decode step does that once for all layers), so a repeated
 * call rewrites the same position. seqs is a host array of distinct slots;
 * qkv and out 16-byte aligned. Synchronises; device-side index checks return
 * INVALID. */
ZYNFER_CU_API int zynfer_cu_attn_decode(ZynferCuCtx *ctx, uint32_t layer, const uint32_t *seqs, uint32_t batch,
                                        const float *qkv, float *out);
/* Per-head RMSNorm (ops.zig:49-67 with the q_norm / k_norm weights,
 * qwen_block.zig:190-191) and split-half RoPE (ops.zig:233-261) of `rows`
 * tokens at positions pos0 .. pos0 + rows - 1, from the fused projection rows
 * qkv [rows][(n_q + 2 n_kv) head_dim] (device). q_out [n_q][rows][head_dim] and
 * k_out [n_kv][rows][head_dim] are heads-major, the layout attentionInto takes
 * (tokensHeadsToHeadsTokens, ops.zig:355-373). Needs the model's RoPE table:
 * pos0 + rows <= max_seq_len. Synchronises. */
ZYNFER_CU_API int zynfer_cu_rmsnorm_qk_rope(ZynferCuCtx *ctx, const float *qkv, uint32_t rows, const float *q_norm,
                                            const float *k_norm, uint32_t pos0, float *q_out, float *k_out);
/* siluMul (ops.zig:36-42): out[i] = silu(gate[i]) * up[i], device pointers,
 * the arithmetic of every SwiGLU epilogue. */
ZYNFER_CU_API int zynfer_cu_swiglu(ZynferCuCtx *ctx, const float *gate, const float *up, uint64_t n, float *out);
/* packRowQ8 (ops.zig:145-162) on the device, bit-exact. */
ZYNFER_CU_API int zynfer_cu_pack_q8(ZynferCuCtx *ctx, const float *w, uint32_t rows, uint32_t cols, int8_t *q,
                      float *scale);
/* rmsNorm (ops.zig:49-67) over rows. */
ZYNFER_CU_API int zynfer_cu_rmsnorm(ZynferCuCtx *ctx, const float *x, const float *w, uint32_t rows, uint32_t cols,
                      float eps, float *y);

/* ---- timing (signpost intervals, bridge.h:94-99) ---- */
/* Per-kernel-class CUDA-event timing of decode steps (eager launches while on). */
ZYNFER_CU_API int zynfer_cu_set_timing(ZynferCuCtx *ctx, int enable);
enum { ZYNFER_CU_K_ATTN = 0, ZYNFER_CU_K_LINEAR = 1, ZYNFER_CU_K_LMHEAD = 2, ZYNFER_CU_K_OTHER = 3 };
ZYNFER_CU_API int zynfer_cu_kernel_time(const ZynferCuCtx *ctx, int kernel_class, uint64_t *launches, double *total_ms);
ZYNFER_CU_API uint64_t zynfer_cu_last_step_ns(const ZynferCuCtx *ctx);
/* Phase timestamps of the last persistent decode step run with timing on
 * (signpost intervals, src/backends/apple/gpu.zig:91-106 pattern): globaltimer
 * ns as seen by CTA 0: [0] start, then (start, end) per phase (QKV, ATT, O,
 * GU, D per layer, then the LM head), then the finish. Copies up to `cap`
 * entries into out and returns how many exist (0 when there is no trace). */
ZYNFER_CU_API int zynfer_cu_phase_trace(const ZynferCuCtx *ctx, uint64_t *out, int cap);
/* Kernels one decode step enqueues (the last one built). */
ZYNFER_CU_API int zynfer_cu_step_launches(const ZynferCuCtx *ctx);
/* Host->device and device->host bytes copied by decode/generate/prefill calls
 * since the last reset (reset != 0 clears after reading). */
ZYNFER_CU_API int zynfer_cu_io_bytes(ZynferCuCtx *ctx, uint64_t *h2d, uint64_t *d2h, int reset);
/* Allocation events since zynfer_cu_model_init ("decode does not allocate",
 * tiny_block.zig:385-401): device = device allocations (cudaMalloc, CUDA
 * graph instantiation), host = growths of host containers past their
 * reserved capacity. The first decode of a batch size captures its graph
 * (one event of each); later decode steps and generate calls of that batch
 * size add none. */
ZYNFER_CU_API int zynfer_cu_alloc_events(const ZynferCuCtx *ctx, uint64_t *device, uint64_t *host);

#ifdef __cplusplus
}
#endif

#endif
