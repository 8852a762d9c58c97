// Host-side launchers for the sm_100a kernels (internal to libzynfer_cuda).
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace zc {

enum WKind : int { kWQ8 = 0, kWBF16 = 1 };

// A byte range of a later kernel's weights to bring into L2 (p null: none).
struct L2Range {
    const void* p;
    uint32_t bytes;
};

// Linear-layer epilogues.
enum Epi : int {
    kEpiNone = 0,     // y = acc * scale
    kEpiResid = 1,    // y = resid + acc * scale
    kEpiSwiGLU = 2,   // rows (2j, 2j+1) = (gate_j, up_j): y[j] = silu(g) * u
    kEpiArgmax = 3,   // optional logits write + argmax key per batch row
};

struct LinearArgs {
    const void* w = nullptr;       // [M][K] int8 or bf16, row-major (HF [out, in])
    const float* scale = nullptr;  // [M] (int8) or nullptr (bf16)
    int wkind = kWQ8;
    int M = 0, K = 0;
    const float* x = nullptr;      // [N][ldx] f32 activations
    int ldx = 0;
    int N = 0;                     // batch rows (tokens / sequences)
    float* y = nullptr;            // [N][ldy] f32 output
    int ldy = 0;
    int epi = kEpiNone;
    const float* resid = nullptr;  // [N][ldy] for kEpiResid (may alias y)
    const float* norm_w = nullptr; // optional RMSNorm applied to x rows first (GEMV only)
    float eps = 1e-6f;
    unsigned long long* argmax_keys = nullptr;  // [N] for kEpiArgmax
    uint32_t* err = nullptr;       // device error word (bounded waits)
    L2Range pf[2] = {};            // the next linear's weights and scales, prefetched into L2
};

// synth.cu
int device_sm_count();  // SMs of the current device (cached)
void configure_kernel(const void* func, size_t dyn_smem);  // once per device, before any launch
void prepare_all_kernels();  // configure every kernel of the library on the current device
void prepare_norm_kernels();
void prepare_gemv_kernels();
void prepare_gemm_simt_kernels();
void prepare_attn_kernels();
void prepare_persistent_kernels();
void prepare_tc_kernels();
void launch_synth_normal(float* out, size_t n, uint64_t seed, uint64_t stream, float k,
                         float add, cudaStream_t st);
void launch_fill(float* out, size_t n, float v, cudaStream_t st);
void launch_pack_q8_rows(const float* w, int rows, int cols, int8_t* q, float* scale,
                         int dst_stride, int dst_offset, cudaStream_t st);
void launch_to_bf16_rows(const float* w, int rows, int cols, uint16_t* out, int dst_stride,
                         int dst_offset, cudaStream_t st);
void launch_copy_rows_i8(const int8_t* src, const float* ssrc, int rows, int cols, int8_t* dst,
                         float* sdst, int dst_stride, int dst_offset, cudaStream_t st);
void launch_copy_rows_u16(const uint16_t* src, int rows, int cols, uint16_t* dst, int dst_stride,
                          int dst_offset, cudaStream_t st);
void launch_unpack_rows_i8(const int8_t* src, const float* ssrc, int rows, int cols, int8_t* dst,
                           float* sdst, int src_stride, int src_offset, cudaStream_t st);
// Seeded stand-in cache of one sequence (positions [0, n) of every layer);
// table_row = that sequence's device block-table row.
void launch_kv_fill(uint16_t* kv, size_t kv_layer_elems, const int* table_row, int n_pool_blocks, int layers,
                    int n_kv, int n, uint64_t seed, uint32_t* err, cudaStream_t st);

// norm.cu
void launch_rmsnorm(const float* x, const float* w, float* y, int rows, int cols, float eps,
                    cudaStream_t st);
void launch_embed(const void* table, const float* scale, int wkind, const uint32_t* ids, int n,
                  int H, int V, float* x, uint32_t* err, cudaStream_t st);
struct QkvArgs {
    const float* qkv;  // [T][ (n_q + 2 n_kv) * d ]
    int T, n_q, n_kv, d;
    const float* q_norm;
    const float* k_norm;
    float eps;
    const float2* rope;  // [max_pos][d/2] (cos, sin)
    int rope_max_pos;
    // positions: row_pos[t] (nullable -> pos0 + t); sequences: row_seq[t] (nullable -> seq0)
    const int* row_pos;
    int pos0;
    const int* row_seq;
    int seq0;
    // paged bf16 cache (nullable: then k and v go only to the staging buffers)
    uint16_t* kv_layer;         // this layer's pool base: [n_kv][blocks][K, V][16][d], kv_swizzle rows
    const int* block_table;     // [seqs][max_blocks]
    int max_blocks;
    int n_pool_blocks;
    // outputs
    float* q_out;          // decode: [T][n_q][d]; prefill: heads-major [n_q][T][d]
    int q_heads_major;
    float* k_stage;        // nullable: [n_kv][T][d] f32 (the op-level entry point)
    float* v_stage;
    int stage_round_bf16;  // staged K/V rounded to bf16 (the values the cache holds)
    // prefill (nullable): K and V as bf16 terms for the tensor-core attention,
    // [4][n_kv][T][d] = K hi, K lo, V hi, V lo with x = hi + lo to 2^-18
    // relative (lo is zero when stage_round_bf16)
    uint16_t* kv_planes;
    uint32_t* err;
};
void launch_qkv_post(const QkvArgs& a, cudaStream_t st);
struct FinalizeArgs {
    unsigned long long* keys;  // [B], reset to 0 after reading
    uint32_t* ids_out;         // [B] argmax ids
    uint32_t* next_tokens;     // [B] (nullable) next step's input ids
    int* positions;            // [B] (nullable) incremented by one
    uint32_t* history;         // (nullable) [steps][B]; row = *step, then *step += 1
    int* step;
    int B;                     // <= 1024 (one CTA)
};
void launch_bf16_to_f32(const uint16_t* src, size_t n, float* dst, cudaStream_t st);
void launch_silu_mul(const float* g, const float* u, size_t n, float* o, cudaStream_t st);
void launch_finalize(const FinalizeArgs& a, cudaStream_t st);

// sample.cu: temperature / top-k / top-p sampling of `rows` rows of logits
struct SampleArgs {
    const float* logits;   // [rows][V]
    int V, rows;
    float inv_t;           // 1 / temperature (> 0)
    int top_k;             // 0 = off (top-p then looks at the 64 largest), else 1..64
    float top_p;           // >= 1 = off
    uint64_t seed;
    const int* seq_of;     // [rows] sequence slot per row (nullable: seq0)
    const int* positions;  // [rows] position of the row's input token (nullable: pos0)
    int seq0, pos0;
    unsigned long long* keys_out;  // nullable [rows]: the id in the argmax-key encoding
    uint32_t* ids_out;             // nullable [rows]
};
void prepare_sample_kernels();
void launch_sample(const SampleArgs& a, cudaStream_t st);

// gemv.cu (N <= 8)
void launch_gemv(const LinearArgs& a, cudaStream_t st);
// The GEMV stages its N activation rows of K values in shared memory: true
// when they fit.
bool gemv_fits(int N, int K);
// fewrow.cu: int8 weights, 2..16 rows, RMSNorm prologue and none / residual /
// SwiGLU epilogues in one launch (results equal the tcgen05 path's)
bool fewrow_fits(const LinearArgs& a);
void prepare_fewrow_kernels();
void launch_fewrow(const LinearArgs& a, cudaStream_t st);
// gemm_simt.cu (any N)
void launch_gemm_simt(const LinearArgs& a, cudaStream_t st);

// attn.cu
// Decode attention splits each (row, kv head) into warp shares of >=
// kMinBlocksPerWarp blocks and a CTA's (at least 4) warps hold consecutive
// shares, so a (row, kv head) meets at most max_blocks / (4 kMinBlocksPerWarp)
// + 2 CTAs: that many records of one (row, kv head) reach global memory.
// Two blocks per warp keeps a one-row step on about half the SMs, so the next
// projection's CTAs start on the others under programmatic dependent launch
// (one block per warp measured 1.03 against 0.95 ms per token; three or four
// were no faster for one row and 1-4 % slower for two).
constexpr int kMinBlocksPerWarp = 2;
inline int decode_max_segs(int max_blocks) { return max_blocks / (4 * kMinBlocksPerWarp) + 2; }
struct AttnDecodeArgs {
    // this step's q, k, v: the raw fused-QKV output [B][(n_q + 2 n_kv) d]; the
    // kernel applies the per-head RMSNorm + RoPE and appends K/V to the cache
    const float* qkv;
    const float* q_norm;        // [d]
    const float* k_norm;        // [d]
    const float2* rope;         // [rope_max_pos][d / 2] (cos, sin)
    int rope_max_pos;
    float eps;
    uint16_t* kv_layer;         // [n_kv][blocks][K, V][16][d], rows chunk-swizzled (kv_swizzle)
    const int* block_table;     // [seqs][max_blocks]
    int max_blocks;
    int n_pool_blocks;
    const int* seq_of;          // [B] sequence slot per batch row
    const int* positions;       // [B] position of the current token (kv_len = pos + 1)
    int B, n_q, n_kv, d;        // B <= 1024, d = 128, n_q = 2 n_kv
    int max_segs;               // decode_max_segs(max_blocks)
    float* partial;             // [B][n_kv][max_segs][group][d + 4] (m, l, pad, pad, acc)
    unsigned int* counters;     // [B][n_kv], zero between launches
    float* out;                 // [B][n_q][d]
    uint32_t* err;
    bool head_clusters;         // B == 1: one 8-CTA cluster per kv head (attn_head_clusters)
};
void launch_attn_decode(const AttnDecodeArgs& a, cudaStream_t st);
// A one-sequence step runs as one 8-CTA cluster per kv head while the
// sequence holds at most kHeadClusterMaxBlocks 16-token blocks (its 64 warps
// then stream at most 10 blocks each); a longer one is spread over every SM.
// Measured on Qwen3-0.6B, batch-1 ms/token clusters vs whole GPU: context
// 4096 0.759 vs 0.809, 8192 0.881 vs 0.891, 16384 1.109 vs 1.002.
constexpr int kHeadClusterMaxBlocks = 640;
inline bool attn_head_clusters(int B, long long max_kv_len) {
    return B == 1 && (max_kv_len + 15) / 16 <= kHeadClusterMaxBlocks;  // 16-token blocks
}

// decode_flow.cu: one decode step of 1..kPersistentMaxBatch rows as one
// cooperative dataflow kernel (int8 weights, hidden 1024, intermediate 3072,
// 16 x 128 query dims, 8 kv heads, at most kFlowMaxLayers layers): weights
// and KV blocks streamed into a shared-memory ring by a producer warp, tagged
// activations instead of grid barriers.
constexpr int kPersistentMaxBatch = 8;
constexpr int kFlowMaxLayers = 62;
struct PersistentLayer {
    const int8_t *wqkv, *wo, *wgu, *wd;
    const float *sqkv, *so, *sgu, *sd;
    const float *input_ln, *post_ln, *q_norm, *k_norm;
};
struct PersistentArgs {
    int B, H, I, V, L, n_q, n_kv;
    float eps;
    const PersistentLayer* layers;  // device array [L]
    const int8_t* embed;            // tied embedding / LM head [V][H]
    const float* sembed;
    const float* final_norm;
    const float2* rope;
    int rope_max_pos;
    uint16_t* kv;                   // pool base; layer l at l * kv_layer_elems
    size_t kv_layer_elems;
    const int* block_table;
    int max_blocks, n_pool_blocks;
    uint32_t* tok;                  // [B] input ids, replaced by the argmax ids
    const int* seq_of;              // [B]
    int* positions;                 // [B], advanced by one
    unsigned long long* keys;       // [B] argmax keys, zero between steps
    uint32_t* ids_out;              // [B]
    uint32_t* history;              // nullable [steps][B]
    int* step;
    float* logits;                  // nullable [B][V]
    unsigned* sync;                 // [3]: unused, finished CTAs, abort flag; zero between launches
    uint32_t* err;
    uint64_t* trace;                // nullable [4 + 10 L] globaltimer ns: start, then per phase (start, end) as
                                    // seen by CTA 0 (phases QKV, ATT, O, GU, D per layer, then HEAD), then finish
    // tagged activations (f32 value | 32-bit tag << 32)
    uint64_t *llx, *llx1;           // [kPersistentMaxBatch][H]
    uint64_t *llqkv, *llattn, *llh; // [..][qkv rows], [..][n_q d], [..][I]
    uint64_t* llrec;                // flow_record_words(ctas): cross-CTA attention records
    uint32_t tag;                   // this step's tag base: a multiple of 64, fresh per launch; layer l uses tag + l + 1
    int stall_layer;                // fault injection: when l >= 1, layer l's QKV input is polled with a tag that
                                    // nothing writes, so its bounded wait runs out (-1: off)
};
inline int persistent_trace_len(int layers) { return 4 + 10 * layers; }
void prepare_flow_kernels();
bool flow_supported(int device);
size_t flow_record_words(int ctas);
cudaError_t launch_decode_flow(const PersistentArgs& a, cudaStream_t st);
struct AttnPrefillArgs {
    const float* q;             // [n_q][T][d]
    const uint16_t* kv_planes;  // [4][n_kv][T][d]: K hi, K lo, V hi, V lo (qkv_post)
    int lo_terms;               // 0: K and V are exact bf16 (the lo planes are zero and skipped)
    int T, n_q, n_kv, d;
    float* out;                 // [T][n_q][d]
    // nullable: the output also as the bf16 hi / lo activation planes of the
    // next linear, [2][t_pad][n_q d] (what the plane kernel would write)
    uint16_t* planes;
    int t_pad;
};
void launch_attn_prefill(const AttnPrefillArgs& a, cudaStream_t st);

}  // namespace zc
