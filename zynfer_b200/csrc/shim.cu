// C ABI of the Zynfer `cuda` backend: context, weights, paged KV cache,
// prefill / decode schedules and CUDA graphs. See include/zynfer_cuda.h.
//
// The host schedule mirrors the reference's Qwen3 forward
// (src/model/qwen_forward.zig:94-175 around src/model/qwen_block.zig:161-235)
// with the B200 layout: fused QKV and interleaved gate/up weights, a paged
// bf16 KV pool of 16-token blocks, token-major activations, and one captured
// CUDA graph per decode batch size.
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <string>
#include <vector>

#include "../../include/zynfer_cuda.h"
#include "common.cuh"
#include "kernels.h"
#include "synth_rng.h"
#include "tc_gemm.h"

using namespace zc;

namespace {

// Which kernel runs a linear layer: the CUDA-core GEMV (few rows), the
// tensor-core tcgen05 path, or the CUDA-core tiled GEMM (kept for A/B checks).
enum LinPath { kPathAuto = 0, kPathGemv = 1, kPathSimt = 2, kPathTc = 3, kPathMma = 4 };
// Decode schedule: separate kernels per op (graph-captured; what auto takes),
// or one persistent dataflow kernel per step for small int8 batches (on request).
enum Schedule { kSchedAuto = 0, kSchedKernels = 1, kSchedPersistent = 2 };
constexpr int kGemvMaxM = 16384;  // model auto policy: largest matrix (output rows) for the batch-1 GEMV
// auto policy: most activation rows for the few-row MMA kernel (measured in a
// decode step: 10 % faster than tcgen05 at 4 rows, level at 6, 13 % slower at 8
// for every linear), and up to 8 rows for the K = 1024 linears alone, whose
// rows it stages fastest (batch 8: 1.45 -> 1.42 ms; slower from 12 rows)
constexpr int kFewRowAutoMax = 6;
constexpr int kFewRowAutoMaxNarrow = 8;
constexpr int kFewRowNarrowK = 1024;

struct LayerDev {
    void* wqkv = nullptr;
    float* sqkv = nullptr;
    void* wo = nullptr;
    float* so = nullptr;
    void* wgu = nullptr;
    float* sgu = nullptr;
    void* wd = nullptr;
    float* sd = nullptr;
    float* input_ln = nullptr;
    float* post_ln = nullptr;
    float* q_norm = nullptr;
    float* k_norm = nullptr;
    // TMA descriptors of the weight matrices (128-row x 128-byte boxes)
    CUtensorMap tm_qkv, tm_o, tm_gu, tm_d;
};

struct TimedEvent {
    cudaEvent_t a, b;
    int cls;
};

// A decode graph of one batch size and the linear kernel families it holds
// (bit kPath* of `paths`), so the path label of a graph launch names them.
struct GraphEntry {
    cudaGraphExec_t exec = nullptr;
    unsigned paths = 0;
};

}  // namespace

struct ZynferCuCtx {
    int device = -1;
    cudaStream_t stream = nullptr;
    std::string err;
    char path[96] = "none";  // label of the last call's kernels; a fixed buffer, written without allocating
    unsigned step_paths = 0;  // linear families (bit kPath*) launched since the last reset
    ZynferCuCaps caps{};
    // allocation events after zynfer_cu_model_init: device allocations
    // (cudaMalloc, graph instantiation) and growth of host containers beyond
    // their reserved capacity. A decode step of a batch size seen before adds
    // neither (tiny_block.zig:385-401 pins the same for host memory).
    uint64_t dev_alloc_events = 0, host_alloc_events = 0;

    // fault injection
    long fail_alloc_at = -1;
    long alloc_count = 0;
    bool fail_upload = false;
    bool fail_launch = false;
    bool fail_wait = false;  // the next persistent decode step stalls on a device wait
    std::vector<void*> allocs;
    std::vector<void*> pinned;

    // model
    bool ready = false;
    ZynferCuModelDesc d{};
    int wkind = kWQ8;
    size_t esz = 1;
    int qd = 0, kvd = 0, qkv_rows = 0;
    std::vector<LayerDev> L;
    void* embed = nullptr;
    float* sembed = nullptr;
    float* final_norm = nullptr;
    float2* rope = nullptr;
    uint16_t* kv = nullptr;
    size_t kv_layer_elems = 0;
    int max_blocks = 0, n_blocks = 0;
    std::vector<int> free_blocks;
    std::vector<uint32_t> block_refs;  // sequences holding each pool block (shared prefixes hold one block several times)
    std::vector<std::vector<int>> seq_blocks;
    std::vector<uint32_t> seq_len;
    std::vector<char> table_dirty;  // host row changed since its last upload
    int* table_host = nullptr;  // pinned [max_seqs][max_blocks]
    int* table_dev = nullptr;

    // decode scratch (max_batch rows)
    float *dx = nullptr, *dx1 = nullptr, *dqkv = nullptr, *dq = nullptr,
          *dattn = nullptr, *dh = nullptr, *dlogits = nullptr, *dpart = nullptr;
    uint32_t* dio = nullptr;  // [tokens B][seq B][pos B] contiguous
    uint32_t* dtok = nullptr;
    int* dseq = nullptr;
    int* dpos = nullptr;
    unsigned long long* dkeys = nullptr;
    uint32_t* dids = nullptr;
    unsigned* dcnt = nullptr;
    uint32_t* dhist = nullptr;
    int* dstep = nullptr;
    size_t hist_cap = 0;  // entries
    // prefill scratch (max_prefill rows)
    float *px = nullptr, *px1 = nullptr, *pqkv = nullptr, *pq = nullptr,
          *pattn = nullptr, *ph = nullptr;
    uint16_t* pkvp = nullptr;  // K and V of a prefill as bf16 terms [4][n_kv][T][d]
    uint32_t* ptok = nullptr;
    // device error word and pinned host staging
    uint32_t* derr = nullptr;
    uint32_t* herr = nullptr;
    uint32_t* hio = nullptr;   // pinned [3 * max_batch]
    uint32_t* hids = nullptr;  // pinned [max_batch]

    CUtensorMap tm_embed;
    // tcgen05 linear scratch: activation planes and per-row exponents, plus
    // B-operand descriptors per (kind, K, NT)
    uint8_t* planes = nullptr;
    // bf16 activation planes that the prefill attention wrote for the O
    // projection, so that linear skips its plane kernel (a buffer of their own:
    // `planes` may still be read by the linear before)
    uint8_t* planes2 = nullptr;
    bool planes_in2 = false;  // set before linear(): x's planes are in planes2
    float* exps = nullptr;  // per-row 2^(e-22) of the int8 digit planes
    int tc_tpad = 0, tc_kmax = 0;
    L2Range pf_next[2] = {};  // prefetch ranges the next linear() passes to its kernel, then clears
    std::map<uint64_t, CUtensorMap> bmaps;
    std::map<std::pair<const void*, uint64_t>, CUtensorMap> amaps;  // op-level weights
    float* simt_xn = nullptr;  // normalised rows for the CUDA-core GEMM path
    size_t simt_xn_elems = 0;
    int path_policy = kPathAuto;
    int schedule = kSchedAuto;
    // next-token rule of decode, generate and prefill: greedy (temperature 0)
    // or sampling (sample.cu)
    float samp_temp = 0.0f;
    uint32_t samp_top_k = 0;
    float samp_top_p = 1.0f;
    uint64_t samp_seed = 0;
    bool persistent_ok = false;          // model shape and device allow the persistent (dataflow) decode kernel
    PersistentLayer* dlayers = nullptr;  // [layers] weight pointers for it
    unsigned* psync = nullptr;           // [3] its unused / finished-CTA / abort words
    uint64_t* ll = nullptr;              // its tagged activation buffers and attention records
    size_t ll_words = 0;
    uint32_t flow_step = 0;              // launches so far: tag base = 64 (1 + step % 2^25)
    uint64_t* ptrace = nullptr;          // its phase timestamps when timing is on
    std::vector<uint64_t> ptrace_host;

    std::map<int, GraphEntry> graphs;  // by 2 B + head_clusters
    bool head_clusters = false;        // the next decode steps' one-sequence attention choice
    int step_launches = 0;  // kernels enqueued by the last decode step
    uint64_t h2d_bytes = 0, d2h_bytes = 0;  // host<->device bytes of decode/generate calls
    cudaEvent_t ev0 = nullptr, ev1 = nullptr;
    uint64_t last_step_ns = 0;

    // per-kernel timing
    bool timing = false;
    std::vector<TimedEvent> tev;
    size_t tev_used = 0;
    uint64_t t_launch[4] = {0, 0, 0, 0};
    double t_ms[4] = {0, 0, 0, 0};
};

namespace {

int fail(ZynferCuCtx* c, int code, const std::string& msg) {
    if (c) c->err = msg;
    return code;
}

int cuda_fail(ZynferCuCtx* c, cudaError_t e, const char* what) {
    std::string m = std::string(what) + ": " + cudaGetErrorString(e);
    int code = e == cudaErrorMemoryAllocation ? ZYNFER_CU_OOM : ZYNFER_CU_LAUNCH;
    if (e == cudaErrorNoDevice || e == cudaErrorInsufficientDriver) code = ZYNFER_CU_NO_DEVICE;
    return fail(c, code, m);
}

#define ZC_CHECK(c, expr, what)                          \
    do {                                                 \
        cudaError_t e_ = (expr);                         \
        if (e_ != cudaSuccess) return cuda_fail(c, e_, what); \
    } while (0)

template <typename T>
int dalloc(ZynferCuCtx* c, T** p, size_t count) {
    *p = nullptr;
    if (c->fail_alloc_at >= 0 && c->alloc_count++ == c->fail_alloc_at) {
        c->fail_alloc_at = -1;
        return fail(c, ZYNFER_CU_OOM, "injected allocation failure (ZYNFER_CUDA_FAIL_AT=alloc)");
    }
    void* v = nullptr;
    const size_t bytes = std::max<size_t>(count * sizeof(T), 16);
    cudaError_t e = cudaMalloc(&v, bytes);
    if (e != cudaSuccess) {
        cudaGetLastError();
        return fail(c, ZYNFER_CU_OOM, std::string("cudaMalloc(") + std::to_string(bytes) + "): " + cudaGetErrorString(e));
    }
    c->dev_alloc_events += 1;
    if (c->allocs.size() == c->allocs.capacity()) c->host_alloc_events += 1;
    c->allocs.push_back(v);
    *p = reinterpret_cast<T*>(v);
    return ZYNFER_CU_OK;
}

template <typename T>
int halloc(ZynferCuCtx* c, T** p, size_t count) {
    void* v = nullptr;
    cudaError_t e = cudaMallocHost(&v, std::max<size_t>(count * sizeof(T), 16));
    if (e != cudaSuccess) return cuda_fail(c, e, "cudaMallocHost");
    c->pinned.push_back(v);
    *p = reinterpret_cast<T*>(v);
    return ZYNFER_CU_OK;
}

void parse_fail_spec(ZynferCuCtx* c, const char* spec) {
    if (!spec || !*spec) return;
    if (strncmp(spec, "alloc:", 6) == 0) {
        c->fail_alloc_at = atol(spec + 6);
        c->alloc_count = 0;
    } else if (strcmp(spec, "upload") == 0) {
        c->fail_upload = true;
    } else if (strcmp(spec, "launch") == 0) {
        c->fail_launch = true;
    } else if (strcmp(spec, "wait") == 0) {
        c->fail_wait = true;
    }
}

bool take_launch_fault(ZynferCuCtx* c) {
    if (!c->fail_launch) return false;
    c->fail_launch = false;
    c->err = "injected launch failure (ZYNFER_CUDA_FAIL_AT=launch)";
    return true;
}

// Path label "<call>:<linear kernel families>[:<mode>]" into the context's
// fixed buffer (no allocation): e.g. "decode:gemv+tcgen05:graph".
void set_path(ZynferCuCtx* c, const char* call, unsigned paths, const char* mode) {
    char fam[48] = "";
    const char* names[5] = {"auto", "gemv", "simt", "tcgen05", "mma"};
    for (int b = 1; b < 5; ++b)
        if (paths & (1u << b)) {
            if (fam[0]) strncat(fam, "+", sizeof(fam) - strlen(fam) - 1);
            strncat(fam, names[b], sizeof(fam) - strlen(fam) - 1);
        }
    snprintf(c->path, sizeof(c->path), "%s%s%s%s%s", call, fam[0] ? ":" : "", fam, mode ? ":" : "", mode ? mode : "");
}

// Map an HF tensor name (qwen3.zig:86-132) to its device destination.
struct Dest {
    enum Kind { None, Vec, Mat } kind = None;
    float* vec = nullptr;
    void* w = nullptr;
    float* s = nullptr;
    int rows = 0, cols = 0;          // HF shape
    int stride = 1, offset = 0;      // destination row = r * stride + offset
};

Dest find_dest(ZynferCuCtx* c, const char* name) {
    Dest d;
    const ZynferCuModelDesc& m = c->d;
    const int H = m.hidden, I = m.inter, hd = m.head_dim;
    if (!strcmp(name, "model.embed_tokens.weight") || !strcmp(name, "lm_head.weight")) {
        d.kind = Dest::Mat; d.w = c->embed; d.s = c->sembed; d.rows = m.vocab; d.cols = H;
        return d;
    }
    if (!strcmp(name, "model.norm.weight")) {
        d.kind = Dest::Vec; d.vec = c->final_norm; d.rows = H; d.cols = 1;
        return d;
    }
    unsigned layer = 0;
    char rest[128];
    if (sscanf(name, "model.layers.%u.%127s", &layer, rest) != 2 || layer >= m.layers) return d;
    LayerDev& Ld = c->L[layer];
    auto vec = [&](float* p, int n) { d.kind = Dest::Vec; d.vec = p; d.rows = n; d.cols = 1; };
    auto mat = [&](void* w, float* s, int r, int cc, int stride, int offset) {
        d.kind = Dest::Mat; d.w = w; d.s = s; d.rows = r; d.cols = cc; d.stride = stride; d.offset = offset;
    };
    if (!strcmp(rest, "input_layernorm.weight")) vec(Ld.input_ln, H);
    else if (!strcmp(rest, "post_attention_layernorm.weight")) vec(Ld.post_ln, H);
    else if (!strcmp(rest, "self_attn.q_norm.weight")) vec(Ld.q_norm, hd);
    else if (!strcmp(rest, "self_attn.k_norm.weight")) vec(Ld.k_norm, hd);
    else if (!strcmp(rest, "self_attn.q_proj.weight")) mat(Ld.wqkv, Ld.sqkv, c->qd, H, 1, 0);
    else if (!strcmp(rest, "self_attn.k_proj.weight")) mat(Ld.wqkv, Ld.sqkv, c->kvd, H, 1, c->qd);
    else if (!strcmp(rest, "self_attn.v_proj.weight")) mat(Ld.wqkv, Ld.sqkv, c->kvd, H, 1, c->qd + c->kvd);
    else if (!strcmp(rest, "self_attn.o_proj.weight")) mat(Ld.wo, Ld.so, H, c->qd, 1, 0);
    else if (!strcmp(rest, "mlp.gate_proj.weight")) mat(Ld.wgu, Ld.sgu, I, H, 2, 0);
    else if (!strcmp(rest, "mlp.up_proj.weight")) mat(Ld.wgu, Ld.sgu, I, H, 2, 1);
    else if (!strcmp(rest, "mlp.down_proj.weight")) mat(Ld.wd, Ld.sd, H, I, 1, 0);
    return d;
}

// Place an f32 HF-layout tensor already on the device into its destination.
void place_f32(ZynferCuCtx* c, const Dest& d, const float* src) {
    if (d.kind == Dest::Vec) {
        cudaMemcpyAsync(d.vec, src, (size_t)d.rows * 4, cudaMemcpyDeviceToDevice, c->stream);
    } else if (c->wkind == kWQ8) {
        launch_pack_q8_rows(src, d.rows, d.cols, reinterpret_cast<int8_t*>(d.w), d.s, d.stride, d.offset,
                            c->stream);
    } else {
        launch_to_bf16_rows(src, d.rows, d.cols, reinterpret_cast<uint16_t*>(d.w), d.stride, d.offset,
                            c->stream);
    }
}

int check_device_error(ZynferCuCtx* c) {
    ZC_CHECK(c, cudaMemcpyAsync(c->herr, c->derr, 4, cudaMemcpyDeviceToHost, c->stream), "read error word");
    c->d2h_bytes += 4;
    ZC_CHECK(c, cudaStreamSynchronize(c->stream), "stream synchronize");
    const uint32_t e = *c->herr;
    if (!e) return ZYNFER_CU_OK;
    cudaMemsetAsync(c->derr, 0, 4, c->stream);
    cudaMemsetAsync(c->dcnt, 0, (size_t)c->d.max_batch * c->d.n_kv * 4, c->stream);
    if (c->psync) cudaMemsetAsync(c->psync, 0, 3 * sizeof(unsigned), c->stream);
    cudaMemsetAsync(c->dkeys, 0, (size_t)c->d.max_batch * 8, c->stream);
    cudaStreamSynchronize(c->stream);
    if (e & kErrTimeout) return fail(c, ZYNFER_CU_TIMEOUT, "device wait timed out (bounded mbarrier wait)");
    return fail(c, ZYNFER_CU_INVALID, "device index check failed (token id, position or KV block)");
}


// --------------------------------------------------------- timing helpers
void tbegin(ZynferCuCtx* c, int cls, TimedEvent** te) {
    *te = nullptr;
    if (!c->timing) return;
    if (c->tev_used == c->tev.size()) {
        // fold completed intervals into the totals, then reuse the pool
        cudaStreamSynchronize(c->stream);
        for (size_t i = 0; i < c->tev_used; ++i) {
            float ms = 0.0f;
            cudaEventElapsedTime(&ms, c->tev[i].a, c->tev[i].b);
            c->t_ms[c->tev[i].cls] += ms;
            c->t_launch[c->tev[i].cls] += 1;
        }
        c->tev_used = 0;
    }
    TimedEvent* e = &c->tev[c->tev_used++];
    e->cls = cls;
    cudaEventRecord(e->a, c->stream);
    *te = e;
}
void tend(ZynferCuCtx* c, TimedEvent* te) {
    if (te) cudaEventRecord(te->b, c->stream);
}

// Grow the tcgen05 scratch to hold `t` activation rows of up to `kmax` columns.
int ensure_tc_scratch(ZynferCuCtx* c, int t, int kmax, int mmax) {
    const int tpad = ((t + 127) / 128) * 128;
    (void)mmax;
    if (tpad <= c->tc_tpad && kmax <= c->tc_kmax) return ZYNFER_CU_OK;
    int rc;
    const int nt = std::max(tpad, c->tc_tpad), nk = std::max(kmax, c->tc_kmax);
    // superseded buffers stay in c->allocs until destroy (scratch only grows)
    if ((rc = dalloc(c, &c->planes, (size_t)4 * nt * nk))) return rc;  // 3 int8 or 2 bf16 planes
    if ((rc = dalloc(c, &c->planes2, (size_t)4 * nt * nk))) return rc;
    if ((rc = dalloc(c, &c->exps, (size_t)nt))) return rc;
    c->tc_tpad = nt;
    c->tc_kmax = nk;
    c->bmaps.clear();
    return ZYNFER_CU_OK;
}

const CUtensorMap* b_map(ZynferCuCtx* c, int wkind, int K, int nt, int second = 0) {
    const uint64_t key = ((uint64_t)second << 56) | ((uint64_t)wkind << 48) | ((uint64_t)K << 16) | (uint64_t)nt;
    auto it = c->bmaps.find(key);
    if (it != c->bmaps.end()) return &it->second;
    CUtensorMap m;
    const int P = wkind == kWQ8 ? 3 : 2;
    if (!make_tmap_k_major(&m, second ? c->planes2 : c->planes, wkind, (uint64_t)K, (uint64_t)P * c->tc_tpad,
                           (uint32_t)nt))
        return nullptr;
    return &(c->bmaps[key] = m);
}

// y = linear(norm_w ? rmsnorm(x) : x) with the epilogue `epi`, on the path the
// policy picks: GEMV (x staged in shared memory) for one row, the few-row
// integer-MMA kernel for 2..16 int8 rows, tcgen05 for more.
// Returns the kernel family it launched (kPathGemv, kPathMma, kPathTc or kPathSimt).
int linear(ZynferCuCtx* c, int cls, const void* w, const float* s, const CUtensorMap* tmA, int M, int K,
           const float* x, int N, float* y, int epi, const float* resid, const float* norm_w,
           unsigned long long* keys, int wkind = -1) {
    if (wkind < 0) wkind = c->wkind;
    LinearArgs a;
    a.w = w; a.scale = s; a.wkind = wkind; a.M = M; a.K = K; a.x = x; a.ldx = K; a.N = N;
    a.y = y; a.ldy = epi == kEpiSwiGLU ? M / 2 : M; a.epi = epi; a.resid = resid; a.norm_w = norm_w;
    a.eps = c->d.eps > 0.0f ? c->d.eps : 1e-6f; a.argmax_keys = keys; a.err = c->derr;
    a.pf[0] = c->pf_next[0]; a.pf[1] = c->pf_next[1];
    c->pf_next[0] = c->pf_next[1] = L2Range{nullptr, 0};
    const bool planes_in2 = c->planes_in2 && wkind == kWBF16;
    c->planes_in2 = false;
    int path = c->path_policy;
    // auto: one activation row -> GEMV (no plane kernel, one launch) except the
    // vocabulary-sized LM head; 2..6 int8 rows -> the few-row kernel (one
    // launch, no plane kernel) up to the same size; more rows -> tcgen05
    if (path == kPathAuto) {
        if (N == 1 && M <= kGemvMaxM) path = kPathGemv;
        else if (N > 1 && (N <= kFewRowAutoMax || (N <= kFewRowAutoMaxNarrow && K <= kFewRowNarrowK)) &&
                 M <= kGemvMaxM && fewrow_fits(a))
            path = kPathMma;
        else path = kPathTc;
    }
    if (path == kPathGemv && !gemv_fits(N, K)) path = kPathTc;
    if (path == kPathMma && !fewrow_fits(a)) path = kPathTc;
    if (path == kPathTc && (!tmA || N > c->tc_tpad || K > c->tc_kmax || K > kPlanesMaxK)) path = kPathSimt;
    TimedEvent* te;
    tbegin(c, cls, &te);
    c->step_paths |= 1u << path;
    if (path == kPathGemv) {
        launch_gemv(a, c->stream);
        c->step_launches += 1;
    } else if (path == kPathMma) {
        launch_fewrow(a, c->stream);
        c->step_launches += 1;
    } else if (path == kPathSimt) {
        if (norm_w) {
            launch_rmsnorm(x, norm_w, c->simt_xn, N, K, a.eps, c->stream);
            a.x = c->simt_xn;
            a.norm_w = nullptr;
            c->step_launches += 1;
        }
        launch_gemm_simt(a, c->stream);
        c->step_launches += 1;
    } else {
        const int nt = tc_tile_tokens(wkind, M, N);
        TcLaunch L;
        L.tmA = tmA;
        L.args = TcArgs{M, K, N, c->tc_tpad, wkind, epi, s, c->exps, y, a.ldy, resid, keys, c->derr, 0,
                        {a.pf[0], a.pf[1]}};
        L.sms = c->caps.sm_count > 0 ? c->caps.sm_count : 148;
        const int S = tc_cluster_size(M, N, K, wkind, epi, L.sms);
        if (!planes_in2) {
            PlanesArgs pa{x, K, N, K, c->tc_tpad, wkind, norm_w, a.eps, c->planes, c->exps};
            launch_prep_planes(pa, c->stream);
            c->step_launches += 1;
        }
        L.tmB = b_map(c, wkind, K, nt, planes_in2 ? 1 : 0);
        if (L.tmB) {
            if (S > 1) launch_tc_cluster(L, S, c->stream);
            else launch_tc_gemm(L, c->stream);
        }
        c->step_launches += 1;
    }
    tend(c, te);
    return path;
}

// One decode step for the rows already staged in dtok/dseq/dpos.
// "auto" takes the kernel graph: it measured faster than the persistent
// dataflow kernel (whose linear phases run on CUDA cores) at every batch size,
// batch 1 included.
bool use_persistent(const ZynferCuCtx* c, int B) {
    return B <= kPersistentMaxBatch && c->persistent_ok && c->schedule == kSchedPersistent && c->samp_temp <= 0.0f;
}

// Replace the argmax keys of `rows` rows by sampled ids (sampling on only;
// the LM head has written the logits).
void enqueue_sample(ZynferCuCtx* c, int rows, const int* seq_of, const int* positions, int seq0, int pos0) {
    SampleArgs sa{};
    sa.logits = c->dlogits; sa.V = (int)c->d.vocab; sa.rows = rows;
    sa.inv_t = 1.0f / c->samp_temp; sa.top_k = (int)c->samp_top_k; sa.top_p = c->samp_top_p; sa.seed = c->samp_seed;
    sa.seq_of = seq_of; sa.positions = positions; sa.seq0 = seq0; sa.pos0 = pos0;
    sa.keys_out = c->dkeys; sa.ids_out = nullptr;
    launch_sample(sa, c->stream);
    c->step_launches += 1;
}

void enqueue_decode_persistent(ZynferCuCtx* c, int B, bool want_logits) {
    const ZynferCuModelDesc& m = c->d;
    PersistentArgs a{};
    a.B = B; a.H = (int)m.hidden; a.I = (int)m.inter; a.V = (int)m.vocab; a.L = (int)m.layers;
    a.n_q = (int)m.n_q; a.n_kv = (int)m.n_kv; a.eps = m.eps;
    a.layers = c->dlayers;
    a.embed = static_cast<const int8_t*>(c->embed); a.sembed = c->sembed; a.final_norm = c->final_norm;
    a.rope = c->rope; a.rope_max_pos = (int)m.max_seq_len;
    a.kv = c->kv; a.kv_layer_elems = c->kv_layer_elems;
    a.block_table = c->table_dev; a.max_blocks = c->max_blocks; a.n_pool_blocks = c->n_blocks;
    a.tok = c->dtok; a.seq_of = c->dseq; a.positions = c->dpos;
    a.keys = c->dkeys; a.ids_out = c->dids; a.history = c->dhist; a.step = c->dstep;
    a.logits = want_logits ? c->dlogits : nullptr;
    a.sync = c->psync; a.err = c->derr;
    const int tl = persistent_trace_len((int)m.layers);
    if (c->timing && !c->ptrace && dalloc(c, &c->ptrace, (size_t)tl) != ZYNFER_CU_OK) c->ptrace = nullptr;
    a.trace = c->timing ? c->ptrace : nullptr;
    const size_t act = (size_t)kPersistentMaxBatch;
    a.llx = c->ll;
    a.llx1 = a.llx + act * m.hidden;
    a.llqkv = a.llx1 + act * m.hidden;
    a.llattn = a.llqkv + act * c->qkv_rows;
    a.llh = a.llattn + act * c->qd;
    a.llrec = a.llh + act * m.inter;
    // tags are unique per (launch, layer): 64 (1 + step) + layer + 1
    a.tag = 64u * (1u + (c->flow_step++ % (1u << 25)));
    a.stall_layer = -1;
    if (c->fail_wait && m.layers >= 2) {
        c->fail_wait = false;
        a.stall_layer = 1;
    }
    launch_decode_flow(a, c->stream);
    c->step_launches = 1;
    if (a.trace) {
        // phase p lasts from its start to the next phase's start (its input wait included)
        c->ptrace_host.resize(tl);
        if (cudaMemcpyAsync(c->ptrace_host.data(), c->ptrace, tl * 8, cudaMemcpyDeviceToHost, c->stream) != cudaSuccess ||
            cudaStreamSynchronize(c->stream) != cudaSuccess)
            return;
        const uint64_t* t = c->ptrace_host.data();
        const int phases = 5 * (int)m.layers + 1;
        auto add = [&](int cls, uint64_t t0, uint64_t t1) {
            c->t_ms[cls] += t1 > t0 ? (double)(t1 - t0) * 1e-6 : 0.0;
            c->t_launch[cls] += 1;
        };
        add(ZYNFER_CU_K_OTHER, t[0], t[1]);
        for (int p = 0; p < phases; ++p) {
            const uint64_t start = t[1 + 2 * p], next = p + 1 < phases ? t[1 + 2 * (p + 1)] : t[3 + 2 * (phases - 1)];
            const int cls = p == phases - 1 ? ZYNFER_CU_K_LMHEAD : (p % 5 == 1 ? ZYNFER_CU_K_ATTN : ZYNFER_CU_K_LINEAR);
            add(cls, start, next);
        }
    }
}

// The next linear() call prefetches into L2 the weights and row scales of the
// linear that follows it in the step (rows x cols), so that one reads them
// from L2 instead of HBM.
void set_prefetch(ZynferCuCtx* c, const void* w, const float* s, size_t rows, size_t cols) {
    c->pf_next[0] = L2Range{w, (uint32_t)(rows * cols * (c->wkind == kWQ8 ? 1 : 2))};
    c->pf_next[1] = L2Range{s, s ? (uint32_t)(rows * sizeof(float)) : 0u};
}

void enqueue_decode(ZynferCuCtx* c, int B, bool want_logits) {
    if (use_persistent(c, B)) {
        enqueue_decode_persistent(c, B, want_logits);
        return;
    }
    const ZynferCuModelDesc& m = c->d;
    const int H = m.hidden, I = m.inter;
    c->step_launches = 0;
    TimedEvent* te;
    tbegin(c, ZYNFER_CU_K_OTHER, &te);
    launch_embed(c->embed, c->sembed, c->wkind, c->dtok, B, H, m.vocab, c->dx, c->derr, c->stream);
    tend(c, te);
    c->step_launches += 1;
    for (uint32_t l = 0; l < m.layers; ++l) {
        const LayerDev& Ld = c->L[l];
        set_prefetch(c, Ld.wo, Ld.so, H, c->qd);
        linear(c, ZYNFER_CU_K_LINEAR, Ld.wqkv, Ld.sqkv, &Ld.tm_qkv, c->qkv_rows, H, c->dx, B, c->dqkv, kEpiNone,
               nullptr, Ld.input_ln, nullptr);
        // per-head RMSNorm + RoPE and the K/V append run inside the attention kernel
        AttnDecodeArgs aa{};
        aa.qkv = c->dqkv; aa.q_norm = Ld.q_norm; aa.k_norm = Ld.k_norm; aa.rope = c->rope;
        aa.rope_max_pos = (int)m.max_seq_len; aa.eps = m.eps;
        aa.kv_layer = c->kv + l * c->kv_layer_elems; aa.block_table = c->table_dev;
        aa.max_blocks = c->max_blocks; aa.n_pool_blocks = c->n_blocks;
        aa.seq_of = c->dseq; aa.positions = c->dpos; aa.B = B; aa.n_q = m.n_q; aa.n_kv = m.n_kv;
        aa.d = m.head_dim; aa.max_segs = decode_max_segs(c->max_blocks); aa.partial = c->dpart;
        aa.counters = c->dcnt; aa.out = c->dattn; aa.err = c->derr; aa.head_clusters = c->head_clusters;
        tbegin(c, ZYNFER_CU_K_ATTN, &te);
        launch_attn_decode(aa, c->stream);
        tend(c, te);
        c->step_launches += 1;
        set_prefetch(c, Ld.wgu, Ld.sgu, 2 * I, H);
        linear(c, ZYNFER_CU_K_LINEAR, Ld.wo, Ld.so, &Ld.tm_o, H, c->qd, c->dattn, B, c->dx1, kEpiResid, c->dx,
               nullptr, nullptr);
        set_prefetch(c, Ld.wd, Ld.sd, H, I);
        linear(c, ZYNFER_CU_K_LINEAR, Ld.wgu, Ld.sgu, &Ld.tm_gu, 2 * I, H, c->dx1, B, c->dh, kEpiSwiGLU, nullptr,
               Ld.post_ln, nullptr);
        if (l + 1 < m.layers) set_prefetch(c, c->L[l + 1].wqkv, c->L[l + 1].sqkv, c->qkv_rows, H);
        linear(c, ZYNFER_CU_K_LINEAR, Ld.wd, Ld.sd, &Ld.tm_d, H, I, c->dh, B, c->dx, kEpiResid, c->dx1, nullptr,
               nullptr);
    }
    const bool sampling = c->samp_temp > 0.0f;
    // the LM head prefetches the next step's first linear
    if (m.layers > 0) set_prefetch(c, c->L[0].wqkv, c->L[0].sqkv, c->qkv_rows, H);
    linear(c, ZYNFER_CU_K_LMHEAD, c->embed, c->sembed, &c->tm_embed, m.vocab, H, c->dx, B,
           want_logits || sampling ? c->dlogits : nullptr, kEpiArgmax, nullptr, c->final_norm, c->dkeys);
    if (sampling) enqueue_sample(c, B, c->dseq, c->dpos, 0, 0);
    FinalizeArgs fa{};
    fa.keys = c->dkeys; fa.ids_out = c->dids; fa.next_tokens = c->dtok; fa.positions = c->dpos;
    fa.history = c->dhist; fa.step = c->dstep; fa.B = B;
    launch_finalize(fa, c->stream);
    c->step_launches += 1;
}

int ensure_blocks(ZynferCuCtx* c, uint32_t seq, uint32_t upto_len) {
    std::vector<int>& bl = c->seq_blocks[seq];
    const size_t need = (upto_len + kKvBlock - 1) / kKvBlock;
    if (need > (size_t)c->max_blocks) return fail(c, ZYNFER_CU_INVALID, "sequence exceeds max_seq_len");
    while (bl.size() < need) {
        if (c->free_blocks.empty()) return fail(c, ZYNFER_CU_OOM, "KV block pool exhausted");
        const int b = c->free_blocks.back();
        c->free_blocks.pop_back();
        c->block_refs[b] = 1;
        c->table_host[(size_t)seq * c->max_blocks + bl.size()] = b;
        if (bl.size() == bl.capacity()) c->host_alloc_events += 1;  // reserved to max_blocks at init
        bl.push_back(b);
        c->table_dirty[seq] = 1;
    }
    return ZYNFER_CU_OK;
}

void release_seq(ZynferCuCtx* c, uint32_t seq) {
    for (int b : c->seq_blocks[seq])
        if (--c->block_refs[b] == 0) c->free_blocks.push_back(b);
    c->seq_blocks[seq].clear();
    c->seq_len[seq] = 0;
    std::fill(c->table_host + (size_t)seq * c->max_blocks, c->table_host + (size_t)(seq + 1) * c->max_blocks, -1);
    c->table_dirty[seq] = 1;
}

// Upload the block-table rows of `seqs` that changed since their last upload.
int upload_table_rows(ZynferCuCtx* c, const uint32_t* seqs, uint32_t n) {
    for (uint32_t i = 0; i < n; ++i) {
        if (!c->table_dirty[seqs[i]]) continue;
        c->table_dirty[seqs[i]] = 0;
        const size_t off = (size_t)seqs[i] * c->max_blocks;
        c->h2d_bytes += (size_t)c->max_blocks * 4;
        ZC_CHECK(c, cudaMemcpyAsync(c->table_dev + off, c->table_host + off, (size_t)c->max_blocks * 4,
                                    cudaMemcpyHostToDevice, c->stream),
                 "block table upload");
    }
    return ZYNFER_CU_OK;
}

int validate_batch(ZynferCuCtx* c, const uint32_t* seqs, uint32_t batch, uint32_t extra) {
    if (!c->ready) return fail(c, ZYNFER_CU_INVALID, "model not initialised");
    if (batch == 0 || batch > c->d.max_batch) return fail(c, ZYNFER_CU_INVALID, "batch must be 1..max_batch");
    for (uint32_t i = 0; i < batch; ++i) {
        if (seqs[i] >= c->d.max_seqs) return fail(c, ZYNFER_CU_INVALID, "sequence id out of range");
        for (uint32_t j = 0; j < i; ++j)
            if (seqs[j] == seqs[i]) return fail(c, ZYNFER_CU_INVALID, "a sequence appears twice in one batch");
        if (c->seq_len[seqs[i]] + extra > c->d.max_seq_len)
            return fail(c, ZYNFER_CU_INVALID, "KV cache full: step would exceed max_seq_len");
    }
    return ZYNFER_CU_OK;
}

int stage_batch(ZynferCuCtx* c, const uint32_t* seqs, const uint32_t* tokens, uint32_t B) {
    for (uint32_t i = 0; i < B; ++i) {
        if (tokens[i] >= c->d.vocab) return fail(c, ZYNFER_CU_INVALID, "token id >= vocab");
        c->hio[i] = tokens[i];
        c->hio[B + i] = seqs[i];
        c->hio[2 * B + i] = c->seq_len[seqs[i]];
    }
    ZC_CHECK(c, cudaMemcpyAsync(c->dio, c->hio, (size_t)3 * B * 4, cudaMemcpyHostToDevice, c->stream), "stage batch");
    c->h2d_bytes += (size_t)3 * B * 4;
    return ZYNFER_CU_OK;
}

void set_io_views(ZynferCuCtx* c, int B) {
    c->dtok = c->dio;
    c->dseq = reinterpret_cast<int*>(c->dio + B);
    c->dpos = reinterpret_cast<int*>(c->dio + 2 * B);
}

int get_graph(ZynferCuCtx* c, int B, GraphEntry* out) {
    const int key = 2 * B + (c->head_clusters ? 1 : 0);
    auto it = c->graphs.find(key);
    if (it != c->graphs.end()) {
        *out = it->second;
        return ZYNFER_CU_OK;
    }
    cudaGraph_t g = nullptr;
    ZC_CHECK(c, cudaStreamBeginCapture(c->stream, cudaStreamCaptureModeRelaxed), "begin capture");
    c->step_paths = 0;
    enqueue_decode(c, B, false);
    cudaError_t e = cudaStreamEndCapture(c->stream, &g);
    if (e != cudaSuccess) return cuda_fail(c, e, "end capture");
    cudaGraphExec_t ge = nullptr;
    e = cudaGraphInstantiate(&ge, g, 0);
    cudaGraphDestroy(g);
    if (e != cudaSuccess) return cuda_fail(c, e, "graph instantiate");
    c->dev_alloc_events += 1;   // the executable graph holds device memory
    c->host_alloc_events += 1;  // and a map node
    GraphEntry ent;
    ent.exec = ge;
    ent.paths = c->step_paths;
    c->graphs[key] = ent;
    *out = ent;
    return ZYNFER_CU_OK;
}

// Prefill scratch-based forward of `t` tokens of `seq` at pos0 = 0 through
// layers [l0, l1). Input rows in px; output rows in px.
void enqueue_prefill_layers(ZynferCuCtx* c, uint32_t seq, int T, uint32_t l0, uint32_t l1) {
    const ZynferCuModelDesc& m = c->d;
    const int H = m.hidden, I = m.inter;
    for (uint32_t l = l0; l < l1; ++l) {
        const LayerDev& Ld = c->L[l];
        linear(c, ZYNFER_CU_K_LINEAR, Ld.wqkv, Ld.sqkv, &Ld.tm_qkv, c->qkv_rows, H, c->px, T, c->pqkv, kEpiNone,
               nullptr, Ld.input_ln, nullptr);
        QkvArgs qa{};
        qa.qkv = c->pqkv; qa.T = T; qa.n_q = m.n_q; qa.n_kv = m.n_kv; qa.d = m.head_dim;
        qa.q_norm = Ld.q_norm; qa.k_norm = Ld.k_norm; qa.eps = m.eps;
        qa.rope = c->rope; qa.rope_max_pos = m.max_seq_len;
        qa.row_pos = nullptr; qa.pos0 = 0; qa.row_seq = nullptr; qa.seq0 = (int)seq;
        qa.kv_layer = c->kv + l * c->kv_layer_elems; qa.block_table = c->table_dev;
        qa.max_blocks = c->max_blocks; qa.n_pool_blocks = c->n_blocks;
        qa.q_out = c->pq; qa.q_heads_major = 1; qa.k_stage = nullptr; qa.v_stage = nullptr;
        qa.kv_planes = c->pkvp;
        qa.stage_round_bf16 = m.prefill_kv_f32 ? 0 : 1; qa.err = c->derr;
        launch_qkv_post(qa, c->stream);
        // bf16 weights: the attention also writes the O projection's activation
        // planes, so O needs no plane kernel (the same from the gate/up epilogue
        // for down measured slower: its scattered 2-byte stores cost more than
        // the launch)
        const bool bf16 = c->wkind == kWBF16 && T <= c->tc_tpad;
        AttnPrefillArgs pa{};
        pa.q = c->pq; pa.kv_planes = c->pkvp; pa.lo_terms = m.prefill_kv_f32 ? 1 : 0; pa.T = T; pa.n_q = m.n_q;
        pa.n_kv = m.n_kv; pa.d = m.head_dim; pa.out = c->pattn;
        pa.planes = bf16 ? reinterpret_cast<uint16_t*>(c->planes2) : nullptr; pa.t_pad = c->tc_tpad;
        launch_attn_prefill(pa, c->stream);
        c->planes_in2 = bf16;
        linear(c, ZYNFER_CU_K_LINEAR, Ld.wo, Ld.so, &Ld.tm_o, H, c->qd, c->pattn, T, c->px1, kEpiResid, c->px,
               nullptr, nullptr);
        linear(c, ZYNFER_CU_K_LINEAR, Ld.wgu, Ld.sgu, &Ld.tm_gu, 2 * I, H, c->px1, T, c->ph, kEpiSwiGLU, nullptr,
               Ld.post_ln, nullptr);
        linear(c, ZYNFER_CU_K_LINEAR, Ld.wd, Ld.sd, &Ld.tm_d, H, I, c->ph, T, c->px, kEpiResid, c->px1, nullptr,
               nullptr);
    }
}

}  // namespace

namespace zc {
int ctx_fail(ZynferCuCtx* c, int code, const char* msg) { return fail(c, code, msg); }

int ctx_check_arch(ZynferCuCtx* c, const ZynferCuModelDesc* w) {
    if (!c || !c->ready) return c ? fail(c, ZYNFER_CU_INVALID, "model not initialised") : ZYNFER_CU_INVALID;
    const ZynferCuModelDesc& m = c->d;
    if (m.vocab != w->vocab || m.hidden != w->hidden || m.inter != w->inter || m.layers != w->layers ||
        m.n_q != w->n_q || m.n_kv != w->n_kv || m.head_dim != w->head_dim)
        return fail(c, ZYNFER_CU_INVALID, "ShapeMismatch: the artifact's architecture is not the model's");
    return ZYNFER_CU_OK;
}
}  // namespace zc

// =================================================================== ABI

extern "C" {

const char* zynfer_cu_build_info(void) {
    return "zynfer_cuda sm_100a (int8/bf16 weight-only Qwen3 decode + prefill, paged bf16 KV)";
}

int zynfer_cu_create(int device, ZynferCuCtx** out) {
    if (!out) return ZYNFER_CU_INVALID;
    *out = nullptr;
    ZynferCuCtx* c = new ZynferCuCtx();
    int n = 0;
    cudaError_t e = cudaGetDeviceCount(&n);
    if (e != cudaSuccess || n == 0) {
        cudaGetLastError();
        c->err = std::string("no CUDA device: ") + (e != cudaSuccess ? cudaGetErrorString(e) : "count is 0");
        *out = c;  // handle kept so the caller can read last_error; destroy it
        return ZYNFER_CU_NO_DEVICE;
    }
    if (device < 0 || device >= n) {
        c->err = "device index out of range";
        *out = c;
        return ZYNFER_CU_NO_DEVICE;
    }
    c->device = device;
    cudaSetDevice(device);
    cudaDeviceProp p{};
    cudaGetDeviceProperties(&p, device);
    snprintf(c->caps.device_name, sizeof(c->caps.device_name), "%s", p.name);
    c->caps.sm_major = p.major;
    c->caps.sm_minor = p.minor;
    c->caps.sm_count = p.multiProcessorCount;
    c->caps.hbm_bytes = p.totalGlobalMem;
    c->caps.l2_bytes = (uint64_t)p.l2CacheSize;
    c->caps.max_smem_per_block = (uint32_t)p.sharedMemPerBlockOptin;
    c->caps.bulk_copy = p.major >= 9;
    c->caps.tcgen05 = p.major == 10 && p.minor == 0;
    if (p.major != 10) {
        c->err = std::string("device ") + p.name + " is not sm_100 (this library is built for sm_100a only)";
        *out = c;
        return ZYNFER_CU_UNSUPPORTED;
    }
    e = cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking);
    if (e != cudaSuccess) {
        c->err = cudaGetErrorString(e);
        *out = c;
        return ZYNFER_CU_LAUNCH;
    }
    cudaEventCreate(&c->ev0);
    cudaEventCreate(&c->ev1);
    prepare_all_kernels();  // function attributes now, never during a graph capture
    parse_fail_spec(c, getenv("ZYNFER_CUDA_FAIL_AT"));
    *out = c;
    return ZYNFER_CU_OK;
}

void zynfer_cu_destroy(ZynferCuCtx* c) {
    if (!c) return;
    // During process teardown the runtime may already be unloading: then the
    // driver reclaims everything and no CUDA call may be made.
    if (c->device >= 0 && cudaSetDevice(c->device) == cudaSuccess) {
        if (c->stream) cudaStreamSynchronize(c->stream);
        for (auto& kv : c->graphs) cudaGraphExecDestroy(kv.second.exec);
        for (auto& t : c->tev) {
            cudaEventDestroy(t.a);
            cudaEventDestroy(t.b);
        }
        if (c->ev0) cudaEventDestroy(c->ev0);
        if (c->ev1) cudaEventDestroy(c->ev1);
        for (void* p : c->allocs) cudaFree(p);
        for (void* p : c->pinned) cudaFreeHost(p);
        if (c->stream) cudaStreamDestroy(c->stream);
    }
    delete c;
}

int zynfer_cu_caps(const ZynferCuCtx* c, ZynferCuCaps* out) {
    if (!c || !out) return ZYNFER_CU_INVALID;
    *out = c->caps;
    return c->device >= 0 ? ZYNFER_CU_OK : ZYNFER_CU_NO_DEVICE;
}

const char* zynfer_cu_last_error(const ZynferCuCtx* c) { return c ? c->err.c_str() : "null context"; }

const char* zynfer_cu_last_path(const ZynferCuCtx* c) { return c ? c->path : "null context"; }

int zynfer_cu_set_fail_at(ZynferCuCtx* c, const char* spec) {
    if (!c) {
        // process-wide: only the allocation-free linear, which has no context
        if (spec && !strcmp(spec, "wait")) {
            static_linear_arm_stall();
            return ZYNFER_CU_OK;
        }
        return ZYNFER_CU_INVALID;
    }
    parse_fail_spec(c, spec);
    return ZYNFER_CU_OK;
}

int zynfer_cu_sync(ZynferCuCtx* c) {
    if (!c || c->device < 0) return ZYNFER_CU_INVALID;
    cudaSetDevice(c->device);
    ZC_CHECK(c, cudaStreamSynchronize(c->stream), "stream synchronize");
    if (c->derr) return check_device_error(c);
    return ZYNFER_CU_OK;
}

int zynfer_cu_model_init(ZynferCuCtx* c, const ZynferCuModelDesc* desc) {
    if (!c || !desc || c->device < 0) return ZYNFER_CU_INVALID;
    if (c->ready) return fail(c, ZYNFER_CU_INVALID, "model already initialised");
    cudaSetDevice(c->device);
    const ZynferCuModelDesc& m = *desc;
    if (m.head_dim != 128 || m.n_kv == 0 || m.n_q != 2 * m.n_kv)
        return fail(c, ZYNFER_CU_UNSUPPORTED, "kernels are built for head_dim 128 and 2 query heads per kv head");
    if (m.hidden % 512 || m.inter % 512 || (m.n_q * m.head_dim) % 512)
        return fail(c, ZYNFER_CU_UNSUPPORTED, "hidden, intermediate and q dims must be multiples of 512");
    if (m.weights != ZYNFER_CU_W_Q8 && m.weights != ZYNFER_CU_W_BF16)
        return fail(c, ZYNFER_CU_INVALID, "unknown weight kind");
    if (m.max_batch == 0 || m.max_batch > 1024 || m.max_seqs == 0 || m.max_seq_len == 0 ||
        m.max_seq_len > m.max_pos || m.layers == 0 || m.vocab == 0)
        return fail(c, ZYNFER_CU_INVALID, "invalid sizes in model descriptor");
    c->d = m;
    if (c->d.max_prefill == 0) c->d.max_prefill = std::min<uint32_t>(m.max_seq_len, 4096);
    c->wkind = m.weights == ZYNFER_CU_W_Q8 ? kWQ8 : kWBF16;
    c->esz = c->wkind == kWQ8 ? 1 : 2;
    const size_t H = m.hidden, I = m.inter, V = m.vocab, hd = m.head_dim;
    c->qd = m.n_q * hd;
    c->kvd = m.n_kv * hd;
    c->qkv_rows = c->qd + 2 * c->kvd;
    const bool q8 = c->wkind == kWQ8;
    int rc;
#define ALLOC(p, n) do { if ((rc = dalloc(c, &(p), (n))) != ZYNFER_CU_OK) return rc; } while (0)
    c->L.resize(m.layers);
    for (auto& Ld : c->L) {
        char* w;
        ALLOC(w, (size_t)c->qkv_rows * H * c->esz); Ld.wqkv = w;
        ALLOC(w, H * (size_t)c->qd * c->esz); Ld.wo = w;
        ALLOC(w, 2 * I * H * c->esz); Ld.wgu = w;
        ALLOC(w, H * I * c->esz); Ld.wd = w;
        if (q8) {
            ALLOC(Ld.sqkv, (size_t)c->qkv_rows);
            ALLOC(Ld.so, H);
            ALLOC(Ld.sgu, 2 * I);
            ALLOC(Ld.sd, H);
        }
        ALLOC(Ld.input_ln, H);
        ALLOC(Ld.post_ln, H);
        ALLOC(Ld.q_norm, hd);
        ALLOC(Ld.k_norm, hd);
    }
    {
        char* w;
        ALLOC(w, V * H * c->esz);
        c->embed = w;
    }
    if (q8) ALLOC(c->sembed, V);
    ALLOC(c->final_norm, H);
    // RoPE table: the reference's f32 formula (ops.zig:250-253) evaluated once
    // on the host: freq = 1 / theta^(i/half), angle = pos * freq.
    {
        const int half = (int)hd / 2;
        std::vector<float2> tab((size_t)m.max_seq_len * half);
        for (int i = 0; i < half; ++i) {
            const float freq = 1.0f / powf(m.theta, (float)i / (float)half);
            for (uint32_t pos = 0; pos < m.max_seq_len; ++pos) {
                const float angle = (float)pos * freq;
                tab[(size_t)pos * half + i] = make_float2(cosf(angle), sinf(angle));
            }
        }
        ALLOC(c->rope, tab.size());
        ZC_CHECK(c, cudaMemcpy(c->rope, tab.data(), tab.size() * sizeof(float2), cudaMemcpyHostToDevice), "rope table");
    }
    // paged KV pool
    c->max_blocks = (int)((m.max_seq_len + kKvBlock - 1) / kKvBlock);
    c->n_blocks = m.kv_blocks ? (int)m.kv_blocks : (int)(m.max_seqs * c->max_blocks);
    c->kv_layer_elems = (size_t)c->n_blocks * 2 * m.n_kv * kKvBlock * hd;
    ALLOC(c->kv, c->kv_layer_elems * m.layers);
    c->free_blocks.clear();
    c->free_blocks.reserve(c->n_blocks);
    c->block_refs.assign(c->n_blocks, 0);
    for (int b = c->n_blocks - 1; b >= 0; --b) c->free_blocks.push_back(b);
    c->seq_blocks.assign(m.max_seqs, {});
    for (auto& bl : c->seq_blocks) bl.reserve(c->max_blocks);  // decode never grows a block list
    c->seq_len.assign(m.max_seqs, 0);
    c->table_dirty.assign(m.max_seqs, 0);
    if ((rc = halloc(c, &c->table_host, (size_t)m.max_seqs * c->max_blocks)) != ZYNFER_CU_OK) return rc;
    std::fill(c->table_host, c->table_host + (size_t)m.max_seqs * c->max_blocks, -1);
    ALLOC(c->table_dev, (size_t)m.max_seqs * c->max_blocks);
    ZC_CHECK(c, cudaMemcpy(c->table_dev, c->table_host, (size_t)m.max_seqs * c->max_blocks * 4, cudaMemcpyHostToDevice), "table");
    // decode scratch
    const size_t B = m.max_batch;
    ALLOC(c->dx, B * H);
    ALLOC(c->dx1, B * H);
    ALLOC(c->dqkv, B * c->qkv_rows);
    ALLOC(c->dq, B * c->qd);
    ALLOC(c->dattn, B * c->qd);
    ALLOC(c->dh, B * I);
    ALLOC(c->dlogits, B * V);
    ALLOC(c->dio, 3 * B);
    ALLOC(c->dkeys, B);
    ALLOC(c->dids, B);
    ALLOC(c->dcnt, B * m.n_kv);
    ALLOC(c->dpart, B * m.n_kv * (size_t)decode_max_segs(c->max_blocks) * 2 * (hd + 4));
    c->hist_cap = std::max<size_t>(B * 4096, 1 << 16);
    ALLOC(c->dhist, c->hist_cap);
    ALLOC(c->dstep, 1);
    // prefill scratch
    const size_t P = c->d.max_prefill;
    ALLOC(c->px, P * H);
    ALLOC(c->px1, P * H);
    ALLOC(c->pqkv, P * c->qkv_rows);
    ALLOC(c->pq, P * c->qd);
    ALLOC(c->pkvp, 4 * P * c->kvd);
    ALLOC(c->pattn, P * c->qd);
    ALLOC(c->ph, P * I);
    ALLOC(c->ptok, P);
    ALLOC(c->derr, 1);
    c->simt_xn_elems = std::max(B, P) * H;
    ALLOC(c->simt_xn, c->simt_xn_elems);
#undef ALLOC
    {
        const int kmax = std::max({(int)H, c->qd, (int)I});
        const int mmax = std::max({c->qkv_rows, 2 * (int)I, (int)H});
        if ((rc = ensure_tc_scratch(c, (int)std::max(B, P), kmax, mmax))) return rc;
    }
    // TMA descriptors of every weight matrix (K-major, 128-row x 128-byte boxes)
    for (auto& Ld : c->L) {
        if (!make_tmap_k_major(&Ld.tm_qkv, Ld.wqkv, c->wkind, H, c->qkv_rows, 128) ||
            !make_tmap_k_major(&Ld.tm_o, Ld.wo, c->wkind, c->qd, H, 128) ||
            !make_tmap_k_major(&Ld.tm_gu, Ld.wgu, c->wkind, H, 2 * I, 128) ||
            !make_tmap_k_major(&Ld.tm_d, Ld.wd, c->wkind, I, H, 128))
            return fail(c, ZYNFER_CU_INTERNAL, "cuTensorMapEncodeTiled failed for a weight matrix");
    }
    if (!make_tmap_k_major(&c->tm_embed, c->embed, c->wkind, H, V, 128))
        return fail(c, ZYNFER_CU_INTERNAL, "cuTensorMapEncodeTiled failed for the embedding");
    // persistent dataflow decode kernel: weight pointers per layer, its sync
    // words, tagged activations [8][H] x2, [8][qkv], [8][qd], [8][I] and the
    // cross-CTA attention records (zero tags are never valid)
    c->persistent_ok = q8 && H == 1024 && I == 3072 && c->qd == 2048 && m.n_kv == 8 &&
                       m.layers <= (uint32_t)kFlowMaxLayers && flow_supported(c->device);
    if (c->persistent_ok) {
        std::vector<PersistentLayer> pl(m.layers);
        for (uint32_t l = 0; l < m.layers; ++l) {
            const LayerDev& Ld = c->L[l];
            pl[l] = PersistentLayer{static_cast<const int8_t*>(Ld.wqkv), static_cast<const int8_t*>(Ld.wo),
                                    static_cast<const int8_t*>(Ld.wgu), static_cast<const int8_t*>(Ld.wd),
                                    Ld.sqkv, Ld.so, Ld.sgu, Ld.sd, Ld.input_ln, Ld.post_ln, Ld.q_norm, Ld.k_norm};
        }
        if ((rc = dalloc(c, &c->dlayers, pl.size())) != ZYNFER_CU_OK) return rc;
        ZC_CHECK(c, cudaMemcpy(c->dlayers, pl.data(), pl.size() * sizeof(PersistentLayer), cudaMemcpyHostToDevice),
                 "persistent layer table");
        if ((rc = dalloc(c, &c->psync, 3)) != ZYNFER_CU_OK) return rc;
        cudaMemset(c->psync, 0, 3 * sizeof(unsigned));
        const int sms = c->caps.sm_count > 0 ? c->caps.sm_count : device_sm_count();
        c->ll_words = (size_t)kPersistentMaxBatch * (2 * H + c->qkv_rows + c->qd + I) + flow_record_words(sms);
        if ((rc = dalloc(c, &c->ll, c->ll_words)) != ZYNFER_CU_OK) return rc;
        cudaMemset(c->ll, 0, c->ll_words * 8);
    }
    if ((rc = halloc(c, &c->herr, 1)) != ZYNFER_CU_OK) return rc;
    if ((rc = halloc(c, &c->hio, 3 * B)) != ZYNFER_CU_OK) return rc;
    if ((rc = halloc(c, &c->hids, B)) != ZYNFER_CU_OK) return rc;
    cudaMemset(c->dkeys, 0, B * 8);
    cudaMemset(c->dcnt, 0, B * m.n_kv * 4);
    cudaMemset(c->derr, 0, 4);
    cudaMemset(c->dstep, 0, 4);
    ZC_CHECK(c, cudaDeviceSynchronize(), "model init");
    c->allocs.reserve(c->allocs.size() + 64);  // op-level scratch growth later does not move the list
    c->dev_alloc_events = 0;
    c->host_alloc_events = 0;
    c->ready = true;
    return ZYNFER_CU_OK;
}

int zynfer_cu_upload_f32(ZynferCuCtx* c, const char* name, const float* data, uint64_t rows, uint64_t cols) {
    if (!c || !c->ready || !name || !data) return c ? fail(c, ZYNFER_CU_INVALID, "bad upload arguments") : ZYNFER_CU_INVALID;
    if (c->fail_upload) {
        c->fail_upload = false;
        return fail(c, ZYNFER_CU_INTERNAL, "injected upload failure (ZYNFER_CUDA_FAIL_AT=upload)");
    }
    cudaSetDevice(c->device);
    Dest d = find_dest(c, name);
    if (d.kind == Dest::None) return fail(c, ZYNFER_CU_INVALID, std::string("unknown tensor ") + name);
    if ((uint64_t)d.rows * d.cols != rows * cols || (d.kind == Dest::Mat && (rows != (uint64_t)d.rows)))
        return fail(c, ZYNFER_CU_INVALID, std::string("shape mismatch for ") + name);
    float* tmp = nullptr;
    ZC_CHECK(c, cudaMalloc(&tmp, rows * cols * 4), "upload staging");
    cudaError_t e = cudaMemcpyAsync(tmp, data, rows * cols * 4, cudaMemcpyHostToDevice, c->stream);
    if (e == cudaSuccess) {
        place_f32(c, d, tmp);
        e = cudaStreamSynchronize(c->stream);
    }
    cudaFree(tmp);
    if (e != cudaSuccess) return cuda_fail(c, e, "upload");
    return ZYNFER_CU_OK;
}

int zynfer_cu_upload_bf16(ZynferCuCtx* c, const char* name, const uint16_t* data, uint64_t rows, uint64_t cols) {
    if (!c || !c->ready || !name || !data) return c ? fail(c, ZYNFER_CU_INVALID, "bad upload arguments") : ZYNFER_CU_INVALID;
    if (c->fail_upload) {
        c->fail_upload = false;
        return fail(c, ZYNFER_CU_INTERNAL, "injected upload failure (ZYNFER_CUDA_FAIL_AT=upload)");
    }
    cudaSetDevice(c->device);
    Dest d = find_dest(c, name);
    if (d.kind == Dest::None) return fail(c, ZYNFER_CU_INVALID, std::string("unknown tensor ") + name);
    if ((uint64_t)d.rows * d.cols != rows * cols) return fail(c, ZYNFER_CU_INVALID, std::string("shape mismatch for ") + name);
    uint16_t* tmp = nullptr;
    float* tmpf = nullptr;
    ZC_CHECK(c, cudaMalloc(&tmp, rows * cols * 2), "upload staging");
    cudaError_t e = cudaMalloc(&tmpf, rows * cols * 4);
    if (e == cudaSuccess) e = cudaMemcpyAsync(tmp, data, rows * cols * 2, cudaMemcpyHostToDevice, c->stream);
    if (e == cudaSuccess) {
        if (d.kind == Dest::Mat && c->wkind == kWBF16) {
            launch_copy_rows_u16(tmp, d.rows, d.cols, reinterpret_cast<uint16_t*>(d.w), d.stride, d.offset, c->stream);
        } else {
            launch_bf16_to_f32(tmp, rows * cols, tmpf, c->stream);
            place_f32(c, d, tmpf);
        }
        e = cudaStreamSynchronize(c->stream);
    }
    cudaFree(tmp);
    if (tmpf) cudaFree(tmpf);
    if (e != cudaSuccess) return cuda_fail(c, e, "upload");
    return ZYNFER_CU_OK;
}

int zynfer_cu_upload_q8(ZynferCuCtx* c, const char* name, const int8_t* q, const float* scale, uint64_t rows,
                        uint64_t cols) {
    if (!c || !c->ready || !name || !q || !scale) return c ? fail(c, ZYNFER_CU_INVALID, "bad upload arguments") : ZYNFER_CU_INVALID;
    if (c->fail_upload) {
        c->fail_upload = false;
        return fail(c, ZYNFER_CU_INTERNAL, "injected upload failure (ZYNFER_CUDA_FAIL_AT=upload)");
    }
    if (c->wkind != kWQ8) return fail(c, ZYNFER_CU_UNSUPPORTED, "int8 upload into a bf16 model");
    cudaSetDevice(c->device);
    Dest d = find_dest(c, name);
    if (d.kind != Dest::Mat) return fail(c, ZYNFER_CU_INVALID, std::string("not an int8 matrix: ") + name);
    if (rows != (uint64_t)d.rows || cols != (uint64_t)d.cols) return fail(c, ZYNFER_CU_INVALID, std::string("shape mismatch for ") + name);
    int8_t* tq = nullptr;
    float* ts = nullptr;
    ZC_CHECK(c, cudaMalloc(&tq, rows * cols), "upload staging");
    cudaError_t e = cudaMalloc(&ts, rows * 4);
    if (e == cudaSuccess) e = cudaMemcpyAsync(tq, q, rows * cols, cudaMemcpyHostToDevice, c->stream);
    if (e == cudaSuccess) e = cudaMemcpyAsync(ts, scale, rows * 4, cudaMemcpyHostToDevice, c->stream);
    if (e == cudaSuccess) {
        launch_copy_rows_i8(tq, ts, d.rows, d.cols, reinterpret_cast<int8_t*>(d.w), d.s, d.stride, d.offset, c->stream);
        e = cudaStreamSynchronize(c->stream);
    }
    cudaFree(tq);
    if (ts) cudaFree(ts);
    if (e != cudaSuccess) return cuda_fail(c, e, "upload");
    return ZYNFER_CU_OK;
}

int zynfer_cu_fill_synthetic(ZynferCuCtx* c, uint64_t seed, float w_std, float norm_std) {
    if (!c || !c->ready) return c ? fail(c, ZYNFER_CU_INVALID, "model not initialised") : ZYNFER_CU_INVALID;
    if (take_launch_fault(c)) return ZYNFER_CU_LAUNCH;
    cudaSetDevice(c->device);
    const ZynferCuModelDesc& m = c->d;
    const size_t maxn = std::max<size_t>((size_t)m.vocab * m.hidden, (size_t)2 * m.inter * m.hidden);
    float* tmp = nullptr;
    ZC_CHECK(c, cudaMalloc(&tmp, maxn * 4), "synthetic staging");
    const float kw = (float)((double)w_std / ZS_IH4_SIGMA);
    const float kn = (float)((double)norm_std / ZS_IH4_SIGMA);
    auto gen = [&](const char* name, uint64_t stream, bool is_norm) {
        Dest d = find_dest(c, name);
        const size_t n = (size_t)d.rows * d.cols;
        if (is_norm) {
            if (norm_std == 0.0f) launch_fill(tmp, n, 1.0f, c->stream);
            else launch_synth_normal(tmp, n, seed, stream, kn, 1.0f, c->stream);
        } else {
            launch_synth_normal(tmp, n, seed, stream, kw, 0.0f, c->stream);
        }
        if (c->wkind == kWBF16 && is_norm) {
            // a bf16 checkpoint stores norm weights in bf16 too (widened on load)
            uint16_t* t16 = reinterpret_cast<uint16_t*>(tmp + n);
            launch_to_bf16_rows(tmp, (int)n, 1, t16, 1, 0, c->stream);
            launch_bf16_to_f32(t16, n, tmp, c->stream);
        }
        place_f32(c, d, tmp);
    };
    gen("model.embed_tokens.weight", ZS_EMBED, false);
    gen("model.norm.weight", ZS_FINAL_NORM, true);
    static const char* names[11] = {"input_layernorm.weight", "self_attn.q_norm.weight", "self_attn.k_norm.weight",
                                    "self_attn.q_proj.weight", "self_attn.k_proj.weight", "self_attn.v_proj.weight",
                                    "self_attn.o_proj.weight", "post_attention_layernorm.weight",
                                    "mlp.gate_proj.weight", "mlp.up_proj.weight", "mlp.down_proj.weight"};
    static const int codes[11] = {ZS_INPUT_LN, ZS_Q_NORM, ZS_K_NORM, ZS_WQ, ZS_WK, ZS_WV, ZS_WO, ZS_POST_LN, ZS_WG, ZS_WU, ZS_WD};
    static const bool norm[11] = {true, true, true, false, false, false, false, true, false, false, false};
    char nm[160];
    for (uint32_t l = 0; l < m.layers; ++l)
        for (int t = 0; t < 11; ++t) {
            snprintf(nm, sizeof(nm), "model.layers.%u.%s", l, names[t]);
            gen(nm, zs_layer_stream(l, (uint32_t)codes[t]), norm[t]);
        }
    cudaError_t e = cudaStreamSynchronize(c->stream);
    cudaFree(tmp);
    if (e != cudaSuccess) return cuda_fail(c, e, "synthetic fill");
    e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(c, e, "synthetic fill launch");
    return ZYNFER_CU_OK;
}

int zynfer_cu_download_q8(ZynferCuCtx* c, const char* name, int8_t* q, float* scale, uint64_t rows, uint64_t cols) {
    if (!c || !c->ready || !name || !q || !scale) return c ? fail(c, ZYNFER_CU_INVALID, "bad download arguments") : ZYNFER_CU_INVALID;
    if (c->wkind != kWQ8) return fail(c, ZYNFER_CU_UNSUPPORTED, "not an int8 model");
    cudaSetDevice(c->device);
    Dest d = find_dest(c, name);
    if (d.kind != Dest::Mat || rows != (uint64_t)d.rows || cols != (uint64_t)d.cols)
        return fail(c, ZYNFER_CU_INVALID, std::string("bad tensor or shape: ") + name);
    int8_t* tq = nullptr;
    float* ts = nullptr;
    ZC_CHECK(c, cudaMalloc(&tq, rows * cols), "download staging");
    cudaError_t e = cudaMalloc(&ts, rows * 4);
    if (e == cudaSuccess) {
        launch_unpack_rows_i8(reinterpret_cast<const int8_t*>(d.w), d.s, d.rows, d.cols, tq, ts, d.stride, d.offset, c->stream);
        e = cudaMemcpyAsync(q, tq, rows * cols, cudaMemcpyDeviceToHost, c->stream);
    }
    if (e == cudaSuccess) e = cudaMemcpyAsync(scale, ts, rows * 4, cudaMemcpyDeviceToHost, c->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(c->stream);
    cudaFree(tq);
    if (ts) cudaFree(ts);
    if (e != cudaSuccess) return cuda_fail(c, e, "download");
    return ZYNFER_CU_OK;
}

int zynfer_cu_seq_reset(ZynferCuCtx* c, uint32_t seq) {
    if (!c || !c->ready) return c ? fail(c, ZYNFER_CU_INVALID, "model not initialised") : ZYNFER_CU_INVALID;
    if (seq >= c->d.max_seqs) return fail(c, ZYNFER_CU_INVALID, "sequence id out of range");
    release_seq(c, seq);
    return ZYNFER_CU_OK;
}

int zynfer_cu_seq_len(const ZynferCuCtx* c, uint32_t seq, uint32_t* len) {
    if (!c || !c->ready || !len || seq >= c->d.max_seqs) return ZYNFER_CU_INVALID;
    *len = c->seq_len[seq];
    return ZYNFER_CU_OK;
}

int zynfer_cu_kv_read(ZynferCuCtx* c, uint32_t seq, uint32_t layer, int which_v, float* out) {
    if (!c || !c->ready || !out) return c ? fail(c, ZYNFER_CU_INVALID, "bad arguments") : ZYNFER_CU_INVALID;
    if (seq >= c->d.max_seqs || layer >= c->d.layers) return fail(c, ZYNFER_CU_INVALID, "index out of range");
    cudaSetDevice(c->device);
    const int d = c->d.head_dim, nkv = c->d.n_kv;
    const uint32_t len = c->seq_len[seq];
    std::vector<uint16_t> blk((size_t)kKvBlock * d);
    for (uint32_t p0 = 0; p0 < len; p0 += kKvBlock) {
        const int b = c->seq_blocks[seq][p0 / kKvBlock];
        for (int h = 0; h < nkv; ++h) {
            const uint16_t* src = c->kv + layer * c->kv_layer_elems + (((size_t)h * c->n_blocks + b) * 2 + (which_v ? 1 : 0)) * kKvBlock * d;
            ZC_CHECK(c, cudaMemcpy(blk.data(), src, blk.size() * 2, cudaMemcpyDeviceToHost), "kv read");
            for (uint32_t i = 0; i < (uint32_t)kKvBlock && p0 + i < len; ++i)
                for (int e = 0; e < d; ++e) {
                    const uint32_t u = (uint32_t)blk[kv_swizzle((int)i, e)] << 16;
                    float f;
                    memcpy(&f, &u, 4);
                    out[((size_t)h * len + p0 + i) * d + e] = f;
                }
        }
    }
    return ZYNFER_CU_OK;
}

int zynfer_cu_kv_fill_synthetic(ZynferCuCtx* c, uint32_t seq, uint32_t n, uint64_t seed) {
    if (!c || !c->ready) return c ? fail(c, ZYNFER_CU_INVALID, "model not initialised") : ZYNFER_CU_INVALID;
    if (seq >= c->d.max_seqs) return fail(c, ZYNFER_CU_INVALID, "sequence id out of range");
    if (n > c->d.max_seq_len) return fail(c, ZYNFER_CU_INVALID, "n exceeds max_seq_len");
    if (c->d.head_dim != 128) return fail(c, ZYNFER_CU_UNSUPPORTED, "head_dim must be 128");
    if (take_launch_fault(c)) return ZYNFER_CU_LAUNCH;
    cudaSetDevice(c->device);
    release_seq(c, seq);
    int rc = ensure_blocks(c, seq, n);
    if (rc) return rc;
    if ((rc = upload_table_rows(c, &seq, 1))) return rc;
    launch_kv_fill(c->kv, c->kv_layer_elems, c->table_dev + (size_t)seq * c->max_blocks, c->n_blocks,
                   (int)c->d.layers, (int)c->d.n_kv, (int)n, seed, c->derr, c->stream);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(c, e, "kv fill launch");
    if ((rc = check_device_error(c))) return rc;
    c->seq_len[seq] = n;
    set_path(c, "kv_fill", 0, nullptr);
    return ZYNFER_CU_OK;
}

int zynfer_cu_seq_fork(ZynferCuCtx* c, uint32_t dst, uint32_t src, uint32_t n) {
    if (!c || !c->ready) return c ? fail(c, ZYNFER_CU_INVALID, "model not initialised") : ZYNFER_CU_INVALID;
    if (dst >= c->d.max_seqs || src >= c->d.max_seqs || dst == src)
        return fail(c, ZYNFER_CU_INVALID, "fork: two different sequence slots");
    if (n > c->seq_len[src]) return fail(c, ZYNFER_CU_INVALID, "fork: n is longer than the source sequence");
    if (take_launch_fault(c)) return ZYNFER_CU_LAUNCH;
    cudaSetDevice(c->device);
    release_seq(c, dst);
    const uint32_t full = n / kKvBlock, rest = n % kKvBlock;
    std::vector<int>& sb = c->seq_blocks[src];
    std::vector<int>& db = c->seq_blocks[dst];
    for (uint32_t i = 0; i < full; ++i) {  // whole blocks are shared: no sequence ever writes a full block again
        const int b = sb[i];
        c->block_refs[b] += 1;
        c->table_host[(size_t)dst * c->max_blocks + i] = b;
        db.push_back(b);
    }
    c->table_dirty[dst] = 1;
    if (rest) {
        // the partly filled block is the one dst appends into next: dst gets its own copy
        int rc = ensure_blocks(c, dst, n);
        if (rc) return rc;
        const int from = sb[full], to = db[full];
        const size_t hd = c->d.head_dim, blk_elems = (size_t)2 * kKvBlock * hd;  // K then V of one head
        for (uint32_t l = 0; l < c->d.layers; ++l) {
            uint16_t* base = c->kv + l * c->kv_layer_elems;
            ZC_CHECK(c, cudaMemcpy2DAsync(base + (size_t)to * blk_elems, (size_t)c->n_blocks * blk_elems * 2,
                                          base + (size_t)from * blk_elems, (size_t)c->n_blocks * blk_elems * 2,
                                          blk_elems * 2, c->d.n_kv, cudaMemcpyDeviceToDevice, c->stream),
                     "fork: copy the partial block");
        }
    }
    int rc = upload_table_rows(c, &dst, 1);
    if (rc) return rc;
    ZC_CHECK(c, cudaStreamSynchronize(c->stream), "fork");
    c->seq_len[dst] = n;
    set_path(c, "seq_fork", 0, nullptr);
    return ZYNFER_CU_OK;
}

int zynfer_cu_extend(ZynferCuCtx* c, uint32_t seq, const uint32_t* tokens, uint32_t n, float* last_logits,
                     uint32_t* argmax) {
    if (!c || !c->ready) return c ? fail(c, ZYNFER_CU_INVALID, "model not initialised") : ZYNFER_CU_INVALID;
    if (!tokens || n == 0) return fail(c, ZYNFER_CU_INVALID, "extend: no tokens");
    if (seq >= c->d.max_seqs) return fail(c, ZYNFER_CU_INVALID, "sequence id out of range");
    if ((uint64_t)c->seq_len[seq] + n > c->d.max_seq_len) return fail(c, ZYNFER_CU_INVALID, "KV cache full");
    uint32_t id = 0;
    for (uint32_t i = 0; i < n; ++i) {
        int rc = zynfer_cu_decode_step(c, &seq, tokens + i, 1, &id, i + 1 == n ? last_logits : nullptr);
        if (rc) return rc;
    }
    if (argmax) *argmax = id;
    set_path(c, "extend", 0, nullptr);
    return ZYNFER_CU_OK;
}

int zynfer_cu_pool_stats(const ZynferCuCtx* c, uint32_t* free_blocks, uint32_t* shared_blocks) {
    if (!c || !c->ready || !free_blocks || !shared_blocks) return ZYNFER_CU_INVALID;
    uint32_t shared = 0;
    for (uint32_t r : c->block_refs) shared += r > 1 ? 1u : 0u;
    *free_blocks = (uint32_t)c->free_blocks.size();
    *shared_blocks = shared;
    return ZYNFER_CU_OK;
}

int zynfer_cu_attn_decode(ZynferCuCtx* c, uint32_t layer, const uint32_t* seqs, uint32_t batch, const float* qkv,
                          float* out) {
    if (!c) return ZYNFER_CU_INVALID;
    if (!seqs || !qkv || !out) return fail(c, ZYNFER_CU_INVALID, "null argument");
    int rc = validate_batch(c, seqs, batch, 1);
    if (rc) return rc;
    if (layer >= c->d.layers) return fail(c, ZYNFER_CU_INVALID, "layer out of range");
    if (reinterpret_cast<uintptr_t>(qkv) % 16 || reinterpret_cast<uintptr_t>(out) % 16)
        return fail(c, ZYNFER_CU_INVALID, "qkv and out must be 16-byte aligned");
    if (take_launch_fault(c)) return ZYNFER_CU_LAUNCH;
    cudaSetDevice(c->device);
    for (uint32_t i = 0; i < batch; ++i)
        if ((rc = ensure_blocks(c, seqs[i], c->seq_len[seqs[i]] + 1))) return rc;
    if ((rc = upload_table_rows(c, seqs, batch))) return rc;
    set_io_views(c, (int)batch);
    for (uint32_t i = 0; i < batch; ++i) {
        c->hio[i] = 0;
        c->hio[batch + i] = seqs[i];
        c->hio[2 * batch + i] = c->seq_len[seqs[i]];
    }
    ZC_CHECK(c, cudaMemcpyAsync(c->dio, c->hio, (size_t)3 * batch * 4, cudaMemcpyHostToDevice, c->stream), "stage");
    const ZynferCuModelDesc& m = c->d;
    const LayerDev& Ld = c->L[layer];
    AttnDecodeArgs aa{};
    aa.qkv = qkv; aa.q_norm = Ld.q_norm; aa.k_norm = Ld.k_norm; aa.rope = c->rope;
    aa.rope_max_pos = (int)m.max_seq_len; aa.eps = m.eps;
    aa.kv_layer = c->kv + layer * c->kv_layer_elems; aa.block_table = c->table_dev;
    aa.max_blocks = c->max_blocks; aa.n_pool_blocks = c->n_blocks;
    aa.seq_of = c->dseq; aa.positions = c->dpos; aa.B = (int)batch; aa.n_q = m.n_q; aa.n_kv = m.n_kv;
    aa.d = m.head_dim; aa.max_segs = decode_max_segs(c->max_blocks); aa.partial = c->dpart;
    aa.counters = c->dcnt; aa.out = out; aa.err = c->derr;
    aa.head_clusters = attn_head_clusters((int)batch, (long long)c->seq_len[seqs[0]] + 1);
    launch_attn_decode(aa, c->stream);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(c, e, "attention launch");
    if ((rc = check_device_error(c))) return rc;
    set_path(c, "attn_decode", 0, nullptr);
    return ZYNFER_CU_OK;
}

int zynfer_cu_rmsnorm_qk_rope(ZynferCuCtx* c, const float* qkv, uint32_t rows, const float* q_norm,
                              const float* k_norm, uint32_t pos0, float* q_out, float* k_out) {
    if (!c || !c->ready) return c ? fail(c, ZYNFER_CU_INVALID, "model not initialised") : ZYNFER_CU_INVALID;
    if (!qkv || !q_norm || !k_norm || !q_out || !k_out || rows == 0) return fail(c, ZYNFER_CU_INVALID, "bad arguments");
    if ((uint64_t)pos0 + rows > c->d.max_seq_len) return fail(c, ZYNFER_CU_INVALID, "positions beyond max_seq_len");
    if (take_launch_fault(c)) return ZYNFER_CU_LAUNCH;
    cudaSetDevice(c->device);
    const ZynferCuModelDesc& m = c->d;
    QkvArgs qa{};
    qa.qkv = qkv; qa.T = (int)rows; qa.n_q = m.n_q; qa.n_kv = m.n_kv; qa.d = m.head_dim;
    qa.q_norm = q_norm; qa.k_norm = k_norm; qa.eps = m.eps;
    qa.rope = c->rope; qa.rope_max_pos = (int)m.max_seq_len;
    qa.row_pos = nullptr; qa.pos0 = (int)pos0; qa.row_seq = nullptr; qa.seq0 = 0;
    qa.kv_layer = nullptr; qa.block_table = nullptr; qa.max_blocks = 0; qa.n_pool_blocks = 0;
    qa.q_out = q_out; qa.q_heads_major = 1; qa.k_stage = k_out; qa.v_stage = nullptr;
    qa.stage_round_bf16 = 0; qa.err = c->derr;
    launch_qkv_post(qa, c->stream);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(c, e, "norm/rope launch");
    int rc = check_device_error(c);
    if (rc) return rc;
    set_path(c, "rmsnorm_qk_rope", 0, nullptr);
    return ZYNFER_CU_OK;
}

int zynfer_cu_swiglu(ZynferCuCtx* c, const float* gate, const float* up, uint64_t n, float* out) {
    if (!c || c->device < 0) return ZYNFER_CU_INVALID;
    if (!gate || !up || !out || n == 0) return fail(c, ZYNFER_CU_INVALID, "bad swiglu arguments");
    if (take_launch_fault(c)) return ZYNFER_CU_LAUNCH;
    cudaSetDevice(c->device);
    launch_silu_mul(gate, up, (size_t)n, out, c->stream);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(c, e, "swiglu launch");
    set_path(c, "swiglu", 0, nullptr);
    return ZYNFER_CU_OK;
}

int zynfer_cu_alloc_events(const ZynferCuCtx* c, uint64_t* device, uint64_t* host) {
    if (!c || !device || !host) return ZYNFER_CU_INVALID;
    *device = c->dev_alloc_events;
    *host = c->host_alloc_events;
    return ZYNFER_CU_OK;
}

int zynfer_cu_prefill(ZynferCuCtx* c, uint32_t seq, const uint32_t* tokens, uint32_t n, float* last_logits,
                      uint32_t* argmax) {
    if (!c || !c->ready) return c ? fail(c, ZYNFER_CU_INVALID, "model not initialised") : ZYNFER_CU_INVALID;
    if (seq >= c->d.max_seqs) return fail(c, ZYNFER_CU_INVALID, "sequence id out of range");
    if (n == 0 || !tokens) return fail(c, ZYNFER_CU_INVALID, "empty prompt");  // qwen_forward.zig:101
    if (n > c->d.max_prefill || n > c->d.max_seq_len) return fail(c, ZYNFER_CU_INVALID, "prompt longer than max_prefill / max_seq_len");
    for (uint32_t i = 0; i < n; ++i)
        if (tokens[i] >= c->d.vocab) return fail(c, ZYNFER_CU_INVALID, "token id >= vocab");  // ops.zig:406
    if (take_launch_fault(c)) return ZYNFER_CU_LAUNCH;
    cudaSetDevice(c->device);
    release_seq(c, seq);  // qwen_forward.zig:110 (reset)
    int rc = ensure_blocks(c, seq, n);
    if (rc) return rc;
    if ((rc = upload_table_rows(c, &seq, 1))) return rc;
    const ZynferCuModelDesc& m = c->d;
    ZC_CHECK(c, cudaMemcpyAsync(c->ptok, tokens, (size_t)n * 4, cudaMemcpyHostToDevice, c->stream), "prompt upload");
    cudaEventRecord(c->ev0, c->stream);
    c->step_paths = 0;
    launch_embed(c->embed, c->sembed, c->wkind, c->ptok, n, m.hidden, m.vocab, c->px, c->derr, c->stream);
    enqueue_prefill_layers(c, seq, (int)n, 0, m.layers);
    const bool sampling = c->samp_temp > 0.0f;
    linear(c, ZYNFER_CU_K_LMHEAD, c->embed, c->sembed, &c->tm_embed, m.vocab, m.hidden, c->px + (size_t)(n - 1) * m.hidden, 1,
           last_logits || sampling ? c->dlogits : nullptr, kEpiArgmax, nullptr, c->final_norm, c->dkeys);
    if (sampling) enqueue_sample(c, 1, nullptr, nullptr, (int)seq, (int)n - 1);
    FinalizeArgs fa{};
    fa.keys = c->dkeys; fa.ids_out = c->dids; fa.B = 1;
    launch_finalize(fa, c->stream);
    cudaEventRecord(c->ev1, c->stream);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(c, e, "prefill launch");
    if (last_logits) ZC_CHECK(c, cudaMemcpyAsync(last_logits, c->dlogits, (size_t)m.vocab * 4, cudaMemcpyDeviceToHost, c->stream), "logits");
    ZC_CHECK(c, cudaMemcpyAsync(c->hids, c->dids, 4, cudaMemcpyDeviceToHost, c->stream), "argmax");
    if ((rc = check_device_error(c))) return rc;
    float ms = 0.0f;
    cudaEventElapsedTime(&ms, c->ev0, c->ev1);
    c->last_step_ns = (uint64_t)(ms * 1e6);
    if (argmax) *argmax = c->hids[0];
    c->seq_len[seq] = n;
    set_path(c, "prefill", c->step_paths, nullptr);
    return ZYNFER_CU_OK;
}

int zynfer_cu_decode_step(ZynferCuCtx* c, const uint32_t* seqs, const uint32_t* tokens, uint32_t batch,
                          uint32_t* argmax, float* logits) {
    if (!c) return ZYNFER_CU_INVALID;
    if (!seqs || !tokens || !argmax) return fail(c, ZYNFER_CU_INVALID, "null argument");
    int rc = validate_batch(c, seqs, batch, 1);
    if (rc) return rc;
    if (take_launch_fault(c)) return ZYNFER_CU_LAUNCH;
    cudaSetDevice(c->device);
    for (uint32_t i = 0; i < batch; ++i)
        if ((rc = ensure_blocks(c, seqs[i], c->seq_len[seqs[i]] + 1))) return rc;
    if ((rc = upload_table_rows(c, seqs, batch))) return rc;
    set_io_views(c, (int)batch);
    if ((rc = stage_batch(c, seqs, tokens, batch))) return rc;
    ZC_CHECK(c, cudaMemsetAsync(c->dstep, 0, 4, c->stream), "step counter");
    c->head_clusters = attn_head_clusters((int)batch, (long long)c->seq_len[seqs[0]] + 1);
    const bool persistent = use_persistent(c, (int)batch);
    const bool eager = logits != nullptr || c->timing || persistent;
    unsigned paths = 0;
    if (!eager) {
        GraphEntry g;
        if ((rc = get_graph(c, (int)batch, &g))) return rc;
        cudaEventRecord(c->ev0, c->stream);
        ZC_CHECK(c, cudaGraphLaunch(g.exec, c->stream), "graph launch");
        paths = g.paths;
    } else {
        cudaEventRecord(c->ev0, c->stream);
        c->step_paths = 0;
        enqueue_decode(c, (int)batch, logits != nullptr);
        paths = c->step_paths;
    }
    cudaEventRecord(c->ev1, c->stream);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(c, e, "decode launch");
    ZC_CHECK(c, cudaMemcpyAsync(c->hids, c->dids, (size_t)batch * 4, cudaMemcpyDeviceToHost, c->stream), "argmax");
    c->d2h_bytes += (size_t)batch * 4;
    if (logits) {
        ZC_CHECK(c, cudaMemcpyAsync(logits, c->dlogits, (size_t)batch * c->d.vocab * 4, cudaMemcpyDeviceToHost, c->stream), "logits");
        c->d2h_bytes += (size_t)batch * c->d.vocab * 4;
    }
    if ((rc = check_device_error(c))) return rc;
    float ms = 0.0f;
    cudaEventElapsedTime(&ms, c->ev0, c->ev1);
    c->last_step_ns = (uint64_t)(ms * 1e6);
    for (uint32_t i = 0; i < batch; ++i) {
        argmax[i] = c->hids[i];
        c->seq_len[seqs[i]] += 1;
    }
    if (persistent) set_path(c, "decode", 0, "persistent");
    else set_path(c, "decode", paths, eager ? "eager" : "graph");
    return ZYNFER_CU_OK;
}

int zynfer_cu_generate(ZynferCuCtx* c, const uint32_t* seqs, const uint32_t* first, uint32_t batch, uint32_t steps,
                       uint32_t* out_ids, float* device_ms) {
    if (!c) return ZYNFER_CU_INVALID;
    if (!seqs || !first || !out_ids) return fail(c, ZYNFER_CU_INVALID, "null argument");
    if (steps == 0) return ZYNFER_CU_OK;
    int rc = validate_batch(c, seqs, batch, steps);
    if (rc) return rc;
    if ((size_t)steps * batch > c->hist_cap) return fail(c, ZYNFER_CU_INVALID, "steps * batch exceeds the on-device history");
    if (take_launch_fault(c)) return ZYNFER_CU_LAUNCH;
    cudaSetDevice(c->device);
    for (uint32_t i = 0; i < batch; ++i)
        if ((rc = ensure_blocks(c, seqs[i], c->seq_len[seqs[i]] + steps))) return rc;
    if ((rc = upload_table_rows(c, seqs, batch))) return rc;
    set_io_views(c, (int)batch);
    if ((rc = stage_batch(c, seqs, first, batch))) return rc;
    ZC_CHECK(c, cudaMemsetAsync(c->dstep, 0, 4, c->stream), "step counter");
    // one sequence: the whole call keeps the choice of its longest step
    c->head_clusters = attn_head_clusters((int)batch, (long long)c->seq_len[seqs[0]] + steps);
    const bool persistent = use_persistent(c, (int)batch);
    GraphEntry g;
    if (!c->timing && !persistent && (rc = get_graph(c, (int)batch, &g))) return rc;
    c->step_paths = 0;
    cudaEventRecord(c->ev0, c->stream);
    for (uint32_t s = 0; s < steps; ++s) {
        if (c->timing || persistent) enqueue_decode(c, (int)batch, false);
        else ZC_CHECK(c, cudaGraphLaunch(g.exec, c->stream), "graph launch");
    }
    const unsigned paths = (c->timing || persistent) ? c->step_paths : g.paths;
    cudaEventRecord(c->ev1, c->stream);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(c, e, "generate launch");
    if ((rc = check_device_error(c))) return rc;
    float ms = 0.0f;
    cudaEventElapsedTime(&ms, c->ev0, c->ev1);
    if (device_ms) *device_ms = ms;
    c->last_step_ns = (uint64_t)(ms * 1e6 / steps);
    ZC_CHECK(c, cudaMemcpy(out_ids, c->dhist, (size_t)steps * batch * 4, cudaMemcpyDeviceToHost), "history");
    for (uint32_t i = 0; i < batch; ++i) c->seq_len[seqs[i]] += steps;
    if (persistent) set_path(c, "generate", 0, "persistent");
    else set_path(c, "generate", paths, c->timing ? "eager" : "graph");
    return ZYNFER_CU_OK;
}

int zynfer_cu_block_forward(ZynferCuCtx* c, uint32_t layer, uint32_t seq, const float* x, uint32_t t, float* out) {
    if (!c || !c->ready) return c ? fail(c, ZYNFER_CU_INVALID, "model not initialised") : ZYNFER_CU_INVALID;
    if (!x || !out || t == 0) return fail(c, ZYNFER_CU_INVALID, "bad arguments");
    if (layer >= c->d.layers || seq >= c->d.max_seqs) return fail(c, ZYNFER_CU_INVALID, "index out of range");
    const uint32_t pos0 = c->seq_len[seq];
    if (pos0 + t > c->d.max_seq_len) return fail(c, ZYNFER_CU_INVALID, "KV cache full");  // qwen_block.zig:176
    if (pos0 == 0 && t > c->d.max_prefill) return fail(c, ZYNFER_CU_INVALID, "t > max_prefill");
    if (take_launch_fault(c)) return ZYNFER_CU_LAUNCH;
    cudaSetDevice(c->device);
    int rc = ensure_blocks(c, seq, pos0 + t);
    if (rc) return rc;
    if ((rc = upload_table_rows(c, &seq, 1))) return rc;
    const ZynferCuModelDesc& m = c->d;
    const int H = m.hidden;
    c->step_paths = 0;
    if (pos0 == 0) {
        ZC_CHECK(c, cudaMemcpyAsync(c->px, x, (size_t)t * H * 4, cudaMemcpyHostToDevice, c->stream), "x upload");
        enqueue_prefill_layers(c, seq, (int)t, layer, layer + 1);
        ZC_CHECK(c, cudaMemcpyAsync(out, c->px, (size_t)t * H * 4, cudaMemcpyDeviceToHost, c->stream), "out");
    } else {
        // tokens after a cached prefix go one at a time through the decode path
        // (prefill == stepwise decode, tiny_block.zig:352-383)
        const LayerDev& Ld = c->L[layer];
        set_io_views(c, 1);
        for (uint32_t i = 0; i < t; ++i) {
            c->hio[0] = 0;
            c->hio[1] = seq;
            c->hio[2] = pos0 + i;
            ZC_CHECK(c, cudaMemcpyAsync(c->dio, c->hio, 12, cudaMemcpyHostToDevice, c->stream), "stage");
            ZC_CHECK(c, cudaMemcpyAsync(c->dx, x + (size_t)i * H, (size_t)H * 4, cudaMemcpyHostToDevice, c->stream), "x");
            linear(c, ZYNFER_CU_K_LINEAR, Ld.wqkv, Ld.sqkv, &Ld.tm_qkv, c->qkv_rows, H, c->dx, 1, c->dqkv, kEpiNone, nullptr, Ld.input_ln, nullptr);
            AttnDecodeArgs aa{};
            aa.qkv = c->dqkv; aa.q_norm = Ld.q_norm; aa.k_norm = Ld.k_norm; aa.rope = c->rope;
            aa.rope_max_pos = (int)m.max_seq_len; aa.eps = m.eps;
            aa.kv_layer = c->kv + layer * c->kv_layer_elems; aa.block_table = c->table_dev;
            aa.max_blocks = c->max_blocks; aa.n_pool_blocks = c->n_blocks; aa.seq_of = c->dseq; aa.positions = c->dpos;
            aa.B = 1; aa.n_q = m.n_q; aa.n_kv = m.n_kv; aa.d = m.head_dim;
            aa.max_segs = decode_max_segs(c->max_blocks); aa.partial = c->dpart;
            aa.counters = c->dcnt; aa.out = c->dattn; aa.err = c->derr;
            aa.head_clusters = attn_head_clusters(1, (long long)pos0 + i + 1);
            launch_attn_decode(aa, c->stream);
            linear(c, ZYNFER_CU_K_LINEAR, Ld.wo, Ld.so, &Ld.tm_o, H, c->qd, c->dattn, 1, c->dx1, kEpiResid, c->dx, nullptr, nullptr);
            linear(c, ZYNFER_CU_K_LINEAR, Ld.wgu, Ld.sgu, &Ld.tm_gu, 2 * m.inter, H, c->dx1, 1, c->dh, kEpiSwiGLU, nullptr, Ld.post_ln, nullptr);
            linear(c, ZYNFER_CU_K_LINEAR, Ld.wd, Ld.sd, &Ld.tm_d, H, m.inter, c->dh, 1, c->dx, kEpiResid, c->dx1, nullptr, nullptr);
            ZC_CHECK(c, cudaMemcpyAsync(out + (size_t)i * H, c->dx, (size_t)H * 4, cudaMemcpyDeviceToHost, c->stream), "out");
            ZC_CHECK(c, cudaStreamSynchronize(c->stream), "block step");
        }
    }
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(c, e, "block launch");
    if ((rc = check_device_error(c))) return rc;
    c->seq_len[seq] = pos0 + t;
    set_path(c, pos0 == 0 ? "block:prefill" : "block:decode", c->step_paths, nullptr);
    return ZYNFER_CU_OK;
}

int zynfer_cu_linear(ZynferCuCtx* c, int wkind, const void* w, const float* scale, const float* x, uint32_t batch,
                     uint32_t m, uint32_t k, float* y) {
    if (!c || c->device < 0) return ZYNFER_CU_INVALID;
    if (!w || !x || !y || batch == 0 || m == 0 || k == 0) return fail(c, ZYNFER_CU_INVALID, "bad linear arguments");
    if (wkind != ZYNFER_CU_W_Q8 && wkind != ZYNFER_CU_W_BF16) return fail(c, ZYNFER_CU_INVALID, "unknown weight kind");
    if (wkind == ZYNFER_CU_W_Q8 && !scale) return fail(c, ZYNFER_CU_INVALID, "int8 weights need scales");
    if (k % 512) return fail(c, ZYNFER_CU_UNSUPPORTED, "k must be a multiple of 512");
    if (reinterpret_cast<uintptr_t>(w) % 16 || reinterpret_cast<uintptr_t>(x) % 16 || reinterpret_cast<uintptr_t>(y) % 8)
        return fail(c, ZYNFER_CU_INVALID, "w and x must be 16-byte and y 8-byte aligned");
    if (m % 128) return fail(c, ZYNFER_CU_UNSUPPORTED, "m must be a multiple of 128");
    if (take_launch_fault(c)) return ZYNFER_CU_LAUNCH;
    cudaSetDevice(c->device);
    const int wk = wkind == ZYNFER_CU_W_Q8 ? kWQ8 : kWBF16;
    int rc = ensure_tc_scratch(c, (int)batch, (int)k, (int)m);
    if (rc) return rc;
    if (c->simt_xn_elems < (size_t)batch * k) {
        if ((rc = dalloc(c, &c->simt_xn, (size_t)batch * k))) return rc;
        c->simt_xn_elems = (size_t)batch * k;
    }
    const auto key = std::make_pair(w, ((uint64_t)wk << 62) | ((uint64_t)m << 32) | (uint64_t)k);
    auto it = c->amaps.find(key);
    if (it == c->amaps.end()) {
        CUtensorMap tm;
        if (!make_tmap_k_major(&tm, w, wk, k, m, 128)) return fail(c, ZYNFER_CU_INTERNAL, "cuTensorMapEncodeTiled failed");
        it = c->amaps.emplace(key, tm).first;
    }
    c->step_launches = 0;
    const int p = linear(c, ZYNFER_CU_K_LINEAR, w, wk == kWQ8 ? scale : nullptr, &it->second, (int)m, (int)k, x,
                         (int)batch, y, kEpiNone, nullptr, nullptr, nullptr, wk);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(c, e, "linear launch");
    set_path(c, "linear", 1u << p, nullptr);
    return ZYNFER_CU_OK;
}

int zynfer_cu_set_sampling(ZynferCuCtx* c, float temperature, uint32_t top_k, float top_p, uint64_t seed) {
    if (!c) return ZYNFER_CU_INVALID;
    if (!(temperature >= 0.0f) || temperature > 1e6f || top_k > 64 || !(top_p > 0.0f) || top_p > 1.0f)
        return fail(c, ZYNFER_CU_INVALID, "sampling: temperature >= 0, top_k <= 64, 0 < top_p <= 1");
    c->samp_temp = temperature;
    c->samp_top_k = top_k;
    c->samp_top_p = top_p;
    c->samp_seed = seed;
    for (auto& kv : c->graphs) cudaGraphExecDestroy(kv.second.exec);  // graphs bake the rule
    c->graphs.clear();
    return ZYNFER_CU_OK;
}

int zynfer_cu_sample(ZynferCuCtx* c, const float* logits, uint32_t rows, uint32_t vocab, const uint32_t* slots,
                     const uint32_t* positions, float temperature, uint32_t top_k, float top_p, uint64_t seed,
                     uint32_t* out_ids) {
    if (!c || !c->ready) return c ? fail(c, ZYNFER_CU_INVALID, "model not initialised") : ZYNFER_CU_INVALID;
    if (!logits || !slots || !positions || !out_ids || rows == 0 || vocab == 0)
        return fail(c, ZYNFER_CU_INVALID, "bad sample arguments");
    if (rows > c->d.max_batch) return fail(c, ZYNFER_CU_INVALID, "rows > max_batch");
    if (!(temperature > 0.0f) || top_k > 64 || !(top_p > 0.0f) || top_p > 1.0f)
        return fail(c, ZYNFER_CU_INVALID, "sampling: temperature > 0, top_k <= 64, 0 < top_p <= 1");
    if (take_launch_fault(c)) return ZYNFER_CU_LAUNCH;
    cudaSetDevice(c->device);
    for (uint32_t i = 0; i < rows; ++i) {
        c->hio[i] = slots[i];
        c->hio[rows + i] = positions[i];
    }
    ZC_CHECK(c, cudaMemcpyAsync(c->dio, c->hio, (size_t)2 * rows * 4, cudaMemcpyHostToDevice, c->stream), "stage");
    SampleArgs sa{};
    sa.logits = logits; sa.V = (int)vocab; sa.rows = (int)rows; sa.inv_t = 1.0f / temperature;
    sa.top_k = (int)top_k; sa.top_p = top_p; sa.seed = seed;
    sa.seq_of = reinterpret_cast<const int*>(c->dio); sa.positions = reinterpret_cast<const int*>(c->dio + rows);
    sa.keys_out = nullptr; sa.ids_out = c->dids;
    launch_sample(sa, c->stream);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(c, e, "sample launch");
    ZC_CHECK(c, cudaMemcpyAsync(c->hids, c->dids, (size_t)rows * 4, cudaMemcpyDeviceToHost, c->stream), "ids");
    int rc = check_device_error(c);
    if (rc) return rc;
    for (uint32_t i = 0; i < rows; ++i) out_ids[i] = c->hids[i];
    set_path(c, "sample", 0, nullptr);
    return ZYNFER_CU_OK;
}

int zynfer_cu_set_linear_path(ZynferCuCtx* c, const char* path) {
    if (!c || !path) return ZYNFER_CU_INVALID;
    if (!strcmp(path, "auto")) c->path_policy = kPathAuto;
    else if (!strcmp(path, "gemv")) c->path_policy = kPathGemv;
    else if (!strcmp(path, "simt")) c->path_policy = kPathSimt;
    else if (!strcmp(path, "tcgen05")) c->path_policy = kPathTc;
    else if (!strcmp(path, "mma")) c->path_policy = kPathMma;
    else return fail(c, ZYNFER_CU_INVALID, std::string("unknown linear path ") + path);
    for (auto& kv : c->graphs) cudaGraphExecDestroy(kv.second.exec);  // graphs bake the old choice
    c->graphs.clear();
    return ZYNFER_CU_OK;
}

int zynfer_cu_set_decode_schedule(ZynferCuCtx* c, const char* schedule) {
    if (!c || !schedule) return ZYNFER_CU_INVALID;
    if (!strcmp(schedule, "auto")) c->schedule = kSchedAuto;
    else if (!strcmp(schedule, "kernels")) c->schedule = kSchedKernels;
    else if (!strcmp(schedule, "persistent")) {
        if (c->ready && !c->persistent_ok)
            return fail(c, ZYNFER_CU_UNSUPPORTED, "the persistent decode kernel needs int8 weights, hidden 1024, "
                                                  "intermediate 3072, 16 x 128 query and 8 x 128 kv dims, at most "
                                                  "62 layers, 100+ SMs and cooperative launch");
        c->schedule = kSchedPersistent;
    } else {
        return fail(c, ZYNFER_CU_INVALID, std::string("unknown decode schedule ") + schedule);
    }
    return ZYNFER_CU_OK;
}

int zynfer_cu_pack_q8(ZynferCuCtx* c, const float* w, uint32_t rows, uint32_t cols, int8_t* q, float* scale) {
    if (!c || c->device < 0) return ZYNFER_CU_INVALID;
    if (!w || !q || !scale || rows == 0 || cols == 0) return fail(c, ZYNFER_CU_INVALID, "bad pack arguments");
    if (take_launch_fault(c)) return ZYNFER_CU_LAUNCH;
    cudaSetDevice(c->device);
    launch_pack_q8_rows(w, (int)rows, (int)cols, q, scale, 1, 0, c->stream);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(c, e, "pack launch");
    return ZYNFER_CU_OK;
}

int zynfer_cu_rmsnorm(ZynferCuCtx* c, const float* x, const float* w, uint32_t rows, uint32_t cols, float eps, float* y) {
    if (!c || c->device < 0) return ZYNFER_CU_INVALID;
    if (!x || !w || !y || rows == 0 || cols % 128) return fail(c, ZYNFER_CU_INVALID, "bad rmsnorm arguments");
    if (take_launch_fault(c)) return ZYNFER_CU_LAUNCH;
    cudaSetDevice(c->device);
    launch_rmsnorm(x, w, y, (int)rows, (int)cols, eps, c->stream);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(c, e, "rmsnorm launch");
    return ZYNFER_CU_OK;
}

int zynfer_cu_set_timing(ZynferCuCtx* c, int enable) {
    if (!c || c->device < 0) return ZYNFER_CU_INVALID;
    cudaSetDevice(c->device);
    if (enable && c->tev.empty()) {
        c->tev.resize(8192);
        for (auto& t : c->tev) {
            cudaEventCreate(&t.a);
            cudaEventCreate(&t.b);
        }
    }
    if (enable) {
        c->tev_used = 0;
        for (int i = 0; i < 4; ++i) {
            c->t_launch[i] = 0;
            c->t_ms[i] = 0.0;
        }
    }
    c->timing = enable != 0;
    return ZYNFER_CU_OK;
}

int zynfer_cu_kernel_time(const ZynferCuCtx* cc, int cls, uint64_t* launches, double* total_ms) {
    ZynferCuCtx* c = const_cast<ZynferCuCtx*>(cc);
    if (!c || cls < 0 || cls > 3 || !launches || !total_ms) return ZYNFER_CU_INVALID;
    cudaSetDevice(c->device);
    cudaStreamSynchronize(c->stream);
    for (size_t i = 0; i < c->tev_used; ++i) {
        float ms = 0.0f;
        cudaEventElapsedTime(&ms, c->tev[i].a, c->tev[i].b);
        c->t_ms[c->tev[i].cls] += ms;
        c->t_launch[c->tev[i].cls] += 1;
    }
    c->tev_used = 0;
    *launches = c->t_launch[cls];
    *total_ms = c->t_ms[cls];
    return ZYNFER_CU_OK;
}

uint64_t zynfer_cu_last_step_ns(const ZynferCuCtx* c) { return c ? c->last_step_ns : 0; }

int zynfer_cu_phase_trace(const ZynferCuCtx* c, uint64_t* out, int cap) {
    if (!c) return 0;
    const int n = (int)c->ptrace_host.size();
    if (out)
        for (int i = 0; i < n && i < cap; ++i) out[i] = c->ptrace_host[i];
    return n;
}

int zynfer_cu_step_launches(const ZynferCuCtx* c) { return c ? c->step_launches : 0; }

int zynfer_cu_io_bytes(ZynferCuCtx* c, uint64_t* h2d, uint64_t* d2h, int reset) {
    if (!c || !h2d || !d2h) return ZYNFER_CU_INVALID;
    *h2d = c->h2d_bytes;
    *d2h = c->d2h_bytes;
    if (reset) c->h2d_bytes = c->d2h_bytes = 0;
    return ZYNFER_CU_OK;
}

}  // extern "C"
