// Sampling of the next token on the device (temperature, top-k, top-p), the
// rule the oracle's zo_sample_row restates. The reference decodes greedily
// (topK, src/model/qwen_forward.zig:177-193); its roadmap's Stage 12
// (docs/roadmap.md:29) names sampling without specifying it, so the rule is
// this backend's:
//
// * temperature only (top_k == 0, top_p >= 1): the Gumbel-max draw
//   argmax_v (l_v (1/T) + g_v), g_v = -log(-log(u_v)): an exact sample of
//   softmax(l / T) in one pass over the vocabulary, first maximum on ties;
// * otherwise the K = top_k (64 when 0) largest logits in topK's order,
//   p_i = exp((l_i - l_0) / T) summed in that order, the shortest prefix whose
//   sum reaches top_p of the total, and the first candidate whose running sum
//   exceeds u times that prefix's sum.
//
// Draws come from the counter generator of synth_rng.h, keyed by (seed,
// sequence slot) and indexed by the token's position, so a sequence's tokens
// do not depend on its batch neighbours and a step repeated at the same
// position draws the same values.
//
// One 1024-thread CTA per row. The top-64 selection keeps each warp's 64 best
// (logit, index) keys in registers (two per lane) with their minimum as the
// admission threshold, so a warp touches its list only for the few logits
// that beat it; warp 0 then merges the 32 lists the same way.
#include "common.cuh"
#include "kernels.h"
#include "synth_rng.h"

namespace zc {

namespace {

constexpr int kSampleThreads = 1024;
constexpr int kSampleWarps = kSampleThreads / kWarp;
constexpr int kMaxTopK = 64;
constexpr unsigned kAll = 0xFFFFFFFFu;

__device__ __forceinline__ unsigned long long umin64(unsigned long long a, unsigned long long b) { return a < b ? a : b; }

// A warp's 64 best keys: slots lane and lane + 32 (a0, a1); empty slots are 0.
struct WarpTop {
    unsigned long long a0 = 0ull, a1 = 0ull;

    __device__ __forceinline__ unsigned long long minimum() const {
        unsigned long long m = umin64(a0, a1);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) m = umin64(m, __shfl_xor_sync(kAll, m, o));
        return m;
    }
    // Every lane holds candidate k (or 0); admit, one at a time, those above
    // the list's minimum mn, each replacing the slot that holds the minimum.
    __device__ __forceinline__ void offer(unsigned long long k, unsigned long long& mn) {
        const int lane = threadIdx.x % kWarp;
        unsigned cand = __ballot_sync(kAll, k > mn);
        while (cand) {
            const int src = __ffs(cand) - 1;
            const unsigned long long kk = __shfl_sync(kAll, k, src);
            const unsigned owner = __ballot_sync(kAll, a0 == mn || a1 == mn);
            if (lane == __ffs(owner) - 1) {
                if (a0 == mn) a0 = kk;
                else a1 = kk;
            }
            mn = minimum();
            cand = __ballot_sync(kAll, k > mn) & ~((2u << src) - 1u);  // lanes after src still above
        }
    }
};

__device__ __forceinline__ uint32_t key_index(unsigned long long k) { return 0xFFFFFFFFu - (uint32_t)(k & 0xFFFFFFFFull); }

__global__ void __launch_bounds__(kSampleThreads) sample_kernel(SampleArgs a) {
    pdl_launch_dependents();
    pdl_wait();
    __shared__ unsigned long long lists[kSampleWarps][kMaxTopK];
    __shared__ unsigned long long best_s[kSampleWarps];
    const int b = blockIdx.x;
    const int warp = threadIdx.x / kWarp, lane = threadIdx.x % kWarp;
    const int V = a.V;
    const float* l = a.logits + (size_t)b * V;
    const uint32_t slot = (uint32_t)(a.seq_of ? a.seq_of[b] : a.seq0);
    const uint32_t pos = (uint32_t)(a.positions ? a.positions[b] : a.pos0);
    const uint64_t key = zs_key(a.seed, ZS_SAMPLE_STREAM(slot));
    const uint64_t base = (uint64_t)pos * (uint64_t)(V + 1);
    uint32_t token = 0;

    if (a.top_k == 0 && !(a.top_p < 1.0f)) {
        // ---- Gumbel-max over the whole vocabulary
        unsigned long long best = 0ull;
        for (int v = threadIdx.x; v < V; v += kSampleThreads) {
            const float u = zs_uniform01(key, base + (uint64_t)v);
            const float g = -logf(-logf(u));
            best = max(best, argmax_key(__fadd_rn(__fmul_rn(l[v], a.inv_t), g), (uint32_t)v));
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) best = max(best, __shfl_xor_sync(kAll, best, o));
        if (lane == 0) best_s[warp] = best;
        __syncthreads();
        if (threadIdx.x == 0) {
            for (int w = 0; w < kSampleWarps; ++w) best = max(best, best_s[w]);
            token = best ? key_index(best) : 0u;
        }
    } else {
        // ---- the 64 largest logits: per-warp lists over contiguous chunks, then merged
        const int chunk = (V + kSampleWarps - 1) / kSampleWarps;
        const int lo = warp * chunk, hi = min(V, lo + chunk);
        WarpTop t;
        unsigned long long mn = 0ull;
        for (int v0 = lo; v0 < hi; v0 += kWarp) {
            const int v = v0 + lane;
            t.offer(v < hi ? argmax_key(l[v], (uint32_t)v) : 0ull, mn);
        }
        lists[warp][lane] = t.a0;
        lists[warp][lane + kWarp] = t.a1;
        __syncthreads();
        if (warp == 0) {
            WarpTop m;
            unsigned long long mm = 0ull;
            for (int j = 0; j < kSampleWarps * kMaxTopK; j += kWarp)
                m.offer(lists[(j + lane) / kMaxTopK][(j + lane) % kMaxTopK], mm);
            __syncwarp();
            lists[0][lane] = m.a0;
            lists[0][lane + kWarp] = m.a1;
            __syncwarp();
            if (lane == 0) {
                unsigned long long* s = lists[0];
                for (int i = 1; i < kMaxTopK; ++i) {  // descending: largest logit, then lowest index
                    const unsigned long long x = s[i];
                    int j = i - 1;
                    while (j >= 0 && s[j] < x) {
                        s[j + 1] = s[j];
                        --j;
                    }
                    s[j + 1] = x;
                }
                int n = 0;
                const int K = a.top_k == 0 || a.top_k > kMaxTopK ? kMaxTopK : a.top_k;
                while (n < K && s[n] != 0ull) ++n;
                if (n > 0) {
                    float p[kMaxTopK];
                    const float l0 = l[key_index(s[0])];
                    float z = 0.0f;
                    for (int i = 0; i < n; ++i) {
                        p[i] = expf(__fmul_rn(__fsub_rn(l[key_index(s[i])], l0), a.inv_t));
                        z = __fadd_rn(z, p[i]);
                    }
                    int m2 = n;
                    if (a.top_p < 1.0f) {
                        const float target = __fmul_rn(a.top_p, z);
                        float c = 0.0f;
                        for (m2 = 0; m2 < n;) {
                            c = __fadd_rn(c, p[m2++]);
                            if (c >= target) break;
                        }
                    }
                    float zm = 0.0f;
                    for (int i = 0; i < m2; ++i) zm = __fadd_rn(zm, p[i]);
                    const float r = __fmul_rn(zs_uniform01(key, base + (uint64_t)V), zm);
                    float c = 0.0f;
                    int pick = m2 - 1;
                    for (int i = 0; i < m2; ++i) {
                        c = __fadd_rn(c, p[i]);
                        if (c > r) {
                            pick = i;
                            break;
                        }
                    }
                    token = key_index(s[pick]);
                }
            }
        }
    }
    if (threadIdx.x == 0) {
        // the finalize kernel reads argmax keys: store the sampled id in that encoding
        if (a.keys_out) a.keys_out[b] = (1ull << 32) | (unsigned long long)(0xFFFFFFFFu - token);
        if (a.ids_out) a.ids_out[b] = token;
    }
}

}  // namespace

void prepare_sample_kernels() { configure_kernel((const void*)sample_kernel, 0); }

void launch_sample(const SampleArgs& a, cudaStream_t st) {
    if (a.rows <= 0) return;
    launch_pdl(sample_kernel, a.rows, kSampleThreads, 0, st, a);
}

}  // namespace zc
