// One greedy decode step of a small batch (1..8 sequences, int8 weights) as a
// single persistent kernel: one CTA per SM, launched cooperatively so every
// CTA is resident, with software grid barriers between the phases that need
// all of the previous phase's output. Per step:
//
//   E     embedding rows (every CTA dequantises them itself; no barrier)
//   per layer (qwen_block.zig:161-235, t = 1):
//   QKV   RMSNorm(input_ln) + fused QKV rows                      | barrier
//   ATT   per-head q/k RMSNorm + RoPE, K/V append, split-K GQA    | barrier
//         attention over the paged bf16 cache with a log-sum-exp merge
//   O     O rows + residual                                       | barrier
//   GU    RMSNorm(post_ln) + gate/up rows + SwiGLU                | barrier
//   D     down rows + residual                                    | barrier
//   HEAD  final RMSNorm + tied LM head rows + argmax; the last CTA to finish
//         turns the keys into next tokens and advances the positions.
//
// Why: at batch 1..8 the work of a layer is ~16 MB of weights and a few MB of
// KV, ~3 us at HBM speed, while a chain of separate kernels costs several
// microseconds per launch boundary. Here a boundary is one atomic arrival and
// an acquire poll, and the weights of the next phase are pulled into L2
// (cp.async.bulk.prefetch) while the current phase runs, so the grid only
// waits for activations that are already in L2.
//
// The linear phases use CUDA cores: each warp streams whole weight rows with
// 16-byte read-only loads (int8 -> f32 by the byte-permute magic number) and
// multiplies them against activations staged once per CTA in shared memory
// (swizzled for conflict-free float4 reads). The attention phase is the
// warp-granular tensor-core kernel of attn.cu restated for this schedule:
// the new token's K/V is computed here, written into the cache and patched
// into the shared-memory copy of its block.
//
// Every wait is bounded: the grid barrier gives up after kSpinLimit polls,
// sets kErrTimeout and an abort flag that releases every other CTA, and
// mbarrier waits drain in-flight copies before a warp leaves.
#include <cuda_runtime.h>

#include "attn_common.cuh"
#include "common.cuh"
#include "kernels.h"

namespace zc {

namespace {

constexpr int kPW = 8;               // warps per CTA
constexpr int kPT = kPW * kWarp;     // threads per CTA
using attn::kBlockBytes;
using attn::kBlockElems;
using attn::kD;
using attn::kG;
using attn::kSlotBytes;
using attn::ldsm_x4;
using attn::ldsm_x4_trans;
using attn::mma_bf16;
using attn::fence_proxy_async_smem;
using attn::pack_terms;
constexpr int kMaxB = kPersistentMaxBatch;
constexpr int kRing = 3;
constexpr int kIdRing = 64;
constexpr size_t kRingBytes = (size_t)kPW * kRing * kSlotBytes;   // 192 KB; the linear phases stage activations here
constexpr uint32_t kSpinLimit = 1u << 22;
constexpr uint32_t kLastBit = 0x80000000u;

// shared-memory layout after the ring
constexpr size_t kOffBars = kRingBytes;                                         // [kPW][kRing] u64
constexpr size_t kOffKidx = kOffBars + kPW * kRing * 8;                         // [kPW][kIdRing] u32
constexpr size_t kOffQ = kOffKidx + kPW * kIdRing * 4;                          // [kPW][kG][kD] f32
constexpr size_t kOffRed = kOffQ + (size_t)kPW * kG * kD * 4;                   // [kPW][kMaxB] f32
constexpr size_t kOffInv = kOffRed + kPW * kMaxB * 4;                           // [kMaxB] f32
constexpr size_t kOffBest = kOffInv + kMaxB * 4;                                // [kPW][kMaxB] u64
constexpr size_t kOffPref = kOffBest + kPW * kMaxB * 8;                         // [kMaxB + 1] i32
constexpr size_t kOffNew = kOffPref + (kMaxB + 1) * 4 + 12;                     // [kPW][2][kD] bf16, 16-aligned
constexpr size_t kPersistSmem = kOffNew + (size_t)kPW * 2 * kD * 2;
static_assert((size_t)kMaxB * 3072 * 4 <= kRingBytes, "activation stage must fit in the ring");
static_assert((size_t)kMaxB * 1024 * 4 + (size_t)kPW * kRing * 4096 <= kRingBytes, "LM head slots must fit");

// ------------------------------------------------------------ helpers

__device__ __forceinline__ unsigned ld_acquire(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void prefetch_l2_bulk(const void* p, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}
// Pull [p, p + bytes) toward L2 in pieces of at most 32 KB (one thread).
__device__ __forceinline__ void prefetch_range(const void* p, size_t bytes) {
    const char* c = reinterpret_cast<const char*>(p);
    const size_t head = (16 - (reinterpret_cast<uintptr_t>(c) & 15)) & 15;
    c += head;
    bytes = bytes > head ? (bytes - head) & ~(size_t)15 : 0;
    while (bytes) {
        const uint32_t n = bytes > 32768 ? 32768u : (uint32_t)bytes;
        prefetch_l2_bulk(c, n);
        c += n;
        bytes -= n;
    }
}
__device__ __forceinline__ float silu(float g) { return g * (1.0f / (1.0f + expf(-g))); }

// Position of activation k in a staged row: the 16-byte reads of one lane
// cover 16 consecutive k (four float4 groups), rotated so a warp's reads
// hit 32 distinct banks.
__device__ __forceinline__ int swz(int k) {
    return (k & ~15) | (((((k >> 2) & 3) + ((k >> 5) & 3)) & 3) << 2) | (k & 3);
}

struct Shared {
    unsigned char* ring;
    uint64_t* bars;
    uint32_t* kidx;
    float* qbuf;
    float* red;
    float* inv;
    unsigned long long* best;
    int* pref;
};

// Software grid barrier number `epoch` (1, 2, ...): every CTA adds one to the
// counter after its writes are fenced; barrier k is complete at k * gridDim.x.
// Returns false when the wait ran out or another CTA gave up.
__device__ __forceinline__ bool grid_sync(const PersistentArgs& a, unsigned epoch) {
    __shared__ int ok_s;
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        atomicAdd(a.sync, 1u);
        const unsigned target = epoch * gridDim.x;
        int ok = 1;
        uint32_t spins = 0;
        while (ld_acquire(a.sync) < target) {
            if (ld_acquire(a.sync + 2)) {
                ok = 0;
                break;
            }
            if (++spins > kSpinLimit) {
                atomicOr(a.err, kErrTimeout);
                atomicExch(a.sync + 2, 1u);
                ok = 0;
                break;
            }
        }
        ok_s = ok;
    }
    __syncthreads();
    return ok_s != 0;
}

// Stage B rows of K activations into the swizzled shared buffer xs, with an
// optional RMSNorm (ops.zig:49-67: (w * x) * 1/sqrt(mean(x^2) + eps)). The
// source is read through L2 (it was written by other CTAs of this grid).
template <int NB, class Src>
__device__ __forceinline__ void stage_rows(const Shared& S, float* xs, int B, int K, const float* norm_w, float eps,
                                           Src src) {
    const int warp = threadIdx.x / kWarp, lane = threadIdx.x % kWarp;
    float ss[NB];
#pragma unroll
    for (int b = 0; b < NB; ++b) ss[b] = 0.0f;
#pragma unroll
    for (int b = 0; b < NB; ++b) {
        if (b >= B) break;
        for (int k = threadIdx.x; k < K; k += kPT) {
            const float v = src(b, k);
            xs[b * K + swz(k)] = v;
            ss[b] += v * v;
        }
    }
    if (norm_w) {
#pragma unroll
        for (int b = 0; b < NB; ++b) {
            if (b >= B) break;
            const float t = warp_sum(ss[b]);
            if (lane == 0) S.red[warp * kMaxB + b] = t;
        }
        __syncthreads();
        if (threadIdx.x < B) {
            float tot = 0.0f;
#pragma unroll
            for (int w = 0; w < kPW; ++w) tot += S.red[w * kMaxB + threadIdx.x];
            S.inv[threadIdx.x] = 1.0f / sqrtf(tot / (float)K + eps);
        }
        __syncthreads();
#pragma unroll
        for (int b = 0; b < NB; ++b) {
            if (b >= B) break;
            const float inv = S.inv[b];
            for (int k = threadIdx.x; k < K; k += kPT) {
                float* p = xs + b * K + swz(k);
                *p = __fmul_rn(__fmul_rn(__ldg(norm_w + k), *p), inv);
            }
        }
    }
    __syncthreads();
}

// R weight rows of an int8 matrix ([M][K], K = 512 KC) held in registers:
// lane l holds bytes [16 (32 c + l), +16) of each row for c < KC.
template <int R, int KC>
struct Rows {
    uint4 w[R][KC];
};
template <int R, int KC>
__device__ __forceinline__ void load_rows(Rows<R, KC>& L, const int8_t* __restrict__ W, int K, int row0, int r1) {
    const int lane = threadIdx.x % kWarp;
#pragma unroll
    for (int r = 0; r < R; ++r) {
        const int row = min(row0 + r, r1 - 1);
#pragma unroll
        for (int c = 0; c < KC; ++c) L.w[r][c] = ldg_stream(W + (size_t)row * K + (size_t)(c * kWarp + lane) * 16);
    }
}
// acc[r][b] = sum_k W[row0 + r, k] xs[b, k], reduced over the warp (every lane holds it).
template <int NB, int R, int KC>
__device__ __forceinline__ void dot_rows(const Rows<R, KC>& L, const float* xs, int K, int B, float (&acc)[R][NB]) {
    const int lane = threadIdx.x % kWarp;
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
        for (int b = 0; b < NB; ++b) acc[r][b] = 0.0f;
#pragma unroll
    for (int c = 0; c < KC; ++c) {
        const int k0 = (c * kWarp + lane) * 16;
#pragma unroll
        for (int r = 0; r < R; ++r) {
            float w[16];
            i8x4_to_f32(L.w[r][c].x, w[0], w[1], w[2], w[3]);
            i8x4_to_f32(L.w[r][c].y, w[4], w[5], w[6], w[7]);
            i8x4_to_f32(L.w[r][c].z, w[8], w[9], w[10], w[11]);
            i8x4_to_f32(L.w[r][c].w, w[12], w[13], w[14], w[15]);
#pragma unroll
            for (int b = 0; b < NB; ++b) {
                if (b >= B) break;
                const float* xb = xs + b * K;
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    const float4 xv = *reinterpret_cast<const float4*>(xb + swz(k0 + 4 * q));
                    acc[r][b] = fmaf(w[4 * q + 0], xv.x, acc[r][b]);
                    acc[r][b] = fmaf(w[4 * q + 1], xv.y, acc[r][b]);
                    acc[r][b] = fmaf(w[4 * q + 2], xv.z, acc[r][b]);
                    acc[r][b] = fmaf(w[4 * q + 3], xv.w, acc[r][b]);
                }
            }
        }
    }
#pragma unroll
    for (int b = 0; b < NB; ++b) {
        if (b >= B) break;
#pragma unroll
        for (int r = 0; r < R; ++r) acc[r][b] = warp_sum(acc[r][b]);
    }
}

// Rows [r0, r1) in units of R rows, unit u on warp u % kPW. `first` already
// holds this warp's first unit (loaded before the grid barrier, so the
// weights are in flight while the grid waits). epi(row0, b, acc, r1) runs in
// lane b.
template <int NB, int R, int KC, class Epi>
__device__ __forceinline__ void linear_rows(Rows<R, KC>& first, const int8_t* __restrict__ W, int K, int r0, int r1,
                                            const float* xs, int B, Epi epi) {
    const int warp = threadIdx.x / kWarp, lane = threadIdx.x % kWarp;
    const int units = (r1 - r0 + R - 1) / R;
    for (int u = warp; u < units; u += kPW) {
        const int row0 = r0 + u * R;
        if (u != warp) load_rows(first, W, K, row0, r1);
        float acc[R][NB];
        dot_rows<NB>(first, xs, K, B, acc);
#pragma unroll
        for (int b = 0; b < NB; ++b) {
            if (b >= B) break;
            if (lane == b) epi(row0, b, acc, r1);
        }
    }
}
template <int R, int KC>
__device__ __forceinline__ void preload_rows(Rows<R, KC>& L, const int8_t* __restrict__ W, int K, int r0, int r1) {
    const int warp = threadIdx.x / kWarp;
    if (r0 + warp * R < r1) load_rows(L, W, K, r0 + warp * R, r1);
}

__device__ __forceinline__ void trace_mark(const PersistentArgs& a, int slot) {
    if (a.trace && blockIdx.x == 0 && threadIdx.x == 0) {
        uint64_t t;
        asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
        a.trace[slot] = t;
    }
}

// CTA c's share [lo, hi) of n items, in multiples of `align`.
__device__ __forceinline__ void cta_share(int n, int align, int& lo, int& hi) {
    const int units = n / align;
    lo = (int)((long)blockIdx.x * units / gridDim.x) * align;
    hi = (int)((long)(blockIdx.x + 1) * units / gridDim.x) * align;
}

struct BlockCursor {
    int b, head, blk, nblk;
};

template <int NB>
__global__ void __launch_bounds__(kPT, 1) decode_persistent_kernel(PersistentArgs a) {
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    Shared S;
    S.ring = smem_raw;
    S.bars = reinterpret_cast<uint64_t*>(smem_raw + kOffBars);
    S.kidx = reinterpret_cast<uint32_t*>(smem_raw + kOffKidx);
    S.qbuf = reinterpret_cast<float*>(smem_raw + kOffQ);
    S.red = reinterpret_cast<float*>(smem_raw + kOffRed);
    S.inv = reinterpret_cast<float*>(smem_raw + kOffInv);
    S.best = reinterpret_cast<unsigned long long*>(smem_raw + kOffBest);
    S.pref = reinterpret_cast<int*>(smem_raw + kOffPref);
    constexpr unsigned kAll = 0xFFFFFFFFu;

    const int warp = threadIdx.x / kWarp, lane = threadIdx.x % kWarp;
    const int B = a.B, H = a.H, I = a.I, V = a.V;
    const int qkv_rows = (a.n_q + 2 * a.n_kv) * kD;
    const int qd = a.n_q * kD;
    const int max_len = a.max_blocks * kKvBlock;
    float* xs = reinterpret_cast<float*>(S.ring);

    // ---- per-step constants: block counts per row, this warp's attention range
    if (threadIdx.x == 0) {
        S.pref[0] = 0;
        for (int b = 0; b < B; ++b) {
            const int len = a.positions[b] + 1;
            if ((len < 1 || len > max_len) && a.err) atomicOr(a.err, kErrBadIndex);
            S.pref[b + 1] = S.pref[b] + (min(max(len, 1), max_len) + kKvBlock - 1) / kKvBlock;
        }
    }
    uint64_t* full = S.bars + warp * kRing;
    uint32_t* kidx = S.kidx + warp * kIdRing;
    if (lane == 0) {
        for (int s = 0; s < kRing; ++s) mbar_init(&full[s], 1);
        fence_barrier_init();
    }
    __syncthreads();
    const int total = S.pref[B] * a.n_kv;
    const int nwarps = gridDim.x * kPW;
    const int per = max((total + nwarps - 1) / nwarps, kMinBlocksPerWarp);
    const int wid = warp * gridDim.x + blockIdx.x;
    const int att_lo = wid * per;
    const int att_n = max(0, min(total, att_lo + per) - att_lo);

    auto locate = [&](int f, BlockCursor& c) {
        int l = 0, h = B - 1;
        while (l < h) {
            const int mid = (l + h + 1) / 2;
            if (a.n_kv * S.pref[mid] <= f) l = mid;
            else h = mid - 1;
        }
        c.b = l;
        c.nblk = S.pref[l + 1] - S.pref[l];
        const int r = f - a.n_kv * S.pref[l];
        c.head = r / c.nblk;
        c.blk = r % c.nblk;
    };
    auto advance = [&](BlockCursor& c) {
        if (++c.blk < c.nblk) return;
        c.blk = 0;
        if (++c.head < a.n_kv) return;
        c.head = 0;
        ++c.b;
        c.nblk = c.b < B ? S.pref[c.b + 1] - S.pref[c.b] : 1;
    };
    // block addresses of this warp's range, 32 at a time (relative to a layer's pool)
    auto fill_chunk = [&](int c) {
        const int j = kWarp * c + lane;
        if (j < att_n) {
            BlockCursor x;
            locate(att_lo + j, x);
            const int seq = a.seq_of[x.b];
            int id = a.block_table[(size_t)seq * a.max_blocks + x.blk];
            if (id < 0 || id >= a.n_pool_blocks) {
                if (a.err) atomicOr(a.err, kErrBadIndex);
                id = 0;
            }
            kidx[j % kIdRing] = (((uint32_t)x.head * (uint32_t)a.n_pool_blocks + (uint32_t)id) * 2u) |
                                (x.blk == x.nblk - 1 ? kLastBit : 0u);
        }
        __syncwarp();
    };
    fill_chunk(0);

    // ---- E: embedding rows (every CTA; CTA 0 also keeps them for the residual)
    const float* x_in_f = nullptr;  // layer input in global memory (nullptr: layer 0, staged from the table)
    if (blockIdx.x == 0) {
        for (int i = threadIdx.x; i < B * H; i += kPT) {
            const int b = i / H, k = i % H;
            const uint32_t id = a.tok[b];
            a.x[i] = id < (uint32_t)V ? __fmul_rn((float)a.embed[(size_t)id * H + k], __ldg(a.sembed + id)) : 0.0f;
        }
    }
    if (threadIdx.x < B && a.tok[threadIdx.x] >= (uint32_t)V && a.err && blockIdx.x == 0)
        atomicOr(a.err, kErrBadIndex);

    unsigned epoch = 0;
    uint32_t uses = 0;  // blocks this warp has pulled through its ring (mbarrier parity)
    int pairs_lo, pairs_hi, h_lo, h_hi, q_lo, q_hi, v_lo, v_hi;
    cta_share(qkv_rows, 1, q_lo, q_hi);
    cta_share(I, 1, pairs_lo, pairs_hi);
    cta_share(H, 1, h_lo, h_hi);
    cta_share(V, 1, v_lo, v_hi);

    trace_mark(a, 0);
    int ph = 0;  // phase index: trace slots 1 + 2 ph (phase start) and 2 + 2 ph (phase end)
    for (int l = 0; l < a.L; ++l) {
        const PersistentLayer& P = a.layers[l];
        uint16_t* kv_layer = a.kv + (size_t)l * a.kv_layer_elems;
        // -------- QKV
        {
            Rows<4, 2> wq;
            preload_rows(wq, P.wqkv, H, q_lo, q_hi);
            if (l > 0 && !grid_sync(a, ++epoch)) return;
            trace_mark(a, 1 + 2 * ph);
            if (threadIdx.x == 0) {
                // the small per-layer vectors the attention phase reads first
                prefetch_l2_bulk(P.q_norm, kD * 4);
                prefetch_l2_bulk(P.k_norm, kD * 4);
                for (int b = 0; b < B; ++b) {
                    const int pos = a.positions[b];
                    if (pos >= 0 && pos < a.rope_max_pos) prefetch_l2_bulk(a.rope + (size_t)pos * (kD / 2), kD * 4);
                }
                prefetch_range(P.wo + (size_t)h_lo * qd, (size_t)(h_hi - h_lo) * qd);
                prefetch_range(P.wgu + (size_t)2 * pairs_lo * H, (size_t)2 * (pairs_hi - pairs_lo) * H);
            }
            if (lane == 0)  // this layer's KV blocks toward L2 (the new rows are patched in shared memory)
                for (int j = 0; j < min(att_n, kWarp); ++j) {
                    const uint16_t* kp = kv_layer + (size_t)(kidx[j % kIdRing] & ~kLastBit) * kBlockElems;
                    prefetch_l2_bulk(kp, kSlotBytes);
                }
            stage_rows<NB>(S, xs, B, H, P.input_ln, a.eps, [&](int b, int k) -> float {
                if (x_in_f) return __ldcg(x_in_f + (size_t)b * H + k);
                const uint32_t id = a.tok[b];
                return id < (uint32_t)V ? __fmul_rn((float)a.embed[(size_t)id * H + k], __ldg(a.sembed + id)) : 0.0f;
            });
            linear_rows<NB>(wq, P.wqkv, H, q_lo, q_hi, xs, B, [&](int row0, int b, float (&acc)[4][NB], int r1) {
#pragma unroll
                for (int r = 0; r < 4; ++r)
                    if (row0 + r < r1)
                        a.qkv[(size_t)b * qkv_rows + row0 + r] = __fmul_rn(acc[r][b], __ldg(P.sqkv + row0 + r));
            });
            trace_mark(a, 2 + 2 * ph++);
        }
        if (!grid_sync(a, ++epoch)) return;
        trace_mark(a, 1 + 2 * ph);

        // -------- ATT
        if (threadIdx.x == 0) prefetch_range(P.wd + (size_t)h_lo * I, (size_t)(h_hi - h_lo) * I);
        if (att_n > 0) {
            unsigned char* ring = S.ring + (size_t)warp * kRing * kSlotBytes;
            float* qb = S.qbuf + warp * kG * kD;
            auto block_k = [&](int j) -> uint16_t* {
                return kv_layer + (size_t)(kidx[j % kIdRing] & ~kLastBit) * kBlockElems;
            };
            auto issue = [&](int j) {
                const int s = (int)((uses + j) % kRing);
                const uint16_t* kp = block_k(j);
                unsigned char* dst = ring + s * kSlotBytes;
                mbar_arrive_expect_tx(&full[s], kSlotBytes);
                bulk_g2s(dst, kp, kSlotBytes, &full[s]);  // K then V of the block: one contiguous 8 KB
            };
            fence_proxy_async_smem();  // the ring held staged activations (generic writes) until the barrier
            const int first = min(kRing, att_n);
            if (lane == 0)
                for (int j = 0; j < first; ++j) issue(j);

            const int g = lane >> 2, t = lane & 3;
            const int mi = lane >> 3, ri = lane & 7;
            const int tok_a = ri + (mi & 1) * 8;
            const int hsel = (lane >> 3) & 1;
            const float scale = 1.0f / sqrtf((float)kD);
            BlockCursor cc;
            locate(att_lo, cc);
            uint32_t qf[8][2];
            float acc[16][4];
            float m_run = -INFINITY, l_run = 0.0f;
            int kv_len = 0, pos = 0;
            bool seg_start = true, has_last = false;
            uint16_t* kvnew = reinterpret_cast<uint16_t*>(smem_raw + kOffNew) + warp * 2 * kD;  // this step's K, V row
            bool alive = true;
            for (int i = 0; i < att_n; ++i) {
                const uint32_t u = uses + i;
                const int s = (int)(u % kRing);
                if (seg_start) {
                    pos = a.positions[cc.b];
                    kv_len = min(max(pos + 1, 1), max_len);
                    const int f_last = a.n_kv * S.pref[cc.b] + cc.head * cc.nblk + cc.nblk - 1;
                    has_last = f_last < att_lo + att_n;  // this warp also holds the row's last block
                    attn::QkvSource src{a.qkv, qkv_rows, qd, a.n_kv, P.q_norm, P.k_norm, a.rope, a.rope_max_pos,
                                        a.eps, a.err};
                    attn::share_setup(src, cc.b, cc.head, pos, has_last, qb, kvnew, qf);
#pragma unroll
                    for (int nt = 0; nt < 16; ++nt) acc[nt][0] = acc[nt][1] = acc[nt][2] = acc[nt][3] = 0.0f;
                    m_run = -INFINITY;
                    l_run = 0.0f;
                    seg_start = false;
                }
                const bool ok = __all_sync(kAll, mbar_wait_bounded(&full[s], (u / kRing) & 1u, a.err));
                if (!ok) {
                    if (lane == 0)
                        for (int j = i; j < min(att_n, i + kRing); ++j)
                            mbar_wait_bounded(&full[(uses + j) % kRing], ((uses + j) / kRing) & 1u, nullptr);
                    __syncwarp();
                    alive = false;
                    break;
                }
                unsigned char* kb = ring + s * kSlotBytes;
                const int nv = min(kKvBlock, kv_len - cc.blk * kKvBlock);
                const bool last = cc.blk == cc.nblk - 1;
                if (last) attn::patch_new_row(block_k(i), kb, nv - 1, kvnew);
                if (nv < kKvBlock) {
                    uint4* vrow = reinterpret_cast<uint4*>(kb + kBlockBytes + nv * kD * 2);
                    for (int x = lane; x < (kKvBlock - nv) * (kD * 2 / 16); x += kWarp) vrow[x] = make_uint4(0, 0, 0, 0);
                }
                __syncwarp();

                float sc[4] = {0.0f, 0.0f, 0.0f, 0.0f}, sd[4] = {0.0f, 0.0f, 0.0f, 0.0f};
                const uint32_t kbase = smem_addr(kb), vbase = kbase + kBlockBytes;
#pragma unroll
                for (int ks = 0; ks < 8; ++ks) {
                    const int ch = 2 * ks + (mi >> 1);
                    uint32_t a0, a1, a2, a3;
                    ldsm_x4(kbase + tok_a * (kD * 2) + ((ch ^ ri) << 4), a0, a1, a2, a3);
                    if (ks & 1) mma_bf16(sd, a0, a1, a2, a3, qf[ks][0], qf[ks][1]);
                    else mma_bf16(sc, a0, a1, a2, a3, qf[ks][0], qf[ks][1]);
                }
#pragma unroll
                for (int e = 0; e < 4; ++e) sc[e] += sd[e];
                float s0 = 0.0f, s1 = 0.0f;
                if (t < 2) {
                    s0 = g < nv ? (sc[0] + sc[1]) * scale : -INFINITY;
                    s1 = g + 8 < nv ? (sc[2] + sc[3]) * scale : -INFINITY;
                }
                float mt = fmaxf(s0, s1);
                mt = fmaxf(mt, __shfl_xor_sync(kAll, mt, 4));
                mt = fmaxf(mt, __shfl_xor_sync(kAll, mt, 8));
                mt = fmaxf(mt, __shfl_xor_sync(kAll, mt, 16));
                const float m_new = fmaxf(m_run, mt);
                if (__any_sync(kAll, m_new > m_run)) {
                    const float corr = expf(m_run - m_new);
                    l_run *= corr;
                    const float ca = __shfl_sync(kAll, corr, hsel);
#pragma unroll
                    for (int nt = 0; nt < 16; ++nt) {
                        acc[nt][0] *= ca;
                        acc[nt][1] *= ca;
                    }
                    m_run = m_new;
                }
                const float p0 = expf(s0 - m_run), p1 = expf(s1 - m_run);
                l_run += p0 + p1;
                const int src0 = 8 * t + hsel, src1 = src0 + 4;
                const float x0 = __shfl_sync(kAll, p0, src0), x8 = __shfl_sync(kAll, p1, src0);
                const float x1 = __shfl_sync(kAll, p0, src1), x9 = __shfl_sync(kAll, p1, src1);
                uint32_t pa0 = 0u, pa2 = 0u;
                if (lane < 16) {
                    pa0 = pack_terms(x0, x1, g & 1);
                    pa2 = pack_terms(x8, x9, g & 1);
                }
#pragma unroll
                for (int np = 0; np < 8; ++np) {
                    const int ch = 2 * np + (mi >> 1);
                    uint32_t b0, b1, b2, b3;
                    ldsm_x4_trans(vbase + tok_a * (kD * 2) + ((ch ^ ri) << 4), b0, b1, b2, b3);
                    mma_bf16(acc[2 * np], pa0, 0u, pa2, 0u, b0, b1);
                    mma_bf16(acc[2 * np + 1], pa0, 0u, pa2, 0u, b2, b3);
                }
                if (nv < kKvBlock || last) fence_proxy_async_smem();
                __syncwarp();
                {
                    const int jn = i + kRing;
                    if (jn < att_n && jn % kWarp == 0) fill_chunk(jn / kWarp);
                    if (lane == 0 && jn < att_n) issue(jn);
                }

                if (last || i == att_n - 1) {
                    const int f0 = a.n_kv * S.pref[cc.b] + cc.head * cc.nblk;
                    const int fw = f0 / per, lw = (f0 + cc.nblk - 1) / per;
                    attn::flush_share(acc, l_run, m_run, cc.b, cc.head, lw - fw + 1, wid - fw, a.max_segs, a.n_q,
                                      a.n_kv, a.partial, a.counters, a.attn, a.err);
                    seg_start = true;
                }
                advance(cc);
            }
            if (!alive) {
                if (lane == 0) atomicExch(a.sync + 2, 1u);
            } else if (att_n > kIdRing) {
                fill_chunk(0);  // the next layer starts from chunk 0 again
            }
            uses += (uint32_t)att_n;
        }
        trace_mark(a, 2 + 2 * ph++);

        // -------- O (+ residual)
        {
            Rows<1, 4> wo;
            preload_rows(wo, P.wo, qd, h_lo, h_hi);
            if (!grid_sync(a, ++epoch)) return;
            trace_mark(a, 1 + 2 * ph);
            if (threadIdx.x == 0 && l + 1 < a.L)
                prefetch_range(a.layers[l + 1].wqkv + (size_t)q_lo * H, (size_t)(q_hi - q_lo) * H);
            stage_rows<NB>(S, xs, B, qd, nullptr, a.eps, [&](int b, int k) { return __ldcg(a.attn + (size_t)b * qd + k); });
            linear_rows<NB>(wo, P.wo, qd, h_lo, h_hi, xs, B, [&](int row0, int b, float (&acc)[1][NB], int) {
                const size_t o = (size_t)b * H + row0;
                a.x1[o] = __fadd_rn(__ldcg(a.x + o), __fmul_rn(acc[0][b], __ldg(P.so + row0)));
            });
            trace_mark(a, 2 + 2 * ph++);
        }

        // -------- GU (+ SwiGLU), three (gate, up) pairs per warp
        {
            Rows<6, 2> wg;
            preload_rows(wg, P.wgu, H, 2 * pairs_lo, 2 * pairs_hi);
            if (!grid_sync(a, ++epoch)) return;
            trace_mark(a, 1 + 2 * ph);
            stage_rows<NB>(S, xs, B, H, P.post_ln, a.eps, [&](int b, int k) { return __ldcg(a.x1 + (size_t)b * H + k); });
            linear_rows<NB>(wg, P.wgu, H, 2 * pairs_lo, 2 * pairs_hi, xs, B,
                        [&](int row0, int b, float (&acc)[6][NB], int r1) {
#pragma unroll
                            for (int p = 0; p < 3; ++p) {
                                const int row = row0 + 2 * p;
                                if (row >= r1) break;
                                const float gate = __fmul_rn(acc[2 * p][b], __ldg(P.sgu + row));
                                const float up = __fmul_rn(acc[2 * p + 1][b], __ldg(P.sgu + row + 1));
                                a.h[(size_t)b * I + (row >> 1)] = __fmul_rn(silu(gate), up);
                            }
                        });
            trace_mark(a, 2 + 2 * ph++);
        }

        // -------- D (+ residual)
        {
            Rows<1, 6> wd;
            preload_rows(wd, P.wd, I, h_lo, h_hi);
            if (!grid_sync(a, ++epoch)) return;
            trace_mark(a, 1 + 2 * ph);
            if (threadIdx.x == 0 && l + 1 == a.L) {  // first rows of every warp's LM head share
                const int rpw = (v_hi - v_lo + kPW - 1) / kPW;
                for (int w = 0; w < kPW; ++w) {
                    const int r = v_lo + w * rpw;
                    if (r < v_hi) prefetch_range(a.embed + (size_t)r * H, (size_t)min(v_hi - r, 32) * H);
                }
            }
            stage_rows<NB>(S, xs, B, I, nullptr, a.eps, [&](int b, int k) { return __ldcg(a.h + (size_t)b * I + k); });
            linear_rows<NB>(wd, P.wd, I, h_lo, h_hi, xs, B, [&](int row0, int b, float (&acc)[1][NB], int) {
                const size_t o = (size_t)b * H + row0;
                a.x[o] = __fadd_rn(__ldcg(a.x1 + o), __fmul_rn(acc[0][b], __ldg(P.sd + row0)));
            });
            trace_mark(a, 2 + 2 * ph++);
        }
        x_in_f = a.x;
    }

    // -------- HEAD: final RMSNorm, tied LM head rows, argmax. Each warp streams
    // a contiguous share of the CTA's rows, two 4-row units in registers and
    // kHeadAhead units ahead toward L2.
    if (!grid_sync(a, ++epoch)) return;
    trace_mark(a, 1 + 2 * ph);
    stage_rows<NB>(S, xs, B, H, a.final_norm, a.eps, [&](int b, int k) { return __ldcg(a.x + (size_t)b * H + k); });
    unsigned long long best[NB];
#pragma unroll
    for (int b = 0; b < NB; ++b) best[b] = 0ull;
    {
        // Each warp streams a contiguous share of the CTA's rows through its own
        // ring of kRing 4-row slots (cp.async.bulk, 4 KB each), kHeadAhead
        // slots further pulled toward L2; the dot products read the slots.
        constexpr int kHeadRows = 4, kHeadAhead = 8;
        constexpr int kSlot = kHeadRows * 1024;  // H = 1024 int8 per row
        unsigned char* hring = S.ring + (size_t)kMaxB * 1024 * 4 + (size_t)warp * kRing * kSlot;
        const int rpw = (v_hi - v_lo + kPW - 1) / kPW;
        const int w0 = min(v_hi, v_lo + warp * rpw), w1 = min(v_hi, w0 + rpw);
        const int units = (w1 - w0 + kHeadRows - 1) / kHeadRows;
        auto hissue = [&](int j) {  // lane 0: unit j into its slot
            const int r = w0 + j * kHeadRows, nr = min(kHeadRows, w1 - r);
            const int s = (int)((uses + j) % kRing);
            mbar_arrive_expect_tx(&full[s], (uint32_t)(nr * H));
            bulk_g2s(hring + s * kSlot, a.embed + (size_t)r * H, (uint32_t)(nr * H), &full[s]);
        };
        auto hprefetch = [&](int j) {
            const int r = w0 + j * kHeadRows;
            prefetch_l2_bulk(a.embed + (size_t)r * H, (uint32_t)(min(kHeadRows, w1 - r) * H));
        };
        fence_proxy_async_smem();  // the slots held staged activations (generic writes) before
        if (lane == 0) {
            for (int j = 0; j < min(kRing, units); ++j) hissue(j);
            for (int j = kRing; j < min(kRing + kHeadAhead, units); ++j) hprefetch(j);
        }
        for (int j = 0; j < units; ++j) {
            const uint32_t u = uses + j;
            const int s = (int)(u % kRing);
            if (!__all_sync(kAll, mbar_wait_bounded(&full[s], (u / kRing) & 1u, a.err))) {
                if (lane == 0)
                    for (int jj = j; jj < min(units, j + kRing); ++jj)
                        mbar_wait_bounded(&full[(uses + jj) % kRing], ((uses + jj) / kRing) & 1u, nullptr);
                __syncwarp();
                if (lane == 0) atomicExch(a.sync + 2, 1u);
                break;
            }
            const int row0 = w0 + j * kHeadRows;
            Rows<kHeadRows, 2> cur;
            const unsigned char* slot = hring + s * kSlot;
#pragma unroll
            for (int r = 0; r < kHeadRows; ++r)
#pragma unroll
                for (int c = 0; c < 2; ++c)
                    cur.w[r][c] = *reinterpret_cast<const uint4*>(slot + r * 1024 + (c * kWarp + lane) * 16);
            float acc[kHeadRows][NB];
            dot_rows<NB>(cur, xs, H, B, acc);
#pragma unroll
            for (int b = 0; b < NB; ++b) {
                if (b >= B) break;
                if (lane != b) continue;
#pragma unroll
                for (int r = 0; r < kHeadRows; ++r) {
                    const int row = row0 + r;
                    if (row >= w1) break;
                    const float val = __fmul_rn(acc[r][b], __ldg(a.sembed + row));
                    if (a.logits) a.logits[(size_t)b * V + row] = val;
                    const unsigned long long key = argmax_key(val, (uint32_t)row);
                    best[b] = key > best[b] ? key : best[b];
                }
            }
            __syncwarp();
            if (lane == 0) {
                if (j + kRing < units) hissue(j + kRing);
                if (j + kRing + kHeadAhead < units) hprefetch(j + kRing + kHeadAhead);
            }
        }
        uses += (uint32_t)units;
    }
    trace_mark(a, 2 + 2 * ph);
#pragma unroll
    for (int b = 0; b < NB; ++b) {
        if (b >= B) break;
        if (lane == b) S.best[warp * kMaxB + b] = best[b];
    }
    __syncthreads();
    if (threadIdx.x < B) {
        unsigned long long m = 0ull;
        for (int w = 0; w < kPW; ++w) m = S.best[w * kMaxB + threadIdx.x] > m ? S.best[w * kMaxB + threadIdx.x] : m;
        if (m) atomicMax(a.keys + threadIdx.x, m);
    }
    __syncthreads();
    // the last CTA to finish turns keys into tokens (finalize_kernel's job in the
    // multi-kernel schedule) and re-arms the step counters
    if (threadIdx.x == 0) {
        __threadfence();
        const unsigned prev = atomicAdd(a.sync + 1, 1u);
        if (prev == gridDim.x - 1) {
            __threadfence();
            const int row = a.history ? *a.step : 0;
            for (int b = 0; b < B; ++b) {
                const unsigned long long key = atomicExch(a.keys + b, 0ull);
                const uint32_t id = key == 0ull ? 0u : argmax_key_index(key);
                a.ids_out[b] = id;
                a.tok[b] = id;
                a.positions[b] += 1;
                if (a.history) a.history[(size_t)row * B + b] = id;
            }
            if (a.history) *a.step = row + 1;
            if (a.trace) {
                uint64_t t;
                asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
                a.trace[3 + 2 * ph] = t;
            }
            a.sync[0] = 0u;
            a.sync[1] = 0u;
            __threadfence();
        }
    }
}

}  // namespace

void prepare_persistent_kernels() {
    configure_kernel((const void*)decode_persistent_kernel<1>, kPersistSmem);
    configure_kernel((const void*)decode_persistent_kernel<2>, kPersistSmem);
    configure_kernel((const void*)decode_persistent_kernel<4>, kPersistSmem);
    configure_kernel((const void*)decode_persistent_kernel<8>, kPersistSmem);
}

bool persistent_supported(int device) {
    int coop = 0;
    if (cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, device) != cudaSuccess || !coop) return false;
    const void* kernels[] = {(const void*)decode_persistent_kernel<1>, (const void*)decode_persistent_kernel<2>,
                             (const void*)decode_persistent_kernel<4>, (const void*)decode_persistent_kernel<8>};
    for (const void* k : kernels) {
        int blocks = 0;
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&blocks, k, kPT, kPersistSmem) != cudaSuccess || blocks < 1)
            return false;
    }
    return true;
}

cudaError_t launch_decode_persistent(const PersistentArgs& a, cudaStream_t st) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(device_sm_count());
    cfg.blockDim = dim3(kPT);
    cfg.dynamicSmemBytes = kPersistSmem;
    cfg.stream = st;
    cudaLaunchAttribute attr;
    attr.id = cudaLaunchAttributeCooperative;
    attr.val.cooperative = 1;
    cfg.attrs = &attr;
    cfg.numAttrs = 1;
    if (a.B <= 1) return cudaLaunchKernelEx(&cfg, decode_persistent_kernel<1>, a);
    if (a.B <= 2) return cudaLaunchKernelEx(&cfg, decode_persistent_kernel<2>, a);
    if (a.B <= 4) return cudaLaunchKernelEx(&cfg, decode_persistent_kernel<4>, a);
    return cudaLaunchKernelEx(&cfg, decode_persistent_kernel<8>, a);
}

}  // namespace zc
