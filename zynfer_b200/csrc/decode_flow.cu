// One greedy decode step of 1..8 sequences (int8 weights, Qwen3-0.6B widths)
// as a single cooperative kernel run as a dataflow pipeline: one CTA per SM,
// eight consumer warps and one producer warp per CTA.
//
// Per step (qwen_block.zig:161-235 per layer, t = 1; qwen_forward.zig:163-193
// for the head):
//
//   QKV   RMSNorm(input_ln) + this CTA's rows of the fused QKV matrix
//   ATT   q/k RMSNorm + RoPE, K/V append, GQA attention over this CTA's range
//         of 16-token KV blocks; partial softmax states merged in shared
//         memory per CTA, then across CTAs by the CTA holding a row's last
//         block (log-sum-exp merge, attentionInto ops.zig:285-354)
//   O     O rows + residual
//   GU    RMSNorm(post_ln) + gate/up rows + SwiGLU
//   D     down rows + residual
//   HEAD  final RMSNorm + tied LM head rows + argmax; the last CTA to finish
//         turns the argmax keys into next tokens and advances the positions.
//
// Why this shape. At batch 1 a token reads ~600 MB of weights and a few
// hundred MB of KV, ~130 us at HBM speed, but the layer chain has 140
// dependent stages; the step is only fast if a stage costs about one L2 round
// trip. Two things make that so:
//
// * Weights and KV blocks do not depend on activations, so the producer warp
//   streams this CTA's slices of every phase, in phase order, into a ring of
//   shared memory with bulk copies (cp.async.bulk, mbarrier completion), as
//   far ahead as the ring allows (~1 layer per SM at batch 1). HBM keeps
//   streaming while the chain waits; a phase finds its weights on chip.
// * Activations travel as 64-bit words (f32 value, 32-bit tag). A consumer
//   polls the words it needs until every tag equals this step's tag for the
//   layer: the data and the "ready" signal arrive in the same load, so a
//   phase boundary costs one L2 round trip and no grid barrier. Tags are
//   unique per (step, layer) (the host passes a fresh base per launch), so
//   the buffers are never cleared. A buffer is rewritten one layer later,
//   and every writer of layer l+1 depends, through the all-to-all phases, on
//   every reader of layer l having finished.
//
// Everything a phase needs besides its input activations (row scales, norm
// weights, RoPE entries, block ids) is loaded before its poll, so that the
// poll is the only dependent global access on the chain.
//
// Every wait is bounded: a poll or mbarrier wait that runs out sets
// kErrTimeout and a global abort flag that ends the other CTAs' waits. The
// consumer warps take every abort decision together (bar.red.and), so no
// named barrier is left half-full; the producer waits, bounded, for its bulk
// copies still in flight before it leaves.
#include <cuda_runtime.h>

#include "attn_common.cuh"
#include "common.cuh"
#include "kernels.h"

namespace zc {

namespace {

using attn::kBlockBytes;
using attn::kBlockElems;
using attn::kD;
using attn::kG;
using attn::kPartHead;
using attn::kPartStride;
using attn::kSlotBytes;

constexpr int kH = 1024, kI = 3072, kQD = 2048, kNKV = 8, kQKV = kQD + 2 * kNKV * kD;
constexpr int kCW = 8;                 // consumer warps
constexpr int kCT = kCW * kWarp;       // consumer threads (named barrier 1)
constexpr int kFT = kCT + kWarp;       // + the producer warp
constexpr int kNF = 32;                // item barriers (full / empty pairs)
constexpr int kHeadRows = 32;          // LM head rows per ring item
constexpr int kMaxRowsCta = 64;        // rows of one linear phase per CTA (needs >= 100 CTAs)
constexpr int kMaxResRows = 16;        // residual rows per CTA (O and D phases)
constexpr int kRecHead = kD + 2;       // record words per query head: m, l, acc[128]
constexpr int kRecWords = kG * kRecHead;
constexpr uint32_t kPollLimit = 1u << 22;
constexpr size_t kSmemMax = 232448;    // sm_100 opt-in shared memory per CTA
constexpr int kMinCtas = 100;
static_assert(kQKV == 4096, "Qwen3-0.6B fused QKV rows");

__host__ __device__ constexpr size_t up(size_t x, size_t a) { return (x + a - 1) / a * a; }

// Shared-memory layout for NB batch rows; the ring takes what is left.
template <int NB>
struct Lay {
    static constexpr size_t xa = 0;                                          // [NB][1024] f32: QKV, GU, HEAD inputs
    static constexpr size_t xb = xa + (size_t)NB * kH * 4;                   // [NB][3072] f32: O, D inputs
    static constexpr size_t part = xb + (size_t)NB * kI * 4;                 // [2][kCW][kPartStride] warp partials
    static constexpr size_t own = part + (size_t)2 * kCW * kPartStride * 4;  // [kPartStride] merger's own partial
    static constexpr size_t qb = own + (size_t)kPartStride * 4;              // [kCW][2][128] f32
    static constexpr size_t kvn = qb + (size_t)kCW * kG * kD * 4;            // [kCW][256] bf16: new K, V rows
    static constexpr size_t res = kvn + (size_t)kCW * 2 * kD * 2;            // [2][NB][kMaxResRows] f32
    static constexpr size_t scl = res + (size_t)2 * NB * kMaxResRows * 4;    // [kMaxRowsCta] f32
    static constexpr size_t red = scl + (size_t)kMaxRowsCta * 4;             // [kCW][NB] f32
    static constexpr size_t best = up(red + (size_t)kCW * NB * 4, 16);       // [kCW][NB] u64
    static constexpr size_t pref = best + (size_t)kCW * NB * 8;              // [NB + 1] i32
    static constexpr size_t iend = up(pref + (size_t)(NB + 1) * 4, 16);      // [kNF] u32 (producer)
    static constexpr size_t flag = iend + (size_t)kNF * 4;                   // abort flag (i32)
    static constexpr size_t shr = flag + 16;                                 // Shares (this CTA's row ranges)
    static constexpr size_t cur = up(shr + 64, 16);                          // [kCW] u32 x2: consumer ring cursors
    static constexpr size_t bars = up(cur + (size_t)kCW * 8, 16);            // [2][kNF] u64: full, empty
    static constexpr size_t ring = up(bars + (size_t)2 * kNF * 8, 1024);
    static constexpr uint32_t ring_bytes = (uint32_t)((kSmemMax - ring) / 1024 * 1024);
    static constexpr size_t total = ring + ring_bytes;
    // attention items hold one KV block per consumer warp while two fit in the ring
    static constexpr int att_item = ring_bytes >= 2u * kCW * kSlotBytes ? kCW : kCW / 2;
    static_assert(total <= kSmemMax, "shared memory");
    static_assert(ring_bytes >= (uint32_t)(kMaxRowsCta * kH), "the largest linear item must fit in the ring");
    static_assert(ring_bytes >= (uint32_t)(kCW / 2 * kSlotBytes), "an attention item must fit in the ring");
};

// ------------------------------------------------------------ tagged words

__device__ __forceinline__ void ll_st(uint64_t* p, float v, uint32_t tag) {
    const uint64_t w = ((uint64_t)tag << 32) | (uint64_t)__float_as_uint(v);
    asm volatile("st.volatile.global.u64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}
__device__ __forceinline__ uint64_t ll_ld(const uint64_t* p) {
    uint64_t v;
    asm volatile("ld.volatile.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void ll_ld2(const uint64_t* p, uint64_t& a, uint64_t& b) {
    asm volatile("ld.volatile.global.v2.u64 {%0,%1}, [%2];" : "=l"(a), "=l"(b) : "l"(p) : "memory");
}
__device__ __forceinline__ bool ll_ok(uint64_t w, uint32_t tag) { return (uint32_t)(w >> 32) == tag; }
__device__ __forceinline__ float ll_val(uint64_t w) { return __uint_as_float((uint32_t)w); }

struct Ctl {
    unsigned* abort_g;      // global: some CTA gave up
    uint32_t* err;
    volatile int* abort_s;  // shared: this CTA gave up
};
__device__ __forceinline__ bool stopped(const Ctl& c) {
    return *c.abort_s || *reinterpret_cast<volatile unsigned*>(c.abort_g);
}
__device__ __noinline__ void give_up(const Ctl& c, bool timed_out) {
    if (timed_out && c.err) atomicOr(c.err, kErrTimeout);
    atomicExch(c.abort_g, 1u);
    *c.abort_s = 1;
}
// One more iteration of a bounded wait; false when the wait has to end.
__device__ __forceinline__ bool keep_waiting(uint32_t& spins, const Ctl& c) {
    ++spins;
    if ((spins & 127u) == 0u && stopped(c)) {
        *c.abort_s = 1;
        return false;
    }
    if (spins > kPollLimit) {
        give_up(c, true);
        return false;
    }
    return true;
}
__device__ __forceinline__ bool mbar_wait_ctl(uint64_t* bar, uint32_t parity, const Ctl& c) {
    uint32_t spins = 0;
    while (!mbar_try_wait(bar, parity))
        if (!keep_waiting(spins, c)) return false;
    return true;
}

// mbarrier wait that suspends the thread for up to `ns` nanoseconds per try
// (it resumes as soon as the phase completes), so a waiting producer warp
// takes no issue slots from the consumer warps of its SM sub-partition.
__device__ __forceinline__ bool mbar_try_wait_sleep(uint64_t* bar, uint32_t parity, uint32_t ns) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_addr(bar)), "r"(parity), "r"(ns)
        : "memory");
    return ok != 0;
}

// Consumer-group barrier (named barrier 1, the 256 consumer threads) that
// also ANDs a flag over them.
__device__ __forceinline__ bool cbar_and(bool ok) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\t"
        "setp.ne.u32 p, %1, 0;\n\t"
        "bar.red.and.pred q, 1, %2, p;\n\t"
        "selp.u32 %0, 1, 0, q;\n\t}"
        : "=r"(r)
        : "r"((uint32_t)ok), "n"(kCT)
        : "memory");
    return r != 0;
}

// Ring placement shared by the producer and the consumers: an item never
// wraps; one that would is placed at the ring's start. Returns the absolute
// start (ring offset = start % RB).
template <uint32_t RB>
__device__ __forceinline__ uint32_t ring_take(uint32_t& head, uint32_t bytes) {
    const uint32_t pos = head % RB;
    const uint32_t start = pos + bytes > RB ? head + (RB - pos) : head;
    head = start + bytes;
    return start;
}
__device__ __forceinline__ uint32_t item_bytes(uint32_t bytes) { return (bytes + 127u) & ~127u; }

// Position of activation k in a staged row: the 16-byte reads of one lane
// cover 16 consecutive k (four float4 groups), rotated so a warp's reads
// hit 32 distinct banks.
__device__ __forceinline__ int swz(int k) {
    return (k & ~15) | (((((k >> 2) & 3) + ((k >> 5) & 3)) & 3) << 2) | (k & 3);
}
__device__ __forceinline__ uint32_t u4get(const uint4& v, int q) {
    return q == 0 ? v.x : q == 1 ? v.y : q == 2 ? v.z : v.w;
}

// CTA c's share [lo, hi) of n items, in multiples of `align`.
__device__ __forceinline__ void cta_share(int n, int align, int& lo, int& hi) {
    const int units = n / align;
    lo = (int)((unsigned)blockIdx.x * (unsigned)units / gridDim.x) * align;
    hi = (int)((unsigned)(blockIdx.x + 1) * (unsigned)units / gridDim.x) * align;
}

struct Shares {
    int q_lo, q_hi;  // fused QKV rows
    int h_lo, h_hi;  // O / down rows (hidden)
    int p_lo, p_hi;  // gate/up pairs
    int v_lo, v_hi;  // LM head rows
    // attention: this CTA's piece, blocks [blk0, blk0 + nb) of (row b, kv
    // head hd) whose cache holds nblk blocks; it is CTA k of the m CTAs
    // first .. first + m - 1 that share that (row, head)
    int b, hd, blk0, nb, nblk, k, m, first;
};

// Attention partition. The (row b, kv head) pairs s = b n_kv + head, in
// order, own contiguous groups of CTAs [first(s), first(s + 1)), at least one
// each, sized in proportion to their KV blocks (P = blocks before s, T = all
// blocks, S = pairs, G = CTAs): first(s) = floor(P (G - S) / T) + s. CTA k of
// a group of m takes blocks [k n / m, (k + 1) n / m) of its pair's n, so no
// CTA holds blocks of two pairs and the group's last CTA holds the last block.
__device__ __forceinline__ int group_first(const int* pref, int B, int s, int T) {
    const int S = B * kNKV;
    if (s >= S) return (int)gridDim.x;
    const int b = s / kNKV, head = s % kNKV;
    const unsigned long long P = (unsigned long long)kNKV * pref[b] + (unsigned long long)head * (pref[b + 1] - pref[b]);
    return (int)(P * (gridDim.x - S) / (unsigned long long)T) + s;
}
// CTA k of a group of m over n blocks holds any (its range is not empty).
__device__ __forceinline__ bool group_live(int k, int n, int m) { return (k + 1) * n / m > k * n / m; }

__device__ __forceinline__ void trace_mark(const PersistentArgs& a, int slot) {
    if (a.trace && blockIdx.x == 0 && threadIdx.x == 0) {
        uint64_t t;
        asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
        a.trace[slot] = t;
    }
}

// ------------------------------------------------------------ shared views

__device__ __forceinline__ unsigned char* smem_base() {
    extern __shared__ __align__(1024) unsigned char flow_smem_raw[];
    return flow_smem_raw;
}
template <int NB, class T>
__device__ __forceinline__ T* at(size_t off) {
    return reinterpret_cast<T*>(smem_base() + off);
}
template <int NB>
__device__ __forceinline__ Ctl ctl_of(const PersistentArgs& a) {
    return Ctl{a.sync + 2, a.err, at<NB, int>(Lay<NB>::flag)};
}
template <int NB>
__device__ __forceinline__ uint64_t* full_bar(int s) { return at<NB, uint64_t>(Lay<NB>::bars) + s; }
template <int NB>
__device__ __forceinline__ uint64_t* empty_bar(int s) { return at<NB, uint64_t>(Lay<NB>::bars) + kNF + s; }

// ------------------------------------------------------------ producer

// The producer warp's ring state; lane 0 does the waiting.
struct Prod {
    uint32_t n, head, oldest, tail;
    int ok;
};
// Room for an item of `bytes` (placement size) at the ring position the
// consumers compute too: waits, suspended, for the oldest items to be freed.
template <int NB>
__device__ __noinline__ uint32_t prod_reserve(Prod& p, uint32_t bytes, Ctl ctl) {
    constexpr uint32_t RB = Lay<NB>::ring_bytes;
    uint32_t* iend = at<NB, uint32_t>(Lay<NB>::iend);
    const int lane = threadIdx.x % kWarp;
    const uint32_t start = ring_take<RB>(p.head, bytes);
    if (lane == 0) {
#pragma unroll 1
        while (p.ok && p.oldest < p.n && (p.head - p.tail > RB || p.n - p.oldest >= (uint32_t)kNF)) {
            const int s = (int)(p.oldest % kNF);
            uint32_t spins = 0;
            bool done;
#pragma unroll 1
            while (!(done = mbar_try_wait_sleep(empty_bar<NB>(s), (p.oldest / kNF) & 1u, 20000u)))
                if (!keep_waiting(spins, ctl)) break;
            if (!done) {
                p.ok = 0;
                break;
            }
            p.tail = iend[s];
            ++p.oldest;
        }
        if (p.ok) iend[p.n % kNF] = p.head;
    }
    p.ok = __shfl_sync(0xFFFFFFFFu, p.ok, 0);
    return start % RB;
}
template <int NB>
__device__ __noinline__ void prod_linear(Prod& p, const int8_t* src, uint32_t bytes, Ctl ctl) {
    if (!bytes || !p.ok) return;
    const uint32_t off = prod_reserve<NB>(p, item_bytes(bytes), ctl);
    if (!p.ok) return;
    unsigned char* ring = at<NB, unsigned char>(Lay<NB>::ring);
    uint64_t* bar = full_bar<NB>((int)(p.n % kNF));
    if (threadIdx.x % kWarp == 0) {
        mbar_arrive_expect_tx(bar, bytes);
#pragma unroll 1
        for (uint32_t o = 0; o < bytes; o += 32768u) bulk_g2s(ring + off + o, src + o, min(32768u, bytes - o), bar);
    }
    __syncwarp();
    ++p.n;
}
template <int NB>
__device__ __noinline__ void prod_att(Prod& p, const PersistentArgs& a, const uint16_t* kv_layer, int b, int hd,
                                      int blk0, int nb, Ctl ctl) {
    if (!p.ok) return;
    const uint32_t off = prod_reserve<NB>(p, item_bytes((uint32_t)nb * kSlotBytes), ctl);
    if (!p.ok) return;
    unsigned char* ring = at<NB, unsigned char>(Lay<NB>::ring);
    uint64_t* bar = full_bar<NB>((int)(p.n % kNF));
    const int lane = threadIdx.x % kWarp;
    if (lane == 0) mbar_arrive_expect_tx(bar, (uint32_t)nb * kSlotBytes);
    __syncwarp();
    if (lane < nb) {
        int id = a.block_table[(size_t)a.seq_of[b] * a.max_blocks + blk0 + lane];
        if (id < 0 || id >= a.n_pool_blocks) {
            if (a.err) atomicOr(a.err, kErrBadIndex);
            id = 0;
        }
        const uint16_t* src = kv_layer + ((size_t)hd * a.n_pool_blocks + id) * 2 * kBlockElems;
        bulk_g2s(ring + off + lane * kSlotBytes, src, kSlotBytes, bar);
    }
    __syncwarp();
    ++p.n;
}

// The producer warp: this CTA's slices of every phase, in phase order.
template <int NB>
__device__ __noinline__ void producer(const PersistentArgs& a) {
    constexpr int A = Lay<NB>::att_item;
    const Shares sh = *at<NB, Shares>(Lay<NB>::shr);
    const Ctl ctl = ctl_of<NB>(a);
    Prod p{0u, 0u, 0u, 0u, 1};
#pragma unroll 1
    for (int l = 0; l < a.L && p.ok; ++l) {
        const PersistentLayer& P = a.layers[l];
        const uint16_t* kv_layer = a.kv + (size_t)l * a.kv_layer_elems;
        prod_linear<NB>(p, P.wqkv + (size_t)sh.q_lo * kH, (uint32_t)(sh.q_hi - sh.q_lo) * kH, ctl);
#pragma unroll 1
        for (int i = 0; i < sh.nb; i += A) prod_att<NB>(p, a, kv_layer, sh.b, sh.hd, sh.blk0 + i, min(A, sh.nb - i), ctl);
        prod_linear<NB>(p, P.wo + (size_t)sh.h_lo * kQD, (uint32_t)(sh.h_hi - sh.h_lo) * kQD, ctl);
        prod_linear<NB>(p, P.wgu + (size_t)2 * sh.p_lo * kH, (uint32_t)(2 * (sh.p_hi - sh.p_lo)) * kH, ctl);
        prod_linear<NB>(p, P.wd + (size_t)sh.h_lo * kI, (uint32_t)(sh.h_hi - sh.h_lo) * kI, ctl);
    }
#pragma unroll 1
    for (int r = sh.v_lo; r < sh.v_hi && p.ok; r += kHeadRows)
        prod_linear<NB>(p, a.embed + (size_t)r * kH, (uint32_t)min(kHeadRows, sh.v_hi - r) * kH, ctl);

    // Before leaving, wait (bounded) until every copy it issued has landed,
    // so that none is in flight into this CTA's shared memory if the
    // consumers stop early.
    if (threadIdx.x % kWarp == 0) {
#pragma unroll 1
        for (uint32_t i = p.oldest; i < p.n; ++i)
            mbar_wait_bounded(full_bar<NB>((int)(i % kNF)), (i / kNF) & 1u, nullptr, 1u << 20);
    }
}

// ------------------------------------------------------------ consumer helpers

// Stage the rows [B][K] of a tagged vector into xs (swizzled rows of K),
// multiplied by the norm weights nw_g when given (thread t's pairs are k =
// 2 t + 512 j), copying rows [r_lo, r_hi) of the raw values into res, and
// publishing each warp's per-row sums of squares of the raw values in
// red[warp][b]. Not inlined: its polling loop runs in registers of its own.
template <int NB, int K>
__device__ __noinline__ bool stage_ll(const uint64_t* src, int B, uint32_t tag, float* xs, const float* nw_g,
                                      float* red, float* res, int r_lo, int r_hi, Ctl c) {
    constexpr int J = K / 512, N = NB * J;
    const int t = threadIdx.x;
    float2 nw[J];
#pragma unroll
    for (int j = 0; j < J; ++j)
        nw[j] = nw_g ? __ldg(reinterpret_cast<const float2*>(nw_g) + t + 256 * j) : make_float2(1.0f, 1.0f);
    float ss[NB];
#pragma unroll
    for (int b = 0; b < NB; ++b) ss[b] = 0.0f;
    bool ok = true;
    // Pairs are polled eight at a time; every pair of a group that is not
    // ready yet is re-read together, so a group completes one round trip
    // after its last pair lands.
#pragma unroll
    for (int i0 = 0; i0 < N; i0 += 8) {
        uint64_t w[8][2];
        uint32_t pending = 0u;
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            const int i = i0 + u, b = i / J, j = i % J;
            if (i < N && b < B) {
                ll_ld2(src + (size_t)b * K + 2 * t + 512 * j, w[u][0], w[u][1]);
                pending |= 1u << u;
            }
        }
        uint32_t spins = 0;
#pragma unroll 1
        while (ok) {
#pragma unroll
            for (int u = 0; u < 8; ++u)
                if (((pending >> u) & 1u) && ll_ok(w[u][0], tag) && ll_ok(w[u][1], tag)) pending &= ~(1u << u);
            if (!pending) break;
            if (!keep_waiting(spins, c)) {
                ok = false;
                break;
            }
#pragma unroll
            for (int u = 0; u < 8; ++u) {
                const int i = i0 + u, b = i / J, j = i % J;
                if ((pending >> u) & 1u) ll_ld2(src + (size_t)b * K + 2 * t + 512 * j, w[u][0], w[u][1]);
            }
        }
        if (!ok) break;
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            const int i = i0 + u, b = i / J, j = i % J;
            if (i >= N || b >= B) continue;
            const int k = 2 * t + 512 * j;
            const float v0 = ll_val(w[u][0]), v1 = ll_val(w[u][1]);
            ss[b] = fmaf(v0, v0, ss[b]);
            ss[b] = fmaf(v1, v1, ss[b]);
            if (res) {
                if (k >= r_lo && k < r_hi) res[b * kMaxResRows + k - r_lo] = v0;
                if (k + 1 >= r_lo && k + 1 < r_hi) res[b * kMaxResRows + k + 1 - r_lo] = v1;
            }
            xs[b * K + swz(k)] = nw_g ? __fmul_rn(nw[j].x, v0) : v0;
            xs[b * K + swz(k + 1)] = nw_g ? __fmul_rn(nw[j].y, v1) : v1;
        }
    }
    if (red) {
        const int warp = threadIdx.x / kWarp, lane = threadIdx.x % kWarp;
#pragma unroll
        for (int b = 0; b < NB; ++b) {
            const float sw = warp_sum(ss[b]);
            if (lane == 0) red[warp * NB + b] = sw;
        }
    }
    return ok;
}

// Layer 0's input: embedding rows dequantised (embeddingGather ops.zig:397-411
// on the int8 table: f32(q) * scale), staged like stage_ll.
template <int NB>
__device__ __noinline__ void stage_embed(const uint32_t* tok, int B, int V, const int8_t* embed, const float* sembed,
                                         uint32_t* err, float* xs, const float* nw_g, float* red, float* res, int r_lo,
                                         int r_hi) {
    const int t = threadIdx.x;
    float2 nw[kH / 512];
#pragma unroll
    for (int j = 0; j < kH / 512; ++j) nw[j] = __ldg(reinterpret_cast<const float2*>(nw_g) + t + 256 * j);
    float ss[NB];
#pragma unroll
    for (int b = 0; b < NB; ++b) {
        ss[b] = 0.0f;
        if (b >= B) continue;
        const uint32_t id = tok[b];
        const bool valid = id < (uint32_t)V;
        if (!valid && t == 0 && blockIdx.x == 0 && err) atomicOr(err, kErrBadIndex);
        const float sc = valid ? __ldg(sembed + id) : 0.0f;
        const int8_t* row = embed + (size_t)(valid ? id : 0) * kH;
#pragma unroll
        for (int j = 0; j < kH / 512; ++j) {
            const int k = 2 * t + 512 * j;
            const char2 q = *reinterpret_cast<const char2*>(row + k);
            const float v0 = valid ? __fmul_rn((float)q.x, sc) : 0.0f;
            const float v1 = valid ? __fmul_rn((float)q.y, sc) : 0.0f;
            ss[b] = fmaf(v0, v0, ss[b]);
            ss[b] = fmaf(v1, v1, ss[b]);
            if (k >= r_lo && k < r_hi) res[b * kMaxResRows + k - r_lo] = v0;
            if (k + 1 >= r_lo && k + 1 < r_hi) res[b * kMaxResRows + k + 1 - r_lo] = v1;
            xs[b * kH + swz(k)] = __fmul_rn(nw[j].x, v0);
            xs[b * kH + swz(k + 1)] = __fmul_rn(nw[j].y, v1);
        }
    }
    const int warp = threadIdx.x / kWarp, lane = threadIdx.x % kWarp;
#pragma unroll
    for (int b = 0; b < NB; ++b) {
        const float sw = warp_sum(ss[b]);
        if (lane == 0) red[warp * NB + b] = sw;
    }
}

// 1 / sqrt(mean(x^2) + eps) per row in every consumer thread, from the
// per-warp sums stage_ll published (after the barrier that follows it).
template <int NB>
__device__ __forceinline__ void read_inv(const float* red, int K, float eps, float (&inv)[NB]) {
#pragma unroll
    for (int b = 0; b < NB; ++b) {
        float s = 0.0f;
#pragma unroll
        for (int w = 0; w < kCW; ++w) s += red[w * NB + b];
        inv[b] = 1.0f / sqrtf(s / (float)K + eps);
    }
}

// 16-byte loads from shared memory by 32-bit shared address (explicit
// ld.shared, whatever the compiler can infer about the pointer it came from).
__device__ __forceinline__ uint4 lds_u4(uint32_t addr) {
    uint4 v;
    asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr));
    return v;
}
__device__ __forceinline__ float4 lds_f4(uint32_t addr) {
    float4 v;
    asm volatile("ld.shared.v4.f32 {%0,%1,%2,%3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "r"(addr));
    return v;
}

// acc[r][b] = sum_k W[r][k] xs[b][k] for R int8 rows of K in shared memory
// (row stride K), nrows of them real; every lane ends with the sums.
template <int NB, int R, int K>
__device__ __forceinline__ void dot_rows(const int8_t* w, int nrows, const float* xs, int B, float (&acc)[R][NB]) {
    const int lane = threadIdx.x % kWarp;
    const uint32_t wa = smem_addr(w), xa = smem_addr(xs);
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
        for (int b = 0; b < NB; ++b) acc[r][b] = 0.0f;
#pragma unroll
    for (int c = 0; c < K / 512; ++c) {
        const int k0 = (c * kWarp + lane) * 16;
        uint4 wv[R];
#pragma unroll
        for (int r = 0; r < R; ++r)
            wv[r] = r < nrows ? lds_u4(wa + (uint32_t)(r * K + k0)) : make_uint4(0u, 0u, 0u, 0u);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            float wf[R][4];
#pragma unroll
            for (int r = 0; r < R; ++r) i8x4_to_f32(u4get(wv[r], q), wf[r][0], wf[r][1], wf[r][2], wf[r][3]);
#pragma unroll
            for (int b = 0; b < NB; ++b) {
                if (b >= B) break;
                const float4 xv = lds_f4(xa + (uint32_t)(b * K + swz(k0 + 4 * q)) * 4u);
#pragma unroll
                for (int r = 0; r < R; ++r) {
                    acc[r][b] = fmaf(wf[r][0], xv.x, acc[r][b]);
                    acc[r][b] = fmaf(wf[r][1], xv.y, acc[r][b]);
                    acc[r][b] = fmaf(wf[r][2], xv.z, acc[r][b]);
                    acc[r][b] = fmaf(wf[r][3], xv.w, acc[r][b]);
                }
            }
        }
    }
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
        for (int b = 0; b < NB; ++b)
            if (b < B) acc[r][b] = warp_sum(acc[r][b]);
}

// The warp's q fragments for (row b, kv head) and, when it holds the row's
// last block, this step's K and V rows (qwen_block.zig:191-205: per-head
// RMSNorm, split-half RoPE, bf16 rounding on append); attn::share_setup with
// the q, k, v words polled from the tagged QKV output.
__device__ __noinline__ bool share_setup_ll(const uint64_t* qkv_row, int head, int pos, bool has_last,
                                            const float* q_norm, const float* k_norm, const float2* rope,
                                            int rope_max_pos, float eps, uint32_t tag, float* qb, uint16_t* kvnew,
                                            Ctl c, uint32_t* err) {
    const int lane = threadIdx.x % kWarp;
    const uint64_t* qsrc = qkv_row + (size_t)(head * kG) * kD;
    const uint64_t* ksrc = qkv_row + kQD + (size_t)head * kD;
    const uint64_t* vsrc = ksrc + (size_t)kNKV * kD;
    const bool rope_ok = pos >= 0 && pos < rope_max_pos;
    const float2* cs = rope + (size_t)(rope_ok ? pos : 0) * (kD / 2);
    uint64_t wq[kG][4], wk[4] = {0, 0, 0, 0}, wv[4] = {0, 0, 0, 0};
    float qn[4], kn[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    float2 c2[2];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
#pragma unroll
        for (int hh = 0; hh < kG; ++hh) wq[hh][j] = ll_ld(qsrc + hh * kD + lane + 32 * j);
        qn[j] = __ldg(q_norm + lane + 32 * j);
        if (has_last) {
            wk[j] = ll_ld(ksrc + lane + 32 * j);
            wv[j] = ll_ld(vsrc + lane + 32 * j);
            kn[j] = __ldg(k_norm + lane + 32 * j);
        }
    }
#pragma unroll
    for (int j = 0; j < 2; ++j) c2[j] = __ldg(cs + lane + 32 * j);
    // words of q (bits 0-7), k (8-11), v (12-15) not ready yet; all of them
    // are re-read together until every tag matches
    uint32_t pending = has_last ? 0xFFFFu : 0xFFu;
    uint32_t spins = 0;
    bool ok = true;
#pragma unroll 1
    while (true) {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
#pragma unroll
            for (int hh = 0; hh < kG; ++hh)
                if (((pending >> (hh * 4 + j)) & 1u) && ll_ok(wq[hh][j], tag)) pending &= ~(1u << (hh * 4 + j));
            if (((pending >> (8 + j)) & 1u) && ll_ok(wk[j], tag)) pending &= ~(1u << (8 + j));
            if (((pending >> (12 + j)) & 1u) && ll_ok(wv[j], tag)) pending &= ~(1u << (12 + j));
        }
        if (!pending) break;
        if (!keep_waiting(spins, c)) {
            ok = false;
            break;
        }
#pragma unroll
        for (int j = 0; j < 4; ++j) {
#pragma unroll
            for (int hh = 0; hh < kG; ++hh)
                if ((pending >> (hh * 4 + j)) & 1u) wq[hh][j] = ll_ld(qsrc + hh * kD + lane + 32 * j);
            if ((pending >> (8 + j)) & 1u) wk[j] = ll_ld(ksrc + lane + 32 * j);
            if ((pending >> (12 + j)) & 1u) wv[j] = ll_ld(vsrc + lane + 32 * j);
        }
    }
    ok = __all_sync(0xFFFFFFFFu, ok);
    if (!ok) return false;
    float qv[kG][4], kr[4], vr[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
#pragma unroll
        for (int hh = 0; hh < kG; ++hh) qv[hh][j] = ll_val(wq[hh][j]);
        kr[j] = has_last ? ll_val(wk[j]) : 0.0f;
        vr[j] = has_last ? ll_val(wv[j]) : 0.0f;
    }
    auto norm_rope = [&](float (&v)[4], const float (&w)[4]) {
        float ss = 0.0f;
#pragma unroll
        for (int j = 0; j < 4; ++j) ss += v[j] * v[j];
        ss = warp_sum(ss);
        const float inv = 1.0f / sqrtf(ss / (float)kD + eps);
#pragma unroll
        for (int j = 0; j < 4; ++j) v[j] = __fmul_rn(__fmul_rn(w[j], v[j]), inv);
        if (rope_ok) {
#pragma unroll
            for (int j = 0; j < 2; ++j) {
                const float x0 = v[j], x1 = v[j + 2];
                v[j] = __fsub_rn(__fmul_rn(x0, c2[j].x), __fmul_rn(x1, c2[j].y));
                v[j + 2] = __fadd_rn(__fmul_rn(x0, c2[j].y), __fmul_rn(x1, c2[j].x));
            }
        }
    };
#pragma unroll
    for (int hh = 0; hh < kG; ++hh) {
        norm_rope(qv[hh], qn);
#pragma unroll
        for (int j = 0; j < 4; ++j) qb[hh * kD + lane + 32 * j] = qv[hh][j];
    }
    if (has_last) {
        norm_rope(kr, kn);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            kvnew[lane + 32 * j] = f32_to_bf16_rne(kr[j]);
            kvnew[kD + lane + 32 * j] = f32_to_bf16_rne(vr[j]);
        }
    }
    if (!rope_ok && lane == 0 && err) atomicOr(err, kErrBadIndex);
    __syncwarp();
    return true;
}

// The tensor-core B fragments of the two query heads in qb: lanes g < 4 hold
// (head g / 2, bf16 term g % 2) at dims 16 ks + 2 t (+1, +8, +9).
__device__ __forceinline__ void q_fragments(const float* qb, uint32_t (&qf)[8][2]) {
    const int lane = threadIdx.x % kWarp;
    const int g = lane >> 2, t = lane & 3;
    if (g < 4) {
        const float* qp = qb + (g >> 1) * kD;
        const bool lo_part = g & 1;
#pragma unroll
        for (int ks = 0; ks < 8; ++ks) {
            qf[ks][0] = attn::pack_terms(qp[16 * ks + 2 * t], qp[16 * ks + 2 * t + 1], lo_part);
            qf[ks][1] = attn::pack_terms(qp[16 * ks + 2 * t + 8], qp[16 * ks + 2 * t + 9], lo_part);
        }
    } else {
#pragma unroll
        for (int ks = 0; ks < 8; ++ks) qf[ks][0] = qf[ks][1] = 0u;
    }
}

// D = A . B + D for an m16n8k16 tile whose A rows 8..15 are zero: only the
// row-g outputs (d0, d1) are kept; the zero rows go to scratch registers.
__device__ __forceinline__ void mma_rows8(float (&d)[2], uint32_t a0, uint32_t a2, uint32_t b0, uint32_t b1) {
    float z2, z3;  // rows 8..15: zero, discarded
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%5}, {%7,%8}, "
        "{%9,%10,%11,%11};"
        : "=f"(d[0]), "=f"(d[1]), "=f"(z2), "=f"(z3)
        : "r"(a0), "r"(0u), "r"(a2), "r"(b0), "r"(b1), "f"(d[0]), "f"(d[1]), "f"(0.0f));
}

// One 16-token KV block in shared memory (K 4 KB then V 4 KB, chunk-swizzled
// rows; nv valid rows) into the warp's online softmax state, on the tensor
// cores: S = K [q_hi q_lo] (exact products), p in f32, O += [p_hi p_lo] V.
__device__ __forceinline__ void attend_block(const unsigned char* kb, int nv, const uint32_t (&qf)[8][2],
                                             float (&acc)[16][2], float& m_run, float& l_run) {
    constexpr unsigned kAll = 0xFFFFFFFFu;
    const int lane = threadIdx.x % kWarp;
    const int g = lane >> 2, t = lane & 3;
    const int mi = lane >> 3, ri = lane & 7;
    const int tok_a = ri + (mi & 1) * 8;
    const int hsel = (lane >> 3) & 1;
    const float scale = 1.0f / sqrtf((float)kD);
    float sc[4] = {0.0f, 0.0f, 0.0f, 0.0f}, sd[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    const uint32_t kbase = smem_addr(kb), vbase = kbase + kBlockBytes;
#pragma unroll
    for (int ks = 0; ks < 8; ++ks) {
        const int ch = 2 * ks + (mi >> 1);
        uint32_t a0, a1, a2, a3;
        attn::ldsm_x4(kbase + tok_a * (kD * 2) + ((ch ^ ri) << 4), a0, a1, a2, a3);
        if (ks & 1) attn::mma_bf16(sd, a0, a1, a2, a3, qf[ks][0], qf[ks][1]);
        else attn::mma_bf16(sc, a0, a1, a2, a3, qf[ks][0], qf[ks][1]);
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
        pa0 = attn::pack_terms(x0, x1, g & 1);
        pa2 = attn::pack_terms(x8, x9, g & 1);
    }
#pragma unroll
    for (int np = 0; np < 8; ++np) {
        const int ch = 2 * np + (mi >> 1);
        uint32_t b0, b1, b2, b3;
        attn::ldsm_x4_trans(vbase + tok_a * (kD * 2) + ((ch ^ ri) << 4), b0, b1, b2, b3);
        mma_rows8(acc[2 * np], pa0, pa2, b0, b1);
        mma_rows8(acc[2 * np + 1], pa0, pa2, b2, b3);
    }
}

// End of a warp's blocks of a piece: l summed over the warp, the hi and lo
// rows of acc combined (attn::share_reduce for the two-register layout), then
// stored as a shared-memory record [head][m, l, -, -, acc[128]].
__device__ __forceinline__ void warp_partial(float (&acc)[16][2], float l_run, float m_run, float* rec) {
    constexpr unsigned kAll = 0xFFFFFFFFu;
    const int lane = threadIdx.x % kWarp;
    const int t = lane & 3, hsel = (lane >> 3) & 1;
    float L = l_run;
    L += __shfl_xor_sync(kAll, L, 4);
    L += __shfl_xor_sync(kAll, L, 8);
    L += __shfl_xor_sync(kAll, L, 16);
    const float Lh = __shfl_sync(kAll, L, hsel);
    const float Mh = __shfl_sync(kAll, m_run, hsel);
#pragma unroll
    for (int nt = 0; nt < 16; ++nt) {
        acc[nt][0] += __shfl_xor_sync(kAll, acc[nt][0], 4);
        acc[nt][1] += __shfl_xor_sync(kAll, acc[nt][1], 4);
    }
    if (!attn::share_writer()) return;
    float* pg = rec + hsel * kPartHead;
    if (t == 0) {
        pg[0] = Mh;
        pg[1] = Lh;
    }
#pragma unroll
    for (int nt = 0; nt < 16; ++nt)
        *reinterpret_cast<float2*>(pg + 4 + nt * 8 + 2 * t) = make_float2(acc[nt][0], acc[nt][1]);
}

// ------------------------------------------------------------ cross-CTA merge

// Merge of `count` shared-memory partials (slots base + j kPartStride, [h][m,
// l, -, -, acc[128]]) in the log-sum-exp sense by all consumer threads at once:
// thread t owns query head t / 128, dim t % 128. Returns that thread's
// (M, L, A); the slot order fixes the result.
__device__ __forceinline__ void merge_slots(const float* base, int count, float& M, float& L, float& A) {
    const int hh = threadIdx.x >> 7, d = threadIdx.x & (kD - 1);
    const float* b = base + hh * kPartHead;
    M = -INFINITY;
#pragma unroll 1
    for (int j = 0; j < count; ++j) M = fmaxf(M, b[j * kPartStride]);
    L = 0.0f;
    A = 0.0f;
#pragma unroll 1
    for (int j = 0; j < count; ++j) {
        const float m = b[j * kPartStride];
        const float c = m == -INFINITY ? 0.0f : expf(m - M);
        L = fmaf(b[j * kPartStride + 1], c, L);
        A = fmaf(b[j * kPartStride + 4 + d], c, A);
    }
}

// The cross-CTA merge of one (row, kv head): records 0 .. nrec - 1 (record k
// from CTA k of the group, none from CTAs of the group that hold no block) and
// this CTA's own partial, combined in the log-sum-exp sense; the normalised
// output of both query heads is published as tagged words. Warp w polls
// records w, w + 8, w + 16 (every pending word of them re-read together, so
// the poll ends one round trip after the last record lands) and folds them
// in order; the warps' partials go to shared memory (slots 0..7 of `part`,
// the own partial after them) and warp 0 merges them in warp order.
// Called by all consumer warps; returns false on a timeout or abort.
__device__ __noinline__ bool merge_across_ctas(const uint64_t* rec_bh, int nrec, int n, int m, const float* own,
                                               float* part, uint64_t* out, uint32_t tag, Ctl ctl) {
    constexpr int kPer = 3;  // records per warp and round
    const int warp = threadIdx.x / kWarp, lane = threadIdx.x % kWarp;
    float M[kG] = {-INFINITY, -INFINITY}, L[kG] = {0.0f, 0.0f};
    float A[kG][4] = {{0.0f, 0.0f, 0.0f, 0.0f}, {0.0f, 0.0f, 0.0f, 0.0f}};
    bool ok = true;
#pragma unroll 1
    for (int k0 = 0; k0 < nrec && ok; k0 += kPer * kCW) {
        // words of record j: [h][m, l] and [h][acc 4 lane .. 4 lane + 3]
        uint64_t w[kPer][kG][3][2];
        uint32_t pending = 0u;
#pragma unroll
        for (int j = 0; j < kPer; ++j) {
            const int k = k0 + warp + kCW * j;
            if (k < nrec && group_live(k, n, m)) pending |= 1u << j;
        }
        const uint32_t live = pending;
        auto load = [&](int j) {
            const uint64_t* r = rec_bh + (size_t)(k0 + warp + kCW * j) * kRecWords;
#pragma unroll
            for (int h = 0; h < kG; ++h) {
                ll_ld2(r + h * kRecHead, w[j][h][0][0], w[j][h][0][1]);
                ll_ld2(r + h * kRecHead + 2 + 4 * lane, w[j][h][1][0], w[j][h][1][1]);
                ll_ld2(r + h * kRecHead + 4 + 4 * lane, w[j][h][2][0], w[j][h][2][1]);
            }
        };
#pragma unroll
        for (int j = 0; j < kPer; ++j)
            if ((live >> j) & 1u) load(j);
        uint32_t spins = 0;
#pragma unroll 1
        while (true) {
#pragma unroll
            for (int j = 0; j < kPer; ++j) {
                if (!((pending >> j) & 1u)) continue;
                bool ready = true;
#pragma unroll
                for (int h = 0; h < kG; ++h)
#pragma unroll
                    for (int q = 0; q < 3; ++q) ready = ready && ll_ok(w[j][h][q][0], tag) && ll_ok(w[j][h][q][1], tag);
                if (ready) pending &= ~(1u << j);
            }
            if (!pending) break;
            if (!keep_waiting(spins, ctl)) {
                ok = false;
                break;
            }
#pragma unroll
            for (int j = 0; j < kPer; ++j)
                if ((pending >> j) & 1u) load(j);
        }
        if (!ok) break;
#pragma unroll
        for (int j = 0; j < kPer; ++j) {
            if (!((live >> j) & 1u)) continue;
#pragma unroll
            for (int h = 0; h < kG; ++h) {
                const float m = ll_val(w[j][h][0][0]), lsum = ll_val(w[j][h][0][1]);
                if (m == -INFINITY) continue;
                if (m > M[h]) {
                    const float cr = expf(M[h] - m);
                    L[h] *= cr;
#pragma unroll
                    for (int e = 0; e < 4; ++e) A[h][e] *= cr;
                    M[h] = m;
                }
                const float ex = expf(m - M[h]);
                L[h] = fmaf(lsum, ex, L[h]);
                A[h][0] = fmaf(ll_val(w[j][h][1][0]), ex, A[h][0]);
                A[h][1] = fmaf(ll_val(w[j][h][1][1]), ex, A[h][1]);
                A[h][2] = fmaf(ll_val(w[j][h][2][0]), ex, A[h][2]);
                A[h][3] = fmaf(ll_val(w[j][h][2][1]), ex, A[h][3]);
            }
        }
    }
    // warp partial -> slot `warp` ([h][m, l, -, -, acc[128]]); the own
    // partial -> slot kCW
    float* rec = part + (size_t)warp * kPartStride;
#pragma unroll
    for (int h = 0; h < kG; ++h) {
        if (lane == 0) {
            rec[h * kPartHead] = M[h];
            rec[h * kPartHead + 1] = L[h];
        }
        *reinterpret_cast<float4*>(rec + h * kPartHead + 4 + 4 * lane) = make_float4(A[h][0], A[h][1], A[h][2], A[h][3]);
    }
    if (warp == 0) {
        float* o = part + (size_t)kCW * kPartStride;
        for (int i = lane; i < kPartStride; i += kWarp) o[i] = own[i];
    }
    if (!cbar_and(ok)) return false;
    float Mm, Lm, Am;
    merge_slots(part, kCW + 1, Mm, Lm, Am);
    ll_st(out + threadIdx.x, Am * (1.0f / Lm), tag);  // thread t: head t / 128, dim t % 128
    return true;
}

// ------------------------------------------------------------ consumer phases
//
// Each phase is a function of its own (not inlined): it holds only its own
// state in registers, and nothing but the layer index lives across phases.
// The consumer warps' ring cursor lives in shared memory. Every phase ends
// with a consumer barrier that ANDs the success flags; a false return ends
// the step for every consumer warp together.

// The consumer side of the ring: the next item's shared-memory address, its
// barrier slot and phase parity, in the order the producer issued them.
template <int NB>
struct Cursor {
    uint32_t n, head;
    __device__ __forceinline__ Cursor() {
        const uint2 c = at<NB, uint2>(Lay<NB>::cur)[threadIdx.x / kWarp];
        n = c.x;
        head = c.y;
    }
    __device__ __forceinline__ void save() const {
        __syncwarp();
        if (threadIdx.x % kWarp == 0) at<NB, uint2>(Lay<NB>::cur)[threadIdx.x / kWarp] = make_uint2(n, head);
        __syncwarp();
    }
    __device__ __forceinline__ const unsigned char* next(uint32_t bytes, int& s, uint32_t& parity) {
        constexpr uint32_t RB = Lay<NB>::ring_bytes;
        const uint32_t start = ring_take<RB>(head, item_bytes(bytes));
        s = (int)(n % kNF);
        parity = (n / kNF) & 1u;
        ++n;
        return at<NB, unsigned char>(Lay<NB>::ring) + start % RB;
    }
};
template <int NB>
__device__ __forceinline__ void release_item(int s) {
    __syncwarp();
    if (threadIdx.x % kWarp == 0) mbar_arrive(empty_bar<NB>(s));
}
template <int NB>
__device__ __forceinline__ bool wait_item(int s, uint32_t parity, const Ctl& ctl) {
    return __all_sync(0xFFFFFFFFu, mbar_wait_ctl(full_bar<NB>(s), parity, ctl));
}

// QKV: RMSNorm(input_ln) + this CTA's fused QKV rows (layer 0 stages the
// embedding rows instead of the previous layer's output).
template <int NB>
__device__ __noinline__ bool qkv_phase(const PersistentArgs& a, int l) {
    using LY = Lay<NB>;
    const Shares sh = *at<NB, Shares>(LY::shr);
    const PersistentLayer& P = a.layers[l];
    const uint32_t tag = a.tag + (uint32_t)l + 1u;
    const Ctl ctl = ctl_of<NB>(a);
    const int tid = threadIdx.x, warp = tid / kWarp, lane = tid % kWarp, B = a.B;
    float* xa = at<NB, float>(LY::xa);
    float* scl = at<NB, float>(LY::scl);
    float* red = at<NB, float>(LY::red);
    float* res0 = at<NB, float>(LY::res);
    const int nq = sh.q_hi - sh.q_lo;
#pragma unroll 1
    for (int i = tid; i < nq; i += kCT) scl[i] = __ldg(P.sqkv + sh.q_lo + i);
    bool ok = true;
    if (l == 0)
        stage_embed<NB>(a.tok, B, a.V, a.embed, a.sembed, a.err, xa, P.input_ln, red, res0, sh.h_lo, sh.h_hi);
    else  // (an injected stall polls a tag that nothing writes, so the bounded wait runs out)
        ok = stage_ll<NB, kH>(a.llx, B, l == a.stall_layer ? (tag - 1u) ^ 0x80000000u : tag - 1u, xa, P.input_ln, red,
                              res0, sh.h_lo, sh.h_hi, ctl);
    if (!cbar_and(ok)) return false;
    trace_mark(a, 1 + 10 * l);
    float inv[NB];
    read_inv<NB>(red, kH, a.eps, inv);
    Cursor<NB> cur;
    if (nq) {
        int s;
        uint32_t par;
        const unsigned char* item = cur.next((uint32_t)nq * kH, s, par);
        constexpr int R = 4;
        const int units = (nq + R - 1) / R;
        if (warp < units) ok = wait_item<NB>(s, par, ctl);
#pragma unroll 1
        for (int u = warp; u < units && ok; u += kCW) {
            const int r0 = u * R;
            float acc[R][NB];
            dot_rows<NB, R, kH>(reinterpret_cast<const int8_t*>(item) + (size_t)r0 * kH, min(R, nq - r0), xa, B, acc);
#pragma unroll
            for (int r = 0; r < R; ++r)
#pragma unroll
                for (int b = 0; b < NB; ++b)
                    if (b < B && r0 + r < nq && lane == ((r * NB + b) & 31))
                        ll_st(a.llqkv + (size_t)b * kQKV + sh.q_lo + r0 + r,
                              __fmul_rn(__fmul_rn(acc[r][b], inv[b]), scl[r0 + r]), tag);
        }
        release_item<NB>(s);
    }
    cur.save();
    trace_mark(a, 2 + 10 * l);
    return cbar_and(ok);  // scl and xa are rewritten by the next phases
}

// ATT: this CTA's piece of one (row, kv head): its KV blocks, one per warp
// per ring item, merged in shared memory, then either published (the CTA
// holds the whole row), written as a record, or merged with the group's
// records (the group's last CTA); see the file comment.
template <int NB>
__device__ __noinline__ bool att_phase(const PersistentArgs& a, int l) {
    using LY = Lay<NB>;
    constexpr int A = LY::att_item;
    const Shares sh = *at<NB, Shares>(LY::shr);
    const PersistentLayer& P = a.layers[l];
    const uint32_t tag = a.tag + (uint32_t)l + 1u;
    const Ctl ctl = ctl_of<NB>(a);
    const int warp = threadIdx.x / kWarp, lane = threadIdx.x % kWarp;
    const int max_len = a.max_blocks * kKvBlock;
    float* part = at<NB, float>(LY::part);
    float* own = at<NB, float>(LY::own);
    float* qb = at<NB, float>(LY::qb) + warp * kG * kD;
    uint16_t* kvnew = at<NB, uint16_t>(LY::kvn) + warp * 2 * kD;
    uint16_t* kv_layer = a.kv + (size_t)l * a.kv_layer_elems;
    trace_mark(a, 3 + 10 * l);
    Cursor<NB> cur;
    bool ok = true;
    if (sh.nb > 0) {
        const int b = sh.b, hd = sh.hd, blk0 = sh.blk0, nb = sh.nb, nblk = sh.nblk;
        const bool starts = blk0 == 0, ends = blk0 + nb == nblk;
        const int pos = a.positions[b];
        const int kv_len = min(max(pos + 1, 1), max_len);
        // this warp's blocks of the piece: i = warp, warp + kCW, ...
        const bool have = warp < nb;
        const bool holds_last = ends && ((nb - 1) % kCW) == warp;
        uint16_t* last_k = nullptr;
        if (holds_last) {
            int id = a.block_table[(size_t)a.seq_of[b] * a.max_blocks + nblk - 1];
            if (id < 0 || id >= a.n_pool_blocks) id = 0;  // the producer reports it
            last_k = kv_layer + ((size_t)hd * a.n_pool_blocks + id) * 2 * kBlockElems;
        }
        uint32_t qf[8][2];
        if (have && ok)
            ok = share_setup_ll(a.llqkv + (size_t)b * kQKV, hd, pos, holds_last, P.q_norm, P.k_norm, a.rope,
                                a.rope_max_pos, a.eps, tag, qb, kvnew, ctl, a.err);
        if (have && ok) q_fragments(qb, qf);
        float acc[16][2];
#pragma unroll
        for (int nt = 0; nt < 16; ++nt) acc[nt][0] = acc[nt][1] = 0.0f;
        float m_run = -INFINITY, l_run = 0.0f;
#pragma unroll 1
        for (int i0 = 0; i0 < nb; i0 += A) {
            int s;
            uint32_t par;
            const unsigned char* item = cur.next((uint32_t)min(A, nb - i0) * kSlotBytes, s, par);
            // this warp's block of the item (at most one: A <= kCW)
            const int mine = i0 + ((warp - i0 % kCW + kCW) % kCW);
            if (mine < min(nb, i0 + A) && ok) {
                ok = wait_item<NB>(s, par, ctl);
                if (ok) {
                    unsigned char* kb = const_cast<unsigned char*>(item) + (size_t)(mine - i0) * kSlotBytes;
                    const int blk = blk0 + mine;
                    const int nv = min(kKvBlock, kv_len - blk * kKvBlock);
                    const bool last = blk == nblk - 1;
                    if (last) attn::patch_new_row(last_k, kb, nv - 1, kvnew);
                    if (nv < kKvBlock) {
                        uint4* vrow = reinterpret_cast<uint4*>(kb + kBlockBytes + nv * kD * 2);
#pragma unroll 1
                        for (int x = lane; x < (kKvBlock - nv) * (kD * 2 / 16); x += kWarp)
                            vrow[x] = make_uint4(0u, 0u, 0u, 0u);
                    }
                    __syncwarp();
                    attend_block(kb, nv, qf, acc, m_run, l_run);
                    if (nv < kKvBlock || last) attn::fence_proxy_async_smem();
                }
            }
            release_item<NB>(s);
        }
        if (have && ok) warp_partial(acc, l_run, m_run, part + warp * kPartStride);
        ok = cbar_and(ok);
        if (ok) {
            // the warps' partials merged by all threads, thread t owning
            // (query head t / 128, dim t % 128)
            float M, L, Av;
            merge_slots(part, min(nb, kCW), M, L, Av);
            const int hh = threadIdx.x >> 7, d = threadIdx.x & (kD - 1);
            if (starts && ends) {
                ll_st(a.llattn + (size_t)b * kQD + (size_t)(hd * kG + hh) * kD + d, Av * (1.0f / L), tag);
            } else if (ends) {
                if (d == 0) {
                    own[hh * kPartHead] = M;
                    own[hh * kPartHead + 1] = L;
                }
                own[hh * kPartHead + 4 + d] = Av;
            } else {
                uint64_t* rec = a.llrec + (((size_t)b * kNKV + hd) * gridDim.x + sh.k) * kRecWords + hh * kRecHead;
                if (d == 0) {
                    ll_st(rec, M, tag);
                    ll_st(rec + 1, L, tag);
                }
                ll_st(rec + 2 + d, Av, tag);
            }
        }
        if (ok && !starts && ends) {
            // the group's last CTA merges the records of the CTAs before it
            // with its own and publishes the output
            ok = cbar_and(ok);  // `own` is written
            if (ok)
                ok = merge_across_ctas(a.llrec + ((size_t)b * kNKV + hd) * gridDim.x * kRecWords, sh.k, nblk, sh.m,
                                       own, part, a.llattn + (size_t)b * kQD + (size_t)hd * kG * kD, tag, ctl);
        }
    }
    cur.save();
    trace_mark(a, 4 + 10 * l);
    return cbar_and(ok);
}

// O (+ residual) and D (+ residual): rows [h_lo, h_hi), one per warp, over
// the staged attention output (K = 2048) or SwiGLU output (K = 3072).
template <int NB, int K>
__device__ __noinline__ bool out_phase(const PersistentArgs& a, int l) {
    using LY = Lay<NB>;
    const Shares sh = *at<NB, Shares>(LY::shr);
    const PersistentLayer& P = a.layers[l];
    constexpr bool is_o = K == kQD;
    const uint32_t tag = a.tag + (uint32_t)l + 1u;
    const Ctl ctl = ctl_of<NB>(a);
    const int tid = threadIdx.x, warp = tid / kWarp, lane = tid % kWarp, B = a.B;
    float* xb = at<NB, float>(LY::xb);
    float* scl = at<NB, float>(LY::scl);
    const float* res = at<NB, float>(LY::res) + (is_o ? 0 : NB * kMaxResRows);
    const int nh = sh.h_hi - sh.h_lo;
    const float* sg = is_o ? P.so : P.sd;
#pragma unroll 1
    for (int i = tid; i < nh; i += kCT) scl[i] = __ldg(sg + sh.h_lo + i);
    bool ok = stage_ll<NB, K>(is_o ? a.llattn : a.llh, B, tag, xb, nullptr, nullptr, nullptr, 0, 0, ctl);
    if (!cbar_and(ok)) return false;
    constexpr int slot = is_o ? 5 : 9;
    trace_mark(a, slot + 10 * l);
    Cursor<NB> cur;
    uint64_t* dst = is_o ? a.llx1 : a.llx;
    if (nh) {
        int s;
        uint32_t par;
        const unsigned char* item = cur.next((uint32_t)nh * K, s, par);
        if (warp < nh) ok = wait_item<NB>(s, par, ctl);
#pragma unroll 1
        for (int u = warp; u < nh && ok; u += kCW) {
            float acc[1][NB];
            dot_rows<NB, 1, K>(reinterpret_cast<const int8_t*>(item) + (size_t)u * K, 1, xb, B, acc);
#pragma unroll
            for (int b = 0; b < NB; ++b)
                if (b < B && lane == b)
                    ll_st(dst + (size_t)b * kH + sh.h_lo + u,
                          __fadd_rn(res[b * kMaxResRows + u], __fmul_rn(acc[0][b], scl[u])), tag);
        }
        release_item<NB>(s);
    }
    cur.save();
    trace_mark(a, slot + 1 + 10 * l);
    return cbar_and(ok);
}

// GU (+ SwiGLU): RMSNorm(post_ln) + gate/up pairs [p_lo, p_hi).
template <int NB>
__device__ __noinline__ bool gu_phase(const PersistentArgs& a, int l) {
    using LY = Lay<NB>;
    const Shares sh = *at<NB, Shares>(LY::shr);
    const PersistentLayer& P = a.layers[l];
    const uint32_t tag = a.tag + (uint32_t)l + 1u;
    const Ctl ctl = ctl_of<NB>(a);
    const int tid = threadIdx.x, warp = tid / kWarp, lane = tid % kWarp, B = a.B;
    float* xa = at<NB, float>(LY::xa);
    float* scl = at<NB, float>(LY::scl);
    float* red = at<NB, float>(LY::red);
    float* res1 = at<NB, float>(LY::res) + NB * kMaxResRows;
    const int np = sh.p_hi - sh.p_lo;
#pragma unroll 1
    for (int i = tid; i < 2 * np; i += kCT) scl[i] = __ldg(P.sgu + 2 * sh.p_lo + i);
    bool ok = stage_ll<NB, kH>(a.llx1, B, tag, xa, P.post_ln, red, res1, sh.h_lo, sh.h_hi, ctl);
    if (!cbar_and(ok)) return false;
    trace_mark(a, 7 + 10 * l);
    float inv[NB];
    read_inv<NB>(red, kH, a.eps, inv);
    Cursor<NB> cur;
    if (np) {
        int s;
        uint32_t par;
        const unsigned char* item = cur.next((uint32_t)(2 * np) * kH, s, par);
        constexpr int R = 6;  // three (gate, up) pairs
        const int rows = 2 * np, units = (rows + R - 1) / R;
        if (warp < units) ok = wait_item<NB>(s, par, ctl);
#pragma unroll 1
        for (int u = warp; u < units && ok; u += kCW) {
            const int r0 = u * R;
            float acc[R][NB];
            dot_rows<NB, R, kH>(reinterpret_cast<const int8_t*>(item) + (size_t)r0 * kH, min(R, rows - r0), xa, B, acc);
#pragma unroll
            for (int p = 0; p < R / 2; ++p)
#pragma unroll
                for (int b = 0; b < NB; ++b) {
                    const int row = r0 + 2 * p;
                    if (b < B && row < rows && lane == ((p * NB + b) & 31)) {
                        const float gate = __fmul_rn(__fmul_rn(acc[2 * p][b], inv[b]), scl[row]);
                        const float upv = __fmul_rn(__fmul_rn(acc[2 * p + 1][b], inv[b]), scl[row + 1]);
                        ll_st(a.llh + (size_t)b * kI + sh.p_lo + (row >> 1), __fmul_rn(silu(gate), upv), tag);
                    }
                }
        }
        release_item<NB>(s);
    }
    cur.save();
    trace_mark(a, 8 + 10 * l);
    return cbar_and(ok);
}

// HEAD: final RMSNorm, this CTA's tied LM head rows, argmax (topK(1),
// qwen_forward.zig:177-193); the last CTA to finish turns the keys into next
// tokens and advances the rows.
template <int NB>
__device__ __noinline__ void head_phase(const PersistentArgs& a, bool ok) {
    using LY = Lay<NB>;
    constexpr unsigned kAll = 0xFFFFFFFFu;
    const Shares sh = *at<NB, Shares>(LY::shr);
    const Ctl ctl = ctl_of<NB>(a);
    const int tid = threadIdx.x, warp = tid / kWarp, lane = tid % kWarp, B = a.B;
    float* xa = at<NB, float>(LY::xa);
    float* red = at<NB, float>(LY::red);
    unsigned long long* bestv = at<NB, unsigned long long>(LY::best);
    const int hslot = 1 + 10 * a.L;
    unsigned long long best[NB];
#pragma unroll
    for (int b = 0; b < NB; ++b) best[b] = 0ull;
    if (ok) {
        ok = stage_ll<NB, kH>(a.llx, B, a.tag + (uint32_t)a.L, xa, a.final_norm, red, nullptr, 0, 0, ctl);
        ok = cbar_and(ok);
    }
    if (ok) {
        trace_mark(a, hslot);
        float inv[NB];
        read_inv<NB>(red, kH, a.eps, inv);
        constexpr int R = kHeadRows / kCW;
        Cursor<NB> cur;
#pragma unroll 1
        for (int r = sh.v_lo; r < sh.v_hi; r += kHeadRows) {
            const int rows = min(kHeadRows, sh.v_hi - r);
            int s;
            uint32_t par;
            const unsigned char* item = cur.next((uint32_t)rows * kH, s, par);
            const int r0 = warp * R;
            const float sc = r0 + (lane & (R - 1)) < rows ? __ldg(a.sembed + r + r0 + (lane & (R - 1))) : 0.0f;
            if (r0 < rows && ok) {
                ok = wait_item<NB>(s, par, ctl);
                if (ok) {
                    float acc[R][NB];
                    dot_rows<NB, R, kH>(reinterpret_cast<const int8_t*>(item) + (size_t)r0 * kH, min(R, rows - r0), xa, B, acc);
#pragma unroll
                    for (int q = 0; q < R; ++q) {
                        const float sq = __shfl_sync(kAll, sc, q);
#pragma unroll
                        for (int b = 0; b < NB; ++b) {
                            if (b >= B || r0 + q >= rows) continue;
                            const float val = __fmul_rn(__fmul_rn(acc[q][b], inv[b]), sq);
                            const uint32_t row = (uint32_t)(r + r0 + q);
                            if (a.logits && lane == b) a.logits[(size_t)b * a.V + row] = val;
                            const unsigned long long key = argmax_key(val, row);
                            best[b] = key > best[b] ? key : best[b];
                        }
                    }
                }
            }
            release_item<NB>(s);
        }
    }
    trace_mark(a, hslot + 1);
#pragma unroll
    for (int b = 0; b < NB; ++b)
        if (lane == 0) bestv[warp * NB + b] = best[b];
    ok = cbar_and(ok);
    if (ok && tid < B) {
        unsigned long long m = 0ull;
#pragma unroll 1
        for (int w = 0; w < kCW; ++w) m = bestv[w * NB + tid] > m ? bestv[w * NB + tid] : m;
        if (m) atomicMax(a.keys + tid, m);
    }
    ok = cbar_and(ok);
    if (ok && tid == 0) {
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
                a.trace[hslot + 2] = t;
            }
            a.sync[1] = 0u;
            __threadfence();
        }
    }
}

// ------------------------------------------------------------ the kernel

template <int NB>
__global__ void __launch_bounds__(kFT, 1) decode_flow_kernel(const __grid_constant__ PersistentArgs a) {
    using LY = Lay<NB>;
    const int warp = threadIdx.x / kWarp;
    const int max_len = a.max_blocks * kKvBlock;
    int* pref = at<NB, int>(LY::pref);
    if (threadIdx.x == 0) {
        *at<NB, int>(LY::flag) = 0;
        pref[0] = 0;
        for (int b = 0; b < a.B; ++b) {
            const int len = a.positions[b] + 1;
            if ((len < 1 || len > max_len) && a.err) atomicOr(a.err, kErrBadIndex);
            pref[b + 1] = pref[b] + (min(max(len, 1), max_len) + kKvBlock - 1) / kKvBlock;
        }
        Shares sh;
        cta_share(kQKV, 1, sh.q_lo, sh.q_hi);
        cta_share(kH, 1, sh.h_lo, sh.h_hi);
        cta_share(kI, 1, sh.p_lo, sh.p_hi);
        cta_share(a.V, 1, sh.v_lo, sh.v_hi);
        // this CTA's attention piece: its (row, kv head) group and share
        const int T = pref[a.B] * kNKV, S = a.B * kNKV, c = (int)blockIdx.x;
        int lo = 0, hi = S - 1;  // the last pair whose group starts at or before c
        while (lo < hi) {
            const int mid = (lo + hi + 1) / 2;
            if (group_first(pref, a.B, mid, T) <= c) lo = mid;
            else hi = mid - 1;
        }
        sh.first = group_first(pref, a.B, lo, T);
        sh.m = group_first(pref, a.B, lo + 1, T) - sh.first;
        sh.k = c - sh.first;
        sh.b = lo / kNKV;
        sh.hd = lo % kNKV;
        sh.nblk = pref[sh.b + 1] - pref[sh.b];
        sh.blk0 = sh.k * sh.nblk / sh.m;
        sh.nb = (sh.k + 1) * sh.nblk / sh.m - sh.blk0;
        *at<NB, Shares>(LY::shr) = sh;
    }
    if (threadIdx.x < kCW) at<NB, uint2>(LY::cur)[threadIdx.x] = make_uint2(0u, 0u);
    if (threadIdx.x == kCT) {
        for (int s = 0; s < kNF; ++s) {
            mbar_init(full_bar<NB>(s), 1);
            mbar_init(empty_bar<NB>(s), kCW);
        }
        fence_barrier_init();
    }
    trace_mark(a, 0);
    __syncthreads();

    if (warp == kCW) {
        producer<NB>(a);
        return;
    }
    bool ok = true;
#pragma unroll 1
    for (int l = 0; l < a.L && ok; ++l) {
        ok = qkv_phase<NB>(a, l);
        if (ok) ok = att_phase<NB>(a, l);
        if (ok) ok = out_phase<NB, kQD>(a, l);
        if (ok) ok = gu_phase<NB>(a, l);
        if (ok) ok = out_phase<NB, kI>(a, l);
    }
    head_phase<NB>(a, ok);
}

template <int NB>
constexpr size_t flow_smem() {
    return Lay<NB>::total;
}

}  // namespace

void prepare_flow_kernels() {
    configure_kernel((const void*)decode_flow_kernel<1>, flow_smem<1>());
    configure_kernel((const void*)decode_flow_kernel<2>, flow_smem<2>());
    configure_kernel((const void*)decode_flow_kernel<4>, flow_smem<4>());
    configure_kernel((const void*)decode_flow_kernel<8>, flow_smem<8>());
}

bool flow_supported(int device) {
    int coop = 0, sms = 0;
    if (cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, device) != cudaSuccess || !coop) return false;
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device) != cudaSuccess || sms < kMinCtas)
        return false;
    const void* kernels[] = {(const void*)decode_flow_kernel<1>, (const void*)decode_flow_kernel<2>,
                             (const void*)decode_flow_kernel<4>, (const void*)decode_flow_kernel<8>};
    const size_t smem[] = {flow_smem<1>(), flow_smem<2>(), flow_smem<4>(), flow_smem<8>()};
    for (int i = 0; i < 4; ++i) {
        int blocks = 0;
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&blocks, kernels[i], kFT, smem[i]) != cudaSuccess ||
            blocks < 1)
            return false;
    }
    return true;
}

size_t flow_record_words(int ctas) { return (size_t)kPersistentMaxBatch * kNKV * ctas * kRecWords; }

cudaError_t launch_decode_flow(const PersistentArgs& a, cudaStream_t st) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(device_sm_count());
    cfg.blockDim = dim3(kFT);
    cfg.stream = st;
    cudaLaunchAttribute attr;
    attr.id = cudaLaunchAttributeCooperative;
    attr.val.cooperative = 1;
    cfg.attrs = &attr;
    cfg.numAttrs = 1;
    if (a.B <= 1) {
        cfg.dynamicSmemBytes = flow_smem<1>();
        return cudaLaunchKernelEx(&cfg, decode_flow_kernel<1>, a);
    }
    if (a.B <= 2) {
        cfg.dynamicSmemBytes = flow_smem<2>();
        return cudaLaunchKernelEx(&cfg, decode_flow_kernel<2>, a);
    }
    if (a.B <= 4) {
        cfg.dynamicSmemBytes = flow_smem<4>();
        return cudaLaunchKernelEx(&cfg, decode_flow_kernel<4>, a);
    }
    cfg.dynamicSmemBytes = flow_smem<8>();
    return cudaLaunchKernelEx(&cfg, decode_flow_kernel<8>, a);
}

}  // namespace zc
