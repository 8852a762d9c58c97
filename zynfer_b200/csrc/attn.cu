// Causal GQA attention (attentionInto, src/backends/cpu/ops.zig:285-354) on
// the B200: a split-K decode kernel over the paged bf16 KV cache with a
// log-sum-exp merge, and a tiled f32 prefill kernel.
#include <algorithm>
#include <type_traits>

#include "attn_common.cuh"
#include "common.cuh"
#include "kernels.h"

namespace zc {

namespace {

// ------------------------------------------------------------- decode
//
// Persistent and warp-granular. The work of one launch is the list of
// (batch row, kv head, 16-token KV block) triples, row-major; every warp of
// the grid takes an equal contiguous range of it (at least
// kMinBlocksPerWarp), so each block of K/V is read exactly once and all
// warps stream the same number of bytes whatever the context lengths. A warp
// owns a private ring of kRing 8 KB slots (K then V of one block and head;
// three slots, two for a one-row step)
// filled by cp.async.bulk on per-slot mbarriers; there is no barrier between
// warps in the main loop.
//
// Per block, on the tensor cores (mma.sync m16n8k16, bf16 in, f32 out):
//   S[16 tok][8] = K[16 tok][128] . Qcols[128][8], columns (h0 hi, h0 lo,
//       h1 hi, h1 lo, 0...): q is split into two bf16 terms, q = hi + lo,
//       |q - hi - lo| <= 2^-18 |q|, and K is exact bf16, so every product is
//       exact and the dot products carry f32 accuracy;
//   online softmax per query head in f32 (max, exp, sum);
//   O[4 rows][128] += P[4 rows][16 tok] . V[16 tok][128], rows (h0 hi, h0 lo,
//       h1 hi, h1 lo): p is split the same way.
// Two consecutive blocks of one (row, kv head) are taken together: their
// score and PV mma chains interleave and share one online-softmax update
// (the running max over both blocks' scores), which keeps a warp issuing
// while one chain waits (4 % faster at 64 rows, where the kernel streams at
// the rate of the same ring without the math).
// A range boundary inside a (row, kv head) leaves partial results
// (max, sum, acc[d]) per query head; the last warp to finish one (atomic
// counter) merges them in segment order:
//   m = max m_s,  l = sum l_s e^(m_s - m),  o = sum acc_s e^(m_s - m) / l.
// A one-sequence step of up to kHeadClusterMaxBlocks blocks runs instead as
// one 8-CTA cluster per kv head: the same per-warp loop over that head's
// blocks, the CTAs' partials merged in the cluster's first CTA after one
// cluster barrier (distributed shared memory, no counter).
//
// KV blocks are stored with their 16-byte chunks XOR-swizzled by token
// (kv_swizzle), so the ldmatrix reads of K rows and the transposing reads of
// V rows hit 32 distinct banks.
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
constexpr int kDecWarps = 8, kDecThreads = kDecWarps * kWarp;
static_assert(kDecWarps >= 4, "decode_max_segs assumes CTA spans of at least 4 warps");
constexpr int kMaxBatch = 1024;
constexpr int kIdRing = 64;                                 // per-warp ring of block addresses (2 chunks of 32)
constexpr size_t align16(size_t x) { return (x + 15) & ~(size_t)15; }
constexpr size_t kWarpScratch = kG * kD * 4 + 2 * kD * 2;    // per warp: q (2 x 128 f32), new K/V row
constexpr int kHeadCtas = 8;                                // CTAs of a kv head's cluster (one-sequence steps)
// Shared-memory layout for RING slots per warp. Three slots keep a block
// loading while a warp computes on a pair (the rate at many rows); a one-row
// step over the whole GPU gives every warp at most one pair (2 blocks), so
// two slots hold its whole share, and the smaller footprint (~163 KB instead
// of ~227 KB) lets the neighbouring one-row GEMV kernels' CTAs be resident on
// the same SM. HEAD (one sequence, one cluster per kv head): the block-count
// prefix has one row, a warp holds one piece of one (row, kv head) and so one
// record, and the first CTA of a cluster receives every CTA's record in cl.
template <int RING, bool HEAD = false>
struct DecLayout {
    static constexpr int kPref = HEAD ? 2 : kMaxBatch + 1;  // block-count prefix entries
    static constexpr int kRecK = HEAD ? 1 : 2;              // records per warp
    static constexpr size_t ring_bytes = (size_t)kDecWarps * RING * kSlotBytes;
    static constexpr size_t scratch_off = align16(ring_bytes + kDecWarps * RING * sizeof(uint64_t) +
                                                  kPref * sizeof(int) + kDecWarps * kIdRing * sizeof(uint32_t));
    static constexpr size_t rec_off = scratch_off + kDecWarps * kWarpScratch;  // [kRecK][kDecWarps] share records
    static constexpr size_t gid_off = rec_off + (size_t)kRecK * kDecWarps * attn::kPartStride * 4;  // [kRecK][kDecWarps]
    static constexpr size_t cl_off = align16(gid_off + kRecK * kDecWarps * sizeof(int));
    static constexpr size_t smem = cl_off + (HEAD ? (size_t)kHeadCtas * attn::kPartStride * 4 : 0);
    static_assert(smem <= 232448, "decode attention shared memory");
    static_assert(scratch_off % 16 == 0 && kWarpScratch % 16 == 0 && rec_off % 16 == 0 &&
                      (attn::kPartStride * 4) % 16 == 0,
                  "records are written and read as float2 / float4");
};

struct BlockCursor {
    int b, head, blk, nblk;
};

// DSMEM address of `p` (this CTA's shared memory) in cluster CTA `rank`.
__device__ __forceinline__ uint32_t map_rank(const void* p, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_addr(p)), "r"(rank));
    return r;
}
__device__ __forceinline__ void st_cluster_f32(uint32_t addr, float v) {
    asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(addr), "f"(v) : "memory");
}
__device__ __forceinline__ void st_cluster_f32x4(uint32_t addr, const float4& v) {
    asm volatile("st.shared::cluster.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "f"(v.x), "f"(v.y), "f"(v.z), "f"(v.w)
                 : "memory");
}
__device__ __forceinline__ void cluster_arrive_relaxed() {
    asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_arrive_release() {
    asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait_acquire() {
    asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// kHead: a one-sequence step launched as one cluster of kHeadCtas CTAs per
// kv head. The cluster's 64 warps split that head's blocks into equal
// contiguous shares, the CTAs' records meet in the first CTA's shared memory
// and it merges them after one cluster barrier: no global records, no
// counter, no second pass through L2.
template <int kRing, bool kHead = false>
__device__ __forceinline__ void attn_decode_body(const AttnDecodeArgs& a) {
    using Lay = DecLayout<kRing, kHead>;
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    const int warp = threadIdx.x / kWarp, lane = threadIdx.x % kWarp;
    unsigned char* ring = smem_raw + (size_t)warp * kRing * kSlotBytes;
    uint64_t* full = reinterpret_cast<uint64_t*>(smem_raw + Lay::ring_bytes) + warp * kRing;
    int* pref = reinterpret_cast<int*>(smem_raw + Lay::ring_bytes + kDecWarps * kRing * sizeof(uint64_t));
    uint32_t* kidx = reinterpret_cast<uint32_t*>(pref + Lay::kPref) + warp * kIdRing;
    float* qb = reinterpret_cast<float*>(smem_raw + Lay::scratch_off + warp * kWarpScratch);
    float* recs = reinterpret_cast<float*>(smem_raw + Lay::rec_off);  // record (warp, k) at (k * kDecWarps + warp)
    auto rec_k = [](int k) { return Lay::kRecK == 1 ? 0 : k; };        // one record per warp in a head cluster
    int (*rec_gid)[kDecWarps] = reinterpret_cast<int (*)[kDecWarps]>(smem_raw + Lay::gid_off);  // (row, kv head) of each record
    uint16_t* kvnew = reinterpret_cast<uint16_t*>(qb + kG * kD);
    constexpr unsigned kAll = 0xFFFFFFFFu;

    const int B = kHead ? 1 : a.B;
    const int max_len = a.max_blocks * kKvBlock;
    // Row-major prefix of KV block counts. Positions and block tables are
    // written before the step starts, never by the kernels this launch may
    // overlap, so they are read before griddepcontrol.wait.
    if (warp == 0) {
        int carry = 0;
        for (int base = 0; base < B; base += kWarp) {
            const int b = base + lane;
            int n = 0;
            if (b < B) {
                const int len = a.positions[b] + 1;
                if ((len < 1 || len > max_len) && a.err) atomicOr(a.err, kErrBadIndex);
                n = (min(max(len, 1), max_len) + kKvBlock - 1) / kKvBlock;
            }
            int x = n;
#pragma unroll
            for (int o = 1; o < kWarp; o <<= 1) {
                const int y = __shfl_up_sync(kAll, x, o);
                if (lane >= o) x += y;
            }
            if (b < B) pref[b + 1] = carry + x;
            carry += __shfl_sync(kAll, x, kWarp - 1);
        }
        if (lane == 0) pref[0] = 0;
    }
    if (lane == 0) {
        for (int s = 0; s < kRing; ++s) mbar_init(&full[s], 1);
        fence_barrier_init();
    }
    __syncthreads();

    const int total = pref[B] * a.n_kv;
    // CTA-major shares: the warps of a CTA hold consecutive shares, so the
    // pieces of a (row, kv head) mostly meet in one CTA and merge in shared
    // memory; only CTA-level records leave the CTA.
    int per, c_lo, c_hi;
    if constexpr (kHead) {
        // every CTA takes part in the cluster barriers, idle or not; the first
        // arrive tells the others this CTA runs before they write into it
        cluster_arrive_relaxed();
        const int head = blockIdx.x / kHeadCtas, rank = blockIdx.x % kHeadCtas;
        const int nblk = pref[1];
        per = max((nblk + kHeadCtas * kDecWarps - 1) / (kHeadCtas * kDecWarps), 1);
        c_lo = head * nblk + min(rank * kDecWarps * per, nblk);
        c_hi = min(head * nblk + nblk, c_lo + kDecWarps * per);
    } else {
        const int nwarps = gridDim.x * kDecWarps;
        per = max((total + nwarps - 1) / nwarps, kMinBlocksPerWarp);
        c_lo = blockIdx.x * kDecWarps * per;
        if (c_lo >= total) return;  // the whole CTA is idle
        c_hi = min(total, c_lo + kDecWarps * per);
    }
    const int lo = c_lo + warp * per;
    const int n = max(0, min(c_hi, lo + per) - lo);
    if (lane < Lay::kRecK) rec_gid[lane][warp] = -1;

    auto locate = [&](int f, BlockCursor& c) {
        int l = 0, h = B - 1;
        while (l < h) {
            const int mid = (l + h + 1) / 2;
            if (a.n_kv * pref[mid] <= f) l = mid;
            else h = mid - 1;
        }
        c.b = l;
        c.nblk = pref[l + 1] - pref[l];
        const int r = f - a.n_kv * pref[l];
        c.head = r / c.nblk;
        c.blk = r % c.nblk;
    };
    auto advance = [&](BlockCursor& c) {
        if (++c.blk < c.nblk) return;
        c.blk = 0;
        if (++c.head < a.n_kv) return;
        c.head = 0;
        do {
            ++c.b;
            c.nblk = c.b < B ? pref[c.b + 1] - pref[c.b] : 1;
        } while (c.nblk == 0);
    };
    // Block addresses of this warp's range, 32 at a time, one lane per block:
    // kidx = K block index in units of kBlockElems (V follows n_kv blocks
    // later), bit 31 = last block of its row.
    constexpr uint32_t kLastBit = 0x80000000u;
    auto fill_chunk = [&](int c) {
        const int j = kWarp * c + lane;
        if (j < n) {
            BlockCursor x;
            locate(lo + j, x);
            const int seq = a.seq_of[x.b];
            int id = a.block_table[(size_t)seq * a.max_blocks + x.blk];
            if (id < 0 || id >= a.n_pool_blocks) {
                if (a.err) atomicOr(a.err, kErrBadIndex);
                id = 0;  // keep the pipeline whole; the error word reports the launch
            }
            kidx[j % kIdRing] = (((uint32_t)x.head * (uint32_t)a.n_pool_blocks + (uint32_t)id) * 2u) |
                                (x.blk == x.nblk - 1 ? kLastBit : 0u);
        }
        __syncwarp();
    };
    auto block_k = [&](int j) -> const uint16_t* {
        return a.kv_layer + (size_t)(kidx[j % kIdRing] & ~kLastBit) * kBlockElems;
    };
    auto issue = [&](int j, int s) {  // lane 0: block j of the range into slot s
        const uint16_t* kp = block_k(j);
        unsigned char* dst = ring + s * kSlotBytes;
        mbar_arrive_expect_tx(&full[s], kSlotBytes);
        // K then V of the block: one contiguous 8 KB, read once per step, so
        // evict-first in L2: the next linears' prefetched weights (evict-last)
        // stay (batch 16 / 64: 3.3 / 1.6 % faster per step)
        bulk_g2s_hint(dst, kp, kSlotBytes, &full[s], l2_evict_first_policy());
    };

    // Fill the ring. The cache holds every earlier token (this step's row is
    // computed here and patched into the shared copy), so the copies start
    // before griddepcontrol.wait; only the QKV output is the previous kernel's.
    BlockCursor cc;
    locate(lo, cc);
    fill_chunk(0);
    const int first = min(kRing, n);
    if (lane == 0)
        for (int j = 0; j < first; ++j) issue(j, j);
    const attn::QkvSource src{a.qkv, (a.n_q + 2 * a.n_kv) * kD, a.n_q * kD, a.n_kv, a.q_norm, a.k_norm,
                              a.rope, a.rope_max_pos, a.eps, a.err};
    int pos = n > 0 ? a.positions[cc.b] : 0;  // the first piece's position and RoPE row, before the wait
    attn::ShareAux aux = attn::share_aux(src, pos);
    pdl_wait();
    pdl_launch_dependents();  // after the wait: the next linear's early weight loads do not delay this one's start

    const int g = lane >> 2, t = lane & 3;
    const int mi = lane >> 3, ri = lane & 7;
    const int tok_a = ri + (mi & 1) * 8;                // row this lane addresses for ldmatrix
    const int hsel = (lane >> 3) & 1;                   // head of this lane's P / O rows (lanes < 16)
    const float scale = 1.0f / sqrtf((float)kD);

    uint32_t qf[8][2];
    float acc[16][4];
    float m_run = -INFINITY, l_run = 0.0f;
    int kv_len = 0;
    bool seg_start = true, has_last = false;

    // Blocks i .. i + NB - 1 of the range, all of one (row, kv head); only the
    // last of them may be the row's last block. With NB = 2 the two blocks'
    // score and PV chains interleave and share one online-softmax update.
    auto run_blocks = [&](int i, auto nb_c) -> bool {
        constexpr int NB = decltype(nb_c)::value;
        bool ok = true;
#pragma unroll
        for (int u = 0; u < NB; ++u)
            ok = mbar_wait_bounded(&full[(i + u) % kRing], (uint32_t)(((i + u) / kRing) & 1), a.err) && ok;
        if (!__all_sync(kAll, ok)) return false;
        uint32_t kbase[NB];
        int nv[NB];
        bool patched = false;
#pragma unroll
        for (int u = 0; u < NB; ++u) {
            unsigned char* kb = ring + ((i + u) % kRing) * kSlotBytes;
            kbase[u] = smem_addr(kb);
            const int blk = cc.blk + u;
            nv[u] = min(kKvBlock, kv_len - blk * kKvBlock);  // valid tokens in this block
            if (blk == cc.nblk - 1) {
                attn::patch_new_row(const_cast<uint16_t*>(block_k(i + u)), kb, nv[u] - 1, kvnew);
                patched = true;
            }
            if (nv[u] < kKvBlock) {
                // rows past the end of the sequence: p = 0 there, but 0 * (stale NaN) is NaN
                uint4* vrow = reinterpret_cast<uint4*>(kb + kBlockBytes + nv[u] * kD * 2);
                for (int x = lane; x < (kKvBlock - nv[u]) * (kD * 2 / 16); x += kWarp) vrow[x] = make_uint4(0, 0, 0, 0);
                patched = true;
            }
        }
        __syncwarp();

        // S = K . Qcols
        float sc[NB][4], sd[NB][4];  // even / odd k-steps
#pragma unroll
        for (int u = 0; u < NB; ++u)
#pragma unroll
            for (int e = 0; e < 4; ++e) sc[u][e] = sd[u][e] = 0.0f;
#pragma unroll
        for (int ks = 0; ks < 8; ++ks) {
            const int ch = 2 * ks + (mi >> 1);
#pragma unroll
            for (int u = 0; u < NB; ++u) {
                uint32_t a0, a1, a2, a3;
                ldsm_x4(kbase[u] + tok_a * (kD * 2) + ((ch ^ ri) << 4), a0, a1, a2, a3);
                if (ks & 1) mma_bf16(sd[u], a0, a1, a2, a3, qf[ks][0], qf[ks][1]);
                else mma_bf16(sc[u], a0, a1, a2, a3, qf[ks][0], qf[ks][1]);
            }
        }
        // lanes t = 0, 1 hold head t's scores for tokens g and g + 8
        float s0[NB], s1[NB];
        float mt = -INFINITY;
#pragma unroll
        for (int u = 0; u < NB; ++u) {
#pragma unroll
            for (int e = 0; e < 4; ++e) sc[u][e] += sd[u][e];
            s0[u] = 0.0f;
            s1[u] = 0.0f;
            if (t < 2) {
                s0[u] = g < nv[u] ? (sc[u][0] + sc[u][1]) * scale : -INFINITY;
                s1[u] = g + 8 < nv[u] ? (sc[u][2] + sc[u][3]) * scale : -INFINITY;
            }
            mt = fmaxf(mt, fmaxf(s0[u], s1[u]));
        }
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
        // P as the A operand: lane (g < 4, t) holds row g = (head g/2, term g%2)
        // at tokens 2t, 2t+1 (a0) and 2t+8, 2t+9 (a2); p(h, tok) sits in lane
        // 4 (tok % 8) + h, register p0 (tok < 8) or p1.
        const int src0 = 8 * t + hsel, src1 = src0 + 4;
        uint32_t pa0[NB], pa2[NB];
#pragma unroll
        for (int u = 0; u < NB; ++u) {
            const float p0 = expf(s0[u] - m_run), p1 = expf(s1[u] - m_run);
            l_run += p0 + p1;
            const float x0 = __shfl_sync(kAll, p0, src0), x8 = __shfl_sync(kAll, p1, src0);
            const float x1 = __shfl_sync(kAll, p0, src1), x9 = __shfl_sync(kAll, p1, src1);
            pa0[u] = 0u;
            pa2[u] = 0u;
            if (lane < 16) {
                pa0[u] = pack_terms(x0, x1, g & 1);
                pa2[u] = pack_terms(x8, x9, g & 1);
            }
        }
        // O += P . V, two 8-dim tiles per transposing ldmatrix
#pragma unroll
        for (int np = 0; np < 8; ++np) {
            const int ch = 2 * np + (mi >> 1);
#pragma unroll
            for (int u = 0; u < NB; ++u) {
                uint32_t b0, b1, b2, b3;
                ldsm_x4_trans(kbase[u] + kBlockBytes + tok_a * (kD * 2) + ((ch ^ ri) << 4), b0, b1, b2, b3);
                mma_bf16(acc[2 * np], pa0[u], 0u, pa2[u], 0u, b0, b1);
                mma_bf16(acc[2 * np + 1], pa0[u], 0u, pa2[u], 0u, b2, b3);
            }
        }
        if (patched) fence_proxy_async_smem();  // generic writes above, bulk copy next
        __syncwarp();
#pragma unroll
        for (int u = 0; u < NB; ++u) {
            const int jn = i + u + kRing;  // next block for this slot
            if (jn < n && jn % kWarp == 0) fill_chunk(jn / kWarp);
            if (lane == 0 && jn < n) issue(jn, (i + u) % kRing);
        }
        return true;
    };

    for (int i = 0; i < n;) {
        if (seg_start) {
            if (i > 0) {
                pos = a.positions[cc.b];
                aux = attn::share_aux(src, pos);
            }
            kv_len = min(max(pos + 1, 1), max_len);
            const int f_last = a.n_kv * pref[cc.b] + cc.head * cc.nblk + cc.nblk - 1;
            has_last = f_last < lo + n;  // this warp also holds the row's last block
            attn::share_setup(src, aux, cc.b, cc.head, has_last, qb, kvnew, qf);
#pragma unroll
            for (int nt = 0; nt < 16; ++nt) acc[nt][0] = acc[nt][1] = acc[nt][2] = acc[nt][3] = 0.0f;
            m_run = -INFINITY;
            l_run = 0.0f;
            seg_start = false;
        }
        const int nb = (i + 1 < n && cc.blk + 1 < cc.nblk) ? 2 : 1;
        const bool ok = nb == 2 ? run_blocks(i, std::integral_constant<int, 2>{})
                                : run_blocks(i, std::integral_constant<int, 1>{});
        if (!ok) {
            // let every copy still in flight land before the warp stops (the
            // error word reports the launch; the CTA merge below still runs)
            if (lane == 0)
                for (int j = i; j < min(n, i + kRing); ++j)
                    mbar_wait_bounded(&full[j % kRing], (uint32_t)((j / kRing) & 1), nullptr);
            __syncwarp();
            break;
        }
        if (nb == 2) advance(cc);
        i += nb;
        const bool last = cc.blk == cc.nblk - 1;
        if (last || i == n) {
            // ---- end of this warp's piece of (row b, kv head): the whole row
            // goes straight to the output, a piece to this warp's record 0 (the
            // row began before this share) or 1 (it goes on past it)
            const int f0 = a.n_kv * pref[cc.b] + cc.head * cc.nblk;
            float Lh, Mh;
            attn::share_reduce(acc, l_run, m_run, Lh, Mh);
            if (f0 >= lo && f0 + cc.nblk <= lo + n) {
                attn::share_store_out(acc, Lh, a.out, cc.b, cc.head, a.n_q);
            } else {
                const int k = rec_k(f0 < lo ? 0 : 1);
                attn::share_store_record(acc, Lh, Mh, recs + (size_t)(k * kDecWarps + warp) * attn::kPartStride);
                if (lane == 0) rec_gid[k][warp] = cc.b * a.n_kv + cc.head;
            }
            seg_start = true;
        }
        advance(cc);
    }

    // ---- CTA merge: every (row, kv head) that meets this CTA's range in more
    // than one warp, or leaves it, is merged from the warps' records (warp
    // order); a row that ends in this CTA is stored, otherwise the CTA's
    // record goes to global memory and the last CTA to arrive merges them
    // (head clusters: to the cluster's first CTA, which merges them).
    __syncthreads();
    bool head_wait_done = false;  // this warp already waited on the first cluster barrier
    {
        BlockCursor gc;
        locate(c_lo, gc);
        int g0 = a.n_kv * pref[gc.b] + gc.head * gc.nblk;
        for (int gi = 0; g0 < c_hi; ++gi) {
            const int g1 = g0 + gc.nblk, gb = gc.b, gh = gc.head;
            if (gi % kDecWarps == warp) {
                const int wa = max(0, (g0 - c_lo) / per), wb = min(kDecWarps - 1, (g1 - 1 - c_lo) / per);
                const int lo_a = c_lo + wa * per;
                const bool whole = wa == wb && g0 >= lo_a && g1 <= lo_a + per;  // already stored by its warp
                if (!whole) {
                    // records of warps wa..wb, in order; shared memory, so read them directly
                    float M[attn::kG] = {-INFINITY, -INFINITY};
                    float L[attn::kG] = {0.0f, 0.0f};
                    float4 A0 = make_float4(0.0f, 0.0f, 0.0f, 0.0f), A1 = A0;
                    if constexpr (kHead) {
                        // one record per warp, in slots wa..wb: every shared-memory
                        // load is issued before any is used (same sums, same order)
                        float rm0[kDecWarps], rm1[kDecWarps], rl0[kDecWarps], rl1[kDecWarps];
                        float4 ru0[kDecWarps], ru1[kDecWarps];
                        bool live[kDecWarps];
#pragma unroll
                        for (int i = 0; i < kDecWarps; ++i) {
                            const int wi = min(wa + i, wb);
                            const float* r = recs + (size_t)wi * attn::kPartStride;
                            live[i] = wa + i <= wb;
                            rm0[i] = live[i] ? r[0] : -INFINITY;
                            rm1[i] = live[i] ? r[attn::kPartHead] : -INFINITY;
                            rl0[i] = r[1];
                            rl1[i] = r[attn::kPartHead + 1];
                            ru0[i] = *reinterpret_cast<const float4*>(r + 4 + 4 * lane);
                            ru1[i] = *reinterpret_cast<const float4*>(r + attn::kPartHead + 4 + 4 * lane);
                            live[i] = live[i] && rec_gid[0][wi] == gb * a.n_kv + gh;  // a warp that stopped early
                        }
#pragma unroll
                        for (int i = 0; i < kDecWarps; ++i) {
                            M[0] = fmaxf(M[0], rm0[i]);
                            M[1] = fmaxf(M[1], rm1[i]);
                        }
#pragma unroll
                        for (int i = 0; i < kDecWarps; ++i) {
                            if (!live[i]) continue;
                            const float c0 = rm0[i] == -INFINITY ? 0.0f : expf(rm0[i] - M[0]);
                            const float c1 = rm1[i] == -INFINITY ? 0.0f : expf(rm1[i] - M[1]);
                            L[0] += rl0[i] * c0;
                            L[1] += rl1[i] * c1;
                            const float4 u0 = ru0[i], u1 = ru1[i];
                            A0.x += u0.x * c0; A0.y += u0.y * c0; A0.z += u0.z * c0; A0.w += u0.w * c0;
                            A1.x += u1.x * c1; A1.y += u1.y * c1; A1.z += u1.z * c1; A1.w += u1.w * c1;
                        }
                    } else {
                        for (int wi = wa; wi <= wb; ++wi) {
                            const int k = (wi == wa && g0 >= c_lo + wi * per) ? 1 : 0;
                            const float* r = recs + (size_t)(k * kDecWarps + wi) * attn::kPartStride;
                            M[0] = fmaxf(M[0], r[0]);
                            M[1] = fmaxf(M[1], r[attn::kPartHead]);
                        }
                        for (int wi = wa; wi <= wb; ++wi) {
                            const int k = (wi == wa && g0 >= c_lo + wi * per) ? 1 : 0;
                            const float* r = recs + (size_t)(k * kDecWarps + wi) * attn::kPartStride;
                            if (rec_gid[k][wi] != gb * a.n_kv + gh) continue;  // a warp that stopped early
                            const float c0 = r[0] == -INFINITY ? 0.0f : expf(r[0] - M[0]);
                            const float c1 = r[attn::kPartHead] == -INFINITY ? 0.0f : expf(r[attn::kPartHead] - M[1]);
                            L[0] += r[1] * c0;
                            L[1] += r[attn::kPartHead + 1] * c1;
                            const float4 u0 = *reinterpret_cast<const float4*>(r + 4 + 4 * lane);
                            const float4 u1 = *reinterpret_cast<const float4*>(r + attn::kPartHead + 4 + 4 * lane);
                            A0.x += u0.x * c0; A0.y += u0.y * c0; A0.z += u0.z * c0; A0.w += u0.w * c0;
                            A1.x += u1.x * c1; A1.y += u1.y * c1; A1.z += u1.z * c1; A1.w += u1.w * c1;
                        }
                    }
                    if (g0 >= c_lo && g1 <= c_hi) {
                        attn::merged_store_out(L, A0, A1, a.out, gb, gh, a.n_q);
                    } else if constexpr (kHead) {
                        // this CTA's record into slot `rank` of the cluster's first CTA
                        cluster_wait_acquire();  // (the first barrier: every CTA runs)
                        const uint32_t rec = map_rank(smem_raw + Lay::cl_off, 0) +
                                             (uint32_t)((blockIdx.x % kHeadCtas) * attn::kPartStride * 4);
                        if (lane == 0) {
                            st_cluster_f32(rec, M[0]);
                            st_cluster_f32(rec + 4, L[0]);
                            st_cluster_f32(rec + attn::kPartHead * 4, M[1]);
                            st_cluster_f32(rec + attn::kPartHead * 4 + 4, L[1]);
                        }
                        st_cluster_f32x4(rec + (4 + 4 * lane) * 4, A0);
                        st_cluster_f32x4(rec + (attn::kPartHead + 4 + 4 * lane) * 4, A1);
                        head_wait_done = true;
                    } else {
                        const int span = kDecWarps * per;
                        const int fc = g0 / span, nseg = (g1 - 1) / span - fc + 1, seg = (int)blockIdx.x - fc;
                        if (seg < a.max_segs && nseg <= a.max_segs) {
                            float* base = a.partial + ((size_t)gb * a.n_kv + gh) * a.max_segs * attn::kPartStride;
                            attn::merged_store_record(M, L, A0, A1, base + (size_t)seg * attn::kPartStride);
                            attn::publish_and_merge(gb, gh, nseg, a.n_q, a.n_kv, base, a.counters, a.out);
                        } else if (lane == 0 && a.err) {
                            atomicOr(a.err, kErrBadIndex);
                        }
                    }
                }
            }
            g0 = g1;
            if (++gc.head == a.n_kv) {
                gc.head = 0;
                ++gc.b;
            }
            gc.nblk = gc.b < B ? pref[gc.b + 1] - pref[gc.b] : 1;
        }
    }
    if constexpr (kHead) {
        if (!head_wait_done) cluster_wait_acquire();
        cluster_arrive_release();  // this CTA's record is in the first CTA
        cluster_wait_acquire();
        const int nblk = pref[1], span = kDecWarps * per;
        const int nseg = (nblk + span - 1) / span;  // CTAs with blocks; their records, in rank order
        if (blockIdx.x % kHeadCtas == 0 && nseg > 1 && warp == 0) {
            float M[kG], L[kG];
            float4 A0, A1;
            attn::merge_records<false, kHeadCtas>(reinterpret_cast<const float*>(smem_raw + Lay::cl_off), nseg, M, L,
                                                  A0, A1);
            attn::merged_store_out(L, A0, A1, a.out, 0, blockIdx.x / kHeadCtas, a.n_q);
        }
    }
}

// The decode kernels: three ring slots for many rows (the register file is
// the kernel's own); for a one-row step over the whole GPU two slots and at
// most 192 registers per thread, so a one-row GEMV CTA (256 threads, <= 64
// registers, <= 48 KB of shared memory) fits on the same SM beside it; a
// one-row step in head clusters (64 SMs, the rest left to the next GEMV) has
// three slots, so a warp's blocks are all requested before the wait while
// shares are at most 3 blocks (contexts up to 3072).
__global__ void __launch_bounds__(kDecThreads, 1) attn_decode_kernel(AttnDecodeArgs a) { attn_decode_body<3>(a); }
__global__ void __maxnreg__(192) attn_decode_row_kernel(AttnDecodeArgs a) { attn_decode_body<2>(a); }
__global__ void __launch_bounds__(kDecThreads, 1) attn_decode_head_kernel(AttnDecodeArgs a) { attn_decode_body<3, true>(a); }

// ------------------------------------------------------------ prefill
//
// Causal GQA prefill attention on the tensor cores (mma.sync m16n8k16, bf16
// in, f32 accumulate), flash-attention style. CTA = (32-query tile, kv head),
// 8 warps: warp w takes query head 2 kvh + (w >> 2), rows 16 ((w >> 1) & 1)
// of the tile, and the key half (w & 1) of every 64-key tile, so both heads
// share each staged K/V tile and a tile's MMAs are spread over twice the
// warps; the two halves' softmax states merge once at the end. f32 q is
// split into two bf16 terms (x = hi + lo to 2^-18 relative) and each product
// is taken as q_hi k_hi + q_hi k_lo + q_lo k_hi (likewise P V), so S and P V
// carry f32-grade accuracy; when K and V are exact bf16 (the cache's
// values) their lo terms are zero and skipped. K and V arrive from qkv_post
// already split into bf16 planes, and each 64-key tile is copied with
// cp.async into a double buffer (16-byte chunks of each row XOR-swizzled by
// row for conflict-free ldmatrix) while the previous tile is computed. Keys
// after the query or past T are masked (kv_len == q_len == T, ops.zig:322).
constexpr int PQ = 32, PK = 64, PTHREADS = 256;
constexpr int kTileBytes = PK * kD * 2;  // one bf16 plane of a K or V tile
constexpr size_t kPrefillSmem = (size_t)2 * 4 * kTileBytes;  // two stages of K hi, K lo, V hi, V lo

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool valid) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(valid ? 16 : 0)
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_1() { asm volatile("cp.async.wait_group 1;" ::: "memory"); }

__global__ void __launch_bounds__(PTHREADS, 1) attn_prefill_kernel(AttnPrefillArgs a) {
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    constexpr unsigned kAll = 0xFFFFFFFFu;
    pdl_wait();
    pdl_launch_dependents();
    const int qt = gridDim.x - 1 - blockIdx.x, kvh = blockIdx.y;  // longest (causal) tiles first
    const int T = a.T;
    const int q0 = qt * PQ;
    const int warp = threadIdx.x / kWarp, lane = threadIdx.x % kWarp;
    const int hs = warp >> 2, kh = warp & 1;
    const int h = kvh * kG + hs;                 // query head of this warp
    const int r0 = q0 + ((warp >> 1) & 1) * 16;  // first query row of this warp
    const int g = lane >> 2, t = lane & 3;
    const int mi = lane >> 3, ri = lane & 7;
    const float scale = 1.0f / sqrtf((float)kD);
    const bool lo = a.lo_terms != 0;
    const int nplanes = lo ? 4 : 2;  // staged planes: K hi, (K lo), V hi, (V lo)
    const int stage_bytes = nplanes * kTileBytes;
    const size_t plane = (size_t)a.n_kv * T * kD;

    // copy the 64-key tile starting at k0 into stage s (keys past T as zeros)
    auto issue = [&](int k0, int s) {
        const uint32_t base = smem_addr(smem_raw) + (uint32_t)(s * stage_bytes);
        const int chunks = nplanes * PK * (kD / 8);
        for (int i = threadIdx.x; i < chunks; i += PTHREADS) {
            const int c = i % (kD / 8), r = (i / (kD / 8)) % PK, sp = i / (PK * (kD / 8));
            const int p = lo ? sp : 2 * sp;  // source plane
            const bool valid = k0 + r < T;
            const uint16_t* src = a.kv_planes + (size_t)p * plane + ((size_t)kvh * T + (valid ? k0 + r : 0)) * kD + 8 * c;
            cp_async16(base + (uint32_t)(sp * kTileBytes + r * kD * 2 + ((c ^ (r & 7)) << 4)), src, valid);
        }
    };

    // Q fragments (A operand, 16 rows x 16 dims per k-step), hi and lo terms
    uint32_t qa[8][4], qb[8][4];
    {
        const float* qh = a.q + (size_t)h * T * kD;
        const int ra = min(r0 + g, T - 1), rb = min(r0 + g + 8, T - 1);
#pragma unroll
        for (int ks = 0; ks < 8; ++ks) {
            const int d0 = 16 * ks + 2 * t;
            const float2 x0 = *reinterpret_cast<const float2*>(qh + (size_t)ra * kD + d0);
            const float2 x1 = *reinterpret_cast<const float2*>(qh + (size_t)rb * kD + d0);
            const float2 x2 = *reinterpret_cast<const float2*>(qh + (size_t)ra * kD + d0 + 8);
            const float2 x3 = *reinterpret_cast<const float2*>(qh + (size_t)rb * kD + d0 + 8);
            qa[ks][0] = attn::pack_terms(x0.x, x0.y, false);
            qa[ks][1] = attn::pack_terms(x1.x, x1.y, false);
            qa[ks][2] = attn::pack_terms(x2.x, x2.y, false);
            qa[ks][3] = attn::pack_terms(x3.x, x3.y, false);
            qb[ks][0] = attn::pack_terms(x0.x, x0.y, true);
            qb[ks][1] = attn::pack_terms(x1.x, x1.y, true);
            qb[ks][2] = attn::pack_terms(x2.x, x2.y, true);
            qb[ks][3] = attn::pack_terms(x3.x, x3.y, true);
        }
    }
    float o[16][4];
#pragma unroll
    for (int nt = 0; nt < 16; ++nt) o[nt][0] = o[nt][1] = o[nt][2] = o[nt][3] = 0.0f;
    float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.0f, l1 = 0.0f;  // rows g and g + 8

    const int last_key = min(q0 + PQ, T);  // keys [0, last_key)
    const int ntiles = (last_key + PK - 1) / PK;
    issue(0, 0);
    cp_async_commit();
    for (int it = 0; it < ntiles; ++it) {
        const int k0 = it * PK;
        if (it + 1 < ntiles) issue(k0 + PK, (it + 1) & 1);
        cp_async_commit();
        cp_async_wait_1();  // this tile's group is complete
        __syncthreads();
        const int kb = k0 + 32 * kh;  // first key of this warp's half
        if (kb <= r0 + 15) {
            const uint32_t st = smem_addr(smem_raw) + (uint32_t)((it & 1) * stage_bytes);
            const uint32_t khi_s = st, klo_s = st + kTileBytes;
            const uint32_t vhi_s = st + (lo ? 2 : 1) * kTileBytes, vlo_s = st + 3 * kTileBytes;
            // S = Q K^T over this warp's 32 keys: 4 n-tiles of 8 keys; ldmatrix.x4 yields two
            float sacc[4][4];
#pragma unroll
            for (int j = 0; j < 4; ++j) sacc[j][0] = sacc[j][1] = sacc[j][2] = sacc[j][3] = 0.0f;
#pragma unroll
            for (int ks = 0; ks < 8; ++ks) {
#pragma unroll
                for (int jp = 0; jp < 2; ++jp) {
                    // matrices: (keys 16jp + 0..7, dims 16ks..+7), (same keys, +8), (keys +8, dims), (keys +8, +8)
                    const int key = 32 * kh + 16 * jp + ri + ((mi >> 1) << 3);
                    const int ch = 2 * ks + (mi & 1);
                    const uint32_t off = (uint32_t)(key * kD * 2 + ((ch ^ (key & 7)) << 4));
                    uint32_t h0, h1, h2, h3;
                    attn::ldsm_x4(khi_s + off, h0, h1, h2, h3);
                    attn::mma_bf16(sacc[2 * jp], qa[ks][0], qa[ks][1], qa[ks][2], qa[ks][3], h0, h1);
                    attn::mma_bf16(sacc[2 * jp], qb[ks][0], qb[ks][1], qb[ks][2], qb[ks][3], h0, h1);
                    attn::mma_bf16(sacc[2 * jp + 1], qa[ks][0], qa[ks][1], qa[ks][2], qa[ks][3], h2, h3);
                    attn::mma_bf16(sacc[2 * jp + 1], qb[ks][0], qb[ks][1], qb[ks][2], qb[ks][3], h2, h3);
                    if (lo) {
                        uint32_t l0b, l1b, l2b, l3b;
                        attn::ldsm_x4(klo_s + off, l0b, l1b, l2b, l3b);
                        attn::mma_bf16(sacc[2 * jp], qa[ks][0], qa[ks][1], qa[ks][2], qa[ks][3], l0b, l1b);
                        attn::mma_bf16(sacc[2 * jp + 1], qa[ks][0], qa[ks][1], qa[ks][2], qa[ks][3], l2b, l3b);
                    }
                }
            }
            // scale, causal mask, online softmax (rows g and g + 8 of the warp's 16)
            const int qa_row = r0 + g, qb_row = r0 + g + 8;
            float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int key = kb + 8 * j + 2 * t;
                sacc[j][0] = (key <= qa_row && key < T) ? sacc[j][0] * scale : -INFINITY;
                sacc[j][1] = (key + 1 <= qa_row && key + 1 < T) ? sacc[j][1] * scale : -INFINITY;
                sacc[j][2] = (key <= qb_row && key < T) ? sacc[j][2] * scale : -INFINITY;
                sacc[j][3] = (key + 1 <= qb_row && key + 1 < T) ? sacc[j][3] * scale : -INFINITY;
                mx0 = fmaxf(mx0, fmaxf(sacc[j][0], sacc[j][1]));
                mx1 = fmaxf(mx1, fmaxf(sacc[j][2], sacc[j][3]));
            }
            mx0 = fmaxf(mx0, __shfl_xor_sync(kAll, mx0, 1));
            mx0 = fmaxf(mx0, __shfl_xor_sync(kAll, mx0, 2));
            mx1 = fmaxf(mx1, __shfl_xor_sync(kAll, mx1, 1));
            mx1 = fmaxf(mx1, __shfl_xor_sync(kAll, mx1, 2));
            const float n0 = fmaxf(m0, mx0), n1 = fmaxf(m1, mx1);
            // a row with no visible key yet keeps max -inf; its terms stay 0
            const float c0 = n0 == -INFINITY ? 1.0f : expf(m0 - n0);
            const float c1 = n1 == -INFINITY ? 1.0f : expf(m1 - n1);
            m0 = n0;
            m1 = n1;
            l0 *= c0;
            l1 *= c1;
#pragma unroll
            for (int nt = 0; nt < 16; ++nt) {
                o[nt][0] *= c0;
                o[nt][1] *= c0;
                o[nt][2] *= c1;
                o[nt][3] *= c1;
            }
            uint32_t pa[2][4], pb[2][4];  // P as the A operand of 2 k-steps of 16 keys, hi and lo
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const float p0 = n0 == -INFINITY ? 0.0f : expf(sacc[j][0] - n0);
                const float p1 = n0 == -INFINITY ? 0.0f : expf(sacc[j][1] - n0);
                const float p2 = n1 == -INFINITY ? 0.0f : expf(sacc[j][2] - n1);
                const float p3 = n1 == -INFINITY ? 0.0f : expf(sacc[j][3] - n1);
                l0 += p0 + p1;
                l1 += p2 + p3;
                // n-tile j = keys 8j..: k-step j / 2, registers (0, 1) for even j, (2, 3) for odd j
                const int kk = j >> 1, hi2 = (j & 1) * 2;
                pa[kk][hi2 + 0] = attn::pack_terms(p0, p1, false);
                pa[kk][hi2 + 1] = attn::pack_terms(p2, p3, false);
                pb[kk][hi2 + 0] = attn::pack_terms(p0, p1, true);
                pb[kk][hi2 + 1] = attn::pack_terms(p2, p3, true);
            }
            // O += P V: 2 k-steps of 16 keys x 16 n-tiles of 8 dims (ldmatrix.trans: two n-tiles each)
#pragma unroll
            for (int kk = 0; kk < 2; ++kk) {
#pragma unroll
                for (int np = 0; np < 8; ++np) {
                    const int key = 32 * kh + 16 * kk + ri + ((mi & 1) << 3);
                    const int ch = 2 * np + (mi >> 1);
                    const uint32_t off = (uint32_t)(key * kD * 2 + ((ch ^ (key & 7)) << 4));
                    uint32_t h0, h1, h2, h3;
                    attn::ldsm_x4_trans(vhi_s + off, h0, h1, h2, h3);
                    attn::mma_bf16(o[2 * np], pa[kk][0], pa[kk][1], pa[kk][2], pa[kk][3], h0, h1);
                    attn::mma_bf16(o[2 * np], pb[kk][0], pb[kk][1], pb[kk][2], pb[kk][3], h0, h1);
                    attn::mma_bf16(o[2 * np + 1], pa[kk][0], pa[kk][1], pa[kk][2], pa[kk][3], h2, h3);
                    attn::mma_bf16(o[2 * np + 1], pb[kk][0], pb[kk][1], pb[kk][2], pb[kk][3], h2, h3);
                    if (lo) {
                        uint32_t l0b, l1b, l2b, l3b;
                        attn::ldsm_x4_trans(vlo_s + off, l0b, l1b, l2b, l3b);
                        attn::mma_bf16(o[2 * np], pa[kk][0], pa[kk][1], pa[kk][2], pa[kk][3], l0b, l1b);
                        attn::mma_bf16(o[2 * np + 1], pa[kk][0], pa[kk][1], pa[kk][2], pa[kk][3], l2b, l3b);
                    }
                }
            }
        }
        __syncthreads();  // the stage is rewritten by the copy issued in the next iteration
    }

    asm volatile("cp.async.wait_group 0;" ::: "memory");  // (only empty groups can remain)
    // merge the two key halves of each (head, row group): half 1 hands its
    // state (quad-summed l, m, o in fragment order) to half 0 through shared
    // memory (the staging buffers are free now)
    l0 += __shfl_xor_sync(kAll, l0, 1);
    l0 += __shfl_xor_sync(kAll, l0, 2);
    l1 += __shfl_xor_sync(kAll, l1, 1);
    l1 += __shfl_xor_sync(kAll, l1, 2);
    float* xch = reinterpret_cast<float*>(smem_raw) + (size_t)(warp >> 1) * kWarp * 68 + lane * 68;
    if (kh == 1) {
#pragma unroll
        for (int nt = 0; nt < 16; ++nt)
            *reinterpret_cast<float4*>(xch + 4 * nt) = make_float4(o[nt][0], o[nt][1], o[nt][2], o[nt][3]);
        *reinterpret_cast<float4*>(xch + 64) = make_float4(m0, m1, l0, l1);
    }
    __syncthreads();
    if (kh == 1) return;
    const float4 ml = *reinterpret_cast<const float4*>(xch + 64);
    const float M0 = fmaxf(m0, ml.x), M1 = fmaxf(m1, ml.y);
    const float ca0 = m0 == -INFINITY ? 0.0f : expf(m0 - M0), cb0 = ml.x == -INFINITY ? 0.0f : expf(ml.x - M0);
    const float ca1 = m1 == -INFINITY ? 0.0f : expf(m1 - M1), cb1 = ml.y == -INFINITY ? 0.0f : expf(ml.y - M1);
    const float L0 = l0 * ca0 + ml.z * cb0, L1 = l1 * ca1 + ml.w * cb1;
    const float i0 = L0 > 0.0f ? 1.0f / L0 : 0.0f, i1 = L1 > 0.0f ? 1.0f / L1 : 0.0f;
    // normalise and store rows g, g + 8: out [T][n_q][d]
    const int ra = r0 + g, rb = r0 + g + 8;
    const size_t K = (size_t)a.n_q * kD, out_plane = (size_t)a.t_pad * K;
    // the plane kernel's bf16 hi / lo split of two consecutive outputs
    auto store_planes = [&](int r, int d, float v0, float v1) {
        const uint16_t h0 = f32_to_bf16_rne(v0), h1 = f32_to_bf16_rne(v1);
        const uint16_t l0 = f32_to_bf16_rne(__fsub_rn(v0, __uint_as_float((uint32_t)h0 << 16)));
        const uint16_t l1 = f32_to_bf16_rne(__fsub_rn(v1, __uint_as_float((uint32_t)h1 << 16)));
        uint16_t* p = a.planes + (size_t)r * K + (size_t)h * kD + d;
        *reinterpret_cast<uint32_t*>(p) = (uint32_t)h0 | ((uint32_t)h1 << 16);
        *reinterpret_cast<uint32_t*>(p + out_plane) = (uint32_t)l0 | ((uint32_t)l1 << 16);
    };
#pragma unroll
    for (int nt = 0; nt < 16; ++nt) {
        const float4 po = *reinterpret_cast<const float4*>(xch + 4 * nt);
        const int d = 8 * nt + 2 * t;
        if (ra < T) {
            const float v0 = (o[nt][0] * ca0 + po.x * cb0) * i0, v1 = (o[nt][1] * ca0 + po.y * cb0) * i0;
            *reinterpret_cast<float2*>(a.out + ((size_t)ra * a.n_q + h) * kD + d) = make_float2(v0, v1);
            if (a.planes) store_planes(ra, d, v0, v1);
        }
        if (rb < T) {
            const float v0 = (o[nt][2] * ca1 + po.z * cb1) * i1, v1 = (o[nt][3] * ca1 + po.w * cb1) * i1;
            *reinterpret_cast<float2*>(a.out + ((size_t)rb * a.n_q + h) * kD + d) = make_float2(v0, v1);
            if (a.planes) store_planes(rb, d, v0, v1);
        }
    }
}

}  // namespace

void prepare_attn_kernels() {
    configure_kernel((const void*)attn_decode_kernel, DecLayout<3>::smem);
    configure_kernel((const void*)attn_decode_row_kernel, DecLayout<2>::smem);
    configure_kernel((const void*)attn_decode_head_kernel, DecLayout<3, true>::smem);
    configure_kernel((const void*)attn_prefill_kernel, kPrefillSmem);
}

void launch_attn_decode(const AttnDecodeArgs& a, cudaStream_t st) {
    if (a.B == 1 && a.head_clusters) {
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(a.n_kv * kHeadCtas);
        cfg.blockDim = dim3(kDecThreads);
        cfg.dynamicSmemBytes = DecLayout<3, true>::smem;
        cfg.stream = st;
        cudaLaunchAttribute attr[2];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = kHeadCtas;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[1].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 2;
        cudaLaunchKernelEx(&cfg, attn_decode_head_kernel, a);
        return;
    }
    if (a.B == 1) launch_pdl(attn_decode_row_kernel, device_sm_count(), kDecThreads, DecLayout<2>::smem, st, a);
    else launch_pdl(attn_decode_kernel, device_sm_count(), kDecThreads, DecLayout<3>::smem, st, a);
}

void launch_attn_prefill(const AttnPrefillArgs& a, cudaStream_t st) {
    dim3 grid((a.T + PQ - 1) / PQ, a.n_kv);
    const size_t smem = a.lo_terms ? kPrefillSmem : kPrefillSmem / 2;
    launch_pdl(attn_prefill_kernel, grid, PTHREADS, smem, st, a);
}

}  // namespace zc
