// Pieces shared by the decode attention kernel (attn.cu) and the persistent
// decode kernel (decode_flow.cu): tensor-core fragment helpers and the
// end-of-share flush with its log-sum-exp merge (attentionInto,
// src/backends/cpu/ops.zig:285-354, split over KV blocks).
#pragma once

#include "common.cuh"

namespace zc {
namespace attn {

constexpr int kD = 128, kG = 2;                  // head dim, query heads per kv head
constexpr int kBlockElems = kKvBlock * kD;       // 2048 bf16 = 4 KB (K or V of one block and head)
constexpr int kBlockBytes = kBlockElems * 2;
constexpr int kSlotBytes = 2 * kBlockBytes;      // K then V
// Partial result of one share, per query head: [m, l, -, -, acc[128]] so the
// accumulator is 16-byte aligned; a share holds kG of them.
constexpr int kPartHead = kD + 4;
constexpr int kPartStride = kG * kPartHead;
static_assert(kD == 128 && kKvBlock == 16, "the fragment mapping assumes 16-token blocks of 128 dims");

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr)
                 : "memory");
}
__device__ __forceinline__ void ldsm_x4_trans(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                              uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr)
                 : "memory");
}
// D = A . B + D for one m16n8k16 tile; A rows 8..15 are zero when a1 = a3 = 0.
__device__ __forceinline__ void mma_bf16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
// Two f32 -> packed bf16x2 (x0 in the low half), round to nearest even.
__device__ __forceinline__ uint32_t cvt_bf16x2(float x0, float x1) {
    uint32_t r;
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(x1), "f"(x0));
    return r;
}
// One bf16 term of (x0, x1): the rounded values (lo_part = 0) or the rounded
// remainders x - bf16(x) (lo_part = 1); hi + lo carries x to 2^-18 relative.
__device__ __forceinline__ uint32_t pack_terms(float x0, float x1, bool lo_part) {
    const uint32_t h = cvt_bf16x2(x0, x1);
    if (!lo_part) return h;
    return cvt_bf16x2(x0 - __uint_as_float(h << 16), x1 - __uint_as_float(h & 0xFFFF0000u));
}

// Where the fused decode attention reads this step's q, k and v: the raw
// fused-QKV linear output [B][qkv_rows] (q heads, then k heads, then v heads)
// with the per-head RMSNorm weights and the RoPE table.
struct QkvSource {
    const float* qkv;
    int qkv_rows, qd, n_kv;
    const float* q_norm;
    const float* k_norm;
    const float2* rope;  // [rope_max_pos][64] (cos, sin)
    int rope_max_pos;
    float eps;
    uint32_t* err;
};

// Set-up of a warp's share of (row b, kv head) at position pos (qkv_post's
// math, qwen_block.zig:191-205): the two query heads, RMSNorm(q_norm) +
// split-half RoPE, become the tensor-core B fragments qf; when the share
// holds the row's last block (has_last), this step's key (RMSNorm(k_norm) +
// RoPE) and value, rounded to bf16, go to kvnew[0..127] / kvnew[128..255].
// Every load is issued before any is used. qb: 2 x 128 f32 of shared memory.
// The norm weights and the RoPE row of pos (ShareAux) come from buffers no
// kernel of the step writes, so they may be loaded before griddepcontrol.wait.
struct ShareAux {
    float qn[4], kn[4];
    float2 c2[2];
    bool rope_ok;
};
__device__ __forceinline__ ShareAux share_aux(const QkvSource& src, int pos) {
    const int lane = threadIdx.x % kWarp;
    ShareAux x;
    x.rope_ok = pos >= 0 && pos < src.rope_max_pos;
    const float2* cs = src.rope + (size_t)(x.rope_ok ? pos : 0) * (kD / 2);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        x.qn[j] = __ldg(src.q_norm + lane + 32 * j);
        x.kn[j] = __ldg(src.k_norm + lane + 32 * j);
    }
#pragma unroll
    for (int j = 0; j < 2; ++j) x.c2[j] = __ldg(cs + lane + 32 * j);
    return x;
}
__device__ __forceinline__ void share_setup(const QkvSource& src, const ShareAux& aux, int b, int head,
                                            bool has_last, float* qb, uint16_t* kvnew, uint32_t (&qf)[8][2]) {
    const int lane = threadIdx.x % kWarp;
    const int g = lane >> 2, t = lane & 3;
    const float* qsrc = src.qkv + (size_t)b * src.qkv_rows + (size_t)(head * kG) * kD;
    const float* ksrc = src.qkv + (size_t)b * src.qkv_rows + src.qd + (size_t)head * kD;
    const float* vsrc = ksrc + (size_t)src.n_kv * kD;
    const bool rope_ok = aux.rope_ok;
    const float(&qn)[4] = aux.qn;
    const float(&kn)[4] = aux.kn;
    const float2(&c2)[2] = aux.c2;
    float qv[kG][4], kr[4], vr[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
#pragma unroll
        for (int hh = 0; hh < kG; ++hh) qv[hh][j] = __ldcg(qsrc + hh * kD + lane + 32 * j);
        kr[j] = has_last ? __ldcg(ksrc + lane + 32 * j) : 0.0f;
        vr[j] = has_last ? __ldcg(vsrc + lane + 32 * j) : 0.0f;
    }
    auto norm_rope = [&](float (&v)[4], const float (&w)[4]) {
        float ss = 0.0f;
#pragma unroll
        for (int j = 0; j < 4; ++j) ss += v[j] * v[j];
        ss = warp_sum(ss);
        const float inv = 1.0f / sqrtf(ss / (float)kD + src.eps);
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
    if (!rope_ok && lane == 0 && src.err) atomicOr(src.err, kErrBadIndex);
    __syncwarp();
    if (g < 4) {
        const float* qp = qb + (g >> 1) * kD;
        const bool lo_part = g & 1;
#pragma unroll
        for (int ks = 0; ks < 8; ++ks) {
            qf[ks][0] = pack_terms(qp[16 * ks + 2 * t], qp[16 * ks + 2 * t + 1], lo_part);
            qf[ks][1] = pack_terms(qp[16 * ks + 2 * t + 8], qp[16 * ks + 2 * t + 9], lo_part);
        }
    } else {
#pragma unroll
        for (int ks = 0; ks < 8; ++ks) qf[ks][0] = qf[ks][1] = 0u;
    }
}

// This step's K/V row (token r of its block) into the cache block (kg: K of
// this head, its V right after) and into the shared copy of the block.
__device__ __forceinline__ void patch_new_row(uint16_t* kg, unsigned char* slot, int r, const uint16_t* kvnew) {
    const int lane = threadIdx.x % kWarp;
    uint16_t* vg = kg + kBlockElems;
    uint16_t* kl = reinterpret_cast<uint16_t*>(slot);
    uint16_t* vl = reinterpret_cast<uint16_t*>(slot + kBlockBytes);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const int e = kv_swizzle(r, lane + 32 * j);
        const uint16_t kbits = kvnew[lane + 32 * j], vbits = kvnew[kD + lane + 32 * j];
        kg[e] = kbits;
        vg[e] = vbits;
        kl[e] = kbits;
        vl[e] = vbits;
    }
}

// ---- end of a warp's share: the fragment-layout state of the block loop
// (lanes (g < 4, t) hold O rows g = (head g/2, term g%2) at dims 8 nt + 2t
// (+1); lanes with t < 2 hold query head t's running max and partial sums)
// folded into a record [head][m, l, -, -, acc[128]] or a normalised output.

// Sum l over the warp, combine the hi and lo rows of acc in place; returns
// this lane's head (hsel) total l and max m.
__device__ __forceinline__ void share_reduce(float (&acc)[16][4], float l_run, float m_run, float& Lh, float& Mh) {
    constexpr unsigned kAll = 0xFFFFFFFFu;
    const int lane = threadIdx.x % kWarp;
    const int hsel = (lane >> 3) & 1;
    float L = l_run;
    L += __shfl_xor_sync(kAll, L, 4);
    L += __shfl_xor_sync(kAll, L, 8);
    L += __shfl_xor_sync(kAll, L, 16);
    Lh = __shfl_sync(kAll, L, hsel);
    Mh = __shfl_sync(kAll, m_run, hsel);
#pragma unroll
    for (int nt = 0; nt < 16; ++nt) {
        acc[nt][0] += __shfl_xor_sync(kAll, acc[nt][0], 4);
        acc[nt][1] += __shfl_xor_sync(kAll, acc[nt][1], 4);
    }
}
__device__ __forceinline__ bool share_writer() {
    const int lane = threadIdx.x % kWarp;
    return lane < 16 && ((lane >> 2) & 1) == 0;  // lanes 0-3: head 0, 8-11: head 1
}
// o = acc / l of both query heads of (b, kv head) into out [B][n_q][d]
__device__ __forceinline__ void share_store_out(const float (&acc)[16][4], float Lh, float* out, int b, int head,
                                                int n_q) {
    const int lane = threadIdx.x % kWarp;
    const int t = lane & 3, hsel = (lane >> 3) & 1;
    if (!share_writer()) return;
    float* op = out + ((size_t)b * n_q + head * kG + hsel) * kD + 2 * t;
    const float inv = 1.0f / Lh;
#pragma unroll
    for (int nt = 0; nt < 16; ++nt)
        *reinterpret_cast<float2*>(op + nt * 8) = make_float2(acc[nt][0] * inv, acc[nt][1] * inv);
}
// the partial (m, l, acc) of both heads into a record (global or shared)
__device__ __forceinline__ void share_store_record(const float (&acc)[16][4], float Lh, float Mh, float* rec) {
    const int lane = threadIdx.x % kWarp;
    const int t = lane & 3, hsel = (lane >> 3) & 1;
    if (!share_writer()) return;
    float* pg = rec + hsel * kPartHead;
    if (t == 0) {
        pg[0] = Mh;
        pg[1] = Lh;
    }
#pragma unroll
    for (int nt = 0; nt < 16; ++nt)
        *reinterpret_cast<float2*>(pg + 4 + nt * 8 + 2 * t) = make_float2(acc[nt][0], acc[nt][1]);
}

// Merge `count` records (base + j * kPartStride, j in order) in the
// log-sum-exp sense: m = max m_j, l = sum l_j e^(m_j - m), acc = sum acc_j
// e^(m_j - m). Lane owns dims 4 lane .. 4 lane + 3 of both heads (A0, A1);
// M and L of both heads are returned in every lane. kGlobal: records written
// by other CTAs (read through L2), else shared memory. The (m, l) of the
// first 32 records and the accumulators of the first kBatch are all requested
// before any of them is used, so up to kBatch records cost one round trip.
template <bool kGlobal, int kBatch>
__device__ __forceinline__ void merge_records(const float* base, int count, float (&M)[kG], float (&L)[kG],
                                              float4& A0, float4& A1) {
    constexpr unsigned kAll = 0xFFFFFFFFu;
    const int lane = threadIdx.x % kWarp;
    auto ld = [](const float* p) { return kGlobal ? __ldcg(p) : *p; };
    auto ld4 = [](const float* p) {
        return kGlobal ? __ldcg(reinterpret_cast<const float4*>(p)) : *reinterpret_cast<const float4*>(p);
    };
    const float* pa = base + 4 + 4 * lane;
    float m0 = -INFINITY, l0 = 0.0f, m1 = -INFINITY, l1 = 0.0f;  // record s0 + lane of the current chunk
    auto load_ml = [&](int s0) {
        if (s0 + lane < count) {
            const float* ps = base + (size_t)(s0 + lane) * kPartStride;
            m0 = ld(ps);
            l0 = ld(ps + 1);
            m1 = ld(ps + kPartHead);
            l1 = ld(ps + kPartHead + 1);
        }
    };
    float4 u0[kBatch], u1[kBatch];
    auto load_batch = [&](int s0, int j0, int cnt) {
#pragma unroll
        for (int j = 0; j < kBatch; ++j) {
            const int jj = s0 + max(0, min(j0 + j, cnt - 1));
            u0[j] = ld4(pa + (size_t)jj * kPartStride);
            u1[j] = ld4(pa + (size_t)jj * kPartStride + kPartHead);
        }
    };
    load_ml(0);
    load_batch(0, 0, min(kWarp, count));
    float M0 = fmaxf(-INFINITY, m0), M1 = fmaxf(-INFINITY, m1);
    for (int s = lane + kWarp; s < count; s += kWarp) {
        M0 = fmaxf(M0, ld(base + (size_t)s * kPartStride));
        M1 = fmaxf(M1, ld(base + (size_t)s * kPartStride + kPartHead));
    }
    M0 = warp_max(M0);
    M1 = warp_max(M1);
    float L0 = 0.0f, L1 = 0.0f;
    A0 = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    A1 = A0;
    for (int s0 = 0; s0 < count; s0 += kWarp) {
        if (s0 > 0) load_ml(s0);
        float c0 = 0.0f, c1 = 0.0f;
        if (s0 + lane < count) {
            c0 = m0 == -INFINITY ? 0.0f : expf(m0 - M0);
            c1 = m1 == -INFINITY ? 0.0f : expf(m1 - M1);
            L0 += l0 * c0;
            L1 += l1 * c1;
        }
        const int cnt = min(kWarp, count - s0);
        for (int j0 = 0; j0 < cnt; j0 += kBatch) {
            if (s0 > 0 || j0 > 0) load_batch(s0, j0, cnt);  // kBatch records in flight before any is used
#pragma unroll
            for (int j = 0; j < kBatch; ++j) {
                const bool live = j0 + j < cnt;
                const float cj0 = __shfl_sync(kAll, c0, (j0 + j) & (kWarp - 1));
                const float cj1 = __shfl_sync(kAll, c1, (j0 + j) & (kWarp - 1));
                if (live) {
                    A0.x += u0[j].x * cj0; A0.y += u0[j].y * cj0; A0.z += u0[j].z * cj0; A0.w += u0[j].w * cj0;
                    A1.x += u1[j].x * cj1; A1.y += u1[j].y * cj1; A1.z += u1[j].z * cj1; A1.w += u1[j].w * cj1;
                }
            }
        }
    }
    M[0] = M0;
    M[1] = M1;
    L[0] = warp_sum(L0);
    L[1] = warp_sum(L1);
}
// A merged result (lane layout of merge_records) as output or as a record.
__device__ __forceinline__ void merged_store_out(const float (&L)[kG], const float4& A0, const float4& A1,
                                                 float* out, int b, int head, int n_q) {
    const int lane = threadIdx.x % kWarp;
    const float i0 = 1.0f / L[0], i1 = 1.0f / L[1];
    float* op = out + ((size_t)b * n_q + head * kG) * kD + 4 * lane;
    *reinterpret_cast<float4*>(op) = make_float4(A0.x * i0, A0.y * i0, A0.z * i0, A0.w * i0);
    *reinterpret_cast<float4*>(op + kD) = make_float4(A1.x * i1, A1.y * i1, A1.z * i1, A1.w * i1);
}
__device__ __forceinline__ void merged_store_record(const float (&M)[kG], const float (&L)[kG], const float4& A0,
                                                    const float4& A1, float* rec) {
    const int lane = threadIdx.x % kWarp;
    if (lane == 0) {
        rec[0] = M[0];
        rec[1] = L[0];
        rec[kPartHead] = M[1];
        rec[kPartHead + 1] = L[1];
    }
    *reinterpret_cast<float4*>(rec + 4 + 4 * lane) = A0;
    *reinterpret_cast<float4*>(rec + kPartHead + 4 + 4 * lane) = A1;
}

// Segment `seg` of `nseg` of (batch row b, kv head) is published in record
// `rec` (global); the last segment to arrive (atomic counter, no spin)
// merges all of them in segment order and stores the output.
template <int kBatch = 8>
__device__ __forceinline__ void publish_and_merge(int b, int head, int nseg, int n_q, int n_kv, const float* base,
                                                  unsigned* counters, float* out) {
    constexpr unsigned kAll = 0xFFFFFFFFu;
    const int lane = threadIdx.x % kWarp;
    __threadfence();
    __syncwarp();
    unsigned prev = 0;
    if (lane == 0) prev = atomicAdd(counters + (size_t)b * n_kv + head, 1u);
    prev = __shfl_sync(kAll, prev, 0);
    if (prev != (unsigned)(nseg - 1)) return;
    __threadfence();
    float M[kG], L[kG];
    float4 A0, A1;
    merge_records<true, kBatch>(base, nseg, M, L, A0, A1);
    merged_store_out(L, A0, A1, out, b, head, n_q);
    if (lane == 0) counters[(size_t)b * n_kv + head] = 0u;
}

// A warp's share as a whole: when it is the whole row (nseg == 1) the output
// directly, else its record in segment `seg` and the merge by the last one.
template <int kBatch = 8>
__device__ __forceinline__ void flush_share(float (&acc)[16][4], float l_run, float m_run, int b, int head,
                                            int nseg, int seg, int max_segs, int n_q, int n_kv, float* partial,
                                            unsigned* counters, float* out, uint32_t* err) {
    float Lh, Mh;
    share_reduce(acc, l_run, m_run, Lh, Mh);
    if (nseg == 1) {
        share_store_out(acc, Lh, out, b, head, n_q);
        return;
    }
    if (seg >= max_segs || nseg > max_segs) {
        if ((threadIdx.x % kWarp) == 0 && err) atomicOr(err, kErrBadIndex);
        return;
    }
    const float* base = partial + ((size_t)b * n_kv + head) * max_segs * kPartStride;
    share_store_record(acc, Lh, Mh, const_cast<float*>(base) + (size_t)seg * kPartStride);
    publish_and_merge<kBatch>(b, head, nseg, n_q, n_kv, base, counters, out);
}

}  // namespace attn
}  // namespace zc
