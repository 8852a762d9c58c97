// Causal GQA attention (attentionInto, src/backends/cpu/ops.zig:285-354) on
// the B200: a split-K decode kernel over the paged bf16 KV cache with a
// log-sum-exp merge, and a tiled f32 prefill kernel.
#include <algorithm>

#include "common.cuh"
#include "kernels.h"

namespace zc {

namespace {

// ------------------------------------------------------------- decode
//
// Grid (split, kv_head, batch row); 128 threads. Each CTA owns `chunk`
// positions of one sequence's K/V for one kv head and both query heads of its
// GQA group. K/V arrive by untiled bulk copies (cp.async.bulk, 4 KB per
// 16-token block and head) into a 4-stage shared-memory ring of 32-token
// stages, completed on mbarriers; warps then compute scores and an online
// softmax over their 8 tokens per stage (4 lanes per token, 32 dims each).
// The CTA writes a partial (max, sum, acc[d]) per query head; the last CTA of
// a (row, kv head) to finish (atomic counter) merges the splits:
//   m = max m_s,  l = sum l_s e^(m_s - m),  o = sum acc_s e^(m_s - m) / l.
constexpr int kD = 128, kG = 2, kStageTok = 32, kStages = 4, kDecThreads = 128;
constexpr int kBlockElems = kKvBlock * kD;                 // 2048 bf16 = 4 KB
constexpr int kStageElems = kStageTok * kD;                // per K (or V) stage

__global__ void __launch_bounds__(kDecThreads) attn_decode_kernel(AttnDecodeArgs a) {
    extern __shared__ __align__(128) unsigned char smem_raw[];
    uint16_t* ks = reinterpret_cast<uint16_t*>(smem_raw);            // [kStages][32][128]
    uint16_t* vs = ks + kStages * kStageElems;                        // [kStages][32][128]
    uint64_t* full = reinterpret_cast<uint64_t*>(vs + kStages * kStageElems);
    __shared__ float red_m[4][kG], red_l[4][kG];
    __shared__ __align__(16) float red_acc[4][kG][kD];
    __shared__ int is_last;

    pdl_launch_dependents();
    pdl_wait();
    const int split = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
    const int tid = threadIdx.x, warp = tid / kWarp, lane = tid % kWarp;
    const int seq = a.seq_of[b];
    const int kv_len = a.positions[b] + 1;
    const int nsplit = (kv_len + a.chunk - 1) / a.chunk;
    if (split >= nsplit) return;
    const int t0 = split * a.chunk;
    const int t1 = min(t0 + a.chunk, kv_len);
    const int nstage = (t1 - t0 + kStageTok - 1) / kStageTok;
    const int last_blk = (kv_len - 1) / kKvBlock;
    const int* table = a.block_table + (size_t)seq * a.max_blocks;

    if (tid == 0) {
        for (int s = 0; s < kStages; ++s) mbar_init(&full[s], 1);
        fence_barrier_init();
    }
    __syncthreads();

    auto issue = [&](int s) {  // thread 0 only
        const int buf = s % kStages;
        const int bi0 = (t0 + s * kStageTok) / kKvBlock;
        uint32_t bytes = 0;
        int blks[2];
        for (int j = 0; j < 2; ++j) {
            const int bi = bi0 + j;
            blks[j] = -1;
            if (bi <= last_blk && bi < a.max_blocks) {
                const int blk = table[bi];
                if (blk >= 0 && blk < a.n_pool_blocks) {
                    blks[j] = blk;
                    bytes += 2 * kBlockElems * 2;
                } else if (a.err) {
                    atomicOr(a.err, kErrBadIndex);
                }
            }
        }
        mbar_arrive_expect_tx(&full[buf], bytes);
        for (int j = 0; j < 2; ++j) {
            if (blks[j] < 0) continue;
            const uint16_t* kp = a.kv_layer + (((size_t)blks[j] * 2 + 0) * a.n_kv + kvh) * kBlockElems;
            const uint16_t* vp = a.kv_layer + (((size_t)blks[j] * 2 + 1) * a.n_kv + kvh) * kBlockElems;
            bulk_g2s(ks + buf * kStageElems + j * kBlockElems, kp, kBlockElems * 2, &full[buf]);
            bulk_g2s(vs + buf * kStageElems + j * kBlockElems, vp, kBlockElems * 2, &full[buf]);
        }
    };
    if (tid == 0)
        for (int s = 0; s < min(kStages, nstage); ++s) issue(s);

    // lane -> (token slot tq, dim quarter j): dims 32 i + 8 j + e, i = 0..3, e = 0..7
    const int tq = lane / 4, j = lane % 4;
    float q[kG][32];
#pragma unroll
    for (int g = 0; g < kG; ++g) {
        const float* qp = a.q + ((size_t)b * a.n_q + kvh * kG + g) * kD;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float4 v0 = *reinterpret_cast<const float4*>(qp + 32 * i + 8 * j);
            const float4 v1 = *reinterpret_cast<const float4*>(qp + 32 * i + 8 * j + 4);
            q[g][8 * i + 0] = v0.x; q[g][8 * i + 1] = v0.y; q[g][8 * i + 2] = v0.z; q[g][8 * i + 3] = v0.w;
            q[g][8 * i + 4] = v1.x; q[g][8 * i + 5] = v1.y; q[g][8 * i + 6] = v1.z; q[g][8 * i + 7] = v1.w;
        }
    }
    const float scale = 1.0f / sqrtf((float)kD);
    float m[kG], l[kG], acc[kG][32];
#pragma unroll
    for (int g = 0; g < kG; ++g) {
        m[g] = -INFINITY;
        l[g] = 0.0f;
#pragma unroll
        for (int e = 0; e < 32; ++e) acc[g][e] = 0.0f;
    }

    for (int s = 0; s < nstage; ++s) {
        const int buf = s % kStages;
        const bool ok = mbar_wait_bounded(&full[buf], (uint32_t)((s / kStages) & 1), a.err);
        if (__syncthreads_or(!ok)) return;  // timed out: error flag set, nothing merged
        const int tok = t0 + s * kStageTok + warp * 8 + tq;
        const bool valid = tok < t1;
        const uint16_t* kr = ks + buf * kStageElems + (warp * 8 + tq) * kD;
        const uint16_t* vr = vs + buf * kStageElems + (warp * 8 + tq) * kD;
        float dot[kG] = {0.0f, 0.0f};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const uint4 kv = *reinterpret_cast<const uint4*>(kr + 32 * i + 8 * j);
            const float kf[8] = {bf16lo(kv.x), bf16hi(kv.x), bf16lo(kv.y), bf16hi(kv.y),
                                 bf16lo(kv.z), bf16hi(kv.z), bf16lo(kv.w), bf16hi(kv.w)};
#pragma unroll
            for (int e = 0; e < 8; ++e)
#pragma unroll
                for (int g = 0; g < kG; ++g) dot[g] = fmaf(q[g][8 * i + e], kf[e], dot[g]);
        }
        float p[kG];
#pragma unroll
        for (int g = 0; g < kG; ++g) {
            dot[g] += __shfl_xor_sync(0xFFFFFFFFu, dot[g], 1);
            dot[g] += __shfl_xor_sync(0xFFFFFFFFu, dot[g], 2);
            const float sc = valid ? dot[g] * scale : -INFINITY;
            float mx = sc;
            mx = fmaxf(mx, __shfl_xor_sync(0xFFFFFFFFu, mx, 4));
            mx = fmaxf(mx, __shfl_xor_sync(0xFFFFFFFFu, mx, 8));
            mx = fmaxf(mx, __shfl_xor_sync(0xFFFFFFFFu, mx, 16));
            const float m_new = fmaxf(m[g], mx);
            const float corr = m_new == -INFINITY ? 1.0f : expf(m[g] - m_new);
            p[g] = valid ? expf(sc - m_new) : 0.0f;
            l[g] = l[g] * corr + p[g];
            m[g] = m_new;
#pragma unroll
            for (int e = 0; e < 32; ++e) acc[g][e] *= corr;
        }
        if (valid) {
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const uint4 vv = *reinterpret_cast<const uint4*>(vr + 32 * i + 8 * j);
                const float vf[8] = {bf16lo(vv.x), bf16hi(vv.x), bf16lo(vv.y), bf16hi(vv.y),
                                     bf16lo(vv.z), bf16hi(vv.z), bf16lo(vv.w), bf16hi(vv.w)};
#pragma unroll
                for (int e = 0; e < 8; ++e)
#pragma unroll
                    for (int g = 0; g < kG; ++g) acc[g][8 * i + e] = fmaf(p[g], vf[e], acc[g][8 * i + e]);
            }
        }
        __syncthreads();  // stage buffer free
        if (tid == 0 && s + kStages < nstage) issue(s + kStages);
    }

    // reduce the 8 token slots of each warp (lanes with equal j)
#pragma unroll
    for (int g = 0; g < kG; ++g) {
#pragma unroll
        for (int o = 4; o < 32; o <<= 1) l[g] += __shfl_xor_sync(0xFFFFFFFFu, l[g], o);
#pragma unroll
        for (int e = 0; e < 32; ++e) {
            float v = acc[g][e];
#pragma unroll
            for (int o = 4; o < 32; o <<= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
            acc[g][e] = v;
        }
    }
    if (lane < 4) {
#pragma unroll
        for (int g = 0; g < kG; ++g) {
            if (lane == 0) {
                red_m[warp][g] = m[g];
                red_l[warp][g] = l[g];
            }
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int e = 0; e < 8; ++e) red_acc[warp][g][32 * i + 8 * lane + e] = acc[g][8 * i + e];
        }
    }
    __syncthreads();

    // combine the 4 warps: thread = (g, dim); 2 x 128 = 256 > 128 threads, loop g
    float* part = a.partial + (((size_t)b * a.n_kv + kvh) * a.max_splits + split) * kG * (kD + 2);
    for (int g = 0; g < kG; ++g) {
        float M = -INFINITY;
        for (int w = 0; w < 4; ++w) M = fmaxf(M, red_m[w][g]);
        float L = 0.0f, A = 0.0f;
        for (int w = 0; w < 4; ++w) {
            const float c = red_m[w][g] == -INFINITY ? 0.0f : expf(red_m[w][g] - M);
            L += red_l[w][g] * c;
            A += red_acc[w][g][tid] * c;
        }
        if (nsplit == 1) {
            a.out[((size_t)b * a.n_q + kvh * kG + g) * kD + tid] = A / L;
        } else {
            float* pg = part + g * (kD + 2);
            if (tid == 0) {
                pg[0] = M;
                pg[1] = L;
            }
            pg[2 + tid] = A;
        }
    }
    if (nsplit == 1) return;

    __threadfence();
    __syncthreads();
    if (tid == 0) {
        const unsigned prev = atomicAdd(a.counters + (size_t)b * a.n_kv + kvh, 1u);
        is_last = prev == (unsigned)(nsplit - 1);
    }
    __syncthreads();
    if (!is_last) return;
    __threadfence();
    const float* base = a.partial + ((size_t)b * a.n_kv + kvh) * a.max_splits * kG * (kD + 2);
    for (int g = 0; g < kG; ++g) {
        float M = -INFINITY;
        for (int sp = 0; sp < nsplit; ++sp) M = fmaxf(M, __ldcg(base + (sp * kG + g) * (kD + 2)));
        float L = 0.0f, A = 0.0f;
        for (int sp = 0; sp < nsplit; ++sp) {
            const float* pg = base + (sp * kG + g) * (kD + 2);
            const float ms = __ldcg(pg);
            const float c = ms == -INFINITY ? 0.0f : expf(ms - M);
            L += __ldcg(pg + 1) * c;
            A += __ldcg(pg + 2 + tid) * c;
        }
        a.out[((size_t)b * a.n_q + kvh * kG + g) * kD + tid] = A / L;
    }
    if (tid == 0) a.counters[(size_t)b * a.n_kv + kvh] = 0u;
}

// ------------------------------------------------------------ prefill
//
// CTA per (64-query tile, query head), 256 threads, f32 throughout:
// S = Q K^T (thread: 4 queries x 4 keys), online softmax (4 threads per
// query row), O += P V (thread: 4 queries x 8 dims). Keys after the query or
// past T are masked (kv_len == q_len == T, ops.zig:322).
constexpr int PQ = 64, PK = 64, PTHREADS = 256;

__global__ void __launch_bounds__(PTHREADS) attn_prefill_kernel(AttnPrefillArgs a) {
    extern __shared__ __align__(16) float sm[];
    float* Qs = sm;                       // [128][PQ]  (d-major)
    float* Ks = Qs + kD * PQ;             // [128][PK]  (d-major)
    float* Vs = Ks + kD * PK;             // [PK][128]
    float* Ps = Vs + PK * kD;             // [PK][PQ]   (key-major)
    float* rowc = Ps + PK * PQ;           // [PQ] correction factors
    float* rowl = rowc + PQ;              // [PQ] final sums

    pdl_launch_dependents();
    pdl_wait();
    const int qt = blockIdx.x, h = blockIdx.y;
    const int kvh = h / (a.n_q / a.n_kv);
    const int q0 = qt * PQ;
    const int tid = threadIdx.x;
    const int T = a.T;
    const float scale = 1.0f / sqrtf((float)kD);

    for (int i = tid; i < PQ * kD; i += PTHREADS) {
        const int r = i / kD, d = i % kD;
        Qs[d * PQ + r] = (q0 + r < T) ? a.q[((size_t)h * T + q0 + r) * kD + d] : 0.0f;
    }
    // S-phase mapping
    const int sx = tid % 16, sy = tid / 16;  // keys sx*4.., queries sy*4..
    // O-phase mapping
    const int ox = tid % 16, oy = tid / 16;  // dims ox*8.., queries oy*4..
    // softmax mapping: row = tid / 4, part = tid % 4 (16 keys each)
    const int srow = tid / 4, spart = tid % 4;
    float m_run = -INFINITY, l_run = 0.0f;
    float o[4][8];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int c = 0; c < 8; ++c) o[i][c] = 0.0f;

    const int last_key = min(q0 + PQ, T);  // keys [0, last_key)
    for (int k0 = 0; k0 < last_key; k0 += PK) {
        __syncthreads();
        for (int i = tid; i < PK * kD; i += PTHREADS) {
            const int r = i / kD, d = i % kD;
            const bool in = k0 + r < T;
            const size_t off = ((size_t)kvh * T + k0 + r) * kD + d;
            Ks[d * PK + r] = in ? a.k[off] : 0.0f;
            Vs[r * kD + d] = in ? a.v[off] : 0.0f;
        }
        __syncthreads();
        float s[4][4];
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
            for (int c = 0; c < 4; ++c) s[i][c] = 0.0f;
#pragma unroll 8
        for (int d = 0; d < kD; ++d) {
            const float4 qv = *reinterpret_cast<const float4*>(Qs + d * PQ + sy * 4);
            const float4 kv = *reinterpret_cast<const float4*>(Ks + d * PK + sx * 4);
            const float qa[4] = {qv.x, qv.y, qv.z, qv.w};
            const float ka[4] = {kv.x, kv.y, kv.z, kv.w};
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int c = 0; c < 4; ++c) s[i][c] = fmaf(qa[i], ka[c], s[i][c]);
        }
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                const int qi = q0 + sy * 4 + i, kj = k0 + sx * 4 + c;
                Ps[(sx * 4 + c) * PQ + sy * 4 + i] = (kj <= qi && kj < T) ? s[i][c] * scale : -INFINITY;
            }
        __syncthreads();
        // online softmax over this tile's 64 keys for row srow
        float mx = -INFINITY;
        for (int c = 0; c < 16; ++c) mx = fmaxf(mx, Ps[(spart * 16 + c) * PQ + srow]);
        mx = fmaxf(mx, __shfl_xor_sync(0xFFFFFFFFu, mx, 1));
        mx = fmaxf(mx, __shfl_xor_sync(0xFFFFFFFFu, mx, 2));
        const float m_new = fmaxf(m_run, mx);
        const float corr = m_new == -INFINITY ? 1.0f : expf(m_run - m_new);
        float sum = 0.0f;
        for (int c = 0; c < 16; ++c) {
            float* pp = Ps + (spart * 16 + c) * PQ + srow;
            const float pv = *pp == -INFINITY ? 0.0f : expf(*pp - m_new);
            *pp = pv;
            sum += pv;
        }
        sum += __shfl_xor_sync(0xFFFFFFFFu, sum, 1);
        sum += __shfl_xor_sync(0xFFFFFFFFu, sum, 2);
        l_run = l_run * corr + sum;
        m_run = m_new;
        if (spart == 0) rowc[srow] = corr;
        __syncthreads();
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float c = rowc[oy * 4 + i];
#pragma unroll
            for (int cc = 0; cc < 8; ++cc) o[i][cc] *= c;
        }
        const int kmax = min(PK, last_key - k0);
        for (int kk = 0; kk < kmax; ++kk) {
            const float4 pv = *reinterpret_cast<const float4*>(Ps + kk * PQ + oy * 4);
            const float4 v0 = *reinterpret_cast<const float4*>(Vs + kk * kD + ox * 8);
            const float4 v1 = *reinterpret_cast<const float4*>(Vs + kk * kD + ox * 8 + 4);
            const float pa[4] = {pv.x, pv.y, pv.z, pv.w};
            const float va[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int cc = 0; cc < 8; ++cc) o[i][cc] = fmaf(pa[i], va[cc], o[i][cc]);
        }
    }
    if (spart == 0) rowl[srow] = l_run;
    __syncthreads();
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int qi = q0 + oy * 4 + i;
        if (qi >= T) continue;
        const float inv = 1.0f / rowl[oy * 4 + i];
        float* op = a.out + ((size_t)qi * a.n_q + h) * kD + ox * 8;
#pragma unroll
        for (int cc = 0; cc < 8; ++cc) op[cc] = o[i][cc] * inv;
    }
}

}  // namespace

constexpr size_t kDecodeSmem = (size_t)2 * kStages * kStageElems * 2 + kStages * sizeof(uint64_t);
constexpr size_t kPrefillSmem = ((size_t)kD * PQ + kD * PK + PK * kD + PK * PQ + 2 * PQ) * sizeof(float);

void prepare_attn_kernels() {
    configure_kernel((const void*)attn_decode_kernel, kDecodeSmem);
    configure_kernel((const void*)attn_prefill_kernel, kPrefillSmem);
}

void launch_attn_decode(const AttnDecodeArgs& a, cudaStream_t st) {
    dim3 grid(a.max_splits, a.n_kv, a.B);
    launch_pdl(attn_decode_kernel, grid, kDecThreads, kDecodeSmem, st, a);
}

void launch_attn_prefill(const AttnPrefillArgs& a, cudaStream_t st) {
    dim3 grid((a.T + PQ - 1) / PQ, a.n_q);
    launch_pdl(attn_prefill_kernel, grid, PTHREADS, kPrefillSmem, st, a);
}

}  // namespace zc
