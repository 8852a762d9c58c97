// int8 weight-only linear for a few activation rows (2..16), in one launch:
//   Y[t, m] = (sum_k W[m, k] X[t, k]) * scale[m]      (matmulQ8, src/backends/cpu/ops.zig:200-228)
// with the optional RMSNorm of X (ops.zig:49-67) and the residual / SwiGLU
// epilogues of the decode block (qwen_block.zig:161-235).
//
// Why a third kernel family: at 2..16 rows the tcgen05 linear needs a
// separate activation-plane launch and a TMA/mbarrier pipeline fill before its
// first MMA, and the CUDA-core GEMV re-reads every activation from shared
// memory once per weight byte and row. Both are latency, not bytes: a decode
// step at these batch sizes is a chain of 28 x 5 dependent launches. This
// kernel keeps the GEMV's shape (every weight load of a warp issued before
// griddepcontrol.wait, one launch per linear) and does the products on the
// integer tensor-core path:
//
// * Each CTA stages the activation rows itself, with the arithmetic of the
//   plane kernel of tc_gemm.cu, operation for operation (the block order of
//   sq4 for the sum of squares, order-free maxima): RMSNorm scale, a
//   per-row power of two 2^e >= max|x|, and the 22-bit fixed-point value
//   split into three signed int8 digits v = d0 2^16 + d1 2^8 + d2. The
//   digits, and so every integer sum below, equal the tcgen05 path's, and the
//   epilogue repeats its f32 operations: the outputs are bit-identical.
// * mma.sync.m16n8k32 s8 x s8 -> s32, activation rows as the 16-row A operand
//   and eight weight rows as the B operand (n = 8). The k order inside each
//   64-byte block is permuted identically for A and B so that a lane's
//   fragments are one 16-byte load of a weight row (from HBM, straight into
//   the B registers) and one 16-byte load per digit plane and activation row
//   (from shared memory, rows padded to K + 64 bytes: the eight lanes of a
//   quarter-warp hit distinct banks).
// * A CTA is 8 warps: KS slices of K per group of weight rows. Each warp
//   recombines its three plane sums exactly in 64-bit integers; the slices
//   are summed in shared memory (exact, so order-free) and one thread per
//   (row, output) applies 2^(e-22) * scale[m] and the epilogue.
//
// No waits, no atomics: the kernel cannot hang, and it reads only the rows
// and columns the host checked.
#include "common.cuh"
#include "kernels.h"

namespace zc {

namespace {

constexpr int kFrThreads = 256;
constexpr int kFrWarps = kFrThreads / kWarp;
constexpr int kFrMaxK = 4096;
constexpr int kFrMaxRows = 16;
constexpr int kFrPad = 64;  // bytes after each staged digit row
constexpr int kFrHeld = 24;  // activation float4 a thread holds (rows x K / 1024)

__device__ __forceinline__ void mma_s8(int (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                       uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t word(const uint4& v, int i) {
    return i == 0 ? v.x : i == 1 ? v.y : i == 2 ? v.z : v.w;
}

template <int NBP, int KS>
constexpr size_t fr_red_bytes(int rows_per_cta) {
    return (size_t)KS * rows_per_cta * NBP * sizeof(long long);
}

// NBP: activation rows the MMA covers (8: rows g only, 16: rows g and g + 8).
// TN: n8 weight tiles per warp. KS: K slices per weight-row group (8 / KS groups per CTA).
// KV: float4 per thread and activation row (K <= 1024 KV).
template <int NBP, int TN, int KS, int KV, int EPI>
__global__ void __launch_bounds__(kFrThreads, TN == 2 ? 2 : 1) fewrow_q8_kernel(LinearArgs a) {
    constexpr int WT = kFrWarps / KS;       // weight-row groups per CTA
    constexpr int ROWS = WT * 8 * TN;       // weight rows per CTA
    constexpr int kMaxBlk = 8 / TN;         // 64-byte blocks per lane and tile held in registers
    extern __shared__ __align__(16) unsigned char smem[];
    __shared__ float red_bs[NBP][kFrMaxK / 128], red_mx[kFrWarps][NBP];
    __shared__ float xscale_s[NBP], inv_s[NBP];
    __shared__ int e_s[NBP];

    const int K = a.K, N = a.N;
    const int S = K + kFrPad;
    int8_t* planes = reinterpret_cast<int8_t*>(smem);                              // [3][NBP][S]
    long long* red = reinterpret_cast<long long*>(smem + (size_t)3 * NBP * S);     // [KS][ROWS][NBP]
    const int warp = threadIdx.x / kWarp, lane = threadIdx.x % kWarp;
    const int g = lane >> 2, t = lane & 3;
    const int ks = warp % KS, wt = warp / KS;
    const int KW = K / KS;                  // multiple of 64
    const int nblk = KW / 64;               // <= kMaxBlk
    const int row0 = blockIdx.x * ROWS;

    // ---- this warp's weights, every load in flight before the dependency wait
    uint4 wv[kMaxBlk][TN];
    const int8_t* wq = static_cast<const int8_t*>(a.w);
#pragma unroll
    for (int blk = 0; blk < kMaxBlk; ++blk) {
        if (blk < nblk) {
#pragma unroll
            for (int tn = 0; tn < TN; ++tn) {
                const int row = row0 + (wt * TN + tn) * 8 + g;
                // evict-first: read once per step (batch 2 / 4: 1.0 / 1.4 % per step;
                // the batch-1 GEMV measured slower with it)
                wv[blk][tn] = ldg_stream_first(wq + (size_t)row * K + ks * KW + blk * 64 + 16 * t);
            }
        }
    }
    prefetch_l2_ranges(a.pf);
    // this thread's first epilogue item: its row scales now (weights), its
    // residual right after the wait, so the epilogue waits for no load
    constexpr int OUTS = EPI == kEpiSwiGLU ? ROWS / 2 : ROWS;
    const bool item0 = threadIdx.x < N * OUTS;
    const int b_0 = threadIdx.x / OUTS, o_0 = threadIdx.x % OUTS;
    float sc0[2] = {1.0f, 1.0f};
    if (item0) {
        if constexpr (EPI == kEpiSwiGLU) {
            sc0[0] = __ldg(a.scale + row0 + 2 * o_0);
            sc0[1] = __ldg(a.scale + row0 + 2 * o_0 + 1);
        } else {
            sc0[0] = __ldg(a.scale + row0 + o_0);
        }
    }
    pdl_wait();
    float rs0 = 0.0f;
    if constexpr (EPI == kEpiResid)
        if (item0) rs0 = a.resid[(size_t)b_0 * a.ldy + row0 + o_0];

    // ---- activation rows -> digit planes, with the plane kernel's thread
    // mapping (thread i holds k = 4 (i + 256 j) of every row) and the
    // sum-of-squares order of sq4. Every row's values are loaded at once and
    // stay in registers for both passes (NBP * KV <= kFrHeld float4).
    float4 wn[KV];
    float4 xv[NBP][KV];
#pragma unroll
    for (int i = 0; i < KV; ++i) {
        const int k = 4 * (threadIdx.x + i * kFrThreads);
        wn[i] = (a.norm_w && k < K) ? __ldg(reinterpret_cast<const float4*>(a.norm_w + k))
                                    : make_float4(1.f, 1.f, 1.f, 1.f);
#pragma unroll
        for (int b = 0; b < NBP; ++b)
            xv[b][i] = (b < N && k < K) ? *reinterpret_cast<const float4*>(a.x + (size_t)b * a.ldx + k)
                                        : make_float4(0.f, 0.f, 0.f, 0.f);
    }
#pragma unroll
    for (int b = 0; b < NBP; ++b) {
        float mx = 0.0f;
#pragma unroll
        for (int i = 0; i < KV; ++i) {
            const float4 x4 = xv[b][i];
            // (warp, lane) holds values 4 lane .. 4 lane + 3 of the 128-value block warp + 8 i
            const float bs = warp_sum(sq4(x4));
            if (lane == 0 && 4 * (threadIdx.x + i * kFrThreads) < K) red_bs[b][warp + kFrWarps * i] = bs;
            const float4 p = a.norm_w ? make_float4(__fmul_rn(wn[i].x, x4.x), __fmul_rn(wn[i].y, x4.y),
                                                    __fmul_rn(wn[i].z, x4.z), __fmul_rn(wn[i].w, x4.w))
                                      : x4;
            mx = fmaxf(mx, fmaxf(fmaxf(fabsf(p.x), fabsf(p.y)), fmaxf(fabsf(p.z), fabsf(p.w))));
        }
        mx = warp_max(mx);
        if (lane == 0) red_mx[warp][b] = mx;
    }
    __syncthreads();
    if (threadIdx.x < N) {
        const int b = threadIdx.x;
        float ss = 0.0f, mx = 0.0f;
        for (int kb = 0; kb < K / 128; ++kb) ss = __fadd_rn(ss, red_bs[b][kb]);  // blocks in k order
#pragma unroll
        for (int i = 0; i < kFrWarps; ++i) mx = fmaxf(mx, red_mx[i][b]);
        float inv = 1.0f;
        if (a.norm_w) {
            inv = 1.0f / sqrtf(ss / (float)K + a.eps);
            mx = __fmul_rn(mx, inv);
        }
        int e = 0;
        if (mx > 0.0f) frexpf(mx, &e);  // max|x| < 2^e
        inv_s[b] = inv;
        e_s[b] = e;
        xscale_s[b] = ldexpf(1.0f, e - 22);  // exact power of two
    }
    __syncthreads();
#pragma unroll
    for (int b = 0; b < NBP; ++b) {
        if (b >= N) break;
        const float inv = inv_s[b];
        const int e = e_s[b];
        int8_t* p0 = planes + (size_t)b * S;
#pragma unroll
        for (int i = 0; i < KV; ++i) {
            const int k = 4 * (threadIdx.x + i * kFrThreads);
            if (k >= K) break;
            const float4 x4 = xv[b][i];
            const float f[4] = {a.norm_w ? __fmul_rn(__fmul_rn(wn[i].x, x4.x), inv) : x4.x,
                                a.norm_w ? __fmul_rn(__fmul_rn(wn[i].y, x4.y), inv) : x4.y,
                                a.norm_w ? __fmul_rn(__fmul_rn(wn[i].z, x4.z), inv) : x4.z,
                                a.norm_w ? __fmul_rn(__fmul_rn(wn[i].w, x4.w), inv) : x4.w};
            uint32_t d0, d1, d2;
            digits4(f, e, d0, d1, d2);
            *reinterpret_cast<uint32_t*>(p0 + k) = d0;
            *reinterpret_cast<uint32_t*>(p0 + (size_t)NBP * S + k) = d1;
            *reinterpret_cast<uint32_t*>(p0 + (size_t)2 * NBP * S + k) = d2;
        }
    }
    __syncthreads();

    // the next kernel may launch now: its CTAs' weight loads and prefetches
    // (issued before its dependency wait) no longer compete with this
    // kernel's activation loads (measured: 4-12 % per decode step at 2-16 rows)
    pdl_launch_dependents();

    // ---- products: per 64-byte block, lane (g, t) owns bytes [16 t, 16 t + 16)
    // of weight row g and of activation rows g and g + 8; MMA j takes bytes
    // 8 j .. 8 j + 7 of each (A words 2j, 2j+1; B words 2j, 2j+1)
    int acc[TN][3][4];
#pragma unroll
    for (int tn = 0; tn < TN; ++tn)
#pragma unroll
        for (int p = 0; p < 3; ++p)
#pragma unroll
            for (int c = 0; c < 4; ++c) acc[tn][p][c] = 0;
#pragma unroll
    for (int blk = 0; blk < kMaxBlk; ++blk) {
        if (blk < nblk) {
            const int kb = ks * KW + blk * 64 + 16 * t;
#pragma unroll
            for (int p = 0; p < 3; ++p) {
                const int8_t* pl = planes + (size_t)p * NBP * S + kb;
                const uint4 ag = *reinterpret_cast<const uint4*>(pl + (size_t)g * S);
                uint4 ag8 = make_uint4(0u, 0u, 0u, 0u);
                if constexpr (NBP == 16) ag8 = *reinterpret_cast<const uint4*>(pl + (size_t)(g + 8) * S);
#pragma unroll
                for (int j = 0; j < 2; ++j) {
#pragma unroll
                    for (int tn = 0; tn < TN; ++tn)
                        mma_s8(acc[tn][p], word(ag, 2 * j), word(ag8, 2 * j), word(ag, 2 * j + 1),
                               word(ag8, 2 * j + 1), word(wv[blk][tn], 2 * j), word(wv[blk][tn], 2 * j + 1));
                }
            }
        }
    }
    // C fragment: c0 (row g, col 2t), c1 (g, 2t + 1), c2 (g + 8, 2t), c3 (g + 8, 2t + 1)
#pragma unroll
    for (int tn = 0; tn < TN; ++tn) {
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            const int b = g + (c >= 2 ? 8 : 0);
            if (b >= NBP) continue;
            const int r = (wt * TN + tn) * 8 + 2 * t + (c & 1);
            const long long v = (long long)acc[tn][0][c] * 65536ll + (long long)acc[tn][1][c] * 256ll +
                                (long long)acc[tn][2][c];
            red[((size_t)ks * ROWS + r) * NBP + b] = v;
        }
    }
    __syncthreads();

    // ---- epilogue: one thread per (activation row, weight row or SwiGLU pair)
    for (int idx = threadIdx.x; idx < N * OUTS; idx += kFrThreads) {
        const int b = idx / OUTS, o = idx % OUTS;
        const bool first = idx == threadIdx.x;
        auto value = [&](int r, float sc) -> float {
            long long v = 0;
#pragma unroll
            for (int s = 0; s < KS; ++s) v += red[((size_t)s * ROWS + r) * NBP + b];
            return __fmul_rn(__fmul_rn(__ll2float_rn(v), xscale_s[b]), sc);
        };
        if constexpr (EPI == kEpiSwiGLU) {
            const float gate = value(2 * o, first ? sc0[0] : a.scale[row0 + 2 * o]);
            const float up = value(2 * o + 1, first ? sc0[1] : a.scale[row0 + 2 * o + 1]);
            a.y[(size_t)b * a.ldy + (row0 >> 1) + o] = __fmul_rn(silu(gate), up);
        } else if constexpr (EPI == kEpiResid) {
            const size_t at = (size_t)b * a.ldy + row0 + o;
            a.y[at] = __fadd_rn(first ? rs0 : a.resid[at], value(o, first ? sc0[0] : a.scale[row0 + o]));
        } else {
            a.y[(size_t)b * a.ldy + row0 + o] = value(o, first ? sc0[0] : a.scale[row0 + o]);
        }
    }
}

// Weight rows per CTA and K slices: 32 rows x 4 slices where that still
// gives a full wave of CTAs, else 8 rows x 8 slices.
struct FrShape {
    int tn, ks, rows;
};
FrShape fr_shape(int M, int K) {
    if (M >= 4096 && M % 32 == 0 && K % 256 == 0 && K / 4 <= 64 * 4) return {2, 4, 32};
    return {1, 8, 8};
}

template <int NBP, int TN, int KS>
size_t fr_smem(int K) {
    constexpr int ROWS = (kFrWarps / KS) * 8 * TN;
    return (size_t)3 * NBP * (K + kFrPad) + fr_red_bytes<NBP, KS>(ROWS);
}

template <int NBP, int TN, int KS, int KV>
void launch_kv(const LinearArgs& a, int rows, cudaStream_t st) {
    const size_t smem = fr_smem<NBP, TN, KS>(a.K);
    const int grid = a.M / rows;
    switch (a.epi) {
        case kEpiResid:
            launch_pdl(fewrow_q8_kernel<NBP, TN, KS, KV, kEpiResid>, grid, kFrThreads, smem, st, a);
            break;
        case kEpiSwiGLU:
            launch_pdl(fewrow_q8_kernel<NBP, TN, KS, KV, kEpiSwiGLU>, grid, kFrThreads, smem, st, a);
            break;
        default: launch_pdl(fewrow_q8_kernel<NBP, TN, KS, KV, kEpiNone>, grid, kFrThreads, smem, st, a); break;
    }
}

template <int NBP, int TN, int KS, int KV>
void prepare_kv() {
    const size_t smem = fr_smem<NBP, TN, KS>(kFrMaxK);
    configure_kernel((const void*)fewrow_q8_kernel<NBP, TN, KS, KV, kEpiNone>, smem);
    configure_kernel((const void*)fewrow_q8_kernel<NBP, TN, KS, KV, kEpiResid>, smem);
    configure_kernel((const void*)fewrow_q8_kernel<NBP, TN, KS, KV, kEpiSwiGLU>, smem);
}

// 32 weight rows x 4 K slices (K <= 1024), or 8 rows x 8 slices; K / 1024
// (rounded up) float4 of every row per thread: 8 rows up to K = 3072, 16 rows
// up to K = 1024
template <int NBP>
void launch_rows(const LinearArgs& a, cudaStream_t st) {
    const FrShape s = fr_shape(a.M, a.K);
    if (s.tn == 2) {
        launch_kv<NBP, 2, 4, 1>(a, s.rows, st);
        return;
    }
    const int kv = (a.K + 1023) / 1024;
    if (kv <= 1) launch_kv<NBP, 1, 8, 1>(a, s.rows, st);
    else if constexpr (NBP * 2 <= kFrHeld) {
        if (kv == 2) launch_kv<NBP, 1, 8, 2>(a, s.rows, st);
        else if constexpr (NBP * 3 <= kFrHeld) launch_kv<NBP, 1, 8, 3>(a, s.rows, st);
    }
}

template <int NBP>
void prepare_rows() {
    prepare_kv<NBP, 2, 4, 1>();
    prepare_kv<NBP, 1, 8, 1>();
    if constexpr (NBP * 2 <= kFrHeld) prepare_kv<NBP, 1, 8, 2>();
    if constexpr (NBP * 3 <= kFrHeld) prepare_kv<NBP, 1, 8, 3>();
}

}  // namespace

bool fewrow_fits(const LinearArgs& a) {
    if (a.wkind != kWQ8 || a.N < 2 || a.N > kFrMaxRows || a.epi == kEpiArgmax || !a.scale) return false;
    if (a.K < 512 || a.K > kFrMaxK || a.K % 512 || a.ldx % 4) return false;
    if ((a.N <= 8 ? 8 : 16) * ((a.K + 1023) / 1024) > kFrHeld) return false;  // rows held in registers
    const FrShape s = fr_shape(a.M, a.K);
    if (a.M % s.rows) return false;
    if ((a.K / (kFrWarps / (s.rows / (8 * s.tn)))) % 64) return false;  // K slice of whole 64-byte blocks
    return true;
}

void prepare_fewrow_kernels() {
    prepare_rows<8>();
    prepare_rows<16>();
}

void launch_fewrow(const LinearArgs& a, cudaStream_t st) {
    if (a.N <= 8) launch_rows<8>(a, st);
    else launch_rows<16>(a, st);
}

}  // namespace zc
