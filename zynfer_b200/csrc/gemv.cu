// Weight-only GEMV for 1..8 activation rows: y[b, r] = (sum_k W[r, k] x[b, k]) * scale[r]
// (matvecQ8, src/backends/cpu/ops.zig:181-197), W int8 (per-row scale) or bf16.
//
// Design (HBM-bound): each warp streams whole weight rows with 16-byte
// read-only loads (one row = K bytes for int8, 2K for bf16; a warp covers 512
// contiguous bytes per instruction), converts int8 with the byte-permute
// magic-number trick, and multiplies against activations staged once per CTA
// in shared memory (optionally RMS-normalised on the way in). The shared
// layout is swizzled so the 16-byte activation reads of a warp hit 32
// distinct banks. A persistent grid (one wave of resident CTAs) walks row
// groups so the activation staging cost is paid once per CTA, not once per
// row group. A warp holds a whole row group's weights in registers (K <= 3072
// for one row per warp): all of its loads are in flight at once, and the
// first group's are issued before griddepcontrol.wait.
// Epilogues: scale, residual add, SwiGLU over interleaved (gate, up) rows,
// and a fused argmax for the LM head (orderable 64-bit key, atomicMax).
#include <algorithm>

#include "common.cuh"
#include "kernels.h"

namespace zc {

namespace {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / kWarp;
constexpr size_t kMaxSmem = 200 * 1024;  // activation staging: 8 rows of K = 6400, 1 row of K = 51200

int padded_rows(int N) { return N <= 1 ? 1 : N <= 2 ? 2 : N <= 4 ? 4 : 8; }

// Position of activation k in the swizzled shared row. int8 lanes read 16
// consecutive k (four float4 groups); bf16 lanes read 8 (two groups).
template <int WK>
__device__ __forceinline__ int swz(int k) {
    if constexpr (WK == kWQ8) {
        return (k & ~15) | (((((k >> 2) & 3) + ((k >> 5) & 3)) & 3) << 2) | (k & 3);
    } else {
        return (k & ~7) | (((((k >> 2) & 1) + ((k >> 5) & 1)) & 1) << 2) | (k & 3);
    }
}


template <int WK, int NB, int R, int EPI>
__global__ void __launch_bounds__(kThreads, NB == 1 ? 4 : 1) gemv_kernel(LinearArgs a) {
    static_assert(EPI != kEpiSwiGLU || R % 2 == 0, "SwiGLU needs (gate, up) row pairs in one unit");
    extern __shared__ float xs[];  // [NB][K] swizzled
    __shared__ float red[kWarps];
    __shared__ unsigned long long best_s[kWarps][NB];
    const int K = a.K;
    const int warp = threadIdx.x / kWarp, lane = threadIdx.x % kWarp;

    constexpr int kElems = WK == kWQ8 ? 16 : 8;     // k values per 16-byte load
    const int row_bytes = WK == kWQ8 ? K : 2 * K;
    const int iters = K / (kElems * kWarp);          // K is a multiple of 512 (int8) / 256 (bf16)
    const int groups = (a.M + R - 1) / R;
    const char* wbase = reinterpret_cast<const char*>(a.w);
    const int g_first = blockIdx.x * kWarps + warp;
    prefetch_l2_ranges(a.pf);

    // A row group of up to kHeld 16-byte loads per lane is read whole into
    // registers, every load in flight at once; the first group's loads are
    // issued before griddepcontrol.wait (the weights do not depend on the
    // previous kernel), so only the activations are read after it.
    constexpr int kHeld = R >= 4 ? 8 : 6;
    constexpr int kMaxIt = kHeld / R;
    const bool held = iters <= kMaxIt;
    uint4 wv[kMaxIt][R];
    auto load_group = [&](int g) {
        const int r0 = g * R;
#pragma unroll
        for (int it = 0; it < kMaxIt; ++it) {
            if (it < iters) {
                const int k0 = it * kElems * kWarp + lane * kElems;
#pragma unroll
                for (int r = 0; r < R; ++r) {
                    const int row = min(r0 + r, a.M - 1);
                    wv[it][r] = ldg_stream(wbase + (size_t)row * row_bytes + (size_t)k0 * (WK == kWQ8 ? 1 : 2));
                }
            }
        }
    };
    if (held) {
        if (g_first < groups) load_group(g_first);
    } else {
        // pull this warp's first row group toward L2 while the previous kernel finishes
        const int r0 = g_first * R;
        for (int r = 0; r < R && r0 + r < a.M; ++r)
            for (int off = lane * 128; off < row_bytes; off += kWarp * 128) prefetch_l2(wbase + (size_t)(r0 + r) * row_bytes + off);
    }
    // the first row group's scales (weights: before the wait) and residuals
    // (after it, issued with the staging loads) are in registers before the
    // products finish, so the epilogue waits for no load
    float sc_first[R];
#pragma unroll
    for (int r = 0; r < R; ++r) {
        const int row = min(g_first * R + r, a.M - 1);
        sc_first[r] = (a.scale && g_first < groups) ? __ldg(a.scale + row) : 1.0f;
    }
    pdl_wait();
    float rs_first[R][NB];
    if constexpr (EPI == kEpiResid) {
#pragma unroll
        for (int b = 0; b < NB; ++b)
#pragma unroll
            for (int r = 0; r < R; ++r) {
                const int row = min(g_first * R + r, a.M - 1);
                rs_first[r][b] = (g_first < groups && b < a.N && lane == b) ? a.resid[(size_t)b * a.ldy + row] : 0.0f;
            }
    }

    // ---- stage activations: every row at once, kWpr warps per row, so the
    // staging latency does not grow with the number of rows (NB <= kWarps).
    // RMSNorm (ops.zig:49-67) is a per-row positive scale, so it is factored
    // out of the dot product: the staged row is w * x, the sum of squares is
    // reduced in the same pass, and inv multiplies each output at the end
    // (one barrier instead of two)
    constexpr int kWpr = kWarps / NB;
    {
        const int b = warp / kWpr, part = warp % kWpr;
        const int t0 = part * kWarp + lane;
        constexpr int nthr = kWpr * kWarp;
        const bool live = b < NB && b < a.N;
        const float* xr = a.x + (size_t)(live ? b : 0) * a.ldx;
        float ss = 0.0f;
        if (b < NB) {
            // four consecutive k stay together under swz, so whole float4s move
            // (x rows are 16-byte aligned: ldx and K are multiples of 4)
            if (live) {
                for (int k = 4 * t0; k < K; k += 4 * nthr) {
                    const float4 v = *reinterpret_cast<const float4*>(xr + k);
                    ss += v.x * v.x;
                    ss += v.y * v.y;
                    ss += v.z * v.z;
                    ss += v.w * v.w;
                    float4 o = v;
                    if (a.norm_w) {
                        const float4 w = __ldg(reinterpret_cast<const float4*>(a.norm_w + k));
                        o = make_float4(__fmul_rn(w.x, v.x), __fmul_rn(w.y, v.y), __fmul_rn(w.z, v.z), __fmul_rn(w.w, v.w));
                    }
                    *reinterpret_cast<float4*>(xs + b * K + swz<WK>(k)) = o;
                }
            } else {
                for (int k = 4 * t0; k < K; k += 4 * nthr)
                    *reinterpret_cast<float4*>(xs + b * K + k) = make_float4(0.f, 0.f, 0.f, 0.f);
            }
        }
        if (a.norm_w) {
            ss = warp_sum(ss);
            if (lane == 0) red[warp] = ss;
        }
    }
    __syncthreads();
    float inv_b[NB];  // RMSNorm scale of each row (1 without a norm)
#pragma unroll
    for (int b = 0; b < NB; ++b) {
        inv_b[b] = 1.0f;
        if (a.norm_w) {
            float tot = 0.0f;
#pragma unroll
            for (int w = 0; w < kWpr; ++w) tot += red[b * kWpr + w];
            inv_b[b] = 1.0f / sqrtf(tot / (float)K + a.eps);
        }
    }

    // the next kernel may launch once the activations are staged: its weight
    // loads then do not compete with this kernel's (batch 1: 0.837 -> 0.808 ms/token)
    pdl_launch_dependents();
    unsigned long long best[NB];
#pragma unroll
    for (int b = 0; b < NB; ++b) best[b] = 0ull;

    // acc[r][b] += W[r0 + r][k0 .. k0 + kElems) . x[b][same]: four k at a
    // time, converted once for every row, each activation float4 read once
    // from shared memory for all R weight rows
    // One activation row: two accumulators per weight row (even and odd
    // groups of four k), which halves the dependent FMA chain of a lane.
    constexpr int kAcc = NB == 1 ? 2 : 1;
    auto dot_chunk = [&](const uint4 (&wr)[R], int k0, float (&acc2)[kAcc][R][NB]) {
#pragma unroll
        for (int q = 0; q < kElems / 4; ++q) {
            float (&acc)[R][NB] = acc2[q % kAcc];
            float w[R][4];
#pragma unroll
            for (int r = 0; r < R; ++r) {
                if constexpr (WK == kWQ8) {
                    const uint32_t word = q == 0 ? wr[r].x : q == 1 ? wr[r].y : q == 2 ? wr[r].z : wr[r].w;
                    i8x4_to_f32(word, w[r][0], w[r][1], w[r][2], w[r][3]);
                } else {
                    const uint32_t lo = q == 0 ? wr[r].x : wr[r].z, hi = q == 0 ? wr[r].y : wr[r].w;
                    w[r][0] = bf16lo(lo); w[r][1] = bf16hi(lo);
                    w[r][2] = bf16lo(hi); w[r][3] = bf16hi(hi);
                }
            }
#pragma unroll
            for (int b = 0; b < NB; ++b) {
                const float4 xv = *reinterpret_cast<const float4*>(xs + b * K + swz<WK>(k0 + 4 * q));
#pragma unroll
                for (int r = 0; r < R; ++r) {
                    acc[r][b] = fmaf(w[r][0], xv.x, acc[r][b]);
                    acc[r][b] = fmaf(w[r][1], xv.y, acc[r][b]);
                    acc[r][b] = fmaf(w[r][2], xv.z, acc[r][b]);
                    acc[r][b] = fmaf(w[r][3], xv.w, acc[r][b]);
                }
            }
        }
    };

    for (int g = g_first; g < groups; g += gridDim.x * kWarps) {
        const int r0 = g * R;
        float accs[kAcc][R][NB];
#pragma unroll
        for (int i = 0; i < kAcc; ++i)
#pragma unroll
            for (int r = 0; r < R; ++r)
#pragma unroll
                for (int b = 0; b < NB; ++b) accs[i][r][b] = 0.0f;

        if (held) {
            if (g != g_first) load_group(g);
#pragma unroll
            for (int it = 0; it < kMaxIt; ++it)
                if (it < iters) dot_chunk(wv[it], it * kElems * kWarp + lane * kElems, accs);
        } else {
            // two chunks in flight: the next chunk's loads are issued before
            // this one's products
            auto load_chunk = [&](int it, uint4 (&wr)[R]) {
                const int k0 = it * kElems * kWarp + lane * kElems;
#pragma unroll
                for (int r = 0; r < R; ++r) {
                    const int row = min(r0 + r, a.M - 1);
                    wr[r] = ldg_stream(wbase + (size_t)row * row_bytes + (size_t)k0 * (WK == kWQ8 ? 1 : 2));
                }
            };
            uint4 cur[R], nxt[R];
            load_chunk(0, cur);
            for (int it = 0; it < iters; ++it) {
                if (it + 1 < iters) load_chunk(it + 1, nxt);
                dot_chunk(cur, it * kElems * kWarp + lane * kElems, accs);
#pragma unroll
                for (int r = 0; r < R; ++r) cur[r] = nxt[r];
            }
        }
        float acc[R][NB];
#pragma unroll
        for (int r = 0; r < R; ++r)
#pragma unroll
            for (int b = 0; b < NB; ++b) {
                float v = accs[0][r][b];
#pragma unroll
                for (int i = 1; i < kAcc; ++i) v += accs[i][r][b];
                acc[r][b] = warp_sum(v);
            }

        // every lane holds the sums; lane b (< NB) writes batch row b
#pragma unroll
        for (int b = 0; b < NB; ++b) {
            if (b >= a.N) break;
#pragma unroll
            for (int r = 0; r < R; ++r) {
                const int row = r0 + r;
                if (row >= a.M) break;
                const bool first = g == g_first;
                const float s = first ? sc_first[r] : (a.scale ? a.scale[row] : 1.0f);
                const float val = __fmul_rn(__fmul_rn(acc[r][b], inv_b[b]), s);
                if constexpr (EPI == kEpiSwiGLU) {
                    if ((r & 1) == 1 && lane == b) {
                        const float sg = first ? sc_first[r - 1] : (a.scale ? a.scale[row - 1] : 1.0f);
                        const float gate = __fmul_rn(__fmul_rn(acc[r - 1][b], inv_b[b]), sg);
                        a.y[(size_t)b * a.ldy + (row >> 1)] = __fmul_rn(silu(gate), val);
                    }
                } else if constexpr (EPI == kEpiResid) {
                    if (lane == b) {
                        const float rs = first ? rs_first[r][b] : a.resid[(size_t)b * a.ldy + row];
                        a.y[(size_t)b * a.ldy + row] = __fadd_rn(rs, val);
                    }
                } else if constexpr (EPI == kEpiArgmax) {
                    if (lane == b && a.y) a.y[(size_t)b * a.ldy + row] = val;
                    const unsigned long long key = argmax_key(val, (uint32_t)row);
                    best[b] = key > best[b] ? key : best[b];
                } else {
                    if (lane == b) a.y[(size_t)b * a.ldy + row] = val;
                }
            }
        }
    }

    if constexpr (EPI == kEpiArgmax) {
        if (lane == 0)
#pragma unroll
            for (int b = 0; b < NB; ++b) best_s[warp][b] = best[b];
        __syncthreads();
        if (threadIdx.x < a.N) {
            unsigned long long m = 0ull;
            for (int w = 0; w < kWarps; ++w) m = best_s[w][threadIdx.x] > m ? best_s[w][threadIdx.x] : m;
            if (m) atomicMax(a.argmax_keys + threadIdx.x, m);
        }
    }
}

template <int WK, int NB, int R>
void launch_nb(const LinearArgs& a, cudaStream_t st) {
    const size_t smem = (size_t)NB * a.K * sizeof(float);
    const int groups = (a.M + R - 1) / R;
    auto pick = [&](auto kern) {
        // resident CTAs per SM (threads, registers, shared memory): the grid
        // never exceeds one wave, and warps loop over the remaining row groups
        int per_sm = 0;
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kThreads, smem) != cudaSuccess || per_sm < 1)
            per_sm = 1;
        const int want = (groups + kWarps - 1) / kWarps;
        launch_pdl(kern, std::min(want, per_sm * device_sm_count()), kThreads, smem, st, a);
    };
    switch (a.epi) {
        case kEpiResid: pick(gemv_kernel<WK, NB, R, kEpiResid>); break;
        case kEpiSwiGLU:
            if constexpr (R % 2 == 0) pick(gemv_kernel<WK, NB, R, kEpiSwiGLU>);
            break;
        case kEpiArgmax: pick(gemv_kernel<WK, NB, R, kEpiArgmax>); break;
        default: pick(gemv_kernel<WK, NB, R, kEpiNone>); break;
    }
}

template <int WK>
void launch_wk(const LinearArgs& a, cudaStream_t st) {
    // one activation row: one weight row per warp (most CTAs, shortest chain),
    // two for SwiGLU, whose (gate, up) rows must meet in one warp
    if (a.N <= 1 && a.epi == kEpiSwiGLU) launch_nb<WK, 1, 2>(a, st);
    else if (a.N <= 1) launch_nb<WK, 1, 1>(a, st);
    else if (a.N <= 2) launch_nb<WK, 2, 4>(a, st);
    else if (a.N <= 4) launch_nb<WK, 4, 4>(a, st);
    else launch_nb<WK, 8, 4>(a, st);
}

template <int WK, int NB, int R>
void prepare_nb() {
    configure_kernel((const void*)gemv_kernel<WK, NB, R, kEpiNone>, kMaxSmem);
    configure_kernel((const void*)gemv_kernel<WK, NB, R, kEpiResid>, kMaxSmem);
    if constexpr (R % 2 == 0) configure_kernel((const void*)gemv_kernel<WK, NB, R, kEpiSwiGLU>, kMaxSmem);
    configure_kernel((const void*)gemv_kernel<WK, NB, R, kEpiArgmax>, kMaxSmem);
}

}  // namespace

bool gemv_fits(int N, int K) { return N >= 1 && N <= 8 && (size_t)padded_rows(N) * K * sizeof(float) <= kMaxSmem; }

void prepare_gemv_kernels() {
    prepare_nb<kWQ8, 1, 1>(); prepare_nb<kWQ8, 1, 2>(); prepare_nb<kWQ8, 2, 4>(); prepare_nb<kWQ8, 4, 4>(); prepare_nb<kWQ8, 8, 4>();
    prepare_nb<kWBF16, 1, 1>(); prepare_nb<kWBF16, 1, 2>(); prepare_nb<kWBF16, 2, 4>(); prepare_nb<kWBF16, 4, 4>(); prepare_nb<kWBF16, 8, 4>();
}

void launch_gemv(const LinearArgs& a, cudaStream_t st) {
    if (a.wkind == kWQ8) launch_wk<kWQ8>(a, st);
    else launch_wk<kWBF16>(a, st);
}

}  // namespace zc
