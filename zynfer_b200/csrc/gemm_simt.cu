// CUDA-core tiled GEMM for many activation rows: Y[n, m] = (sum_k W[m, k] X[n, k]) * scale[m]
// with W int8 (per-row scale) or bf16, X and Y f32 token-major. Same epilogues
// as the GEMV. Exact f32 products (int8 and bf16 widen exactly), f32 FMA
// accumulation. Used for prefill and for decode batches above 8 rows.
#include <algorithm>

#include "common.cuh"
#include "kernels.h"

namespace zc {

namespace {

constexpr int BM = 128, BN = 64, BK = 32, THREADS = 256;
constexpr int WPAD = BM + 4, XPAD = BN + 4;


template <int WK, int EPI>
__global__ void __launch_bounds__(THREADS) gemm_simt_kernel(LinearArgs a) {
    __shared__ __align__(16) float Ws[BK][WPAD];
    __shared__ __align__(16) float Xs[BK][XPAD];
    __shared__ unsigned long long best_s[BN];
    pdl_launch_dependents();
    pdl_wait();
    const int tid = threadIdx.x;
    const int tx = tid % 16, ty = tid / 16;
    const int m0 = blockIdx.x * BM, n0 = blockIdx.y * BN;
    const char* wb = reinterpret_cast<const char*>(a.w);
    const int esz = WK == kWQ8 ? 1 : 2;

    if constexpr (EPI == kEpiArgmax) {
        if (tid < BN) best_s[tid] = 0ull;
    }

    float acc[8][4];
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = 0.0f;

    // per-thread load slots
    const int wrow = tid / 2, wk = (tid % 2) * 16;  // 16 k of one weight row
    const int xrow = tid / 4, xk = (tid % 4) * 8;   // 8 k of one activation row

    for (int k0 = 0; k0 < a.K; k0 += BK) {
        float wv[16];
        {
            const int m = min(m0 + wrow, a.M - 1);
            const char* p = wb + ((size_t)m * a.K + k0 + wk) * esz;
            if constexpr (WK == kWQ8) {
                const uint4 u = *reinterpret_cast<const uint4*>(p);
                i8x4_to_f32(u.x, wv[0], wv[1], wv[2], wv[3]);
                i8x4_to_f32(u.y, wv[4], wv[5], wv[6], wv[7]);
                i8x4_to_f32(u.z, wv[8], wv[9], wv[10], wv[11]);
                i8x4_to_f32(u.w, wv[12], wv[13], wv[14], wv[15]);
            } else {
                const uint4 u0 = *reinterpret_cast<const uint4*>(p);
                const uint4 u1 = *reinterpret_cast<const uint4*>(p + 16);
                const uint32_t w32[8] = {u0.x, u0.y, u0.z, u0.w, u1.x, u1.y, u1.z, u1.w};
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    wv[2 * i] = bf16lo(w32[i]);
                    wv[2 * i + 1] = bf16hi(w32[i]);
                }
            }
        }
        float xv[8];
        {
            const int n = n0 + xrow;
            if (n < a.N) {
                const float* p = a.x + (size_t)n * a.ldx + k0 + xk;
                const float4 v0 = *reinterpret_cast<const float4*>(p);
                const float4 v1 = *reinterpret_cast<const float4*>(p + 4);
                xv[0] = v0.x; xv[1] = v0.y; xv[2] = v0.z; xv[3] = v0.w;
                xv[4] = v1.x; xv[5] = v1.y; xv[6] = v1.z; xv[7] = v1.w;
            } else {
#pragma unroll
                for (int i = 0; i < 8; ++i) xv[i] = 0.0f;
            }
        }
        __syncthreads();
#pragma unroll
        for (int i = 0; i < 16; ++i) Ws[wk + i][wrow] = wv[i];
#pragma unroll
        for (int i = 0; i < 8; ++i) Xs[xk + i][xrow] = xv[i];
        __syncthreads();
#pragma unroll
        for (int k = 0; k < BK; ++k) {
            const float4 a0 = *reinterpret_cast<const float4*>(&Ws[k][tx * 8]);
            const float4 a1 = *reinterpret_cast<const float4*>(&Ws[k][tx * 8 + 4]);
            const float4 b0 = *reinterpret_cast<const float4*>(&Xs[k][ty * 4]);
            const float av[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
            const float bv[4] = {b0.x, b0.y, b0.z, b0.w};
#pragma unroll
            for (int i = 0; i < 8; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
        }
    }

    // epilogue
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const int n = n0 + ty * 4 + j;
        if (n >= a.N) continue;
        float out[8];
        unsigned long long best = 0ull;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int m = m0 + tx * 8 + i;
            const float s = (a.scale && m < a.M) ? a.scale[m] : 1.0f;
            out[i] = __fmul_rn(acc[i][j], s);
        }
        if constexpr (EPI == kEpiSwiGLU) {
            const int mj = (m0 + tx * 8) / 2;
            float* yp = a.y + (size_t)n * a.ldy + mj;
#pragma unroll
            for (int p = 0; p < 4; ++p)
                if (m0 + tx * 8 + 2 * p + 1 < a.M) yp[p] = __fmul_rn(silu(out[2 * p]), out[2 * p + 1]);
        } else {
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const int m = m0 + tx * 8 + i;
                if (m >= a.M) break;
                const size_t o = (size_t)n * a.ldy + m;
                if constexpr (EPI == kEpiResid) {
                    a.y[o] = __fadd_rn(a.resid[o], out[i]);
                } else if constexpr (EPI == kEpiArgmax) {
                    if (a.y) a.y[o] = out[i];
                    const unsigned long long key = argmax_key(out[i], (uint32_t)m);
                    best = key > best ? key : best;
                } else {
                    a.y[o] = out[i];
                }
            }
        }
        if constexpr (EPI == kEpiArgmax) {
            if (best) atomicMax(&best_s[ty * 4 + j], best);
        }
    }
    if constexpr (EPI == kEpiArgmax) {
        __syncthreads();
        if (tid < BN && n0 + tid < a.N && best_s[tid]) atomicMax(a.argmax_keys + n0 + tid, best_s[tid]);
    }
}

template <int WK>
void launch_wk(const LinearArgs& a, cudaStream_t st) {
    dim3 grid((a.M + BM - 1) / BM, (a.N + BN - 1) / BN);
    switch (a.epi) {
        case kEpiResid: launch_pdl(gemm_simt_kernel<WK, kEpiResid>, grid, THREADS, 0, st, a); break;
        case kEpiSwiGLU: launch_pdl(gemm_simt_kernel<WK, kEpiSwiGLU>, grid, THREADS, 0, st, a); break;
        case kEpiArgmax: launch_pdl(gemm_simt_kernel<WK, kEpiArgmax>, grid, THREADS, 0, st, a); break;
        default: launch_pdl(gemm_simt_kernel<WK, kEpiNone>, grid, THREADS, 0, st, a); break;
    }
}

}  // namespace

void prepare_gemm_simt_kernels() {
    configure_kernel((const void*)gemm_simt_kernel<kWQ8, kEpiNone>, 0);
    configure_kernel((const void*)gemm_simt_kernel<kWQ8, kEpiResid>, 0);
    configure_kernel((const void*)gemm_simt_kernel<kWQ8, kEpiSwiGLU>, 0);
    configure_kernel((const void*)gemm_simt_kernel<kWQ8, kEpiArgmax>, 0);
    configure_kernel((const void*)gemm_simt_kernel<kWBF16, kEpiNone>, 0);
    configure_kernel((const void*)gemm_simt_kernel<kWBF16, kEpiResid>, 0);
    configure_kernel((const void*)gemm_simt_kernel<kWBF16, kEpiSwiGLU>, 0);
    configure_kernel((const void*)gemm_simt_kernel<kWBF16, kEpiArgmax>, 0);
}

void launch_gemm_simt(const LinearArgs& a, cudaStream_t st) {
    if (a.wkind == kWQ8) launch_wk<kWQ8>(a, st);
    else launch_wk<kWBF16>(a, st);
}

}  // namespace zc
