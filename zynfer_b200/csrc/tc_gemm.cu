// Tensor-core (tcgen05 / TMEM / TMA) weight-only linear for sm_100a:
//   Y[t, m] = (sum_k W[m, k] X[t, k]) * scale[m]      (matvecQ8, src/backends/cpu/ops.zig:181-197)
//
// The weight tile is the MMA's A operand (M = 128 output rows per CTA, the
// "swap-AB" form: batch rows ride on N), streamed HBM -> shared memory by TMA
// with the 128-byte swizzle and fed to tcgen05.mma without any conversion.
//
// int8 weights (kind::i8, s32 accumulators in TMEM): every activation row is
// written as a 22-bit fixed-point integer v = rint(x * 2^(22-e)) with a
// per-row power-of-two scale 2^e >= max|x|, split into three signed int8
// digits v = d0 2^16 + d1 2^8 + d2. The three digit planes are stacked along
// N, so one MMA computes sum_k q[m,k] d_p[t,k] exactly in s32 for p = 0,1,2;
// the epilogue recombines them exactly in 64-bit integers and applies
// 2^(e-22) * scale[m] with one f32 rounding. The only approximation is the
// 22-bit fixed point of each activation (error <= 2^-23 max|x| per element),
// below f32 accumulation noise.
//
// bf16 weights (kind::f16, f32 accumulators): activations split into
// hi = bf16(x) and lo = bf16(x - hi) planes (x = hi + lo to 2^-16 relative);
// the weights are exact bf16, so the product is f32-accumulate grade.
//
// Persistent and warp-specialised (320 threads, one CTA per SM walking the
// (M tile, N tile, K split) units): warp 0 issues TMA loads, warp 1 owns TMEM
// and issues MMAs (one elected lane), warps 2..9 drain TMEM (two warps per
// 32-lane quarter, alternate 16-token chunks) and run the epilogue. TMEM holds
// two accumulators so the epilogue of one unit overlaps the loads and MMAs of
// the next. Shared-memory stages are recycled through mbarriers (full: TMA
// transaction bytes; empty: tcgen05.commit). No multicast anywhere. Every wait
// is bounded and reports through the device error word. When there are too
// few (M, N) tiles to fill the GPU, K is split: each unit stores its exact
// 64-bit partial values with plain stores and the last unit of a tile to
// finish sums them in split order (deterministic) before the epilogue.
#include <cuda.h>

#include <algorithm>

#include "common.cuh"
#include "kernels.h"
#include "tc_gemm.h"

namespace zc {

namespace {

constexpr int kTcThreads = 320;  // warp 0 TMA, warp 1 MMA, warps 2..9 epilogue
constexpr int kBM = 128;      // weight rows per CTA (MMA M)
constexpr int kKB = 128;      // bytes of K per stage (one 128-byte swizzle atom)

// ---------------------------------------------------------------- PTX

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::
            "r"(smem_addr(dst)),
        "l"(map), "r"(x), "r"(y), "r"(smem_addr(bar))
        : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// K-major operand, 128-byte swizzle: 8-row groups of 1024 bytes (SBO), version 1.
__device__ __forceinline__ uint64_t sdesc_sw128(uint32_t saddr) {
    uint64_t d = 0;
    d |= (uint64_t)((saddr & 0x3FFFFu) >> 4);
    d |= (uint64_t)1u << 16;
    d |= (uint64_t)(1024u >> 4) << 32;
    d |= (uint64_t)1u << 46;
    d |= (uint64_t)2u << 61;
    return d;
}

template <int WK>
__device__ __forceinline__ void mma_issue(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                          uint32_t accumulate) {
    if constexpr (WK == kWQ8) {
        asm volatile(
            "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
            "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
            "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
            : "memory");
    } else {
        asm volatile(
            "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
            "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
            "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
            : "memory");
    }
}

__device__ __forceinline__ void mma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     smem_addr(bar))
                 : "memory");
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ void epi_bar() { asm volatile("bar.sync 1, 256;" ::: "memory"); }

__device__ __forceinline__ float silu(float g) { return g * (1.0f / (1.0f + expf(-g))); }

template <int WK>
constexpr uint32_t make_idesc(int N) {
    // c_format [4,6): s32 = 2 / f32 = 1; a/b format [7,10)/[10,13): int8 signed = 1 / bf16 = 1;
    // K-major A and B; n_dim [17,23) = N >> 3; m_dim [24,29) = M >> 4.
    return (uint32_t)((WK == kWQ8 ? 2u : 1u) << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) |
           ((uint32_t)(kBM >> 4) << 24);
}

// ------------------------------------------------------------- kernel

template <int WK, int NT, int EPI>
__global__ void __launch_bounds__(kTcThreads, 1) tc_gemm_kernel(const __grid_constant__ CUtensorMap tmA,
                                                               const __grid_constant__ CUtensorMap tmB,
                                                               TcArgs a) {
    constexpr int P = WK == kWQ8 ? 3 : 2;  // activation planes
    constexpr int N = P * NT;              // MMA N
    constexpr int A_BYTES = kBM * kKB;
    constexpr int B_BYTES = N * kKB;
    constexpr int STAGE = A_BYTES + B_BYTES;
    constexpr int STAGES = (200 * 1024) / STAGE > 8 ? 8 : (200 * 1024) / STAGE;
    constexpr uint32_t ACC_COLS = N <= 32 ? 32 : (N <= 64 ? 64 : (N <= 128 ? 128 : 256));
    constexpr uint32_t TMEM_COLS = 2 * ACC_COLS;  // two accumulators: epilogue of one overlaps the next tile
    constexpr int KSTEP = 32;  // bytes of K per MMA instruction (i8: K = 32, bf16: K = 16)
    static_assert(NT % 16 == 0 && N <= 256 && STAGES >= 2, "tile shape");

    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * STAGE);
    uint64_t* empty = full + STAGES;
    uint64_t* tmem_full = empty + STAGES;   // [2]
    uint64_t* tmem_empty = tmem_full + 2;   // [2]
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tmem_empty + 2);
    __shared__ unsigned long long best_s[NT];
    __shared__ int last_flag;

    const int warp = threadIdx.x / kWarp, lane = threadIdx.x % kWarp;
    pdl_launch_dependents();
    const int m_tiles = a.M / kBM;
    const int n_tiles = (a.T + NT - 1) / NT;
    const int splits = a.splits;
    const int units = m_tiles * n_tiles * splits;
    const int nkb = a.K * (WK == kWQ8 ? 1 : 2) / kKB;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&tmem_full[b], 1);
            mbar_init(&tmem_empty[b], 8);  // one arrival per epilogue warp
        }
        fence_barrier_init();
    }
    if constexpr (EPI == kEpiArgmax) {
        for (int i = threadIdx.x; i < NT; i += kTcThreads) best_s[i] = 0ull;
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(tmem_slot)),
                     "r"(TMEM_COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    // unit u -> (m_tile, n_tile, split); consecutive CTAs stream consecutive weight tiles
    auto unit_coords = [&](int u, int& mt, int& nt, int& sp) {
        mt = u % m_tiles;
        nt = (u / m_tiles) % n_tiles;
        sp = u / (m_tiles * n_tiles);
    };
    auto kb_range = [&](int sp, int& kb0, int& kb1) {
        kb0 = (int)((long)sp * nkb / splits);
        kb1 = (int)((long)(sp + 1) * nkb / splits);
    };

    if (warp == 0) {
        if (lane == 0) {
            // ---------------- TMA producer: every k-block of every unit of this CTA.
            // The weights do not depend on the previous kernel, so the first
            // STAGES weight tiles are requested before griddepcontrol.wait; the
            // activation tiles (written by the previous kernel) only after it.
            int npre = 0;
            {
                int u = blockIdx.x;
                if (u < units) {
                    int mt, nt, sp, kb0, kb1;
                    unit_coords(u, mt, nt, sp);
                    kb_range(sp, kb0, kb1);
                    for (int kb = kb0; kb < kb1 && npre < STAGES; ++kb, ++npre) {
                        mbar_arrive_expect_tx(&full[npre], STAGE);
                        tma_load_2d(smem + npre * STAGE, &tmA, kb * (WK == kWQ8 ? kKB : kKB / 2), mt * kBM,
                                    &full[npre]);
                    }
                }
            }
            pdl_wait();
            int i = 0;
            bool alive = true;
            for (int u = blockIdx.x; u < units && alive; u += gridDim.x) {
                int mt, nt, sp, kb0, kb1;
                unit_coords(u, mt, nt, sp);
                kb_range(sp, kb0, kb1);
                for (int kb = kb0; kb < kb1; ++kb, ++i) {
                    const int s = i % STAGES, round = i / STAGES;
                    uint8_t* as = smem + s * STAGE;
                    uint8_t* bs = as + A_BYTES;
                    const int kx = kb * (WK == kWQ8 ? kKB : kKB / 2);
                    if (i >= npre) {
                        if (!mbar_wait_bounded(&empty[s], (uint32_t)((round & 1) ^ 1), a.err)) {
                            alive = false;
                            break;
                        }
                        mbar_arrive_expect_tx(&full[s], STAGE);
                        tma_load_2d(as, &tmA, kx, mt * kBM, &full[s]);
                    }
#pragma unroll
                    for (int p = 0; p < P; ++p)
                        tma_load_2d(bs + p * NT * kKB, &tmB, kx, p * a.t_pad + nt * NT, &full[s]);
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            // ---------------- MMA issuer
            constexpr uint32_t idesc = make_idesc<WK>(N);
            int i = 0, j = 0;
            bool alive = true;
            for (int u = blockIdx.x; u < units && alive; u += gridDim.x, ++j) {
                int mt, nt, sp, kb0, kb1;
                unit_coords(u, mt, nt, sp);
                kb_range(sp, kb0, kb1);
                const int acc = j & 1;
                if (!mbar_wait_bounded(&tmem_empty[acc], (uint32_t)(((j >> 1) & 1) ^ 1), a.err)) break;
                tc_fence_after();
                const uint32_t tmem_d = tmem_base + acc * ACC_COLS;
                for (int kb = kb0; kb < kb1; ++kb, ++i) {
                    const int s = i % STAGES, round = i / STAGES;
                    if (!mbar_wait_bounded(&full[s], (uint32_t)(round & 1), a.err)) {
                        alive = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t as = smem_addr(smem + s * STAGE);
                    const uint32_t bs = as + A_BYTES;
#pragma unroll
                    for (int kk = 0; kk < kKB / KSTEP; ++kk)
                        mma_issue<WK>(tmem_d, sdesc_sw128(as + kk * KSTEP), sdesc_sw128(bs + kk * KSTEP), idesc,
                                      (kb > kb0 || kk > 0) ? 1u : 0u);
                    mma_commit(&empty[s]);
                }
                mma_commit(&tmem_full[acc]);
            }
        }
    } else {
        // ---------------- epilogue (warps 2..9; TMEM lane quarter = warp % 4).
        // Reads the activations' row scales and the residual, written by
        // earlier kernels: wait for them first.
        pdl_wait();
        const int q = warp & 3;          // TMEM lane quarter
        const int h = (warp - 2) >> 2;   // which half of the 16-token chunks
        int j = 0;
        for (int u = blockIdx.x; u < units; u += gridDim.x, ++j) {
            int mt, nt, sp;
            unit_coords(u, mt, nt, sp);
            const int m0 = mt * kBM, n0 = nt * NT;
            const int acc = j & 1;
            const int row = m0 + q * 32 + lane;
            const bool ok = mbar_wait_bounded(&tmem_full[acc], (uint32_t)((j >> 1) & 1), a.err);
            tc_fence_after();
            const uint32_t tbase = tmem_base + acc * ACC_COLS + ((uint32_t)(q * 32) << 16);
            const float sc = (a.scale && row < a.M) ? a.scale[row] : 1.0f;
            const bool split_k = splits > 1;
            // Per (token, row) value of this unit's K range, exact: int8 digits
            // recombined in 64-bit integers; bf16 hi + lo planes summed in f64.
            auto tile_values = [&](int t0, long long (&v)[16]) {
                uint32_t r[P][16];
#pragma unroll
                for (int p = 0; p < P; ++p) tmem_ld16(tbase + p * NT + t0, r[p]);
                tmem_wait_ld();
#pragma unroll
                for (int jj = 0; jj < 16; ++jj) {
                    if constexpr (WK == kWQ8) {
                        v[jj] = (long long)(int)r[0][jj] * 65536ll + (long long)(int)r[1][jj] * 256ll +
                                (long long)(int)r[2][jj];
                    } else {
                        v[jj] = __double_as_longlong((double)__uint_as_float(r[0][jj]) +
                                                     (double)__uint_as_float(r[1][jj]));
                    }
                }
            };
            auto release_acc = [&]() {  // TMEM buffer free for the MMA of the unit after next
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&tmem_empty[acc]);
            };
            bool do_final = !split_k;
            long long* part = reinterpret_cast<long long*>(a.acc);
            if (split_k) {
                // store this unit's values (plain coalesced stores); the last unit
                // of the tile to finish sums the splits in split order
                for (int t0 = 16 * h; t0 < NT; t0 += 32) {
                    long long v[16];
                    tile_values(t0, v);
                    if (ok && row < a.M) {
#pragma unroll
                        for (int jj = 0; jj < 16; ++jj) {
                            const int t = n0 + t0 + jj;
                            if (t < a.T) part[((size_t)sp * kAccT + t) * a.M + row] = v[jj];
                        }
                    }
                }
                release_acc();
                __threadfence();
                epi_bar();
                if (threadIdx.x == 64) {
                    const unsigned prev = atomicAdd(a.counters + (size_t)nt * m_tiles + mt, 1u);
                    last_flag = prev == (unsigned)(splits - 1);
                }
                epi_bar();
                do_final = last_flag != 0;
                if (do_final) __threadfence();
            }
            if (do_final) {
                for (int t0 = 16 * h; t0 < NT; t0 += 32) {
                    long long v[16];
                    if (!split_k) {
                        tile_values(t0, v);
                    } else {
#pragma unroll
                        for (int jj = 0; jj < 16; ++jj) {
                            const int t = min(n0 + t0 + jj, a.T - 1);
                            long long si = 0;
                            double sd = 0.0;
                            for (int s = 0; s < splits; ++s) {
                                const long long e = __ldcg(part + ((size_t)s * kAccT + t) * a.M + row);
                                if constexpr (WK == kWQ8) si += e;
                                else sd += __longlong_as_double(e);
                            }
                            v[jj] = WK == kWQ8 ? si : __double_as_longlong(sd);
                        }
                    }
                    // every load of the chunk is issued before any store (the
                    // output may alias the residual, which blocks reordering)
                    float y[16], rs[16];
#pragma unroll
                    for (int jj = 0; jj < 16; ++jj) {
                        const int t = min(n0 + t0 + jj, a.T - 1);
                        if constexpr (WK == kWQ8) y[jj] = __ldg(a.xscale + t);
                        if constexpr (EPI == kEpiResid) rs[jj] = a.resid[(size_t)t * a.ldy + row];
                    }
#pragma unroll
                    for (int jj = 0; jj < 16; ++jj) {
                        if constexpr (WK == kWQ8) y[jj] = __fmul_rn(__fmul_rn(__ll2float_rn(v[jj]), y[jj]), sc);
                        else y[jj] = (float)__longlong_as_double(v[jj]);
                    }
                    if (!ok) continue;
#pragma unroll
                    for (int jj = 0; jj < 16; ++jj) {
                        const int t = n0 + t0 + jj;
                        const bool live = t < a.T && row < a.M;
                        if constexpr (EPI == kEpiSwiGLU) {
                            const float up = __shfl_xor_sync(0xFFFFFFFFu, y[jj], 1);
                            if (live && (lane & 1) == 0)
                                a.y[(size_t)t * a.ldy + (row >> 1)] = __fmul_rn(silu(y[jj]), up);
                        } else if constexpr (EPI == kEpiResid) {
                            if (live) a.y[(size_t)t * a.ldy + row] = __fadd_rn(rs[jj], y[jj]);
                        } else if constexpr (EPI == kEpiArgmax) {
                            if (live && a.y) a.y[(size_t)t * a.ldy + row] = y[jj];
                            // warp argmax over 32 rows with two redux.sync: the
                            // largest orderable value, then the lowest row among
                            // lanes holding it (key low word = ~row)
                            const unsigned long long key = live ? argmax_key(y[jj], (uint32_t)row) : 0ull;
                            const uint32_t hi = (uint32_t)(key >> 32);
                            const uint32_t mx = __reduce_max_sync(0xFFFFFFFFu, hi);
                            const uint32_t lo = __reduce_max_sync(0xFFFFFFFFu, hi == mx ? (uint32_t)key : 0u);
                            const unsigned long long best = ((unsigned long long)mx << 32) | lo;
                            if (lane == 0 && mx) atomicMax(&best_s[t0 + jj], best);
                        } else {
                            if (live) a.y[(size_t)t * a.ldy + row] = y[jj];
                        }
                    }
                }
                if (!split_k) release_acc();
                if constexpr (EPI == kEpiArgmax) {
                    epi_bar();
                    const int e = threadIdx.x - 64;  // 0 .. 255
                    for (int t = e; t < NT; t += 256) {
                        if (n0 + t < a.T && best_s[t]) atomicMax(a.argmax_keys + n0 + t, best_s[t]);
                        best_s[t] = 0ull;
                    }
                    epi_bar();
                }
                if (split_k && threadIdx.x == 64) a.counters[(size_t)nt * m_tiles + mt] = 0u;
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(TMEM_COLS)
                     : "memory");
    }
}


// --------------------------------------------------- activation planes

template <int WK>
__global__ void __launch_bounds__(256) prep_planes_kernel(PlanesArgs a) {
    pdl_launch_dependents();
    pdl_wait();
    const int t = blockIdx.x;
    const int K = a.K;
    const float* xr = a.x + (size_t)t * a.ldx;
    __shared__ float red[8];
    __shared__ float bcast;
    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    float inv = 1.0f;
    if (a.norm_w) {  // RMSNorm prologue (ops.zig:49-67)
        float acc = 0.0f;
        for (int k = threadIdx.x; k < K; k += 256) acc += xr[k] * xr[k];
        acc = warp_sum(acc);
        if (lane == 0) red[warp] = acc;
        __syncthreads();
        if (threadIdx.x == 0) {
            float tot = 0.0f;
            for (int w = 0; w < 8; ++w) tot += red[w];
            bcast = 1.0f / sqrtf(tot / (float)K + a.eps);
        }
        __syncthreads();
        inv = bcast;
    }
    auto val = [&](int k) -> float {
        const float v = xr[k];
        return a.norm_w ? __fmul_rn(__fmul_rn(a.norm_w[k], v), inv) : v;
    };
    if constexpr (WK == kWQ8) {
        float mx = 0.0f;
        for (int k = threadIdx.x; k < K; k += 256) mx = fmaxf(mx, fabsf(val(k)));
        mx = warp_max(mx);
        __syncthreads();
        if (lane == 0) red[warp] = mx;
        __syncthreads();
        if (threadIdx.x == 0) {
            float m = 0.0f;
            for (int w = 0; w < 8; ++w) m = fmaxf(m, red[w]);
            bcast = m;
        }
        __syncthreads();
        int e = 0;
        if (bcast > 0.0f) frexpf(bcast, &e);  // max|x| < 2^e
        if (threadIdx.x == 0) a.xscale[t] = ldexpf(1.0f, e - 22);  // exact power of two
        int8_t* p0 = reinterpret_cast<int8_t*>(a.planes) + (size_t)t * K;
        const size_t plane = (size_t)a.t_pad * K;
        for (int k = threadIdx.x; k < K; k += 256) {
            const int v = __float2int_rn(ldexpf(val(k), 22 - e));  // |v| <= 2^22
            const int d2 = (int)(int8_t)(v & 0xFF);
            const int v1 = (v - d2) >> 8;
            const int d1 = (int)(int8_t)(v1 & 0xFF);
            const int d0 = (v1 - d1) >> 8;  // |d0| <= 64
            p0[k] = (int8_t)d0;
            p0[plane + k] = (int8_t)d1;
            p0[2 * plane + k] = (int8_t)d2;
        }
    } else {
        uint16_t* p0 = reinterpret_cast<uint16_t*>(a.planes) + (size_t)t * K;
        const size_t plane = (size_t)a.t_pad * K;
        for (int k = threadIdx.x; k < K; k += 256) {
            const float v = val(k);
            const uint16_t hi = f32_to_bf16_rne(v);
            const float hif = __uint_as_float((uint32_t)hi << 16);
            p0[k] = hi;
            p0[plane + k] = f32_to_bf16_rne(__fsub_rn(v, hif));
        }
    }
}

template <int WK, int NT>
constexpr size_t tile_smem() {
    constexpr int P = WK == kWQ8 ? 3 : 2;
    constexpr int STAGE = kBM * kKB + P * NT * kKB;
    constexpr int STAGES = (200 * 1024) / STAGE > 8 ? 8 : (200 * 1024) / STAGE;
    return (size_t)STAGES * STAGE + 1024 + (2 * STAGES + 4) * 8 + 16;
}

template <int WK, int NT>
void prepare_tile() {
    configure_kernel((const void*)tc_gemm_kernel<WK, NT, kEpiNone>, tile_smem<WK, NT>());
    configure_kernel((const void*)tc_gemm_kernel<WK, NT, kEpiResid>, tile_smem<WK, NT>());
    configure_kernel((const void*)tc_gemm_kernel<WK, NT, kEpiSwiGLU>, tile_smem<WK, NT>());
    configure_kernel((const void*)tc_gemm_kernel<WK, NT, kEpiArgmax>, tile_smem<WK, NT>());
}

template <int WK, int NT, int EPI>
void launch_tile(const TcLaunch& L, cudaStream_t st) {
    constexpr size_t smem = tile_smem<WK, NT>();
    auto kern = tc_gemm_kernel<WK, NT, EPI>;
    // persistent: one CTA per SM (at most one per work unit) walks the units
    TcArgs args = L.args;
    args.splits = L.splits;
    const int units = (args.M / kBM) * ((args.T + NT - 1) / NT) * L.splits;
    const int grid = std::min(units, L.sms > 0 ? L.sms : 148);
    launch_pdl(kern, grid, kTcThreads, smem, st, *L.tmA, *L.tmB, args);
}

template <int WK, int NT>
void launch_epi(const TcLaunch& L, cudaStream_t st) {
    switch (L.args.epi) {
        case kEpiResid: launch_tile<WK, NT, kEpiResid>(L, st); break;
        case kEpiSwiGLU: launch_tile<WK, NT, kEpiSwiGLU>(L, st); break;
        case kEpiArgmax: launch_tile<WK, NT, kEpiArgmax>(L, st); break;
        default: launch_tile<WK, NT, kEpiNone>(L, st); break;
    }
}

}  // namespace

int tc_tile_tokens(int wkind, int T) {
    if (T <= 16) return 16;
    if (T <= 32) return 32;
    return (wkind == kWQ8 || T <= 64) ? 64 : 128;
}

void prepare_tc_kernels() {
    prepare_tile<kWQ8, 16>(); prepare_tile<kWQ8, 32>(); prepare_tile<kWQ8, 64>();
    prepare_tile<kWBF16, 16>(); prepare_tile<kWBF16, 32>(); prepare_tile<kWBF16, 64>(); prepare_tile<kWBF16, 128>();
    configure_kernel((const void*)prep_planes_kernel<kWQ8>, 0);
    configure_kernel((const void*)prep_planes_kernel<kWBF16>, 0);
}

void launch_prep_planes(const PlanesArgs& a, cudaStream_t st) {
    if (a.wkind == kWQ8) launch_pdl(prep_planes_kernel<kWQ8>, a.T, 256, 0, st, a);
    else launch_pdl(prep_planes_kernel<kWBF16>, a.T, 256, 0, st, a);
}

void launch_tc_gemm(const TcLaunch& L, cudaStream_t st) {
    const int nt = tc_tile_tokens(L.args.wkind, L.args.T);
    if (L.args.wkind == kWQ8) {
        switch (nt) {
            case 16: launch_epi<kWQ8, 16>(L, st); break;
            case 32: launch_epi<kWQ8, 32>(L, st); break;
            default: launch_epi<kWQ8, 64>(L, st); break;
        }
    } else {
        switch (nt) {
            case 16: launch_epi<kWBF16, 16>(L, st); break;
            case 32: launch_epi<kWBF16, 32>(L, st); break;
            case 64: launch_epi<kWBF16, 64>(L, st); break;
            default: launch_epi<kWBF16, 128>(L, st); break;
        }
    }
}

// ------------------------------------------------------ tensor maps

namespace {
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    if (!fn) {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    }
    return fn;
}
}  // namespace

bool make_tmap_k_major(CUtensorMap* map, const void* base, int wkind, uint64_t k_elems, uint64_t rows,
                       uint32_t box_rows) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return false;
    const uint32_t esz = wkind == kWQ8 ? 1 : 2;
    const cuuint64_t dims[2] = {k_elems, rows};
    const cuuint64_t strides[1] = {k_elems * esz};
    const cuuint32_t box[2] = {kKB / esz, box_rows};
    const cuuint32_t estr[2] = {1, 1};
    const CUresult r = fn(map, wkind == kWQ8 ? CU_TENSOR_MAP_DATA_TYPE_UINT8 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2,
                          const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                          CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

int tc_splits(int M, int T, int K, int wkind, int sms) {
    const int nt = tc_tile_tokens(wkind, T);
    const int tiles = (M / kBM) * ((T + nt - 1) / nt);
    const int nkb = K * (wkind == kWQ8 ? 1 : 2) / kKB;
    // The last unit of a tile re-reads splits x NT partial values per row on
    // its critical path, so split only narrow tiles, and only a few ways.
    if (nt > 16) return 1;
    int s = (sms + tiles - 1) / tiles;
    s = std::min(s, std::max(1, nkb / 2));  // at least two K blocks per split
    return std::max(1, std::min(s, 4));
}

}  // namespace zc
