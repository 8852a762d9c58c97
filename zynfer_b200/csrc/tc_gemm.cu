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
// (M tile, N tile) units): warp 0 issues TMA loads, warp 1 owns TMEM
// and issues MMAs (one elected lane), warps 2..9 drain TMEM (two warps per
// 32-lane quarter, alternate 16-token chunks) and run the epilogue. TMEM holds
// two accumulators so the epilogue of one unit overlaps the loads and MMAs of
// the next. Shared-memory stages are recycled through mbarriers (full: TMA
// transaction bytes; empty: tcgen05.commit). No multicast anywhere. Every wait
// is bounded and reports through the device error word. When there are too
// few (M, N) tiles to fill the GPU, tc_cluster_kernel (below) splits K over a
// thread-block cluster instead.
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

// The same with an L2 evict-first policy: weight tiles, read once per decode
// step, should not push out the next linear's prefetched weights (batch 16 /
// 64: 0.5 % per step).
__device__ __forceinline__ void tma_load_2d_first(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
    uint64_t pol;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1, {%2, %3}], [%4], %5;" ::
            "r"(smem_addr(dst)),
        "l"(map), "r"(x), "r"(y), "r"(smem_addr(bar)), "l"(pol)
        : "memory");
}
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

    const int warp = threadIdx.x / kWarp, lane = threadIdx.x % kWarp;
    pdl_launch_dependents();
    prefetch_l2_ranges(a.pf);
    const int m_tiles = a.M / kBM;
    const int n_tiles = (a.T + NT - 1) / NT;
    const int units = m_tiles * n_tiles;
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

    // unit u -> (m_tile, n_tile); consecutive CTAs stream consecutive weight tiles
    auto unit_coords = [&](int u, int& mt, int& nt) {
        mt = u % m_tiles;
        nt = (u / m_tiles) % n_tiles;
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
                    int mt, nt;
                    unit_coords(u, mt, nt);
                    const int kb0 = 0, kb1 = nkb;
                    for (int kb = kb0; kb < kb1 && npre < STAGES; ++kb, ++npre) {
                        if (a.stall && npre == 0) continue;  // stage 0 never arrives
                        mbar_arrive_expect_tx(&full[npre], STAGE);
                        tma_load_2d_first(smem + npre * STAGE, &tmA, kb * (WK == kWQ8 ? kKB : kKB / 2), mt * kBM,
                                    &full[npre]);
                    }
                }
            }
            pdl_wait();
            int i = 0;
            bool alive = true;
            for (int u = blockIdx.x; u < units && alive; u += gridDim.x) {
                int mt, nt;
                unit_coords(u, mt, nt);
                const int kb0 = 0, kb1 = nkb;
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
                        tma_load_2d_first(as, &tmA, kx, mt * kBM, &full[s]);
                    }
                    if (a.stall && i == 0) continue;
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
                int mt, nt;
                unit_coords(u, mt, nt);
                const int kb0 = 0, kb1 = nkb;
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
            int mt, nt;
            unit_coords(u, mt, nt);
            const int m0 = mt * kBM, n0 = nt * NT;
            const int acc = j & 1;
            const int row = m0 + q * 32 + lane;
            const bool ok = mbar_wait_bounded(&tmem_full[acc], (uint32_t)((j >> 1) & 1), a.err);
            tc_fence_after();
            const uint32_t tbase = tmem_base + acc * ACC_COLS + ((uint32_t)(q * 32) << 16);
            const float sc = (a.scale && row < a.M) ? a.scale[row] : 1.0f;
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
            {
                for (int t0 = 16 * h; t0 < NT; t0 += 32) {
                    long long v[16];
                    tile_values(t0, v);
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
                release_acc();
                if constexpr (EPI == kEpiArgmax) {
                    // Keep the per-token best over every M tile this CTA takes and
                    // publish it once per N tile: one global atomic per token and
                    // CTA instead of one per tile (the vocabulary has ~1200 tiles).
                    const int un = u + (int)gridDim.x;
                    const bool flush = un >= units || (un / m_tiles) % n_tiles != nt;
                    if (flush) {
                        epi_bar();
                        const int e = threadIdx.x - 64;  // 0 .. 255
                        for (int t = e; t < NT; t += 256) {
                            if (n0 + t < a.T && best_s[t]) atomicMax(a.argmax_keys + n0 + t, best_s[t]);
                            best_s[t] = 0ull;
                        }
                        epi_bar();
                    }
                }
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


// ------------------------------------------------- cluster split-K kernel
//
// For linears with few (M, N) tiles (batched decode: M = 1024..6144 rows,
// T <= 64 tokens), one tile per thread-block cluster of S CTAs along K: CTA
// `rank` runs the same TMA -> tcgen05 pipeline over its K blocks
// [rank nkb / S, (rank + 1) nkb / S) into its own TMEM accumulator, writes
// the exact per-(token, row) values (int8: 64-bit integers; bf16: f64) to
// its shared memory, and after a cluster barrier reduces rows
// [r0(rank), r0(rank + 1)) of the tile by reading all S copies through
// distributed shared memory (ld.shared::cluster) in rank order. The result
// equals the single-CTA kernel's bit for bit. No global scratch, no atomics.

__device__ __forceinline__ uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
__device__ __forceinline__ uint32_t cluster_size() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_nctarank;" : "=r"(r));
    return r;
}
__device__ __forceinline__ void cluster_sync_all() {
    __syncwarp();  // the .aligned barrier wants every warp converged
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ uint32_t map_rank(uint32_t saddr, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
    return r;
}
__device__ __forceinline__ void ld_cluster_s64x2(uint32_t addr, long long& v0, long long& v1) {
    asm volatile("ld.shared::cluster.v2.s64 {%0, %1}, [%2];" : "=l"(v0), "=l"(v1) : "r"(addr) : "memory");
}
constexpr int kMaxCluster = 8;  // portable cluster size

// Rows [r0(rank), r0(rank + 1)) of the cluster's (M, N) tile: sum the S
// ranks' exact values (part: [NT][kBM] in every rank's shared memory) in rank
// order, then scale and store with the epilogue. Epilogue threads 64..319.
// Row scales 2^(e - 22) of the int8 digit planes come from xsc (shared
// memory) when given, else from a.xscale. Each thread takes U (token, row
// pair) items at a time and issues all their remote loads before any sum.
template <int WK, int NT, int EPI, int SMAX, int U>
__device__ __forceinline__ void cluster_reduce_items(const TcArgs& a, long long* part, int rank, int S, int mt,
                                                     int nt, const float* xsc) {
    const int e = threadIdx.x - 64;  // 0 .. 255
    const int r0 = 2 * ((rank * (kBM / 2)) / S), r1 = 2 * (((rank + 1) * (kBM / 2)) / S);
    const int pairs = (r1 - r0) / 2;
    const int n0 = nt * NT, m0 = mt * kBM;
    uint32_t rb[SMAX];  // every rank's partial tile in the cluster's shared window
#pragma unroll
    for (int s2 = 0; s2 < SMAX; ++s2) rb[s2] = s2 < S ? map_rank(smem_addr(part), (uint32_t)s2) : 0u;
    const int items = pairs * NT;
    for (int base = e; base < items; base += 256 * U) {
        long long x0[U][SMAX], x1[U][SMAX];
        // every load of the U items (remote partials, row scales, activation
        // scales, residuals) is issued before any store: the output may alias
        // the residual, so a load after a store could not be moved ahead of it
        float xs_u[U], sc_u[U][2];
        float2 rs_u[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int idx = min(base + 256 * u, items - 1);
            const int t = idx / pairs, row = r0 + 2 * (idx % pairs);
            const uint32_t off = (uint32_t)((t * kBM + row) * 8);
#pragma unroll
            for (int s2 = 0; s2 < SMAX; ++s2)
                if (s2 < S) ld_cluster_s64x2(rb[s2] + off, x0[u][s2], x1[u][s2]);
            const int tt = min(n0 + t, a.T - 1);
            if constexpr (WK == kWQ8) {
                xs_u[u] = xsc ? xsc[t] : __ldg(a.xscale + tt);
                sc_u[u][0] = __ldg(a.scale + m0 + row);
                sc_u[u][1] = __ldg(a.scale + m0 + row + 1);
            }
            if constexpr (EPI == kEpiResid)
                rs_u[u] = *reinterpret_cast<const float2*>(a.resid + (size_t)tt * a.ldy + m0 + row);
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int idx = base + 256 * u;
            if (idx >= items) break;
            const int t = idx / pairs, row = r0 + 2 * (idx % pairs);
            if (n0 + t >= a.T) continue;
            long long vi[2] = {0, 0};
            double vd[2] = {0.0, 0.0};
#pragma unroll
            for (int s2 = 0; s2 < SMAX; ++s2) {
                if (s2 >= S) break;
                if constexpr (WK == kWQ8) {
                    vi[0] += x0[u][s2];
                    vi[1] += x1[u][s2];
                } else {
                    vd[0] += __longlong_as_double(x0[u][s2]);
                    vd[1] += __longlong_as_double(x1[u][s2]);
                }
            }
            float y[2];
            if constexpr (WK == kWQ8) {
#pragma unroll
                for (int v = 0; v < 2; ++v) y[v] = __fmul_rn(__fmul_rn(__ll2float_rn(vi[v]), xs_u[u]), sc_u[u][v]);
            } else {
#pragma unroll
                for (int v = 0; v < 2; ++v) y[v] = (float)vd[v];
            }
            const size_t o = (size_t)(n0 + t) * a.ldy;
            if constexpr (EPI == kEpiSwiGLU) {
                a.y[o + ((m0 + row) >> 1)] = __fmul_rn(silu(y[0]), y[1]);
            } else if constexpr (EPI == kEpiResid) {
                *reinterpret_cast<float2*>(a.y + o + m0 + row) =
                    make_float2(__fadd_rn(rs_u[u].x, y[0]), __fadd_rn(rs_u[u].y, y[1]));
            } else {
                *reinterpret_cast<float2*>(a.y + o + m0 + row) = make_float2(y[0], y[1]);
            }
        }
    }
}
template <int WK, int NT, int EPI>
__device__ __forceinline__ void cluster_reduce_store(const TcArgs& a, long long* part, int rank, int S, int mt,
                                                     int nt, const float* xsc) {
    if (S <= 2) cluster_reduce_items<WK, NT, EPI, 2, 8>(a, part, rank, S, mt, nt, xsc);
    else if (S <= 4) cluster_reduce_items<WK, NT, EPI, 4, 4>(a, part, rank, S, mt, nt, xsc);
    else cluster_reduce_items<WK, NT, EPI, kMaxCluster, 2>(a, part, rank, S, mt, nt, xsc);
}

template <int WK, int NT, int EPI>
__global__ void __launch_bounds__(kTcThreads, 1) tc_cluster_kernel(const __grid_constant__ CUtensorMap tmA,
                                                                  const __grid_constant__ CUtensorMap tmB,
                                                                  TcArgs a) {
    constexpr int P = WK == kWQ8 ? 3 : 2;
    constexpr int N = P * NT;
    constexpr int A_BYTES = kBM * kKB;
    constexpr int B_BYTES = N * kKB;
    constexpr int STAGE = A_BYTES + B_BYTES;
    constexpr int STAGES = (200 * 1024) / STAGE > 8 ? 8 : (200 * 1024) / STAGE;
    constexpr uint32_t TMEM_COLS = N <= 32 ? 32 : (N <= 64 ? 64 : (N <= 128 ? 128 : 256));
    constexpr int KSTEP = 32;
    static_assert(NT % 16 == 0 && N <= 256 && STAGES >= 2, "tile shape");
    static_assert((size_t)NT * kBM * 8 <= (size_t)STAGES * STAGE, "partial tile must fit in the stages");
    static_assert(EPI != kEpiArgmax, "the cluster kernel has no argmax epilogue");

    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * STAGE);
    uint64_t* empty = full + STAGES;
    uint64_t* tmem_full = empty + STAGES;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tmem_full + 1);
    long long* part = reinterpret_cast<long long*>(smem);  // [NT][kBM], after the last MMA

    const int warp = threadIdx.x / kWarp, lane = threadIdx.x % kWarp;
    pdl_launch_dependents();
    prefetch_l2_ranges(a.pf);
    const int S = (int)cluster_size(), rank = (int)cluster_rank();
    const int m_tiles = a.M / kBM;
    const int tile = blockIdx.x / S;
    const int mt = tile % m_tiles, nt = tile / m_tiles;
    const int nkb = a.K * (WK == kWQ8 ? 1 : 2) / kKB;
    const int kb0 = (int)((long)rank * nkb / S), kb1 = (int)((long)(rank + 1) * nkb / S);

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        mbar_init(tmem_full, 1);
        fence_barrier_init();
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

    if (warp == 0) {
        if (lane == 0) {
            // weights first (they do not depend on the previous kernel), then the planes
            const int npre = min(STAGES, kb1 - kb0);
            for (int i = 0; i < npre; ++i) {
                mbar_arrive_expect_tx(&full[i], STAGE);
                tma_load_2d_first(smem + i * STAGE, &tmA, (kb0 + i) * (WK == kWQ8 ? kKB : kKB / 2), mt * kBM, &full[i]);
            }
            pdl_wait();
            for (int i = 0; kb0 + i < kb1; ++i) {
                const int kb = kb0 + i, s = i % STAGES, round = i / STAGES;
                uint8_t* as = smem + s * STAGE;
                uint8_t* bs = as + A_BYTES;
                const int kx = kb * (WK == kWQ8 ? kKB : kKB / 2);
                if (i >= npre) {
                    if (!mbar_wait_bounded(&empty[s], (uint32_t)((round & 1) ^ 1), a.err)) break;
                    mbar_arrive_expect_tx(&full[s], STAGE);
                    tma_load_2d_first(as, &tmA, kx, mt * kBM, &full[s]);
                }
#pragma unroll
                for (int p = 0; p < P; ++p) tma_load_2d(bs + p * NT * kKB, &tmB, kx, p * a.t_pad + nt * NT, &full[s]);
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            constexpr uint32_t idesc = make_idesc<WK>(N);
            for (int i = 0; kb0 + i < kb1; ++i) {
                const int s = i % STAGES, round = i / STAGES;
                if (!mbar_wait_bounded(&full[s], (uint32_t)(round & 1), a.err)) break;
                tc_fence_after();
                const uint32_t as = smem_addr(smem + s * STAGE);
                const uint32_t bs = as + A_BYTES;
#pragma unroll
                for (int kk = 0; kk < kKB / KSTEP; ++kk)
                    mma_issue<WK>(tmem_base, sdesc_sw128(as + kk * KSTEP), sdesc_sw128(bs + kk * KSTEP), idesc,
                                  (i > 0 || kk > 0) ? 1u : 0u);
                mma_commit(&empty[s]);
            }
            mma_commit(tmem_full);  // also fires when no MMA was issued
        }
    } else {
        // this CTA's exact values -> shared memory [t][row]
        const int q = warp & 3, h = (warp - 2) >> 2;
        const bool ok = mbar_wait_bounded(tmem_full, 0u, a.err);
        tc_fence_after();
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // stages were TMA / MMA operands
        const uint32_t tbase = tmem_base + ((uint32_t)(q * 32) << 16);
        const int row = q * 32 + lane;
        for (int t0 = 16 * h; t0 < NT; t0 += 32) {
            uint32_t r[P][16];
#pragma unroll
            for (int p = 0; p < P; ++p) tmem_ld16(tbase + p * NT + t0, r[p]);
            tmem_wait_ld();
#pragma unroll
            for (int jj = 0; jj < 16; ++jj) {
                long long v;
                if constexpr (WK == kWQ8) {
                    v = (long long)(int)r[0][jj] * 65536ll + (long long)(int)r[1][jj] * 256ll + (long long)(int)r[2][jj];
                } else {
                    v = __double_as_longlong((double)__uint_as_float(r[0][jj]) + (double)__uint_as_float(r[1][jj]));
                }
                part[(t0 + jj) * kBM + row] = ok ? v : 0ll;
            }
        }
        tc_fence_before();
    }
    cluster_sync_all();  // every rank's values are in its shared memory

    if (warp >= 2) {
        pdl_wait();  // residual and row scales come from earlier kernels
        cluster_reduce_store<WK, NT, EPI>(a, part, rank, S, mt, nt, nullptr);
    }
    tc_fence_before();
    cluster_sync_all();  // no rank leaves while another still reads its shared memory
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(TMEM_COLS)
                     : "memory");
    }
}

// --------------------------------------------------- activation planes

// One CTA per activation row, every value loaded once into registers
// (K <= kPrepMaxK): warp reductions give sum(x^2) (in the block order of sq4)
// and max|w x| (the
// RMSNorm scale is a positive constant and rounding keeps the order, so
// max |(w x) inv| = max|w x| * inv exactly), then the planes are written from
// the registers. RMSNorm as ops.zig:49-67: (w * x) * 1/sqrt(mean(x^2) + eps).
constexpr int kPrepThreads = 256;
constexpr int kPrepMaxK = kPlanesMaxK;
constexpr int kPrepVec = kPrepMaxK / (4 * kPrepThreads);  // float4 per thread
template <int WK>
__global__ void __launch_bounds__(kPrepThreads) prep_planes_kernel(PlanesArgs a) {
    pdl_launch_dependents();
    pdl_wait();
    __shared__ float red_bs[kPrepMaxK / 128], red_mx[kPrepThreads / kWarp];
    const int warp = threadIdx.x / kWarp, lane = threadIdx.x % kWarp;
    const int t = blockIdx.x;
    const int K = a.K;  // multiple of 128, <= kPrepMaxK
    const float* xr = a.x + (size_t)t * a.ldx;
    float4 v[kPrepVec], w[kPrepVec];
    float mx = 0.0f;
#pragma unroll
    for (int i = 0; i < kPrepVec; ++i) {
        const int k = 4 * (threadIdx.x + i * kPrepThreads);
        if (k < K) {
            v[i] = *reinterpret_cast<const float4*>(xr + k);
            w[i] = a.norm_w ? __ldg(reinterpret_cast<const float4*>(a.norm_w + k)) : make_float4(1.f, 1.f, 1.f, 1.f);
        } else {
            v[i] = make_float4(0.f, 0.f, 0.f, 0.f);
            w[i] = v[i];
        }
    }
#pragma unroll
    for (int i = 0; i < kPrepVec; ++i) {
        // thread (warp, lane) holds values 4 lane .. 4 lane + 3 of the 128-value block warp + 8 i
        const float bs = warp_sum(sq4(v[i]));
        if (lane == 0 && 4 * (threadIdx.x + i * kPrepThreads) < K) red_bs[warp + (kPrepThreads / kWarp) * i] = bs;
        const float4 p = a.norm_w ? make_float4(__fmul_rn(w[i].x, v[i].x), __fmul_rn(w[i].y, v[i].y),
                                                __fmul_rn(w[i].z, v[i].z), __fmul_rn(w[i].w, v[i].w))
                                  : v[i];
        mx = fmaxf(mx, fmaxf(fmaxf(fabsf(p.x), fabsf(p.y)), fmaxf(fabsf(p.z), fabsf(p.w))));
    }
    mx = warp_max(mx);
    if (lane == 0) red_mx[warp] = mx;
    __syncthreads();
    float ss = 0.0f;
    for (int kb = 0; kb < K / 128; ++kb) ss = __fadd_rn(ss, red_bs[kb]);  // blocks in k order
    mx = 0.0f;
#pragma unroll
    for (int i = 0; i < kPrepThreads / kWarp; ++i) mx = fmaxf(mx, red_mx[i]);
    float inv = 1.0f;
    if (a.norm_w) {
        inv = 1.0f / sqrtf(ss / (float)K + a.eps);
        mx = __fmul_rn(mx, inv);
    }
    auto val = [&](float wv, float xv) -> float { return a.norm_w ? __fmul_rn(__fmul_rn(wv, xv), inv) : xv; };
    const size_t plane = (size_t)a.t_pad * K;
    if constexpr (WK == kWQ8) {
        int e = 0;
        if (mx > 0.0f) frexpf(mx, &e);  // max|x| < 2^e
        if (threadIdx.x == 0) a.xscale[t] = ldexpf(1.0f, e - 22);  // exact power of two
        int8_t* p0 = reinterpret_cast<int8_t*>(a.planes) + (size_t)t * K;
#pragma unroll
        for (int i = 0; i < kPrepVec; ++i) {
            const int k = 4 * (threadIdx.x + i * kPrepThreads);
            if (k >= K) break;
            const float f[4] = {val(w[i].x, v[i].x), val(w[i].y, v[i].y), val(w[i].z, v[i].z), val(w[i].w, v[i].w)};
            uint32_t d0, d1, d2;
            digits4(f, e, d0, d1, d2);
            *reinterpret_cast<uint32_t*>(p0 + k) = d0;
            *reinterpret_cast<uint32_t*>(p0 + plane + k) = d1;
            *reinterpret_cast<uint32_t*>(p0 + 2 * plane + k) = d2;
        }
    } else {
        uint16_t* p0 = reinterpret_cast<uint16_t*>(a.planes) + (size_t)t * K;
#pragma unroll
        for (int i = 0; i < kPrepVec; ++i) {
            const int k = 4 * (threadIdx.x + i * kPrepThreads);
            if (k >= K) break;
            const float f[4] = {val(w[i].x, v[i].x), val(w[i].y, v[i].y), val(w[i].z, v[i].z), val(w[i].w, v[i].w)};
            ushort4 hi, lo;
            uint16_t* h = &hi.x;
            uint16_t* l = &lo.x;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                h[j] = f32_to_bf16_rne(f[j]);
                l[j] = f32_to_bf16_rne(__fsub_rn(f[j], __uint_as_float((uint32_t)h[j] << 16)));
            }
            *reinterpret_cast<ushort4*>(p0 + k) = hi;
            *reinterpret_cast<ushort4*>(p0 + plane + k) = lo;
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

template <int WK, int NT, int EPI>
void launch_cluster_tile(const TcLaunch& L, int S, cudaStream_t st) {
    constexpr size_t smem = tile_smem<WK, NT>();
    const TcArgs& args = L.args;
    const int tiles = (args.M / kBM) * ((args.T + NT - 1) / NT);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(tiles * S);
    cfg.blockDim = dim3(kTcThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = (unsigned)S;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    cudaLaunchKernelEx(&cfg, tc_cluster_kernel<WK, NT, EPI>, *L.tmA, *L.tmB, args);
}

template <int WK, int NT>
void launch_cluster_epi(const TcLaunch& L, int S, cudaStream_t st) {
    switch (L.args.epi) {
        case kEpiResid: launch_cluster_tile<WK, NT, kEpiResid>(L, S, st); break;
        case kEpiSwiGLU: launch_cluster_tile<WK, NT, kEpiSwiGLU>(L, S, st); break;
        default: launch_cluster_tile<WK, NT, kEpiNone>(L, S, st); break;
    }
}

template <int WK, int NT>
void prepare_cluster_tile() {
    configure_kernel((const void*)tc_cluster_kernel<WK, NT, kEpiNone>, tile_smem<WK, NT>());
    configure_kernel((const void*)tc_cluster_kernel<WK, NT, kEpiResid>, tile_smem<WK, NT>());
    configure_kernel((const void*)tc_cluster_kernel<WK, NT, kEpiSwiGLU>, tile_smem<WK, NT>());
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
    const TcArgs& args = L.args;
    const int units = (args.M / kBM) * ((args.T + NT - 1) / NT);
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

int tc_tile_tokens(int wkind, int M, int T) {
    if (T <= 16) return 16;
    if (T <= 32) return 32;
    if (wkind == kWQ8 || T <= 64) return 64;
    // bf16 with many tokens: 128-token tiles, unless they would leave more
    // than half the SMs idle (a 1024-row projection of 512 tokens: 32 tiles);
    // then 64-token tiles, which tc_cluster_size can also split along K
    return 2 * (M / kBM) * ((T + 127) / 128) <= device_sm_count() ? 64 : 128;
}

void prepare_tc_kernels() {
    prepare_cluster_tile<kWQ8, 16>(); prepare_cluster_tile<kWQ8, 32>(); prepare_cluster_tile<kWQ8, 64>();
    prepare_cluster_tile<kWBF16, 16>(); prepare_cluster_tile<kWBF16, 32>(); prepare_cluster_tile<kWBF16, 64>();
    prepare_tile<kWQ8, 16>(); prepare_tile<kWQ8, 32>(); prepare_tile<kWQ8, 64>();
    prepare_tile<kWBF16, 16>(); prepare_tile<kWBF16, 32>(); prepare_tile<kWBF16, 64>(); prepare_tile<kWBF16, 128>();
    configure_kernel((const void*)prep_planes_kernel<kWQ8>, 0);
    configure_kernel((const void*)prep_planes_kernel<kWBF16>, 0);
}

void launch_prep_planes(const PlanesArgs& a, cudaStream_t st) {
    if (a.wkind == kWQ8) launch_pdl(prep_planes_kernel<kWQ8>, a.T, kPrepThreads, 0, st, a);
    else launch_pdl(prep_planes_kernel<kWBF16>, a.T, kPrepThreads, 0, st, a);
}

void launch_tc_gemm(const TcLaunch& L, cudaStream_t st) {
    const int nt = tc_tile_tokens(L.args.wkind, L.args.M, L.args.T);
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

int tc_cluster_size(int M, int T, int K, int wkind, int epi, int sms) {
    const int nt = tc_tile_tokens(wkind, M, T);
    if (nt > 64 || epi == kEpiArgmax) return 1;
    const int tiles = (M / kBM) * ((T + nt - 1) / nt);
    if (2 * tiles > sms) return 1;  // enough tiles to fill the GPU without splitting K
    const int nkb = K * (wkind == kWQ8 ? 1 : 2) / kKB;
    // powers of two pack into the GPCs without leaving clusters for a second wave
    int S = 1;
    while (2 * S <= std::min({sms / tiles, kMaxCluster, nkb})) S *= 2;
    return S;
}

void launch_tc_cluster(const TcLaunch& L, int S, cudaStream_t st) {
    const int nt = tc_tile_tokens(L.args.wkind, L.args.M, L.args.T);
    if (L.args.wkind == kWQ8) {
        switch (nt) {
            case 16: launch_cluster_epi<kWQ8, 16>(L, S, st); break;
            case 32: launch_cluster_epi<kWQ8, 32>(L, S, st); break;
            default: launch_cluster_epi<kWQ8, 64>(L, S, st); break;
        }
    } else {
        switch (nt) {
            case 16: launch_cluster_epi<kWBF16, 16>(L, S, st); break;
            case 32: launch_cluster_epi<kWBF16, 32>(L, S, st); break;
            default: launch_cluster_epi<kWBF16, 64>(L, S, st); break;
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

}  // namespace zc
