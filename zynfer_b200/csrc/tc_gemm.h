// tcgen05 weight-only linear (internal to libzynfer_cuda). See tc_gemm.cu.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "kernels.h"

namespace zc {

// Activation planes: rows [0, T) of X (f32, optionally RMS-normalised) ->
// planes [P][t_pad][K]: int8 digits (P = 3, plus exps[T]) or bf16 hi/lo (P = 2).
struct PlanesArgs {
    const float* x;
    int ldx;
    int T, K, t_pad;
    int wkind;
    const float* norm_w;  // nullable
    float eps;
    void* planes;
    float* xscale;  // int8 only: 2^(e - 22) per row
};

constexpr int kPlanesMaxK = 4096;  // activation rows the plane kernel holds in registers

struct TcArgs {
    int M, K, T, t_pad;
    int wkind;
    int epi;
    const float* scale;  // [M] (int8) or nullptr
    const float* xscale; // [T] (int8): 2^(e - 22) of each activation row
    float* y;            // [T][ldy]
    int ldy;
    const float* resid;
    unsigned long long* argmax_keys;
    uint32_t* err;
    int stall;  // fault injection: 1 = no CTA loads its first stage, so the MMA warp's bounded wait runs out
    L2Range pf[2];  // the next linear's weights and scales, prefetched into L2
};

struct TcLaunch {
    const CUtensorMap* tmA;  // weights [M][K], box 128 B x 128 rows
    const CUtensorMap* tmB;  // planes [P * t_pad][K], box 128 B x NT rows
    TcArgs args;
    int sms;  // persistent grid size
};

int tc_tile_tokens(int wkind, int M, int T);  // NT: tokens per N tile of an M x K by T linear
bool make_tmap_k_major(CUtensorMap* map, const void* base, int wkind, uint64_t k_elems, uint64_t rows,
                       uint32_t box_rows);
void launch_prep_planes(const PlanesArgs& a, cudaStream_t st);
void launch_tc_gemm(const TcLaunch& L, cudaStream_t st);
// Cluster split-K variant for problems with too few (M, N) tiles to fill the
// GPU: CTAs per cluster along K (1 = use launch_tc_gemm), and its launcher
// (one tile per cluster, tiles of at most 64 tokens, no argmax epilogue).
int tc_cluster_size(int M, int T, int K, int wkind, int epi, int sms);
void launch_tc_cluster(const TcLaunch& L, int S, cudaStream_t st);
// The next allocation-free linear call launches with TcArgs::stall set.
void static_linear_arm_stall();

}  // namespace zc
