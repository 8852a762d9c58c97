// Row kernels: RMSNorm, embedding gather, fused QK-norm + RoPE + paged KV
// append, and the per-step argmax finalisation.
#include "common.cuh"
#include "kernels.h"

namespace zc {

// RMSNorm (ops.zig:49-67): inv = 1 / sqrt(mean(x^2) + eps); y = (w * x) * inv.
// One warp per row; the sum of squares is a warp tree (order differs from the
// reference's sequential sum, within f32 rounding).
__global__ void rmsnorm_kernel(const float* __restrict__ x, const float* __restrict__ w,
                               float* __restrict__ y, int rows, int cols, float eps) {
    pdl_launch_dependents();
    pdl_wait();
    const int row = (blockIdx.x * blockDim.x + threadIdx.x) / kWarp;
    const int lane = threadIdx.x % kWarp;
    if (row >= rows) return;
    const float* xr = x + (size_t)row * cols;
    float acc = 0.0f;
    for (int c = lane * 4; c < cols; c += kWarp * 4) {
        const float4 v = *reinterpret_cast<const float4*>(xr + c);
        acc += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
    }
    acc = warp_sum(acc);
    const float inv = 1.0f / sqrtf(acc / (float)cols + eps);
    float* yr = y + (size_t)row * cols;
    for (int c = lane * 4; c < cols; c += kWarp * 4) {
        const float4 v = *reinterpret_cast<const float4*>(xr + c);
        const float4 g = *reinterpret_cast<const float4*>(w + c);
        float4 o;
        o.x = __fmul_rn(__fmul_rn(g.x, v.x), inv);
        o.y = __fmul_rn(__fmul_rn(g.y, v.y), inv);
        o.z = __fmul_rn(__fmul_rn(g.z, v.z), inv);
        o.w = __fmul_rn(__fmul_rn(g.w, v.w), inv);
        *reinterpret_cast<float4*>(yr + c) = o;
    }
}

void launch_rmsnorm(const float* x, const float* w, float* y, int rows, int cols, float eps,
                    cudaStream_t st) {
    const int threads = 256;
    const int blocks = (rows * kWarp + threads - 1) / threads;
    launch_pdl(rmsnorm_kernel, blocks, threads, 0, st, x, w, y, rows, cols, eps);
}

// Embedding rows (ops.zig:397-411). int8 tables are dequantised as
// f32(q) * scale (one rounding, the same value the host computes).
__global__ void embed_kernel(const void* __restrict__ table, const float* __restrict__ scale,
                             int wkind, const uint32_t* __restrict__ ids, int n, int H, int V,
                             float* __restrict__ x, uint32_t* err) {
    pdl_launch_dependents();
    pdl_wait();
    const int row = blockIdx.x;
    if (row >= n) return;
    const uint32_t id = ids[row];
    float* xr = x + (size_t)row * H;
    if (id >= (uint32_t)V) {
        if (threadIdx.x == 0 && err) atomicOr(err, kErrBadIndex);
        for (int c = threadIdx.x; c < H; c += blockDim.x) xr[c] = 0.0f;
        return;
    }
    if (wkind == kWQ8) {
        const int8_t* q = reinterpret_cast<const int8_t*>(table) + (size_t)id * H;
        const float s = scale[id];
        for (int c = threadIdx.x; c < H; c += blockDim.x) xr[c] = __fmul_rn((float)q[c], s);
    } else {
        const uint16_t* b = reinterpret_cast<const uint16_t*>(table) + (size_t)id * H;
        for (int c = threadIdx.x; c < H; c += blockDim.x) xr[c] = __uint_as_float((uint32_t)b[c] << 16);
    }
}

void launch_embed(const void* table, const float* scale, int wkind, const uint32_t* ids, int n, int H,
                  int V, float* x, uint32_t* err, cudaStream_t st) {
    if (n <= 0) return;
    launch_pdl(embed_kernel, n, 256, 0, st, table, scale, wkind, ids, n, H, V, x, err);
}

// One warp per (row, head) over the fused QKV output. q and k heads get the
// per-head RMSNorm (qwen_block.zig:191-192) and split-half RoPE
// (ops.zig:233-261, cos/sin from a host-built table of the same f32 values);
// k and v heads are rounded to bf16 and written into the paged cache at
// their position; prefill also stages them in f32 for the prefill attention.
// head_dim is 128: lane holds elements lane + 32 j, j = 0..3, so the RoPE
// pairs (i, i + 64) sit in one lane.
__global__ void qkv_post_kernel(QkvArgs a) {
    pdl_launch_dependents();
    pdl_wait();
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) / kWarp;
    const int lane = threadIdx.x % kWarp;
    const int heads = a.n_q + 2 * a.n_kv;
    if (warp >= a.T * heads) return;
    const int t = warp / heads;
    const int h = warp % heads;
    const int d = a.d;  // 128
    const float* src = a.qkv + (size_t)t * heads * d + (size_t)h * d;
    float v[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) v[j] = src[lane + 32 * j];
    const int pos = a.row_pos ? a.row_pos[t] : a.pos0 + t;
    if (h < a.n_q + a.n_kv) {
        const float* nw = h < a.n_q ? a.q_norm : a.k_norm;
        float ss = 0.0f;
#pragma unroll
        for (int j = 0; j < 4; ++j) ss += v[j] * v[j];
        ss = warp_sum(ss);
        const float inv = 1.0f / sqrtf(ss / (float)d + a.eps);
#pragma unroll
        for (int j = 0; j < 4; ++j) v[j] = __fmul_rn(__fmul_rn(nw[lane + 32 * j], v[j]), inv);
        if (pos < a.rope_max_pos) {
            const float2* cs = a.rope + (size_t)pos * (d / 2);
#pragma unroll
            for (int j = 0; j < 2; ++j) {
                const float2 c = cs[lane + 32 * j];
                const float x0 = v[j], x1 = v[j + 2];
                v[j] = __fsub_rn(__fmul_rn(x0, c.x), __fmul_rn(x1, c.y));
                v[j + 2] = __fadd_rn(__fmul_rn(x0, c.y), __fmul_rn(x1, c.x));
            }
        } else if (lane == 0 && a.err) {
            atomicOr(a.err, kErrBadIndex);
        }
    }
    if (h < a.n_q) {
        float* dst = a.q_heads_major ? a.q_out + ((size_t)h * a.T + t) * d
                                     : a.q_out + ((size_t)t * a.n_q + h) * d;
#pragma unroll
        for (int j = 0; j < 4; ++j) dst[lane + 32 * j] = v[j];
        return;
    }
    const int which = (h - a.n_q) / a.n_kv;  // 0 = k, 1 = v
    const int kvh = (h - a.n_q) % a.n_kv;
    if (a.kv_layer) {
        const int seq = a.row_seq ? a.row_seq[t] : a.seq0;
        const int bi = pos / kKvBlock;
        int blk = -1;
        if (bi < a.max_blocks) blk = a.block_table[(size_t)seq * a.max_blocks + bi];
        if (blk < 0 || blk >= a.n_pool_blocks) {
            if (lane == 0 && a.err) atomicOr(a.err, kErrBadIndex);
        } else {
            uint16_t* dst = a.kv_layer + (((size_t)kvh * a.n_pool_blocks + blk) * 2 + which) * kKvBlock * d;
#pragma unroll
            for (int j = 0; j < 4; ++j) dst[kv_swizzle(pos % kKvBlock, lane + 32 * j)] = f32_to_bf16_rne(v[j]);
        }
    }
    float* stage = which == 0 ? a.k_stage : a.v_stage;
    if (stage) {
        float* dst = stage + ((size_t)kvh * a.T + t) * d;
#pragma unroll
        for (int j = 0; j < 4; ++j) dst[lane + 32 * j] = a.stage_round_bf16 ? bf16_round(v[j]) : v[j];
    }
    if (a.kv_planes) {
        const size_t plane = (size_t)a.n_kv * a.T * d;
        uint16_t* hi = a.kv_planes + (size_t)(2 * which) * plane + ((size_t)kvh * a.T + t) * d;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const float x = a.stage_round_bf16 ? bf16_round(v[j]) : v[j];
            const uint16_t h = f32_to_bf16_rne(x);
            hi[lane + 32 * j] = h;
            hi[plane + lane + 32 * j] = f32_to_bf16_rne(x - __uint_as_float((uint32_t)h << 16));
        }
    }
}

// siluMul (ops.zig:36-42): o = silu(g) * u, elementwise.
__global__ void silu_mul_kernel(const float* __restrict__ g, const float* __restrict__ u, size_t n,
                                float* __restrict__ o) {
    pdl_launch_dependents();
    pdl_wait();
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        o[i] = __fmul_rn(silu(g[i]), u[i]);
}

void launch_silu_mul(const float* g, const float* u, size_t n, float* o, cudaStream_t st) {
    size_t blocks = (n + 255) / 256;
    if (blocks > (size_t)device_sm_count() * 8) blocks = (size_t)device_sm_count() * 8;
    launch_pdl(silu_mul_kernel, (int)(blocks ? blocks : 1), 256, 0, st, g, u, n, o);
}

void launch_qkv_post(const QkvArgs& a, cudaStream_t st) {
    const int warps = a.T * (a.n_q + 2 * a.n_kv);
    const int threads = 256;
    launch_pdl(qkv_post_kernel, (warps * kWarp + threads - 1) / threads, threads, 0, st, a);
}

// Turn argmax keys into ids, feed them to the next step, advance positions,
// and append to the on-device history. One CTA.
__global__ void finalize_kernel(FinalizeArgs a) {
    pdl_launch_dependents();
    pdl_wait();
    const int b = threadIdx.x;
    const int row = a.history ? *a.step : 0;
    __syncthreads();
    if (b < a.B) {
        const unsigned long long key = a.keys[b];
        const uint32_t id = key == 0ull ? 0u : argmax_key_index(key);
        a.keys[b] = 0ull;
        a.ids_out[b] = id;
        if (a.next_tokens) a.next_tokens[b] = id;
        if (a.positions) a.positions[b] += 1;
        if (a.history) a.history[(size_t)row * a.B + b] = id;
    }
    if (b == 0 && a.history) *a.step = row + 1;
}

void launch_finalize(const FinalizeArgs& a, cudaStream_t st) {
    const int threads = ((a.B + 31) / 32) * 32;
    launch_pdl(finalize_kernel, 1, threads, 0, st, a);
}

__global__ void bf16_to_f32_kernel(const uint16_t* __restrict__ src, size_t n, float* __restrict__ dst) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n;
         i += (size_t)gridDim.x * blockDim.x)
        dst[i] = __uint_as_float((uint32_t)src[i] << 16);
}

void launch_bf16_to_f32(const uint16_t* src, size_t n, float* dst, cudaStream_t st) {
    size_t g = (n + 255) / 256;
    if (g > 148 * 64) g = 148 * 64;
    bf16_to_f32_kernel<<<(int)(g ? g : 1), 256, 0, st>>>(src, n, dst);
}

void prepare_norm_kernels() {
    configure_kernel((const void*)rmsnorm_kernel, 0);
    configure_kernel((const void*)embed_kernel, 0);
    configure_kernel((const void*)qkv_post_kernel, 0);
    configure_kernel((const void*)finalize_kernel, 0);
    configure_kernel((const void*)silu_mul_kernel, 0);
}

}  // namespace zc
