// Synthetic weight generation and weight packing on the device.
//
// pack_q8_rows restates packRowQ8 (src/backends/cpu/ops.zig:145-162) so that
// the int8 weights and scales are bit-identical to the host oracle's:
// max|w| is order-independent, and every other step is one IEEE f32 operation
// (division, reciprocal, multiply, roundf, clamp).
#include <mutex>
#include <set>
#include <utility>

#include "common.cuh"
#include "kernels.h"
#include "synth_rng.h"

namespace zc {

__global__ void synth_normal_kernel(float* out, size_t n, uint64_t key, float k, float add) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n;
         i += (size_t)gridDim.x * blockDim.x) {
        const float v = zs_normal(key, i, k);
        out[i] = add != 0.0f ? __fadd_rn(add, v) : v;
    }
}

__global__ void fill_kernel(float* out, size_t n, float v) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n;
         i += (size_t)gridDim.x * blockDim.x)
        out[i] = v;
}

// Function attributes, set once per device before any launch (so never
// during stream capture): the opt-in dynamic shared-memory ceiling, and the
// same L1/shared split (maximum shared memory) for every kernel so that
// consecutive kernels do not make the SM reconfigure its carveout.
void configure_kernel(const void* func, size_t dyn_smem) {
    static std::mutex mu;
    static std::set<std::pair<int, const void*>> done;
    int dev = 0;
    cudaGetDevice(&dev);
    std::lock_guard<std::mutex> lock(mu);
    if (!done.insert({dev, func}).second) return;
    if (dyn_smem > 48 * 1024) cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)dyn_smem);
    cudaFuncSetAttribute(func, cudaFuncAttributePreferredSharedMemoryCarveout, cudaSharedmemCarveoutMaxShared);
}

void prepare_all_kernels() {
    prepare_norm_kernels();
    prepare_gemv_kernels();
    prepare_gemm_simt_kernels();
    prepare_attn_kernels();
    prepare_flow_kernels();
    prepare_tc_kernels();
    prepare_sample_kernels();
    prepare_fewrow_kernels();
}

int device_sm_count() {
    static int cached[64] = {0};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return 148;
    if (!cached[dev]) {
        int sms = 0;
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        cached[dev] = sms > 0 ? sms : 148;
    }
    return cached[dev];
}

static int grid_for(size_t n) {
    size_t g = (n + 255) / 256;
    return (int)(g > 148 * 64 ? 148 * 64 : (g ? g : 1));
}

void launch_synth_normal(float* out, size_t n, uint64_t seed, uint64_t stream, float k, float add,
                         cudaStream_t st) {
    synth_normal_kernel<<<grid_for(n), 256, 0, st>>>(out, n, zs_key(seed, stream), k, add);
}

void launch_fill(float* out, size_t n, float v, cudaStream_t st) {
    fill_kernel<<<grid_for(n), 256, 0, st>>>(out, n, v);
}

// Seeded stand-in for a prefilled cache of one sequence: positions [0, n) of
// every layer. K (code 100) and V (code 101) of layer l draw from key(seed,
// layer_stream(l, code)); element (kv head h, position p, dim j) is
// normal(key, (h n + p) d + j, 1) rounded to bf16, written into the paged
// block of position p at its swizzled place. One thread per 16-byte chunk
// (8 dims) of one row.
__global__ void kv_fill_kernel(uint16_t* __restrict__ kv, size_t kv_layer_elems, const int* __restrict__ table,
                               int n_pool_blocks, int layers, int n_kv, int n, uint64_t seed, float k,
                               uint32_t* err) {
    constexpr int d = 128, chunks_per_row = d / 8;
    const size_t total = (size_t)layers * 2 * n_kv * n * chunks_per_row;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
        const int c = (int)(i % chunks_per_row);
        size_t r = i / chunks_per_row;
        const int p = (int)(r % n);
        r /= n;
        const int h = (int)(r % n_kv);
        r /= n_kv;
        const int which = (int)(r % 2);
        const int l = (int)(r / 2);
        const int blk = table[p / kKvBlock];
        if (blk < 0 || blk >= n_pool_blocks) {
            if (err) atomicOr(err, kErrBadIndex);
            continue;
        }
        const uint64_t key = zs_key(seed, zs_layer_stream((uint32_t)l, (uint32_t)(100 + which)));
        const uint64_t base = ((uint64_t)h * n + p) * d + 8 * c;
        uint32_t w[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const uint32_t lo = f32_to_bf16_rne(zs_normal(key, base + 2 * e, k));
            const uint32_t hi = f32_to_bf16_rne(zs_normal(key, base + 2 * e + 1, k));
            w[e] = lo | (hi << 16);
        }
        uint16_t* dst = kv + (size_t)l * kv_layer_elems + (((size_t)h * n_pool_blocks + blk) * 2 + which) * kKvBlock * d +
                        kv_swizzle(p % kKvBlock, 8 * c);
        *reinterpret_cast<uint4*>(dst) = make_uint4(w[0], w[1], w[2], w[3]);
    }
}

void launch_kv_fill(uint16_t* kv, size_t kv_layer_elems, const int* table_row, int n_pool_blocks, int layers,
                    int n_kv, int n, uint64_t seed, uint32_t* err, cudaStream_t st) {
    if (n <= 0) return;
    const size_t total = (size_t)layers * 2 * n_kv * n * 16;
    const float k = (float)(1.0 / ZS_IH4_SIGMA);
    kv_fill_kernel<<<grid_for(total), 256, 0, st>>>(kv, kv_layer_elems, table_row, n_pool_blocks, layers, n_kv, n,
                                                    seed, k, err);
}

// One warp per source row.
__global__ void pack_q8_rows_kernel(const float* __restrict__ w, int rows, int cols,
                                    int8_t* __restrict__ q, float* __restrict__ scale,
                                    int dst_stride, int dst_offset) {
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) / kWarp;
    const int lane = threadIdx.x % kWarp;
    if (warp >= rows) return;
    const float* row = w + (size_t)warp * cols;
    float m = 0.0f;
    for (int c = lane; c < cols; c += kWarp) m = fmaxf(m, fabsf(row[c]));
    m = warp_max(m);
    const float s = m == 0.0f ? 1.0f : m / 127.0f;
    const float inv = 1.0f / s;
    const size_t dr = (size_t)warp * dst_stride + dst_offset;
    if (lane == 0) scale[dr] = s;
    int8_t* qr = q + dr * cols;
    for (int c = lane; c < cols; c += kWarp) {
        const float r = roundf(__fmul_rn(row[c], inv));
        qr[c] = (int8_t)fmaxf(-127.0f, fminf(127.0f, r));
    }
}

void launch_pack_q8_rows(const float* w, int rows, int cols, int8_t* q, float* scale,
                         int dst_stride, int dst_offset, cudaStream_t st) {
    const int threads = 256;
    const int blocks = (rows * kWarp + threads - 1) / threads;
    pack_q8_rows_kernel<<<blocks, threads, 0, st>>>(w, rows, cols, q, scale, dst_stride, dst_offset);
}

__global__ void to_bf16_rows_kernel(const float* __restrict__ w, int rows, int cols,
                                    uint16_t* __restrict__ out, int dst_stride, int dst_offset) {
    const size_t n = (size_t)rows * cols;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n;
         i += (size_t)gridDim.x * blockDim.x) {
        const size_t r = i / cols, c = i % cols;
        out[(r * dst_stride + dst_offset) * cols + c] = f32_to_bf16_rne(w[i]);
    }
}

void launch_to_bf16_rows(const float* w, int rows, int cols, uint16_t* out, int dst_stride,
                         int dst_offset, cudaStream_t st) {
    to_bf16_rows_kernel<<<grid_for((size_t)rows * cols), 256, 0, st>>>(w, rows, cols, out, dst_stride,
                                                                      dst_offset);
}

__global__ void copy_rows_i8_kernel(const int8_t* __restrict__ src, const float* __restrict__ ssrc,
                                    int rows, int cols, int8_t* __restrict__ dst,
                                    float* __restrict__ sdst, int dst_stride, int dst_offset) {
    const size_t n = (size_t)rows * cols;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n;
         i += (size_t)gridDim.x * blockDim.x) {
        const size_t r = i / cols, c = i % cols;
        const size_t dr = r * dst_stride + dst_offset;
        dst[dr * cols + c] = src[i];
        if (c == 0) sdst[dr] = ssrc[r];
    }
}

void launch_copy_rows_i8(const int8_t* src, const float* ssrc, int rows, int cols, int8_t* dst,
                         float* sdst, int dst_stride, int dst_offset, cudaStream_t st) {
    copy_rows_i8_kernel<<<grid_for((size_t)rows * cols), 256, 0, st>>>(src, ssrc, rows, cols, dst,
                                                                       sdst, dst_stride, dst_offset);
}

__global__ void copy_rows_u16_kernel(const uint16_t* __restrict__ src, int rows, int cols,
                                     uint16_t* __restrict__ dst, int dst_stride, int dst_offset) {
    const size_t n = (size_t)rows * cols;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n;
         i += (size_t)gridDim.x * blockDim.x) {
        const size_t r = i / cols, c = i % cols;
        dst[(r * dst_stride + dst_offset) * cols + c] = src[i];
    }
}

void launch_copy_rows_u16(const uint16_t* src, int rows, int cols, uint16_t* dst, int dst_stride,
                          int dst_offset, cudaStream_t st) {
    copy_rows_u16_kernel<<<grid_for((size_t)rows * cols), 256, 0, st>>>(src, rows, cols, dst,
                                                                        dst_stride, dst_offset);
}

// Inverse of copy_rows_i8: gather rows (r * src_stride + src_offset) back into a dense tensor.
__global__ void unpack_rows_i8_kernel(const int8_t* __restrict__ src, const float* __restrict__ ssrc,
                                      int rows, int cols, int8_t* __restrict__ dst,
                                      float* __restrict__ sdst, int src_stride, int src_offset) {
    const size_t n = (size_t)rows * cols;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n;
         i += (size_t)gridDim.x * blockDim.x) {
        const size_t r = i / cols, c = i % cols;
        const size_t sr = r * src_stride + src_offset;
        dst[i] = src[sr * cols + c];
        if (c == 0) sdst[r] = ssrc[sr];
    }
}

void launch_unpack_rows_i8(const int8_t* src, const float* ssrc, int rows, int cols, int8_t* dst,
                           float* sdst, int src_stride, int src_offset, cudaStream_t st) {
    unpack_rows_i8_kernel<<<grid_for((size_t)rows * cols), 256, 0, st>>>(src, ssrc, rows, cols, dst,
                                                                         sdst, src_stride, src_offset);
}

}  // namespace zc
