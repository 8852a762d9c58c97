// A tensor-core int8 linear that allocates nothing, for callers that cannot
// call cudaMalloc (an embedder that owns all device memory, a custom
// allocator that must not be bypassed, or code that runs where allocation is
// forbidden). It is the tcgen05 linear of tc_gemm.cu; its only scratch, the
// int8 digit planes of the activations and their per-row scales, lives in the
// file-scope arrays below instead of context memory, and so does the error
// word its bounded device waits report through.
#include <cuda.h>
#include <cuda_runtime.h>

#include <atomic>
#include <climits>
#include <mutex>

#include "../../include/zynfer_cuda.h"
#include "common.cuh"
#include "kernels.h"
#include "tc_gemm.h"

namespace {

constexpr int kMaxRows = ZYNFER_CU_STATIC_MAX_ROWS;  // 64
constexpr int kMaxK = ZYNFER_CU_STATIC_MAX_K;        // 4096
constexpr int kPadRows = 64;                         // planes are padded to one 64-row tile

// Three int8 digit planes [3][kPadRows][kMaxK] (768 KiB), one scale per row
// and the device error word (kErrTimeout when a bounded wait ran out). Every
// device that loads the library holds them until the process exits.
static __device__ __align__(256) int8_t g_planes[3 * kPadRows * kMaxK];
static __device__ __align__(256) float g_xscale[kPadRows];
static __device__ __align__(256) uint32_t g_err;

struct DeviceScratch {
    bool ready = false;
    int8_t* planes = nullptr;
    float* xscale = nullptr;
    uint32_t* err = nullptr;
    int sms = 0;
};

std::mutex g_mu;
DeviceScratch g_dev[64];
std::atomic<bool> g_stall_next{false};  // armed by zynfer_cu_set_fail_at(NULL, "wait")

// Once per device, with that device current: resolve the arrays' device
// addresses (in host code their names are only host-side stand-ins) and set
// the kernels' function attributes. Nothing here allocates memory.
int setup_device(int dev, DeviceScratch** out) {
    if (dev < 0 || dev >= 64) return ZYNFER_CU_INVALID;
    std::lock_guard<std::mutex> lock(g_mu);
    DeviceScratch& d = g_dev[dev];
    if (!d.ready) {
        void* p = nullptr;
        if (cudaGetSymbolAddress(&p, g_planes) != cudaSuccess) return ZYNFER_CU_INTERNAL;
        d.planes = static_cast<int8_t*>(p);
        if (cudaGetSymbolAddress(&p, g_xscale) != cudaSuccess) return ZYNFER_CU_INTERNAL;
        d.xscale = static_cast<float*>(p);
        if (cudaGetSymbolAddress(&p, g_err) != cudaSuccess) return ZYNFER_CU_INTERNAL;
        d.err = static_cast<uint32_t*>(p);
        if (cudaDeviceGetAttribute(&d.sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return ZYNFER_CU_INTERNAL;
        zc::prepare_all_kernels();
        d.ready = true;
    }
    *out = &d;
    return ZYNFER_CU_OK;
}

}  // namespace

namespace zc {
void static_linear_arm_stall() { g_stall_next.store(true); }
}  // namespace zc

extern "C" int zynfer_cu_linear_q8_static(const int8_t* w, const float* scale, const float* x, uint32_t batch,
                                          uint32_t m, uint32_t k, float* y, void* stream) {
    if (!w || !scale || !x || !y) return ZYNFER_CU_INVALID;
    if (reinterpret_cast<uintptr_t>(x) % 16) return ZYNFER_CU_INVALID;  // rows are read as float4
    if (reinterpret_cast<uintptr_t>(y) % 4 || reinterpret_cast<uintptr_t>(scale) % 4)
        return ZYNFER_CU_INVALID;  // the epilogue reads scales and stores outputs as f32
    if (batch == 0 || batch > (uint32_t)kMaxRows || k == 0 || k > (uint32_t)kMaxK || k % 128 || m == 0 || m % 128)
        return ZYNFER_CU_INVALID;
    if (m > (uint32_t)INT_MAX) return ZYNFER_CU_INVALID;  // rows, tiles and strides are int in the kernels
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return ZYNFER_CU_NO_DEVICE;
    DeviceScratch* d = nullptr;
    int rc = setup_device(dev, &d);
    if (rc) return rc;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    // Rows [0, batch) of the planes and scales are rewritten by every call;
    // pad rows keep an earlier call's values, which only reach output columns
    // that are never stored, so nothing has to start at zero.
    zc::PlanesArgs pa{x, (int)k, (int)batch, (int)k, kPadRows, zc::kWQ8, nullptr, 1e-6f, d->planes, d->xscale};
    CUtensorMap tmA, tmB;
    const int nt = zc::tc_tile_tokens(zc::kWQ8, (int)m, (int)batch);
    if (!zc::make_tmap_k_major(&tmA, w, zc::kWQ8, k, m, 128) ||
        !zc::make_tmap_k_major(&tmB, d->planes, zc::kWQ8, k, (uint64_t)3 * kPadRows, (uint32_t)nt))
        return ZYNFER_CU_INTERNAL;
    zc::TcLaunch L;
    L.tmA = &tmA;
    L.tmB = &tmB;
    L.args = zc::TcArgs{(int)m, (int)k, (int)batch, kPadRows, zc::kWQ8, zc::kEpiNone, scale, d->xscale, y, (int)m,
                        nullptr, nullptr, d->err, g_stall_next.exchange(false) ? 1 : 0, {}};
    L.sms = d->sms;
    zc::launch_prep_planes(pa, st);
    zc::launch_tc_gemm(L, st);
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? ZYNFER_CU_OK : ZYNFER_CU_LAUNCH;
}

extern "C" int zynfer_cu_linear_q8_static_status(int clear) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return ZYNFER_CU_NO_DEVICE;
    DeviceScratch* d = nullptr;
    int rc = setup_device(dev, &d);
    if (rc) return rc;
    uint32_t word = 0;
    // synchronous copies of one word between the library's own arrays and the stack: nothing is allocated
    if (cudaMemcpy(&word, d->err, sizeof(word), cudaMemcpyDeviceToHost) != cudaSuccess) return ZYNFER_CU_LAUNCH;
    if (word && clear) {
        const uint32_t zero = 0;
        if (cudaMemcpy(d->err, &zero, sizeof(zero), cudaMemcpyHostToDevice) != cudaSuccess) return ZYNFER_CU_LAUNCH;
    }
    if (word & zc::kErrTimeout) return ZYNFER_CU_TIMEOUT;
    return word ? ZYNFER_CU_INTERNAL : ZYNFER_CU_OK;
}
