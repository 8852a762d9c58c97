// Shared device helpers for the sm_100a Qwen3 kernels.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "kernels.h"

namespace zc {

constexpr int kWarp = 32;
constexpr int kKvBlock = 16;  // tokens per paged KV block

// Element index of (token t, dim e) inside one paged block of K (or V) for
// one kv head: 16 rows of 128 bf16 (256 B) whose 16-byte chunks are
// XOR-swizzled by (t & 7). Eight consecutive tokens then keep any logical
// chunk in eight different bank groups, so row-wise and transposing
// ldmatrix reads of a block are free of bank conflicts.
__host__ __device__ __forceinline__ int kv_swizzle(int t, int e) {
    return t * 128 + ((((e >> 3) ^ (t & 7)) << 3) | (e & 7));
}

// Device error word, set instead of trapping. Codes (bitwise OR):
enum : uint32_t {
    kErrTimeout = 1u,       // a bounded mbarrier wait ran out
    kErrBadIndex = 2u,      // an index check failed (token id, block id)
};

// ---------------------------------------------------------------- numerics

// bf16 bits -> f32 (exact).
__device__ __forceinline__ float bf16lo(uint32_t two) { return __uint_as_float(two << 16); }
__device__ __forceinline__ float bf16hi(uint32_t two) { return __uint_as_float(two & 0xFFFF0000u); }

// f32 -> bf16 bits, round to nearest even (NaN kept quiet), written out so the
// rounding is explicit and identical to the host restatement.
__device__ __forceinline__ uint16_t f32_to_bf16_rne(float x) {
    uint32_t u = __float_as_uint(x);
    if ((u & 0x7FFFFFFFu) > 0x7F800000u) return (uint16_t)((u >> 16) | 0x40u);
    u += 0x7FFFu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}
__device__ __forceinline__ float bf16_round(float x) {
    return __uint_as_float((uint32_t)f32_to_bf16_rne(x) << 16);
}

// Four packed int8 -> four exact f32, without the int->float converter:
// bias each byte to unsigned (xor 0x80), place it in the low mantissa byte of
// 2^23 (0x4B000000), and subtract 2^23 + 128 (Kim et al., "Who Says Elephants
// Can't Run", 2022, applied to f32). Exact for every int8 value.
__device__ __forceinline__ void i8x4_to_f32(uint32_t w, float& f0, float& f1, float& f2, float& f3) {
    const uint32_t u = w ^ 0x80808080u;
    const float magic = 8388736.0f;  // 2^23 + 128
    f0 = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7540)) - magic;
    f1 = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7541)) - magic;
    f2 = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7542)) - magic;
    f3 = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7543)) - magic;
}

// siluScalar (ops.zig:44-46): x * (1 / (1 + e^-x)), the one definition every
// SwiGLU epilogue and the standalone siluMul kernel use.
__device__ __forceinline__ float silu(float g) { return g * (1.0f / (1.0f + expf(-g))); }

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
    return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xFFFFFFFFu, v, o));
    return v;
}

// The int8 digit planes of four activation values f (|f| < 2^e, 2^e a row's
// power-of-two scale): q = rint(f 2^(22-e)),
// |q| <= 2^22, written q = d0 2^16 + d1 2^8 + d2 with d1, d2 in [-128, 127].
// 2^(22-e) is a float whenever 22 - e <= 127, and then f * 2^(22-e) is the
// same correctly rounded product ldexpf returns; with u = q + 0x8080, d2 and
// d1 are bytes 0 and 1 of u minus 128 (the unique such digits) and d0 is
// u >> 16, whose low byte is byte 2 of u. d0, d1, d2 receive the four
// values' digits as packed int8.
__device__ __forceinline__ void digits4(const float (&f)[4], int e, uint32_t& d0, uint32_t& d1, uint32_t& d2) {
    uint32_t u[4];
    if (22 - e <= 127) {
        const float p2 = __int_as_float((22 - e + 127) << 23);
#pragma unroll
        for (int j = 0; j < 4; ++j) u[j] = (uint32_t)(__float2int_rn(__fmul_rn(f[j], p2)) + 0x8080);
    } else {
#pragma unroll
        for (int j = 0; j < 4; ++j) u[j] = (uint32_t)(__float2int_rn(ldexpf(f[j], 22 - e)) + 0x8080);
    }
    const uint32_t lo01 = __byte_perm(u[0], u[1], 0x5140), lo23 = __byte_perm(u[2], u[3], 0x5140);
    const uint32_t hi01 = __byte_perm(u[0], u[1], 0x7362), hi23 = __byte_perm(u[2], u[3], 0x7362);
    d2 = __byte_perm(lo01, lo23, 0x5410) ^ 0x80808080u;
    d1 = __byte_perm(lo01, lo23, 0x7632) ^ 0x80808080u;
    d0 = __byte_perm(hi01, hi23, 0x5410);
}

// RMSNorm sum of squares in the order every kernel that digitises activation
// rows uses, so their row scales agree bit for bit however they split K:
// within each 128-value block, lane l of a warp takes values 4l .. 4l + 3
// (sq4: rounded fused multiply-adds in that order) and the warp adds the 32
// lanes with the xor butterfly of warp_sum; the blocks' sums are then added
// one after another in k order.
__device__ __forceinline__ float sq4(const float4 v) {
    return __fmaf_rn(v.w, v.w, __fmaf_rn(v.z, v.z, __fmaf_rn(v.y, v.y, __fmul_rn(v.x, v.x))));
}

// Orderable key for a (logit, index) pair: a larger key is a larger logit,
// and among equal logits the lower index (the reference's topK keeps the
// first maximum, qwen_forward.zig:177-193). topK starts from (id 0, -inf) and
// takes a logit only when it is strictly greater, so NaN and -inf never win:
// they map to key 0, and an all-zero key decodes to id 0.
__device__ __forceinline__ unsigned long long argmax_key(float v, uint32_t idx) {
    const uint32_t u = __float_as_uint(v);
    if ((u & 0x7FFFFFFFu) > 0x7F800000u || u == 0xFF800000u) return 0ull;  // NaN, -inf
    const uint32_t ord = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
    return ((unsigned long long)ord << 32) | (unsigned long long)(0xFFFFFFFFu - idx);
}
__device__ __forceinline__ uint32_t argmax_key_index(unsigned long long key) {
    return 0xFFFFFFFFu - (uint32_t)(key & 0xFFFFFFFFull);
}

// 16-byte read-only global load that does not allocate in L1 (streamed once).
__device__ __forceinline__ uint4 ldg_stream(const void* p) {
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
    return r;
}
// The same, evict-first in L2 (data read once per step).
__device__ __forceinline__ uint4 ldg_stream_first(const void* p) {
    uint4 r;
    uint64_t pol;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
    asm volatile("ld.global.nc.L1::no_allocate.L2::cache_hint.v4.u32 {%0,%1,%2,%3}, [%4], %5;"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p), "l"(pol));
    return r;
}

// ------------------------------------------------------ mbarrier + bulk copy

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count));
}

__device__ __forceinline__ void fence_barrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)),
                 "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_addr(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Bounded wait: gives up after `limit` polls (each try_wait itself blocks for
// a hardware-defined interval), sets kErrTimeout in *err and returns false.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity, uint32_t* err,
                                                  uint32_t limit = (1u << 22)) {
    for (uint32_t i = 0; i < limit; ++i)
        if (mbar_try_wait(bar, parity)) return true;
    if (err) atomicOr(err, kErrTimeout);
    return false;
}

// Untiled bulk copy global -> this CTA's shared memory, completing on `bar`.
// Both addresses 16-byte aligned, bytes a multiple of 16. No multicast.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_addr(dst)),
        "l"(src), "r"(bytes), "r"(smem_addr(bar))
        : "memory");
}

// The same with an L2 cache policy (createpolicy), e.g. evict-first for data read once.
__device__ __forceinline__ void bulk_g2s_hint(void* dst, const void* src, uint32_t bytes, uint64_t* bar, uint64_t pol) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
            smem_addr(dst)),
        "l"(src), "r"(bytes), "r"(smem_addr(bar)), "l"(pol)
        : "memory");
}
__device__ __forceinline__ uint64_t l2_evict_first_policy() {
    uint64_t pol;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
    return pol;
}

// Programmatic dependent launch: let the next kernel in the stream start its
// prologue, and wait for the previous kernel's results before reading them.
__device__ __forceinline__ void pdl_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// Launch with programmatic dependent launch allowed: the kernel may be
// scheduled while its predecessor in the stream is still running, so every
// kernel launched this way calls pdl_wait() before it reads anything a
// predecessor wrote (griddepcontrol.wait returns once the previous grid has
// completed and its writes are visible).
template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                              Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr;
    attr.id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr.val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = &attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, args...);
}

// L2 prefetch of one cache line (weights that do not depend on a predecessor).
__device__ __forceinline__ void prefetch_l2(const void* p) {
    asm volatile("prefetch.global.L2 [%0];" ::"l"(p));
}

// Every thread of the grid prefetches its share of the ranges' 128-byte lines
// into L2 with the evict-last priority, so they survive the KV streaming of an
// attention launch in between. Weights never depend on an earlier kernel, so
// this runs before griddepcontrol.wait.
__device__ __forceinline__ void prefetch_l2_ranges(const L2Range (&r)[2]) {
    const size_t tid = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
    const size_t step = (size_t)gridDim.x * blockDim.x * 128;
#pragma unroll
    for (int i = 0; i < 2; ++i) {
        if (!r[i].p) continue;
        const char* base = static_cast<const char*>(r[i].p);
        for (size_t off = tid * 128; off < r[i].bytes; off += step)
            asm volatile("prefetch.global.L2::evict_last [%0];" ::"l"(base + off));
    }
}

}  // namespace zc
