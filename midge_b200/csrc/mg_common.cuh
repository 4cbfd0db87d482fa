// mg_common.cuh -- shared device helpers for the sm_100a MoE hot path.
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "midgecuda.h"

namespace mg {

// ------------------------------------------------------------ error state
// Host-side: the last error message (thread-local) and a status code.
void set_error(const char *fmt, ...);
#define MG_CUDA(call)                                                                       \
    do {                                                                                    \
        cudaError_t _e = (call);                                                            \
        if (_e != cudaSuccess) {                                                            \
            ::mg::set_error("%s:%d %s: %s", __FILE__, __LINE__, #call, cudaGetErrorString(_e)); \
            return MG_ERR_CUDA;                                                             \
        }                                                                                   \
    } while (0)
#define MG_CHECK_LAUNCH() MG_CUDA(cudaGetLastError())
#define TRY(expr)                     \
    do {                              \
        int _rc = (expr);             \
        if (_rc != MG_OK) return _rc; \
    } while (0)
#define MG_REQUIRE(cond, code, ...)          \
    do {                                     \
        if (!(cond)) {                       \
            ::mg::set_error(__VA_ARGS__);    \
            return (code);                   \
        }                                    \
    } while (0)

// ------------------------------------------------------------ numerics
// ue8m0 scale byte -> float.  Code 0 is reserved for an exact zero scale (an
// f16 scale can never be 2^-127, so no real code collides with it).
__device__ __forceinline__ float ue8m0_to_f32(uint32_t u) { return __uint_as_float(u << 23); }

// IEEE half bits -> float (exact; hardware conversion).
__device__ __forceinline__ float h2f(uint16_t h) { return __half2float(__ushort_as_half(h)); }

// float -> half, round to nearest even, subnormal results flushed to signed
// zero, overflow to infinity: the KV-cache store of engine/mkern.h:261-273.
// Built from the hardware RNE conversion: a result below the smallest normal
// half (2^-14) is replaced by zero; values whose RNE result is the smallest
// normal stay.  Rounding of a value just below 2^-14 that RNE would carry up
// into 2^-14 matches the reference, which also rounds the mantissa first.
__device__ __forceinline__ uint16_t f2h_ftz(float f) {
    uint32_t x = __float_as_uint(f);
    uint32_t sign = (x >> 16) & 0x8000u;
    int e = (int)((x >> 23) & 0xff) - 112;  // half exponent field before rounding
    if (e <= 0) return (uint16_t)sign;       // the reference flushes on the pre-rounding exponent
    if (e >= 31) return (uint16_t)(sign | 0x7c00u);  // includes NaN, which the reference maps to inf
    return __half_as_ushort(__float2half_rn(f));
}

// fp32 -> f16 hi/lo pair with hi + lo == x to ~22 significant bits.
__device__ __forceinline__ void split_f16(float x, __half &hi, __half &lo) {
    hi = __float2half_rn(x);
    lo = __float2half_rn(x - __half2float(hi));
}

__device__ __forceinline__ uint32_t pack_h2(__half a, __half b) {
    return (uint32_t)__half_as_ushort(a) | ((uint32_t)__half_as_ushort(b) << 16);
}

// two e2m1 codes (one byte, low nibble first) -> f16x2, exact
__device__ __forceinline__ uint32_t e2m1x2_to_h2(uint32_t byte) {
    uint32_t r;
    asm("{\n .reg .b8 b;\n cvt.u8.u32 b, %1;\n cvt.rn.f16x2.e2m1x2 %0, b;\n}" : "=r"(r) : "r"(byte));
    return r;
}

// four e2m1 byte pairs of a word -> four f16x2 (byte i -> out[i])
__device__ __forceinline__ void e2m1x8_to_h2(uint32_t w, uint32_t out[4]) {
    asm("{\n .reg .b8 b0, b1, b2, b3;\n mov.b32 {b0, b1, b2, b3}, %4;\n"
        " cvt.rn.f16x2.e2m1x2 %0, b0;\n cvt.rn.f16x2.e2m1x2 %1, b1;\n"
        " cvt.rn.f16x2.e2m1x2 %2, b2;\n cvt.rn.f16x2.e2m1x2 %3, b3;\n}"
        : "=r"(out[0]), "=r"(out[1]), "=r"(out[2]), "=r"(out[3])
        : "r"(w));
}

// four signed int8 of a word -> two f16x2: (b0,b1) and (b2,b3), exact.
// Each byte is biased to unsigned, placed under the half exponent of 1024
// (unit spacing), and 1024+128 subtracted.
__device__ __forceinline__ void s8x4_to_h2(uint32_t w, uint32_t &lo, uint32_t &hi) {
    uint32_t u = w ^ 0x80808080u;
    uint32_t a = __byte_perm(u, 0x64646464u, 0x5140);
    uint32_t b = __byte_perm(u, 0x64646464u, 0x7362);
    const __half2 bias = __halves2half2(__ushort_as_half(0x6480), __ushort_as_half(0x6480));
    __half2 ha = __hsub2(*reinterpret_cast<__half2 *>(&a), bias);
    __half2 hb = __hsub2(*reinterpret_cast<__half2 *>(&b), bias);
    lo = *reinterpret_cast<uint32_t *>(&ha);
    hi = *reinterpret_cast<uint32_t *>(&hb);
}

// nibble pairs (i, i+4) of a word as unsigned 4-bit ints minus 8 -> f16x2, exact
__device__ __forceinline__ uint32_t u4pair_minus8_h2(uint32_t w_shifted) {
    uint32_t t = (w_shifted & 0x000F000Fu) | 0x64006400u;
    const __half2 bias = __halves2half2(__ushort_as_half(0x6408), __ushort_as_half(0x6408));
    __half2 h = __hsub2(*reinterpret_cast<__half2 *>(&t), bias);
    return *reinterpret_cast<uint32_t *>(&h);
}

// D(16x8 f32) += A(16x16 f16) * B(16x8 f16)
__device__ __forceinline__ void mma_16816(float d[4], const uint32_t a[4], uint32_t b0, uint32_t b1) {
    asm(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};\n"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t ldg_nc_u32(const void *p) {
    uint32_t v;
    asm("ld.global.nc.L1::no_allocate.b32 %0, [%1];" : "=r"(v) : "l"(p));
    return v;
}
__device__ __forceinline__ uint4 ldg_nc_u128(const void *p) {
    uint4 v;
    asm("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}
__device__ __forceinline__ uint32_t ldg_u32_l1(const void *p) {
    uint32_t v;
    asm("ld.global.nc.b32 %0, [%1];" : "=r"(v) : "l"(p));
    return v;
}

// ------------------------------------------------ async copies and mbarriers
__device__ __forceinline__ uint32_t smem_u32(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
// Bounded wait on an mbarrier phase: false if it did not complete within the
// poll budget (each try_wait also suspends for a hardware-defined interval).
constexpr uint32_t MBAR_POLLS = 1u << 22;
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity) {
    for (uint32_t i = 0; i < MBAR_POLLS; i++)
        if (mbar_try_wait(bar, parity)) return true;
    return false;
}
// global -> shared bulk copy completing on an mbarrier (16 B aligned, size % 16 == 0)
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     smem_u32(dst)),
                 "l"(src), "r"(bytes), "r"(smem_u32(bar))
                 : "memory");
}
__device__ __forceinline__ void named_bar_sync(int id, int nthreads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}
__device__ __forceinline__ uint32_t lds32(const void *p) { return *reinterpret_cast<const uint32_t *>(p); }

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// Block-wide sum (blockDim.x multiple of 32, <= 1024); scratch >= 32 floats.
__device__ __forceinline__ float block_sum(float v, float *scratch) {
    int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
    v = warp_sum(v);
    __syncthreads();
    if (lane == 0) scratch[wid] = v;
    __syncthreads();
    float t = lane < nw ? scratch[lane] : 0.f;
    t = warp_sum(t);
    return t;
}

inline int ceil_div(int64_t a, int64_t b) { return (int)((a + b - 1) / b); }

// Programmatic dependent launch.  pdl_trigger: the next grid on the stream,
// when launched with the programmatic attribute, may start once every CTA of
// this grid has triggered or exited.  pdl_wait: blocks until the previous grid
// has completed and its memory operations are visible (returns at once when
// this grid was launched without the attribute).  A dependent reads nothing
// the previous grid (or a grid still running before it) writes, and writes
// nothing, before its wait; and it waits in every CTA, so that its completion
// implies the previous grid's for the normally launched kernels after it.
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// Launch with the programmatic-serialization attribute when pdl is set.
template <typename... KArgs, typename... Args>
inline cudaError_t launch_k(bool pdl, void (*kfn)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                            Args... args) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kfn, args...);
}

// Number of SMs of the current device (cached per device).
int num_sms();

// Raise a kernel's dynamic shared memory limit once per (kernel, device).
// Keyed by the kernel's address: template instances of one signature are
// different kernels.
int ensure_smem_attr(const void *fn, size_t bytes);
template <typename K>
inline int ensure_smem(K kfn, size_t bytes) {
    return ensure_smem_attr(reinterpret_cast<const void *>(kfn), bytes);
}

}  // namespace mg
