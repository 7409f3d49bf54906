// Device helpers shared by the kernels of the path.
#pragma once
#include <cuda_runtime.h>
#include <cstdint>

namespace llmx {

static __device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
static __device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// a: two signed int16 (low half = even k); b: bytes; .lo uses bytes 0,1 (unsigned)
static __device__ __forceinline__ int dp2a_lo_su(uint32_t a, uint32_t b, int c) {
    int d;
    asm("dp2a.lo.s32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}
// .hi uses bytes 2,3 (signed)
static __device__ __forceinline__ int dp2a_hi_ss(uint32_t a, uint32_t b, int c) {
    int d;
    asm("dp2a.hi.s32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}
static __device__ __forceinline__ uint4 ld_stream(const uint4 *p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}
static __device__ __forceinline__ int32_t add_sat(int32_t a, int32_t b) {
    int32_t d;
    asm("add.sat.s32 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
}
static __device__ __forceinline__ int64_t shfl_xor64(int64_t v, int o) {
    return __shfl_xor_sync(0xffffffffu, v, o);
}


// Bulk L2 prefetch (cp.async.bulk.prefetch.L2) of slice `part` of `parts` equal,
// 16-byte aligned slices of [p, p + n): p 16-byte aligned, n a multiple of 16.
constexpr unsigned kPrefetchChunk = 64 * 1024;  // bytes per prefetch instruction
static __device__ __forceinline__ void l2_prefetch_slice(const char *p, unsigned long long n, unsigned part,
                                                         unsigned parts) {
    const unsigned long long per = ((n + parts - 1) / parts + 15) & ~15ull;
    const unsigned long long b0 = part * per, b1 = min(b0 + per, n);
    for (unsigned long long b = b0; b < b1; b += kPrefetchChunk) {
        const unsigned c = (unsigned)min((unsigned long long)kPrefetchChunk, b1 - b);
        asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p + b), "r"(c) : "memory");
    }
}

static __device__ __forceinline__ int32_t lo16(uint32_t w) { return (int32_t)(int16_t)(w & 0xffffu); }
static __device__ __forceinline__ int32_t hi16(uint32_t w) { return (int32_t)(int16_t)(w >> 16); }
// product of a Q8.8 (or raw Q2.14 payload) value and a Q4.12 value rounded to
// Q16.16 on its own (golden_accum_t(a * weight), host:3249-3252 / 3719-3722)
static __device__ __forceinline__ int32_t qk_prod(int32_t q, int32_t k) { return (q * k + 8) >> 4; }
// Q8.8 -> Q4.12 with saturation (golden_weight_t(fm))
static __device__ __forceinline__ int32_t q412(int32_t fm) {
    const int32_t v = fm * 16;
    return v > 32767 ? 32767 : (v < -32768 ? -32768 : v);
}

cudaError_t launch_pdl(const void *fn, dim3 grid, dim3 block, void **args, cudaStream_t s);

}  // namespace llmx
