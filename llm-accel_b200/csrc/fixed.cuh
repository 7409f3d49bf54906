// Fixed-point arithmetic of the resident decoder-layer path, device side.
//
// The formats and rounding rules are those of include/datatypes.hpp:8-15 in
// the LLM-ACCEL tree (ap_fixed with AP_RND / AP_SAT):
//   Q8.8 activations (int16), Q4.12 weights (int16), Q16.16 accumulators
//   (int32), Q2.14 softmax probabilities (int16).
// AP_RND dropping k fraction bits is floor(v / 2^k + 1/2); AP_SAT clamps.
#pragma once
#include <cstdint>

namespace llmx {

__host__ __device__ __forceinline__ int64_t rnd(int64_t v, int k) {
    return (v + ((int64_t)1 << (k - 1))) >> k;
}
__host__ __device__ __forceinline__ int32_t sat32(int64_t v) {
    return v > INT32_MAX ? INT32_MAX : (v < INT32_MIN ? INT32_MIN : (int32_t)v);
}
__host__ __device__ __forceinline__ int32_t sat16(int64_t v) {
    return v > 32767 ? 32767 : (v < -32768 ? -32768 : (int32_t)v);
}
// Exact MAC total -> Q16.16 (rnd4, sat) -> Q8.8 (rnd8, sat):
// kernel/mm_stream_8x64_fused_mac.cpp:89-96 + compute_core_8x64_unified.cpp:31-35.
// The ap_int<48> total is sign-extended from 48 bits first (never reached).
__host__ __device__ __forceinline__ int32_t round_mac(int64_t s) {
    s = (int64_t)((uint64_t)s << 16) >> 16;
    const int32_t acc = sat32(rnd(s, 4));
    return sat16(rnd(acc, 8));
}

// recip_approx: kernel/compute_stream.cpp:15-48 (golden_recip host:537-576).
__host__ __device__ inline int32_t recip_q88(int32_t x) {
    const int64_t safe = x < 0 ? 0 : x;
    int64_t e;
    if (safe >= 64 * 256) e = 4;
    else if (safe >= 32 * 256) e = 8;
    else if (safe >= 16 * 256) e = 16;
    else if (safe >= 8 * 256) e = 32;
    else if (safe >= 4 * 256) e = 64;
    else if (safe >= 2 * 256) e = 128;
    else if (safe >= 256) e = 256;
    else if (safe >= 128) e = 512;
    else if (safe >= 64) e = 1024;
    else if (safe >= 32) e = 2048;
    else e = 4096;
#pragma unroll
    for (int i = 0; i < 3; i++) e = sat16(rnd(e * (2 * 65536 - safe * e), 16));
    return e < 0 ? 0 : (e > 64 * 256 ? 64 * 256 : (int32_t)e);
}

// rsqrt_approx: kernel/compute_stream.cpp:57-86 (golden_rsqrt host:621-656).
// 0.5*safe*square needs up to 77 bits; it is formed as a 128-bit product.
__host__ __device__ inline int32_t rsqrt_q1616(int32_t x) {
    const int64_t safe = x < 16 ? 16 : x;
    int64_t e;
    if (safe >= ((int64_t)64 << 16)) e = 32;
    else if (safe >= ((int64_t)16 << 16)) e = 64;
    else if (safe >= ((int64_t)4 << 16)) e = 128;
    else if (safe >= ((int64_t)1 << 16)) e = 256;
    else if (safe >= 16384) e = 512;
    else if (safe >= 4096) e = 1024;
    else e = 2048;
    for (int i = 0; i < 3; i++) {
        const int64_t ea = e * 256;
        const int64_t square = sat32(rnd(ea * ea, 16));
        // t = 1.5*2^48 - 2^15 * safe * square, rounded by 2^32 and saturated.
        // safe*square < 2^62; split the 2^15 factor to stay in 128 bits.
        const __int128 t = ((__int128)3 << 47) - (((__int128)(safe * square)) << 15);
        const __int128 r = (t + ((__int128)1 << 31)) >> 32;
        const int64_t refine = r > INT32_MAX ? INT32_MAX : (r < INT32_MIN ? INT32_MIN : (int64_t)r);
        e = sat16(rnd(ea * refine, 24));
    }
    return e < 0 ? 0 : (e > 32 * 256 ? 32 * 256 : (int32_t)e);
}

// RMSNorm scalar chain of stream_rmsnorm kernel/compute_stream.cpp:227-288:
// sum (saturating; order-free because every term is >= 0), mean = sum*recip(fm(n)),
// inv_rms = rsqrt(mean + accum(1e-6)); accum(1e-6) rounds to raw 0.
__host__ __device__ inline int32_t inv_rms_q88(int32_t sum_sq, int32_t inv_elems_q88) {
    const int32_t mean = sat32(rnd((int64_t)sum_sq * ((int64_t)inv_elems_q88 * 256), 16));
    return rsqrt_q1616(mean);
}
__host__ __device__ inline int32_t fm_from_count(int n) { return n >= 128 ? 32767 : n * 256; }

// floor(2^32 / s) for 16 <= s < 2^31 (the quotient of accum(1) / safe_sum,
// host:3727-3730: (1.0 << 16) / s with 16 fraction bits, truncated)
__host__ __device__ __forceinline__ uint32_t recip_q16(int32_t s) {
    const uint32_t u = (uint32_t)s;
    return 0xffffffffu / u + ((u & (u - 1)) == 0 ? 1u : 0u);
}

}  // namespace llmx
