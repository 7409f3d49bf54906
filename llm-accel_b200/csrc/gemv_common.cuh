// Device pieces shared by the projection kernels: mbarrier / bulk-copy
// primitives of the weight ring, exact int16 x int16 dot products on the dp2a
// pipe, warp reductions and the SiLU x up epilogue.
#pragma once
#include <cuda_runtime.h>

#include "device_util.cuh"
#include "fixed.cuh"
#include "kernels.cuh"

namespace llmx {

constexpr int kMaxStages = 32;
constexpr uint32_t kSpinLimit = 1u << 26;           // bounded mbarrier waits (seconds of polling)

// ---- mbarrier / bulk-copy primitives ---------------------------------------
static __device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}
static __device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
static __device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}
static __device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
static __device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
// Bounded wait: false when the limit expired (the caller records an error).
static __device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity) {
    for (uint32_t i = 0; i < kSpinLimit; i++)
        if (mbar_try_wait(bar, parity)) return true;
    return false;
}
// Bounded wait that also gives up as soon as any CTA has recorded an error.
static __device__ __forceinline__ bool mbar_wait_err(uint64_t *bar, uint32_t parity, const int *err) {
    for (uint32_t i = 0; i < kSpinLimit; i++) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((i & 255u) == 255u && *reinterpret_cast<const volatile int *>(err) != 0) return false;
    }
    return false;
}
static __device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     smem_u32(dst)),
                 "l"(src), "r"(bytes), "r"(smem_u32(bar))
                 : "memory");
}
// Weight copies that should not displace what the kernels re-read from L2
// (KV cache, activations): the weight stream is read once per step.
static __device__ __forceinline__ uint64_t evict_first_policy() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}
static __device__ __forceinline__ void bulk_g2s_hint(void *dst, const void *src, uint32_t bytes, uint64_t *bar,
                                                     uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}
// ---- peer all-reduce words (layout and tags: ArPeers in kernels.cuh) -------
static __device__ __forceinline__ uint64_t ar_pack(int64_t sum, uint32_t tag) {
    return ((uint64_t)sum << 16) | (tag & 0xffffu);
}
static __device__ __forceinline__ int64_t ar_value(uint64_t w) { return (int64_t)w >> 16; }
static __device__ __forceinline__ void ar_store(uint64_t *p, uint64_t w) {
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}
static __device__ __forceinline__ uint64_t ar_load(const uint64_t *p) {
    uint64_t w;
    asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(w) : "l"(p) : "memory");
    return w;
}
static __device__ __forceinline__ void ar_load2(const uint64_t *p, uint64_t &a, uint64_t &b) {
    asm volatile("ld.relaxed.sys.global.v2.u64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(p) : "memory");
}
// Exact sums of elements (r, e..e+3) over every rank's contribution to
// all-reduce (slot, tag), read from this rank's exchange region; e a multiple
// of 4.  The 16-byte loads of up to four ranks are in flight before any tag is
// checked (one round trip up to 4 ranks, two at 8).
// Each word is waited for at most ar.poll_limit polls; false when one did not
// arrive (or when *fail was set by another thread of the block, so that a
// block gives up once).
static __device__ __forceinline__ bool ar_gather4(const ArPeers &ar, int slot, uint32_t tag, int r, int e,
                                                  const volatile int *fail, int64_t (&sum)[4]) {
    constexpr int PB = 4;  // ranks per round trip
    const uint64_t *words = reinterpret_cast<const uint64_t *>(ar.base[ar.me] + kArHeader);
#pragma unroll
    for (int j = 0; j < 4; j++) sum[j] = 0;
    for (int p0 = 0; p0 < ar.n; p0 += PB) {
        uint64_t w[PB][4];
#pragma unroll
        for (int b = 0; b < PB; b++)
            if (p0 + b < ar.n) {
                const uint64_t *q = words + ar_word_index(slot, p0 + b, r, ar.hidden, e);
                ar_load2(q, w[b][0], w[b][1]);
                ar_load2(q + 2, w[b][2], w[b][3]);
            }
#pragma unroll
        for (int b = 0; b < PB; b++) {
            if (p0 + b >= ar.n) break;
#pragma unroll
            for (int j = 0; j < 4; j++) {
                for (uint32_t it = 0; (uint32_t)(w[b][j] & 0xffffu) != tag; it++) {
                    if (it >= ar.poll_limit || *fail) return false;
                    __nanosleep(64);
                    const uint64_t *q = words + ar_word_index(slot, p0 + b, r, ar.hidden, e + (j & ~1));
                    ar_load2(q, w[b][j & ~1], w[b][j | 1]);
                }
                sum[j] += ar_value(w[b][j]);
            }
        }
    }
    return true;
}

// Named barrier over the consumer warps (the producer warp is the last warp).
static __device__ __forceinline__ void consumer_sync() {
    asm volatile("bar.sync 1, %0;" ::"r"(blockDim.x - 32) : "memory");
}

// golden_silu host:658-668 / cu_silu_approx kernel/compute_stream.cpp:88-96,
// then x up with one rounding (stream_silu_mul :123-164).
// etab: the Q8.8 exp table in global or shared memory (generic loads).
static __device__ __forceinline__ int32_t silu_mul(int32_t g, int32_t u, const int16_t *etab) {
    int32_t s;
    if (g >= 0) {
        const int32_t e = etab[g > 2048 ? 0 : 2048 - g];
        const int32_t r = recip_q88(sat16(256 + e));
        s = sat16(rnd((int64_t)g * r, 8));
    } else {
        const int32_t e = etab[g < -2048 ? 0 : g + 2048];
        const int32_t r = recip_q88(sat16(256 + e));
        s = sat16(rnd((int64_t)g * e * r, 16));
    }
    return sat16(rnd((int64_t)s * u, 8));
}

// Halving ("transpose") warp reduction of N int64 values: afterwards lane L
// holds the warp total of value index idx(L); lanes that differ only in the
// bits below 32/N hold the same index.  N <= 16.
template <int N>
static __device__ __forceinline__ int64_t warp_reduce_n(int64_t (&v)[N], int lane, int &idx) {
    idx = 0;
#pragma unroll
    for (int n = N, o = 16; n > 1; n >>= 1, o >>= 1) {
        const bool up = (lane & o) != 0;
#pragma unroll
        for (int i = 0; i < n / 2; i++) {
            const int64_t send = up ? v[i] : v[i + n / 2];
            const int64_t keep = up ? v[i + n / 2] : v[i];
            v[i] = keep + shfl_xor64(send, o);
        }
        if (up) idx += n / 2;
    }
    int64_t t = v[0];
#pragma unroll
    for (int o = 16 / N; o >= 1; o >>= 1) t += shfl_xor64(t, o);
    return t;
}

// One unit's dot products against R activation rows, accumulated exactly.
// VPL > 0: K == 256 * VPL, every lane takes VPL 16-byte vectors per row (fully
// unrolled, no predicates; K = 2048 -> 8, K = 11008 -> 43); VPL == 0: any K,
// 16-vector chunks.  The int32 partials are flushed to int64 every 16 vectors:
//   |lo| <= 16*8*255*32768 < 2^30, |hi| <= 16*8*128*32768 = 2^29 per flush.
// P > 1: the unit is shared by P warps; warp `part` takes every P-th group of
// 32 vectors, and the P partial sums are added afterwards (exact int64).
template <int R, int U, int VPL, int P>
static __device__ __forceinline__ void unit_dots(const uint4 *__restrict__ wv, const uint4 *__restrict__ xs4,
                                                 const uint4 (&xr)[8], int KV8, int lane, int part,
                                                 int64_t (&acc)[U * R]) {
    constexpr int N = U * R;
#pragma unroll
    for (int i = 0; i < N; i++) acc[i] = 0;
    if constexpr (VPL > 0) {
        int lo[N], hi[N];
#pragma unroll
        for (int i = 0; i < N; i++) lo[i] = hi[i] = 0;
        constexpr int KI = ((VPL > 0 ? VPL : 1) + P - 1) / P;  // vector groups of this warp
#pragma unroll
        for (int ki = 0; ki < KI; ki++) {
            const int k = P == 1 ? ki : ki * P + part;
            if (P > 1 && ki == KI - 1 && k >= VPL) break;
            if (ki > 0 && ki % 16 == 0) {  // flush the int32 partials every 16 vectors
#pragma unroll
                for (int i = 0; i < N; i++) {
                    acc[i] += (int64_t)hi[i] * 256 + lo[i];
                    lo[i] = hi[i] = 0;
                }
            }
            const int v = k * 32 + lane;
            uint4 w[U];
#pragma unroll
            for (int u = 0; u < U; u++) w[u] = wv[u * KV8 + v];
#pragma unroll
            for (int r = 0; r < R; r++) {
                const uint4 x = (R == 1 && VPL <= 8 && P == 1) ? xr[k < 8 ? k : 0] : xs4[r * KV8 + v];
#pragma unroll
                for (int u = 0; u < U; u++) {
                    const int i = r * U + u;
                    lo[i] = dp2a_lo_su(x.x, w[u].x, lo[i]);
                    hi[i] = dp2a_hi_ss(x.x, w[u].x, hi[i]);
                    lo[i] = dp2a_lo_su(x.y, w[u].y, lo[i]);
                    hi[i] = dp2a_hi_ss(x.y, w[u].y, hi[i]);
                    lo[i] = dp2a_lo_su(x.z, w[u].z, lo[i]);
                    hi[i] = dp2a_hi_ss(x.z, w[u].z, hi[i]);
                    lo[i] = dp2a_lo_su(x.w, w[u].w, lo[i]);
                    hi[i] = dp2a_hi_ss(x.w, w[u].w, hi[i]);
                }
            }
        }
#pragma unroll
        for (int i = 0; i < N; i++) acc[i] += (int64_t)hi[i] * 256 + lo[i];
    } else {
    for (int v0 = part * 32; v0 < KV8; v0 += 16 * 32 * P) {
        int lo[N], hi[N];
#pragma unroll
        for (int i = 0; i < N; i++) lo[i] = hi[i] = 0;
#pragma unroll 4
        for (int k = 0; k < 16; k++) {
            const int v = v0 + k * 32 * P + lane;
            if (v < KV8) {
                uint4 w[U];
#pragma unroll
                for (int u = 0; u < U; u++) w[u] = wv[u * KV8 + v];
#pragma unroll
                for (int r = 0; r < R; r++) {
                    const uint4 x = xs4[r * KV8 + v];
#pragma unroll
                    for (int u = 0; u < U; u++) {
                        const int i = r * U + u;
                        lo[i] = dp2a_lo_su(x.x, w[u].x, lo[i]);
                        hi[i] = dp2a_hi_ss(x.x, w[u].x, hi[i]);
                        lo[i] = dp2a_lo_su(x.y, w[u].y, lo[i]);
                        hi[i] = dp2a_hi_ss(x.y, w[u].y, hi[i]);
                        lo[i] = dp2a_lo_su(x.z, w[u].z, lo[i]);
                        hi[i] = dp2a_hi_ss(x.z, w[u].z, hi[i]);
                        lo[i] = dp2a_lo_su(x.w, w[u].w, lo[i]);
                        hi[i] = dp2a_hi_ss(x.w, w[u].w, hi[i]);
                    }
                }
            }
        }
#pragma unroll
        for (int i = 0; i < N; i++) acc[i] += (int64_t)hi[i] * 256 + lo[i];
    }
    }
}


}  // namespace llmx
